// Row-sharded multi-GPU building blocks.  Each GPU holds a contiguous slice of
// the database rows and returns its exact top-8 with global labels; after an
// all-gather of those lists the k-way merge below reproduces the single-GPU
// scan order, (distance, global row).  The blend then needs the winning
// vectors, which live on their owners: every shard writes the vectors it owns
// and -0.0 elsewhere, so a sum over shards (a reduce-scatter) delivers each
// vector bit-exactly (x + -0.0 == x for every x, including -0.0).
#include "exact_common.cuh"
#include "kernels.h"

namespace vfr {
namespace {

__global__ void merge_topk_kernel(const float *__restrict__ dist, const int64_t *__restrict__ labels, int shards,
                                  long long frames, float *__restrict__ out_dist, int64_t *__restrict__ out_labels) {
    long long f = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (f >= frames) return;
    int head[64];
    for (int s = 0; s < shards; ++s) head[s] = 0;
    for (int k = 0; k < 8; ++k) {
        int pick = -1;
        uint32_t best_bits = 0xffffffffu;
        int64_t best_label = INT64_MAX;
        for (int s = 0; s < shards; ++s) {
            if (head[s] >= 8) continue;
            size_t at = (static_cast<size_t>(s) * frames + f) * 8 + head[s];
            int64_t label = labels[at];
            if (label < 0) continue;  // shard list exhausted
            uint32_t bits = total_order_bits(dist[at]);
            if (bits < best_bits || (bits == best_bits && label < best_label)) {
                best_bits = bits;
                best_label = label;
                pick = s;
            }
        }
        if (pick >= 0) {
            ++head[pick];
            out_dist[f * 8 + k] = from_total_order_bits(best_bits);
            out_labels[f * 8 + k] = best_label;
        } else {
            out_dist[f * 8 + k] = __int_as_float(0x7f800000);
            out_labels[f * 8 + k] = -1;
        }
    }
}

__global__ void gather_owned_kernel(const float *__restrict__ vectors, const int32_t *__restrict__ row_of_id,
                                    int64_t n, int64_t label_base, int d, const int64_t *__restrict__ labels,
                                    float *__restrict__ out) {
    const long long slot = blockIdx.x;  // frame * 8 + k
    const int64_t label = labels[slot];
    const int64_t local = label - label_base;
    const bool owned = label >= 0 && local >= 0 && local < n;
    float *dst = out + slot * d;
    if (owned) {
        const float *src = vectors + static_cast<size_t>(row_of_id[local]) * d;
        for (int i = threadIdx.x; i < d; i += blockDim.x) dst[i] = src[i];
    } else {
        for (int i = threadIdx.x; i < d; i += blockDim.x) dst[i] = -0.0f;
    }
}

// neighbours: [frames][8][d] when slot_rows is null; otherwise [rows][d],
// with slot (f, k) reading row slot_rows[f * 8 + k] (rows outside [0, rows)
// read as zero; the host never produces them for a valid slot).
__global__ void blend_gathered_kernel(const float *__restrict__ queries, float *out, const float *__restrict__ dist,
                                      const float *__restrict__ neighbours, const int32_t *__restrict__ slot_rows,
                                      long long rows, int d, const float *index_rate) {
    __shared__ double weights[8];
    __shared__ double weight_sum;
    __shared__ int count_s;
    const long long f = blockIdx.x;
    const float *src = queries + f * d;
    float *dst = out + f * d;
    const float ratio = load_ratio(index_rate);
    if (threadIdx.x == 0) {
        float dd[8];
        double w[8];
        int count = 0;
        for (int k = 0; k < 8; ++k) {
            dd[k] = dist[f * 8 + k];
            if (count == k && dd[k] < __int_as_float(0x7f800000)) ++count;
        }
        weight_sum = reference_weights(dd, count, w);
        for (int k = 0; k < 8; ++k) weights[k] = w[k];
        count_s = count;
    }
    __syncthreads();
    const int count = count_s;
    if (!(ratio > 0.0f) || count == 0) {
        if (dst != src)
            for (int i = threadIdx.x; i < d; i += blockDim.x) dst[i] = src[i];
        return;
    }
    double w[8];
    for (int k = 0; k < 8; ++k) w[k] = weights[k];
    const WeightDivisor sum = weight_divisor(weight_sum);
    const float *nb[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        long long row = f * 8 + k;
        if (slot_rows != nullptr) {
            const int32_t r = slot_rows[f * 8 + k];
            row = (r >= 0 && r < rows) ? r : -1;
        }
        nb[k] = (k < count && row >= 0) ? neighbours + row * static_cast<long long>(d) : nullptr;
    }
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = nb[k] != nullptr ? nb[k][i] : 0.f;
        dst[i] = reference_blend_element(src[i], v, w, sum, count, ratio);
    }
}

}  // namespace

void launch_merge_topk(const float *dist, const int64_t *labels, int shards, long long frames, float *out_dist,
                       int64_t *out_labels, cudaStream_t stream) {
    if (frames <= 0) return;
    const int threads = 128;
    merge_topk_kernel<<<static_cast<unsigned>((frames + threads - 1) / threads), threads, 0, stream>>>(
        dist, labels, shards, frames, out_dist, out_labels);
}

void launch_gather_owned(const float *vectors, const int32_t *row_of_id, int64_t n, int64_t label_base, int d,
                         const int64_t *labels, long long frames, float *out, cudaStream_t stream) {
    if (frames <= 0) return;
    gather_owned_kernel<<<static_cast<unsigned>(frames * 8), 128, 0, stream>>>(vectors, row_of_id, n, label_base, d,
                                                                               labels, out);
}

void launch_blend_gathered(const float *queries, float *out, const float *dist, const float *neighbours,
                           long long frames, int d, const float *index_rate, cudaStream_t stream) {
    if (frames <= 0) return;
    blend_gathered_kernel<<<static_cast<unsigned>(frames), 256, 0, stream>>>(queries, out, dist, neighbours, nullptr,
                                                                             0, d, index_rate);
}

void launch_blend_gathered_rows(const float *queries, float *out, const float *dist, const float *rows_buf,
                                const int32_t *slot_rows, long long rows, long long frames, int d,
                                const float *index_rate, cudaStream_t stream) {
    if (frames <= 0) return;
    blend_gathered_kernel<<<static_cast<unsigned>(frames), 256, 0, stream>>>(queries, out, dist, rows_buf, slot_rows,
                                                                             rows, d, index_rate);
}

}  // namespace vfr
