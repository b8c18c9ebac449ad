// Exact SIMT search + blend.  One CTA per frame; the scan is split across
// "octets" (8 consecutive threads) that each compute one row's squared
// distance in the reference's AVX2 order.  This is the engine for
// VFR_ENGINE_EXACT, the re-run path for frames the tensor-core candidate
// stage cannot certify, and the coarse stage of small IVF indexes.
//
// It reproduces crates/vocal-cpu/src/retrieval.rs:27-83:
//   coarse: every centroid's distance, ordered by (total_cmp, list id), first
//           nprobe lists (retrieval.rs:45-51);
//   scan:   probed lists in coarse order, rows in storage order, top-8 where a
//           distance tie keeps the earlier-scanned row (:52-64) -- expressed
//           as the total order on (distance, scan position), so the parallel
//           split cannot change the result;
//   blend:  f64 weights and f32 blend (:65-81).
// Differences taken from the reference CUDA kernels (retrieval_block.cuh):
// a frame with no candidate keeps its query, index_rate is clamped to [0,1]
// and r <= 0 leaves the frame untouched.
#include <stdexcept>
#include <string>

#include "exact_common.cuh"
#include "kernels.h"
#include "pdl.cuh"

namespace vfr {
namespace {

constexpr int kThreads = 256;
constexpr int kOctets = kThreads / 8;

__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        unsigned long long o = __shfl_xor_sync(kFullMask, v, s);
        v = o < v ? o : v;
    }
    return v;
}

// Bitonic sort of one u64 per lane, ascending across lanes 0..31.
__device__ __forceinline__ unsigned long long warp_sort_u64(unsigned long long v, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            unsigned long long o = __shfl_xor_sync(kFullMask, v, j);
            bool ascending = (lane & k) == 0;
            bool lower = (lane & j) == 0;
            unsigned long long lo = o < v ? o : v, hi = o < v ? v : o;
            v = (lower == ascending) ? lo : hi;
        }
    }
    return v;
}

__device__ void exact_frame(const ExactArgs &a, const long long frame) {
    extern __shared__ float q[];  // [d] copy of the frame
    __shared__ unsigned long long probe_keys[kMaxProbe];
    __shared__ unsigned long long wave_keys[kOctets];
    __shared__ int probe_list[kMaxProbe];
    __shared__ uint32_t probe_base[kMaxProbe + 1];
    __shared__ unsigned long long octet_best[kOctets * 8];
    __shared__ unsigned long long best[8];
    __shared__ int32_t best_row[8];
    __shared__ double weights[8];
    __shared__ double weight_sum;

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int octet = tid >> 3;
    const int j = tid & 7;
    const int octet_base = lane & ~7;
    const int d = a.d;
    const float *src = a.queries + frame * d;
    float *dst = a.out + frame * d;

    if (tid == 0 && a.frame_list && a.counters) atomicAdd(&a.counters->fallback_frames, 1ull);
    float ratio = 1.0f;
    if (a.mode == kModeBlend) {
        ratio = load_ratio(a.index_rate);
        if (!(ratio > 0.0f)) {
            if (dst != src)
                for (int i = tid; i < d; i += kThreads) dst[i] = src[i];
            return;
        }
    }
    for (int i = tid; i < d; i += kThreads) q[i] = src[i];
    __syncthreads();

    // ---- coarse stage ---------------------------------------------------
    int probes = a.nprobe < a.nlist ? a.nprobe : a.nlist;
    if (a.nlist == 1) {
        if (tid == 0) probe_list[0] = 0;
        probes = 1;
    } else {
        if (tid < kMaxProbe) probe_keys[tid] = kEmptyKey;
        __syncthreads();
        for (int base = 0; base < a.nlist; base += kOctets) {
            const int list = base + octet;
            const int clamped = list < a.nlist ? list : a.nlist - 1;
            float dist = octet_l2(q, a.centroids + static_cast<size_t>(clamped) * d, d, j, octet_base, kFullMask);
            if (j == 0) wave_keys[octet] = list < a.nlist ? make_key(dist, static_cast<uint32_t>(list)) : kEmptyKey;
            __syncthreads();
            if (warp == 0) {
                // merge the sorted running top-`probes` with this wave's keys
                unsigned long long nk = warp_sort_u64(wave_keys[lane], lane);
                unsigned long long ok = lane < probes ? probe_keys[lane] : kEmptyKey;
                int rank_new = 0, rank_old = 0;
                for (int i = 0; i < probes; ++i) rank_new += probe_keys[i] < nk;
                for (int i = 0; i < 32; ++i) {
                    unsigned long long other = __shfl_sync(kFullMask, nk, i);
                    rank_old += other <= ok;
                }
                __syncwarp();
                int pn = lane + rank_new;
                int po = lane + rank_old;
                if (pn < probes) probe_keys[pn] = nk;
                if (lane < probes && po < probes) probe_keys[po] = ok;
            }
            __syncthreads();
        }
        if (tid < probes) probe_list[tid] = static_cast<int>(key_pos(probe_keys[tid]));
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0;
        for (int r = 0; r < probes; ++r) {
            probe_base[r] = acc;
            acc += static_cast<uint32_t>(a.offsets[probe_list[r] + 1] - a.offsets[probe_list[r]]);
        }
        probe_base[probes] = acc;
    }
    __syncthreads();

    // ---- list scan ------------------------------------------------------
    Top8 top;
    top.init();
    for (int r = 0; r < probes; ++r) {
        const int list = probe_list[r];
        const int begin = a.offsets[list];
        const int end = a.offsets[list + 1];
        const uint32_t base = probe_base[r];
        for (int row0 = begin; row0 < end; row0 += 4 * kOctets) {
            const float *xs[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int row = row0 + octet + k * kOctets;
                xs[k] = a.vectors + static_cast<size_t>(row < end ? row : begin) * d;
            }
            float dist[4];
            octet_l2n<4>(q, xs, d, j, octet_base, kFullMask, dist);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int row = row0 + octet + k * kOctets;
                // the reference never admits +inf (best starts at +inf, `>=` rejects)
                if (row < end && dist[k] < __int_as_float(0x7f800000))
                    top.insert(make_key(dist[k], base + static_cast<uint32_t>(row - begin)));
            }
        }
    }
    if (j == 0)
#pragma unroll
        for (int i = 0; i < 8; ++i) octet_best[octet * 8 + i] = top.k[i];
    __syncthreads();
    if (warp == 0) {
        int head = 0;
        for (int i = 0; i < 8; ++i) {
            unsigned long long mine = head < 8 ? octet_best[lane * 8 + head] : kEmptyKey;
            unsigned long long m = warp_min_u64(mine);
            if (mine == m && m != kEmptyKey) ++head;
            if (lane == 0) best[i] = m;
        }
        if (lane < 8) {
            unsigned long long key = best[lane];
            int32_t row = -1;
            if (key != kEmptyKey) {
                uint32_t pos = key_pos(key);
                int r = 0;
                while (r + 1 < probes && probe_base[r + 1] <= pos) ++r;
                row = a.offsets[probe_list[r]] + static_cast<int32_t>(pos - probe_base[r]);
            }
            best_row[lane] = row;
        }
    }
    __syncthreads();
    int count = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) count += best_row[i] >= 0;

    if (a.mode == kModeSearch) {
        if (tid < a.k) {
            const bool have = tid < count;
            a.dist_out[frame * a.k + tid] = have ? key_dist(best[tid]) : __int_as_float(0x7f800000);
            a.label_out[frame * a.k + tid] = have ? static_cast<int64_t>(a.ids[best_row[tid]]) + a.label_base : -1;
        }
        return;
    }
    if (count == 0) {
        if (tid == 0 && a.counters) atomicAdd(&a.counters->empty_frames, 1ull);
        if (dst != src)
            for (int i = tid; i < d; i += kThreads) dst[i] = q[i];
        return;
    }
    if (tid == 0) {
        float dist[8];
        double w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) dist[i] = key_dist(best[i]);
        weight_sum = reference_weights(dist, count, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) weights[i] = w[i];
    }
    __syncthreads();
    double w[8];
    int32_t rows[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        w[i] = weights[i];
        rows[i] = best_row[i];
    }
    const WeightDivisor sum = weight_divisor(weight_sum);
    for (int i = tid; i < d; i += kThreads) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = k < count ? __ldg(a.vectors + static_cast<size_t>(rows[k]) * d + i) : 0.f;
        dst[i] = reference_blend_element(q[i], v, w, sum, count, ratio);
    }
}

// One CTA per frame, or, with a device frame list (the frames the
// tensor-core engine could not certify), a fixed grid striding over it.
__global__ void __launch_bounds__(kThreads) exact_kernel(ExactArgs a) {
    grid_dependency_wait();  // the frame list and the outputs belong to the kernel before
    if (a.frame_list) {
        const int count = *a.frame_count;
        for (int i = blockIdx.x; i < count; i += gridDim.x) {
            exact_frame(a, a.frame_list[i]);
            __syncthreads();
        }
    } else {
        exact_frame(a, blockIdx.x);
    }
}

}  // namespace

void launch_exact(const ExactArgs &args, long long frames, cudaStream_t stream, bool after_kernel) {
    if (frames <= 0) return;
    size_t smem = static_cast<size_t>(args.d) * sizeof(float);
    unsigned grid = static_cast<unsigned>(frames);
    if (args.frame_list) grid = static_cast<unsigned>(frames < 1184 ? frames : 1184);
    if (after_kernel) {
        const cudaError_t rc = launch_pdl(exact_kernel, dim3(grid), dim3(kThreads), smem, stream, args);
        if (rc != cudaSuccess) throw std::runtime_error(std::string("exact kernel launch: ") + cudaGetErrorString(rc));
    } else {
        exact_kernel<<<grid, kThreads, smem, stream>>>(args);
    }
}

}  // namespace vfr
