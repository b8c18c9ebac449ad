// Row-sharded blend over peer memory.
//
// After the all-gather and k-way merge of the per-shard top-8 lists every
// rank knows, for each of its frames, the global labels of the 8 winners;
// their fp32 rows live on the GPUs that own those shards.  Instead of
// packing the rows and exchanging them with a collective, each rank maps the
// other ranks' row arrays into its address space once (CUDA IPC; the GPUs
// of one node reach each other's HBM over NVLink / NVSwitch) and the blend
// kernel reads every winner straight from its owner with ordinary loads:
// one kernel moves the bytes and does the arithmetic, with no host wait and
// no staging buffer.  Each winner crosses NVLink once; winners this rank
// owns come from local HBM.  Loads are plain ld.global (no TMA, no
// multicast), so nothing here issues a bulk or tensor copy from another
// GPU's memory.
//
// Arithmetic: the reference's f64 weights and f32 blend
// (crates/vocal-cpu/src/retrieval.rs:65-81) through the same helpers as the
// single-GPU kernels, so the output equals a single index's bit for bit.
#include <cstring>
#include <vector>

#include "exact_common.cuh"
#include "index_build.h"
#include "peer_table.h"
#include "vfr_common.h"

namespace vfr {
namespace {

constexpr int kPeerWarps = 8;  // frames per CTA (one warp each)

__device__ __forceinline__ const float *winner_row(const PeerTable &t, int64_t label) {
    if (label < t.bounds[0] || label >= t.bounds[t.shards]) return nullptr;
    int lo = 0, hi = t.shards;  // bounds[lo] <= label < bounds[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (label >= t.bounds[mid]) lo = mid;
        else hi = mid;
    }
    const int64_t local = label - t.bounds[lo];
    const int64_t row = t.row_of_id[lo] ? static_cast<int64_t>(t.row_of_id[lo][local]) : local;
    return t.rows[lo] + row * static_cast<int64_t>(t.d);
}

// One warp per frame.  Lanes 0-7 resolve slot k = lane (distance, weight,
// owner row), the warp shares them, then every lane blends the elements
// lane, lane + 32, ... (float4 lanes when d % 4 == 0 and the rows are
// 16-byte aligned), all 8 winners' loads of an element group in flight.
template <bool kVec4>
__global__ void __launch_bounds__(32 * kPeerWarps) blend_peer_kernel(const __grid_constant__ PeerTable t,
                                                                     const float *__restrict__ queries,
                                                                     float *out, const float *__restrict__ dist,
                                                                     const int64_t *__restrict__ labels,
                                                                     long long frames, const float *index_rate) {
    const int lane = threadIdx.x & 31;
    const long long f = static_cast<long long>(blockIdx.x) * kPeerWarps + (threadIdx.x >> 5);
    if (f >= frames) return;
    const int d = t.d;
    const float *src = queries + f * d;
    float *dst = out + f * d;
    const float ratio = load_ratio(index_rate);
    // slot k on lane k: its distance (the count is the number of leading
    // finite distances, as the single-GPU merge reports them)
    const float dk = lane < 8 ? dist[f * 8 + lane] : __int_as_float(0x7f800000);
    const unsigned finite = __ballot_sync(kFullMask, lane < 8 && dk < __int_as_float(0x7f800000));
    const int count = __ffs(~finite) - 1;  // leading ones of the 8-bit mask
    if (!(ratio > 0.0f) || count == 0) {
        if (dst != src)
            for (int i = lane; i < d; i += 32) dst[i] = src[i];
        return;
    }
    const double wk = lane < count ? reference_weight(dk) : 0.0;
    const float *mine = lane < count ? winner_row(t, labels[f * 8 + lane]) : nullptr;
    double w[8];
    const float *rows[8];
    double wsum = -0.0;  // the reference's order: S = w0 + w1 + ... (zeros past count)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        w[k] = __shfl_sync(kFullMask, wk, k);
        rows[k] = reinterpret_cast<const float *>(
            __shfl_sync(kFullMask, reinterpret_cast<unsigned long long>(mine), k));
        wsum = __dadd_rn(wsum, w[k]);
    }
    // a label outside every shard (never produced by the merge) counts as
    // missing: the frame keeps its query rather than reading a wrong row
    bool ok = true;
#pragma unroll
    for (int k = 0; k < 8; ++k) ok = ok && (k >= count || rows[k] != nullptr);
    if (!ok) {
        if (dst != src)
            for (int i = lane; i < d; i += 32) dst[i] = src[i];
        return;
    }
    const WeightDivisor sum = weight_divisor(wsum);
    if constexpr (kVec4) {
        const int d4 = d >> 2;
        for (int i4 = lane; i4 < d4; i4 += 32) {
            float4 v4[8];
#pragma unroll
            for (int k = 0; k < 8; ++k)
                v4[k] = k < count ? __ldg(reinterpret_cast<const float4 *>(rows[k]) + i4) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 q4 = __ldg(reinterpret_cast<const float4 *>(src) + i4);
            const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
            float res[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float4 x = v4[k];
                    v[k] = e == 0 ? x.x : e == 1 ? x.y : e == 2 ? x.z : x.w;
                }
                res[e] = reference_blend_element<true>(qv[e], v, w, sum, count, ratio);
            }
            reinterpret_cast<float4 *>(dst)[i4] = make_float4(res[0], res[1], res[2], res[3]);
        }
    } else {
        for (int i = lane; i < d; i += 32) {
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = k < count ? __ldg(rows[k] + i) : 0.f;
            dst[i] = reference_blend_element<true>(src[i], v, w, sum, count, ratio);
        }
    }
}

}  // namespace

void launch_blend_peer(const PeerTable &t, const float *queries, float *out, const float *dist,
                       const int64_t *labels, long long frames, const float *index_rate, cudaStream_t s) {
    require(frames <= static_cast<long long>(INT32_MAX) * kPeerWarps, "frame count exceeds CUDA grid limit");
    if (frames <= 0) return;
    bool vec4 = t.d % 4 == 0 && reinterpret_cast<uintptr_t>(queries) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(out) % 16 == 0;
    for (int k = 0; k < t.shards; ++k) vec4 = vec4 && reinterpret_cast<uintptr_t>(t.rows[k]) % 16 == 0;
    const unsigned grid = static_cast<unsigned>((frames + kPeerWarps - 1) / kPeerWarps);
    if (vec4)
        blend_peer_kernel<true><<<grid, 32 * kPeerWarps, 0, s>>>(t, queries, out, dist, labels, frames, index_rate);
    else
        blend_peer_kernel<false><<<grid, 32 * kPeerWarps, 0, s>>>(t, queries, out, dist, labels, frames, index_rate);
    cuda_check(cudaGetLastError());
}

}  // namespace vfr

// ---------------------------------------------------------------- host side
struct VfrPeerRows {
    int device = 0;
    int self = 0;
    vfr::PeerTable table{};
    std::vector<void *> opened;  // IPC mappings this object closes
};

namespace vfr {
namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(VfrIpcRows::rows_handle), "IPC handle size");

cudaStream_t call_stream(VfrStream *stream) {
    require(stream && stream->stream, "invalid FAISS CUDA stream");
    return static_cast<cudaStream_t>(stream->stream);
}

void close_mappings(VfrPeerRows *p) noexcept {
    for (void *m : p->opened) cudaIpcCloseMemHandle(m);
    p->opened.clear();
}

}  // namespace
}  // namespace vfr

extern "C" int vfr_index_ipc_export(VfrIndex *index, VfrIpcRows *out, char **error) {
    return vfr::guarded(error, [&] {
        vfr::require(index && out, "invalid IPC export arguments");
        vfr::DeviceGuard guard(index->device);
        std::memset(out, 0, sizeof(*out));
        cudaIpcMemHandle_t h{};
        vfr::cuda_check(cudaIpcGetMemHandle(&h, index->vectors), "cudaIpcGetMemHandle(rows)");
        std::memcpy(out->rows_handle, &h, sizeof(h));
        if (index->row_of_id) {
            vfr::cuda_check(cudaIpcGetMemHandle(&h, index->row_of_id), "cudaIpcGetMemHandle(row ids)");
            std::memcpy(out->ids_handle, &h, sizeof(h));
            out->has_ids = 1;
        }
        out->label_base = index->label_base;
        out->rows = index->n;
        out->width = index->d;
        out->device = index->device;
    });
}

extern "C" int vfr_peer_rows_open(VfrIndex *local, int32_t shards, const VfrIpcRows *descs, int32_t self,
                                  VfrPeerRows **out, char **error) {
    return vfr::guarded(error, [&] {
        vfr::require(local && descs && out, "invalid peer-rows arguments");
        vfr::require(shards >= 1 && shards <= vfr::kMaxPeerShards, "shard count out of range (1..64)");
        vfr::require(self >= 0 && self < shards, "own shard index out of range");
        vfr::require(local->nlist == 1, "peer-row blend needs flat shards");
        *out = nullptr;
        vfr::DeviceGuard guard(local->device);
        auto p = std::make_unique<VfrPeerRows>();
        p->device = local->device;
        p->self = self;
        p->table.shards = shards;
        p->table.d = local->d;
        p->table.bounds[0] = descs[0].label_base;
        for (int s = 0; s < shards; ++s) {
            vfr::require(descs[s].width == local->d, "shard widths differ");
            vfr::require(descs[s].label_base == p->table.bounds[s], "row shards must be contiguous and in order");
            vfr::require(descs[s].rows > 0, "empty row shard");
            p->table.bounds[s + 1] = descs[s].label_base + descs[s].rows;
        }
        vfr::require(descs[self].label_base == local->label_base && descs[self].rows == local->n,
                     "own descriptor does not describe the local index");
        try {
            for (int s = 0; s < shards; ++s) {
                if (s == self) {
                    p->table.rows[s] = local->vectors;
                    p->table.row_of_id[s] = descs[s].has_ids ? local->row_of_id : nullptr;
                    continue;
                }
                cudaIpcMemHandle_t h{};
                void *mapped = nullptr;
                std::memcpy(&h, descs[s].rows_handle, sizeof(h));
                vfr::cuda_check(cudaIpcOpenMemHandle(&mapped, h, cudaIpcMemLazyEnablePeerAccess),
                                "cudaIpcOpenMemHandle(rows)");
                p->opened.push_back(mapped);
                p->table.rows[s] = static_cast<const float *>(mapped);
                if (descs[s].has_ids) {
                    std::memcpy(&h, descs[s].ids_handle, sizeof(h));
                    vfr::cuda_check(cudaIpcOpenMemHandle(&mapped, h, cudaIpcMemLazyEnablePeerAccess),
                                    "cudaIpcOpenMemHandle(row ids)");
                    p->opened.push_back(mapped);
                    p->table.row_of_id[s] = static_cast<const int32_t *>(mapped);
                }
            }
        } catch (...) {
            vfr::close_mappings(p.get());
            throw;
        }
        *out = p.release();
    });
}

extern "C" void vfr_peer_rows_close(VfrPeerRows *peers) {
    if (!peers) return;
    int previous = 0;
    cudaGetDevice(&previous);
    cudaSetDevice(peers->device);
    vfr::close_mappings(peers);
    cudaSetDevice(previous);
    delete peers;
}

extern "C" int vfr_blend_peer(VfrPeerRows *peers, const float *queries, float *out, const float *dist,
                              const int64_t *labels, size_t frames, int32_t width, const float *index_rate,
                              VfrStream *stream, char **error) {
    return vfr::guarded(error, [&] {
        vfr::require(peers && queries && out && dist && labels && index_rate, "invalid blend arguments");
        vfr::require(width == peers->table.d, "FAISS feature width mismatch");
        vfr::require(frames <= static_cast<size_t>(INT32_MAX), "frame count exceeds CUDA grid limit");
        if (frames == 0) return;
        vfr::DeviceGuard guard(peers->device);
        vfr::launch_blend_peer(peers->table, queries, out, dist, labels, static_cast<long long>(frames), index_rate,
                               vfr::call_stream(stream));
    });
}
