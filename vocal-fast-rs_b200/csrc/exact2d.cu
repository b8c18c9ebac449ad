// Exact SIMT engine over a 2-D grid, for small IVF batches (realtime blocks
// against a voice index), where the per-frame chain of the one-CTA-per-frame
// exact kernel and the launch chain of the tensor-core IVF path both cost
// more than the arithmetic.  Three launches, the last two chained with
// programmatic dependent launch:
//
//   1. coarse: CTA (16-centroid slice, 8-frame group) stages both in shared
//      memory once, computes the exact distances (the reference's AVX2
//      order) and keeps each frame's first nprobe keys of the slice
//      (distance total order, list id);
//   2. fine: CTA (part, frame) merges the frame's slice lists into the
//      first nprobe lists -- the reference's coarse sort,
//      crates/vocal-cpu/src/retrieval.rs:45-51 -- and scans its 64 scan
//      positions of those lists (probe rank major, storage row minor,
//      :52-64), keeping its 8 best (distance, scan position) keys;
//   3. finish: CTA frame merges its parts' lists into the top 8 (ties keep
//      the earlier scan position, as the reference's insertion does), then
//      writes the search outputs or blends (f64 weights, f32 blend, :65-81).
//
// Every distance is the exact one, so no certificate or re-run is needed;
// the result is the reference's by construction.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "exact2d.h"
#include "exact_common.cuh"
#include "pdl.cuh"

namespace vfr {
namespace {

constexpr int kT = 256;
constexpr int kOct = kT / 8;                 // octets per CTA
constexpr int kRowsPerOctet = 2;
constexpr int kFinePart = kOct * kRowsPerOctet;  // scan positions per fine CTA

// Bitonic sort of one key per lane, ascending across lanes 0..31.
__device__ __forceinline__ unsigned long long sort32(unsigned long long v, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const unsigned long long o = __shfl_xor_sync(kFullMask, v, j);
            const bool up = (lane & k) == 0, low = (lane & j) == 0;
            const unsigned long long lo = o < v ? o : v, hi = o < v ? v : o;
            v = (low == up) ? lo : hi;
        }
    }
    return v;
}

__device__ __forceinline__ unsigned long long min64(unsigned long long v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        const unsigned long long o = __shfl_xor_sync(kFullMask, v, s);
        v = o < v ? o : v;
    }
    return v;
}

// The first `want` keys of `lists` sorted lists of `len` keys each (keys[l *
// len + i], ascending, kEmptyKey past a list's end; keys distinct), by
// warp 0: one warp minimum over the lists' heads per output key.  head is
// shared scratch of `lists` ints.  out[i] = kEmptyKey past the real keys.
__device__ void merge_sorted_lists(const unsigned long long *keys, int lists, int len, int want, int *head,
                                   unsigned long long *out) {
    const int lane = threadIdx.x & 31;
    for (int l = lane; l < lists; l += 32) head[l] = 0;
    __syncwarp();
    for (int r = 0; r < want; ++r) {
        unsigned long long cand = kEmptyKey;
        int owner = -1;
        for (int l = lane; l < lists; l += 32) {
            const int h = head[l];
            const unsigned long long k = h < len ? keys[static_cast<size_t>(l) * len + h] : kEmptyKey;
            if (k < cand) {
                cand = k;
                owner = l;
            }
        }
        const unsigned long long m = min64(cand);
        if (cand == m && m != kEmptyKey) ++head[owner];  // one owner: keys are distinct
        if (lane == 0) out[r] = m;
        __syncwarp();
    }
}


__device__ __forceinline__ bool ratio_off(const ExactArgs &e) {
    return e.mode == kModeBlend && !(load_ratio(e.index_rate) > 0.f);
}

// ---------------------------------------------------------------- 1. coarse
// CTA (slice, frame group): the slice's kSlice centroid rows and the group's
// kGroup frames are staged in shared memory once; octet o computes centroid
// o % kSlice against frames 4 (o / kSlice) .. +3 (the reference's AVX2 order;
// (a - b)^2 == (b - a)^2 exactly, so the operand roles may swap), and warp f
// keeps frame f's first nprobe keys (distance total order, list id).
constexpr int kSlice = 16;                     // centroids per coarse CTA
constexpr int kGroup = 8;                      // frames per coarse CTA
constexpr int kFramesPerOctet = kGroup * kSlice / kOct;
static_assert(kFramesPerOctet == 4 && kGroup == kT / 32, "one warp per frame of the group");
constexpr int kExact2dMaxWidth = 2048;  // (kSlice + kGroup) rows of this width fit the opt-in shared memory

__global__ void __launch_bounds__(kT) exact2d_coarse_kernel(Exact2dArgs a, long long frames) {
    extern __shared__ float cs[];  // [kSlice][stride] centroids, then [kGroup][stride] frames
    __shared__ unsigned long long keys[kGroup][kSlice];
    const ExactArgs &e = a.e;
    launch_dependents();
    if (ratio_off(e)) return;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, octet = tid >> 3, j = tid & 7;
    const int d = e.d, stride = (d + 3) & ~3;
    const int c0 = static_cast<int>(blockIdx.x) * kSlice;
    const long long f0 = static_cast<long long>(blockIdx.y) * kGroup;
    float *cent = cs, *fr = cs + static_cast<size_t>(kSlice) * stride;
    // rows staged whole (16-byte lanes when the width allows), zero past
    // the last centroid or frame
    const bool vec = (d & 3) == 0 && (reinterpret_cast<uintptr_t>(e.centroids) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(e.queries) & 15) == 0;
    auto stage = [&](float *dst, const float *src, bool real) {
        if (vec) {
            const float4 *s4 = reinterpret_cast<const float4 *>(src);
            float4 *d4 = reinterpret_cast<float4 *>(dst);
            for (int k = tid; k < (d >> 2); k += kT) d4[k] = real ? __ldg(s4 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            for (int k = tid; k < d; k += kT) dst[k] = real ? __ldg(src + k) : 0.f;
        }
    };
#pragma unroll 1
    for (int c = 0; c < kSlice; ++c)
        stage(cent + c * stride, e.centroids + static_cast<size_t>(c0 + c < e.nlist ? c0 + c : 0) * d,
              c0 + c < e.nlist);
#pragma unroll 1
    for (int g = 0; g < kGroup; ++g)
        stage(fr + g * stride, e.queries + (f0 + g < frames ? f0 + g : 0) * d, f0 + g < frames);
    __syncthreads();
    const int c = octet % kSlice, g0 = (octet / kSlice) * kFramesPerOctet;
    const float *xs[kFramesPerOctet];
#pragma unroll
    for (int k = 0; k < kFramesPerOctet; ++k) xs[k] = fr + (g0 + k) * stride;
    float dist[kFramesPerOctet];
    octet_l2n<kFramesPerOctet, false>(cent + c * stride, xs, d, j, lane & ~7, kFullMask, dist);
    if (j == 0)
#pragma unroll
        for (int k = 0; k < kFramesPerOctet; ++k)
            keys[g0 + k][c] = c0 + c < e.nlist ? make_key(dist[k], static_cast<uint32_t>(c0 + c)) : kEmptyKey;
    __syncthreads();
    const long long frame = f0 + warp;
    if (frame < frames) {
        const unsigned long long v = sort32(lane < kSlice ? keys[warp][lane] : kEmptyKey, lane);
        if (lane < a.probes) a.coarse_keys[(frame * a.slices + blockIdx.x) * a.probes + lane] = v;
    }
}

// ---------------------------------------------------------------- 2. fine
struct FineSmem {
    int32_t plist[kMaxProbe];
    uint32_t pbase[kMaxProbe + 1];
    int32_t pstart[kMaxProbe];
    unsigned long long top[kMaxProbe];
    unsigned long long keys[kFinePart];
};

__global__ void __launch_bounds__(kT) exact2d_fine_kernel(Exact2dArgs a) {
    extern __shared__ float q[];  // [d], then the merge heads
    __shared__ FineSmem sm;
    const ExactArgs &e = a.e;
    launch_dependents();
    if (ratio_off(e)) return;
    const int tid = threadIdx.x, lane = tid & 31, octet = tid >> 3, j = tid & 7;
    const long long frame = blockIdx.y;
    const int part = blockIdx.x;
    const int d = e.d, P = a.probes;
    // the caller's frames were complete before the coarse launch began
    for (int i = tid; i < d; i += kT) q[i] = e.queries[frame * d + i];
    grid_dependency_wait();  // the coarse keys
    if (e.nlist > 1) {
        if (tid < 32) {
            int *head = reinterpret_cast<int *>(q + ((d + 1) & ~1));
            merge_sorted_lists(a.coarse_keys + frame * a.slices * P, a.slices, P, P, head, sm.top);
        }
        __syncthreads();
        if (tid < P) sm.plist[tid] = static_cast<int32_t>(key_pos(sm.top[tid]));
    } else if (tid == 0) {
        sm.plist[0] = 0;
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0;
        for (int r = 0; r < P; ++r) {
            const int32_t lo = e.offsets[sm.plist[r]], hi = e.offsets[sm.plist[r] + 1];
            sm.pstart[r] = lo;
            sm.pbase[r] = acc;
            acc += static_cast<uint32_t>(hi - lo);
        }
        sm.pbase[P] = acc;
        if (part == 0) {
            for (int r = 0; r < P; ++r) a.probe_list[frame * P + r] = sm.plist[r];
            for (int r = 0; r <= P; ++r) a.probe_base[frame * (P + 1) + r] = sm.pbase[r];
        }
    }
    __syncthreads();
    const uint32_t total = sm.pbase[P];
    const float *xs[kRowsPerOctet];
    uint32_t pos[kRowsPerOctet];
#pragma unroll
    for (int k = 0; k < kRowsPerOctet; ++k) {
        pos[k] = static_cast<uint32_t>(part) * kFinePart + octet + k * kOct;
        int r = 0;
        while (r + 1 < P && sm.pbase[r + 1] <= pos[k]) ++r;
        const uint32_t p = pos[k] < total ? pos[k] : 0u;
        const int row = sm.pstart[r] + static_cast<int>(p - sm.pbase[r]);
        xs[k] = e.vectors + static_cast<size_t>(pos[k] < total ? row : 0) * d;  // row 0: a valid dummy
    }
    float dist[kRowsPerOctet];
    if (total > 0) octet_l2n<kRowsPerOctet>(q, xs, d, j, lane & ~7, kFullMask, dist);
    if (j == 0) {
#pragma unroll
        for (int k = 0; k < kRowsPerOctet; ++k)
            sm.keys[octet * kRowsPerOctet + k] = pos[k] < total && dist[k] < __int_as_float(0x7f800000)
                                                     ? make_key(dist[k], pos[k])
                                                     : kEmptyKey;
    }
    __syncthreads();
    if (tid < 32) {
        // this part's 8 best of its 64 keys: two sorted halves, then 8 pops
        unsigned long long x = sort32(sm.keys[lane], lane), y = sort32(sm.keys[32 + lane], lane);
        for (int r = 0; r < 8; ++r) {
            const unsigned long long hx = __shfl_sync(kFullMask, x, 0), hy = __shfl_sync(kFullMask, y, 0);
            const bool take_x = hx <= hy;
            if (lane == 0) a.fine_keys[(frame * a.parts + part) * 8 + r] = take_x ? hx : hy;
            // pop the taken head: shift that half down one lane
            const unsigned long long nx = __shfl_down_sync(kFullMask, x, 1), ny = __shfl_down_sync(kFullMask, y, 1);
            if (take_x) x = lane == 31 ? kEmptyKey : nx;
            else y = lane == 31 ? kEmptyKey : ny;
        }
    }
}

// ---------------------------------------------------------------- 3. finish
__global__ void __launch_bounds__(kT) exact2d_finish_kernel(Exact2dArgs a) {
    extern __shared__ float q[];  // merge heads
    __shared__ unsigned long long best[8];
    __shared__ int32_t best_row[8];
    __shared__ double weights[8];
    const ExactArgs &e = a.e;
    const int tid = threadIdx.x, lane = tid & 31;
    const long long frame = blockIdx.x;
    const int d = e.d, P = a.probes;
    const float *src = e.queries + frame * d;
    float *dst = e.out + frame * d;
    if (ratio_off(e)) {
        if (dst != src)
            for (int i = tid; i < d; i += kT) dst[i] = src[i];
        return;
    }
    const float ratio = e.mode == kModeBlend ? load_ratio(e.index_rate) : 1.f;
    grid_dependency_wait();  // the parts' keys and the probe lists
    if (tid < 32) {
        merge_sorted_lists(a.fine_keys + frame * a.parts * 8, a.parts, 8, 8, reinterpret_cast<int *>(q), best);
        if (lane < 8) {
            const unsigned long long key = best[lane];
            int32_t row = -1;
            if (key != kEmptyKey) {
                const uint32_t p = key_pos(key);
                const uint32_t *pb = a.probe_base + frame * (P + 1);
                int r = 0;
                while (r + 1 < P && pb[r + 1] <= p) ++r;
                row = e.offsets[a.probe_list[frame * P + r]] + static_cast<int32_t>(p - pb[r]);
            }
            best_row[lane] = row;
            weights[lane] = row >= 0 ? reference_weight(key_dist(key)) : 0.0;
        }
    }
    __syncthreads();
    int count = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) count += best_row[i] >= 0;
    if (e.mode == kModeSearch) {
        if (tid < e.k) {
            const bool have = tid < count;
            e.dist_out[frame * e.k + tid] = have ? key_dist(best[tid]) : __int_as_float(0x7f800000);
            e.label_out[frame * e.k + tid] = have ? static_cast<int64_t>(e.ids[best_row[tid]]) + e.label_base : -1;
        }
        return;
    }
    if (count == 0) {
        if (tid == 0 && e.counters) atomicAdd(&e.counters->empty_frames, 1ull);
        if (dst != src)
            for (int i = tid; i < d; i += kT) dst[i] = src[i];
        return;
    }
    double w[8];
    double wsum = -0.0;  // the reference's order: S = w0 + w1 + ... (zeros past count)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        w[i] = weights[i];
        wsum = __dadd_rn(wsum, w[i]);
    }
    const WeightDivisor sum = weight_divisor(wsum);
    const float *rows[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) rows[k] = e.vectors + static_cast<size_t>(k < count ? best_row[k] : best_row[0]) * d;
    for (int i = tid; i < d; i += kT) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = k < count ? __ldg(rows[k] + i) : 0.f;
        dst[i] = reference_blend_element<true>(src[i], v, w, sum, count, ratio);
    }
}

}  // namespace

int exact2d_max_width() { return kExact2dMaxWidth; }

Exact2dLayout exact2d_layout(size_t frames, int nlist, int nprobe, int64_t max_probed) {
    Exact2dLayout l{};
    l.probes = std::min(nprobe, nlist);
    l.slices = nlist > 1 ? (nlist + kSlice - 1) / kSlice : 0;
    l.parts = static_cast<int>(std::max<int64_t>(1, (max_probed + kFinePart - 1) / kFinePart));
    size_t off = 0;
    auto take = [&](size_t &field, size_t bytes) {
        field = off;
        off = (off + bytes + 255) & ~size_t(255);
    };
    take(l.coarse_keys, frames * std::max(1, l.slices) * l.probes * sizeof(unsigned long long));
    take(l.fine_keys, frames * static_cast<size_t>(l.parts) * 8 * sizeof(unsigned long long));
    take(l.probe_list, frames * l.probes * sizeof(int32_t));
    take(l.probe_base, frames * (l.probes + 1) * sizeof(uint32_t));
    l.total = off;
    return l;
}

void launch_exact2d(const ExactArgs &e, void *workspace, const Exact2dLayout &l, long long frames, cudaStream_t s) {
    if (frames <= 0) return;
    if (frames > 65535) throw std::runtime_error("2-D exact engine: at most 65535 frames per call");
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    Exact2dArgs a{};
    a.e = e;
    a.slices = l.slices;
    a.parts = l.parts;
    a.probes = l.probes;
    a.coarse_keys = reinterpret_cast<unsigned long long *>(ws + l.coarse_keys);
    a.fine_keys = reinterpret_cast<unsigned long long *>(ws + l.fine_keys);
    a.probe_list = reinterpret_cast<int32_t *>(ws + l.probe_list);
    a.probe_base = reinterpret_cast<uint32_t *>(ws + l.probe_base);
    const size_t qbytes = static_cast<size_t>((e.d + 1) & ~1) * sizeof(float);
    const size_t heads = static_cast<size_t>(std::max(l.slices, l.parts)) * sizeof(int);
    const unsigned f = static_cast<unsigned>(frames);
    if (e.nlist > 1) {
        // not a programmatic launch: the frames (possibly blended in place by
        // the previous call) are read before any dependency wait
        const size_t cbytes = static_cast<size_t>(kSlice + kGroup) * ((e.d + 3) & ~3) * sizeof(float);
        cudaError_t at = cudaFuncSetAttribute(exact2d_coarse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(cbytes));
        if (at != cudaSuccess) throw std::runtime_error(std::string("exact2d coarse: ") + cudaGetErrorString(at));
        exact2d_coarse_kernel<<<dim3(static_cast<unsigned>(l.slices), (f + kGroup - 1) / kGroup), kT, cbytes, s>>>(
            a, frames);
        cudaError_t rc = cudaGetLastError();
        if (rc != cudaSuccess) throw std::runtime_error(std::string("exact2d coarse: ") + cudaGetErrorString(rc));
        rc = launch_pdl(exact2d_fine_kernel, dim3(static_cast<unsigned>(l.parts), f), dim3(kT), qbytes + heads, s, a);
        if (rc != cudaSuccess) throw std::runtime_error(std::string("exact2d fine: ") + cudaGetErrorString(rc));
    } else {
        exact2d_fine_kernel<<<dim3(static_cast<unsigned>(l.parts), f), kT, qbytes, s>>>(a);
        cudaError_t rc = cudaGetLastError();
        if (rc != cudaSuccess) throw std::runtime_error(std::string("exact2d fine: ") + cudaGetErrorString(rc));
    }
    const cudaError_t rc = launch_pdl(exact2d_finish_kernel, dim3(f), dim3(kT), heads, s, a);
    if (rc != cudaSuccess) throw std::runtime_error(std::string("exact2d finish: ") + cudaGetErrorString(rc));
}

}  // namespace vfr
