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
constexpr uint64_t kSplitRows = 128;  // rows per slice at least: one pass of the scan

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

// Shared state of one CTA's frame (declared once in the kernel).
struct FrameSmem {
    unsigned long long probe_keys[kMaxProbe];
    unsigned long long wave_keys[kOctets];
    int probe_list[kMaxProbe];
    uint32_t probe_base[kMaxProbe + 1];
    uint32_t scan_base[kMaxProbe + 1];  // probe_base over the probes being scanned only
    unsigned long long octet_best[kOctets * 8];
    unsigned long long best[8];
    unsigned long long red[kThreads / 32];
    int32_t best_row[8];
    double weights[8];
    double weight_sum;
    int last;
};

// The coarse stage: the first nprobe lists in (distance, list id) order and
// the scan position where each starts (probe_base[probes] = rows scanned);
// scan_base is the same over the probes in scan_mask only (the rows this
// call scans).  Returns the number of probed lists.  Called by every thread.
__device__ int coarse_stage(const ExactArgs &a, long long frame, const float *q, FrameSmem &sm,
                            uint32_t scan_mask = ~0u) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, octet = tid >> 3, j = tid & 7;
    const int octet_base = lane & ~7;
    const int d = a.d;
    int probes = a.nprobe < a.nlist ? a.nprobe : a.nlist;
    if (a.nlist == 1) {
        if (tid == 0) sm.probe_list[0] = 0;
        probes = 1;
    } else if (a.probes && a.probe_ok[frame]) {
        // the tensor-core coarse stage certified this frame's lists (the same
        // exact order): only its fine stage was left open
        if (tid < probes) sm.probe_list[tid] = a.probes[frame * a.nprobe + tid];
    } else {
        if (tid < kMaxProbe) sm.probe_keys[tid] = kEmptyKey;
        __syncthreads();
        for (int base = 0; base < a.nlist; base += kOctets) {
            const int list = base + octet;
            const int clamped = list < a.nlist ? list : a.nlist - 1;
            float dist = octet_l2(q, a.centroids + static_cast<size_t>(clamped) * d, d, j, octet_base, kFullMask);
            if (j == 0) sm.wave_keys[octet] = list < a.nlist ? make_key(dist, static_cast<uint32_t>(list)) : kEmptyKey;
            __syncthreads();
            if (warp == 0) {
                // merge the sorted running top-`probes` with this wave's keys
                unsigned long long nk = warp_sort_u64(sm.wave_keys[lane], lane);
                unsigned long long ok = lane < probes ? sm.probe_keys[lane] : kEmptyKey;
                int rank_new = 0, rank_old = 0;
                for (int i = 0; i < probes; ++i) rank_new += sm.probe_keys[i] < nk;
                for (int i = 0; i < 32; ++i) {
                    unsigned long long other = __shfl_sync(kFullMask, nk, i);
                    rank_old += other <= ok;
                }
                __syncwarp();
                int pn = lane + rank_new;
                int po = lane + rank_old;
                if (pn < probes) sm.probe_keys[pn] = nk;
                if (lane < probes && po < probes) sm.probe_keys[po] = ok;
            }
            __syncthreads();
        }
        if (tid < probes) sm.probe_list[tid] = static_cast<int>(key_pos(sm.probe_keys[tid]));
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0, scanned = 0;
        for (int r = 0; r < probes; ++r) {
            const uint32_t len = static_cast<uint32_t>(a.offsets[sm.probe_list[r] + 1] - a.offsets[sm.probe_list[r]]);
            sm.probe_base[r] = acc;
            sm.scan_base[r] = scanned;
            acc += len;
            if ((scan_mask >> r) & 1u) scanned += len;
        }
        sm.probe_base[probes] = acc;
        sm.scan_base[probes] = scanned;
    }
    __syncthreads();
    return probes;
}

// Squared L2 distance in the AVX2 order from a pair of threads (lanes 2p
// and 2p+1, h = lane & 1): thread h owns lanes 4h..4h+3 of the eight and
// reads its half of every 8-float block as one float4, so a thread keeps
// eight 16-byte row loads in flight where an octet thread keeps 4-byte ones.
// Each lane's sum still runs over the blocks in order from +0, and the eight
// lane sums are added in lane order from -0 before the tail, so the value is
// octet_l2's bit for bit.  Needs d % 4 == 0 and 16-byte aligned q and rows;
// both threads of the pair return it.
__device__ __forceinline__ float pair_l2(const float *__restrict__ q, const float *__restrict__ x, int d, int h) {
    const int blocks = d >> 3;
    float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, c3 = 0.0f;
    const float4 *xv = reinterpret_cast<const float4 *>(x) + h;
    const float4 *qv = reinterpret_cast<const float4 *>(q) + h;
#pragma unroll 8
    for (int b = 0; b < blocks; ++b) {
        const float4 xx = __ldg(xv + 2 * b);
        const float4 qq = qv[2 * b];
        const float t0 = __fsub_rn(qq.x, xx.x), t1 = __fsub_rn(qq.y, xx.y);
        const float t2 = __fsub_rn(qq.z, xx.z), t3 = __fsub_rn(qq.w, xx.w);
        c0 = __fadd_rn(c0, __fmul_rn(t0, t0));
        c1 = __fadd_rn(c1, __fmul_rn(t1, t1));
        c2 = __fadd_rn(c2, __fmul_rn(t2, t2));
        c3 = __fadd_rn(c3, __fmul_rn(t3, t3));
    }
    const float o0 = __shfl_xor_sync(kFullMask, c0, 1), o1 = __shfl_xor_sync(kFullMask, c1, 1);
    const float o2 = __shfl_xor_sync(kFullMask, c2, 1), o3 = __shfl_xor_sync(kFullMask, c3, 1);
    const float l[8] = {h ? o0 : c0, h ? o1 : c1, h ? o2 : c2, h ? o3 : c3,
                        h ? c0 : o0, h ? c1 : o1, h ? c2 : o2, h ? c3 : o3};
    float s = -0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = __fadd_rn(s, l[i]);
    float tail = -0.0f;
    for (int i = blocks * 8; i < d; ++i) {
        const float t = __fsub_rn(q[i], __ldg(x + i));
        tail = __fadd_rn(tail, __fmul_rn(t, t));
    }
    return __fadd_rn(s, tail);
}

// scan_range with pair_l2: 128 rows per pass (one per thread pair), each
// pair keeping its own top 8; the pairs' lists are merged per warp in
// registers, then across the warps.
__device__ void scan_range_pairs(const ExactArgs &a, const float *q, FrameSmem &sm, int probes, uint32_t p0,
                                 uint32_t p1) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, pair = tid >> 1, h = tid & 1;
    const int d = a.d;
    Top8 top;
    top.init();
    for (int r = 0; r < probes; ++r) {
        // [p0, p1) counts the scanned probes' rows only; keys carry the
        // full scan position lb + (row - first)
        const uint32_t lb = sm.probe_base[r], cb = sm.scan_base[r], ce = sm.scan_base[r + 1];
        const uint32_t from = cb > p0 ? cb : p0, to = ce < p1 ? ce : p1;
        if (from >= to) continue;
        const int first = a.offsets[sm.probe_list[r]];
        const int begin = first + static_cast<int>(from - cb);
        const int end = first + static_cast<int>(to - cb);
        for (int row0 = begin; row0 < end; row0 += kThreads / 2) {
            const int row = row0 + pair;
            const float dist = pair_l2(q, a.vectors + static_cast<size_t>(row < end ? row : begin) * d, d, h);
            // the reference never admits +inf (best starts at +inf, `>=` rejects)
            if (row < end && dist < __int_as_float(0x7f800000))
                top.insert(make_key(dist, lb + static_cast<uint32_t>(row - first)));
        }
    }
    // the warp's 16 lists (even lanes): eight rounds of a warp minimum, the
    // owner of each minimum advancing its head (keys are distinct)
    int head = 0;
    for (int i = 0; i < 8; ++i) {
        unsigned long long mine = kEmptyKey;
#pragma unroll
        for (int e = 0; e < 8; ++e) mine = (h == 0 && e == head) ? top.k[e] : mine;
        const unsigned long long m = warp_min_u64(mine);
        if (mine == m && m != kEmptyKey) ++head;
        if (lane == 0) sm.octet_best[warp * 8 + i] = m;
    }
    __syncthreads();
    if (warp == 0) {
        head = 0;
        for (int i = 0; i < 8; ++i) {
            const unsigned long long mine =
                lane < kThreads / 32 && head < 8 ? sm.octet_best[lane * 8 + head] : kEmptyKey;
            const unsigned long long m = warp_min_u64(mine);
            if (mine == m && m != kEmptyKey) ++head;
            if (lane == 0) sm.best[i] = m;
        }
    }
    __syncthreads();
}

// Scans positions [p0, p1) of the scanned probes' rows (probe r covers
// scan_base[r] .. scan_base[r + 1], rows in storage order; with every probe
// scanned these are the scan positions) and leaves the CTA's top 8 keys
// (distance, scan position probe_base[r] + row offset) in sm.best.
__device__ void scan_range(const ExactArgs &a, const float *q, FrameSmem &sm, int probes, uint32_t p0, uint32_t p1) {
    if ((a.d & 3) == 0 && (reinterpret_cast<uintptr_t>(a.vectors) & 15) == 0) {
        scan_range_pairs(a, q, sm, probes, p0, p1);
        return;
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, octet = tid >> 3, j = tid & 7;
    const int octet_base = lane & ~7;
    const int d = a.d;
    Top8 top;
    top.init();
    for (int r = 0; r < probes; ++r) {
        // [p0, p1) counts the scanned probes' rows only; keys carry the
        // full scan position lb + (row - first)
        const uint32_t lb = sm.probe_base[r], cb = sm.scan_base[r], ce = sm.scan_base[r + 1];
        const uint32_t from = cb > p0 ? cb : p0, to = ce < p1 ? ce : p1;
        if (from >= to) continue;
        const int first = a.offsets[sm.probe_list[r]];
        const int begin = first + static_cast<int>(from - cb);
        const int end = first + static_cast<int>(to - cb);
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
                    top.insert(make_key(dist[k], lb + static_cast<uint32_t>(row - first)));
            }
        }
    }
    if (j == 0)
#pragma unroll
        for (int i = 0; i < 8; ++i) sm.octet_best[octet * 8 + i] = top.k[i];
    __syncthreads();
    if (warp == 0) {
        int head = 0;
        for (int i = 0; i < 8; ++i) {
            unsigned long long mine = head < 8 ? sm.octet_best[lane * 8 + head] : kEmptyKey;
            unsigned long long m = warp_min_u64(mine);
            if (mine == m && m != kEmptyKey) ++head;
            if (lane == 0) sm.best[i] = m;
        }
    }
    __syncthreads();
}

// From the frame's top 8 keys in sm.best: rows, then the search outputs or
// the blend (retrieval.rs:65-81).
__device__ void finish_frame(const ExactArgs &a, long long frame, const float *q, float ratio, FrameSmem &sm,
                             int probes) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int d = a.d;
    const float *src = a.queries + frame * d;
    float *dst = a.out + frame * d;
    if (warp == 0 && lane < 8) {
        unsigned long long key = sm.best[lane];
        int32_t row = -1;
        if (key != kEmptyKey) {
            uint32_t pos = key_pos(key);
            int r = 0;
            while (r + 1 < probes && sm.probe_base[r + 1] <= pos) ++r;
            row = a.offsets[sm.probe_list[r]] + static_cast<int32_t>(pos - sm.probe_base[r]);
        }
        sm.best_row[lane] = row;
    }
    __syncthreads();
    int count = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) count += sm.best_row[i] >= 0;

    if (a.mode == kModeSearch) {
        if (tid < a.k) {
            const bool have = tid < count;
            a.dist_out[frame * a.k + tid] = have ? key_dist(sm.best[tid]) : __int_as_float(0x7f800000);
            a.label_out[frame * a.k + tid] =
                have ? static_cast<int64_t>(a.ids[sm.best_row[tid]]) + a.label_base : -1;
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
        for (int i = 0; i < 8; ++i) dist[i] = key_dist(sm.best[i]);
        sm.weight_sum = reference_weights(dist, count, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) sm.weights[i] = w[i];
    }
    __syncthreads();
    double w[8];
    int32_t rows[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        w[i] = sm.weights[i];
        rows[i] = sm.best_row[i];
    }
    const WeightDivisor sum = weight_divisor(sm.weight_sum);
    for (int i = tid; i < d; i += kThreads) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = k < count ? __ldg(a.vectors + static_cast<size_t>(rows[k]) * d + i) : 0.f;
        dst[i] = reference_blend_element(q[i], v, w, sum, count, ratio);
    }
}

// Loads the frame into q; false when a blend at index_rate <= 0 leaves it
// as it is (then dst holds the frame).
__device__ bool frame_prologue(const ExactArgs &a, long long frame, float *q, float &ratio, bool copy_through) {
    const int tid = threadIdx.x;
    const int d = a.d;
    const float *src = a.queries + frame * d;
    float *dst = a.out + frame * d;
    ratio = 1.0f;
    if (a.mode == kModeBlend) {
        ratio = load_ratio(a.index_rate);
        if (!(ratio > 0.0f)) {
            if (copy_through && dst != src)
                for (int i = tid; i < d; i += kThreads) dst[i] = src[i];
            return false;
        }
    }
    for (int i = tid; i < d; i += kThreads) q[i] = src[i];
    __syncthreads();
    return true;
}

__device__ void exact_frame(const ExactArgs &a, const long long frame, float *q, FrameSmem &sm) {
    if (threadIdx.x == 0 && a.frame_list && a.counters) atomicAdd(&a.counters->fallback_frames, 1ull);
    float ratio;
    if (!frame_prologue(a, frame, q, ratio, true)) return;
    const int probes = coarse_stage(a, frame, q, sm);
    if (threadIdx.x == 0 && a.frame_list && a.counters)
        atomicAdd(&a.counters->rerun_rows, static_cast<unsigned long long>(sm.scan_base[probes]));
    scan_range(a, q, sm, probes, 0u, sm.probe_base[probes]);
    finish_frame(a, frame, q, ratio, sm, probes);
}

// Slice `s` of fallback frame `i` (of at most kSplitFrames), which has up to
// `nsplit` CTAs and uses as many as its scan has passes of rows: the
// CTA scans its share of the frame's probed rows and stores its top 8; the
// last CTA of the frame to finish (device-scope fence and counter, no
// waiting) merges the slices' lists and finishes the frame.  The keys carry
// scan positions, so the merged list is the whole scan's top 8.
__device__ void exact_split(const ExactArgs &a, long long frame, int i, int s, int nsplit, float *q, FrameSmem &sm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float ratio;
    if (!frame_prologue(a, frame, q, ratio, s == 0)) return;
    // the fine stage's hint (IVF): scan only the probes it marks; every CTA
    // of the frame reads it before the frame's counter below, and the last
    // one clears it after use
    const RerunHint *hint = nullptr;
    if (a.hints != nullptr && i < kSplitFrames && a.probe_ok != nullptr && a.probe_ok[frame] &&
        __ldcg(&a.hints[i].frame) == static_cast<int32_t>(frame))
        hint = a.hints + i;
    const int probes = coarse_stage(a, frame, q, sm, hint ? __ldcg(&hint->scan_mask) : ~0u);
    const uint64_t total = sm.scan_base[probes];
    // slices of at least one pass of rows each: a small scan (a partial IVF
    // re-run) takes a few CTAs, and the rest of the frame's CTAs leave
    // without touching the frame's counter (every CTA computes the same
    // count from the same scan length)
    const int used = static_cast<int>(min(static_cast<uint64_t>(nsplit),
                                          max(uint64_t{1}, (total + kSplitRows - 1) / kSplitRows)));
    if (s >= used) return;
    const uint32_t p0 = static_cast<uint32_t>(total * s / used);
    const uint32_t p1 = static_cast<uint32_t>(total * (s + 1) / used);
    if (tid == 0 && a.counters && p1 > p0) atomicAdd(&a.counters->rerun_rows, static_cast<unsigned long long>(p1 - p0));
    scan_range(a, q, sm, probes, p0, p1);
    unsigned long long *slot = a.split_keys + (static_cast<size_t>(i) * kExactSplitGrid + s) * 8;
    if (tid < 8) slot[tid] = sm.best[tid];
    __threadfence();
    __syncthreads();
    if (tid == 0) sm.last = atomicAdd(a.split_done + i, 1) == used - 1;
    __syncthreads();
    if (!sm.last) return;
    __threadfence();
    if (tid == 0) {
        a.split_done[i] = 0;  // ready for the next call
        if (hint != nullptr) a.hints[i].frame = -1;
        if (a.counters) atomicAdd(&a.counters->fallback_frames, 1ull);
    }
    // the slices' lists, merged: each thread keeps the top 8 of a strided
    // share, then eight rounds of a block-wide minimum
    Top8 mine;
    mine.init();
    const unsigned long long *all = a.split_keys + static_cast<size_t>(i) * kExactSplitGrid * 8;
    for (int e = tid; e < used * 8; e += kThreads) mine.insert(__ldcg(all + e));
    if (hint != nullptr && tid < 8) mine.insert(__ldcg(&hint->keys[tid]));  // the other probes' top 8
    int head = 0;
    for (int r = 0; r < 8; ++r) {
        unsigned long long cand = kEmptyKey;
#pragma unroll
        for (int h = 0; h < 8; ++h) cand = h == head ? mine.k[h] : cand;
        const unsigned long long wmin = warp_min_u64(cand);
        if (lane == 0) sm.red[warp] = wmin;
        __syncthreads();
        unsigned long long m = lane < kThreads / 32 ? sm.red[lane] : kEmptyKey;
        m = warp_min_u64(m);
        if (cand == m && m != kEmptyKey) ++head;  // keys are distinct: one owner
        if (tid == 0) sm.best[r] = m;
        __syncthreads();
    }
    finish_frame(a, frame, q, ratio, sm, probes);
}

// One CTA per frame, or, with a device frame list (the frames the
// tensor-core engine could not certify), a fixed grid over it: with at most
// kSplitFrames listed frames (and split scratch), every frame gets
// gridDim.x / count CTAs, each scanning a slice; otherwise one CTA per frame.
__global__ void __launch_bounds__(kThreads, 3) exact_kernel(ExactArgs a) {
    extern __shared__ __align__(16) float q[];  // [d] copy of the frame
    __shared__ FrameSmem sm;
    grid_dependency_wait();  // the frame list and the outputs belong to the kernel before
    if (a.frame_list) {
        const int count = *a.frame_count;
        if (count > 0 && count <= kSplitFrames && a.split_keys && static_cast<int>(gridDim.x) >= 2 * count) {
            const int nsplit = static_cast<int>(gridDim.x) / count;
            const int i = static_cast<int>(blockIdx.x) % count, s = static_cast<int>(blockIdx.x) / count;
            if (s < nsplit) exact_split(a, a.frame_list[i], i, s, nsplit, q, sm);
        } else {
            for (int i = blockIdx.x; i < count; i += gridDim.x) {
                // full scans: a hint of this entry is not needed
                if (a.hints != nullptr && i < kSplitFrames && threadIdx.x == 0) a.hints[i].frame = -1;
                exact_frame(a, a.frame_list[i], q, sm);
                __syncthreads();
            }
        }
    } else {
        exact_frame(a, blockIdx.x, q, sm);
    }
}

}  // namespace

void launch_exact(const ExactArgs &args, long long frames, cudaStream_t stream, bool after_kernel) {
    if (frames <= 0) return;
    size_t smem = static_cast<size_t>(args.d) * sizeof(float);
    unsigned grid = static_cast<unsigned>(frames);
    if (args.frame_list) grid = static_cast<unsigned>(frames < kExactSplitGrid ? frames : kExactSplitGrid);
    if (after_kernel) {
        const cudaError_t rc = launch_pdl(exact_kernel, dim3(grid), dim3(kThreads), smem, stream, args);
        if (rc != cudaSuccess) throw std::runtime_error(std::string("exact kernel launch: ") + cudaGetErrorString(rc));
    } else {
        exact_kernel<<<grid, kThreads, smem, stream>>>(args);
    }
}

}  // namespace vfr
