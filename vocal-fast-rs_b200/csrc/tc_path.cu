// Tensor-core engine for flat indexes.
//
// Per call:
//   1. prep_queries: fp32 frames -> fp16 (scaled by the index's power-of-two
//      scale s), plus ||q||^2, ||q^|| and ||q - q^|| for the certificate.
//   2. cand_kernel (persistent, warp-specialised, tcgen05 + TMA + TMEM): for
//      each work item (128-frame tile, database segment) the approximate
//      distance d~ = ||x||^2 - (2/s^2) * (q~ . x~) of every row is formed in the
//      epilogue straight out of TMEM and filtered per frame against a running
//      threshold into a shared-memory buffer; the item's 32 smallest
//      (d~, row) keys per frame go to the workspace.  No frame x row matrix is
//      written to HBM.
//   3. merge_kernel: per frame, sort the items' keys, take the 64 smallest,
//      re-rank them with exact fp32 distances in the reference AVX2 order
//      (crates/vocal-cpu/src/retrieval.rs:10-26), keep the top 8 in scan
//      order, and certify that no dropped row can beat the 8th: every dropped
//      row has d~ >= T, and |d - (d~ + ||q||^2)| <= E with E from the fp16
//      rounding residuals, fp32 accumulation and norm rounding.  Certified
//      frames are blended (or their top-k written) exactly like the
//      reference; the rest are listed for
//   4. the exact SIMT kernel, which re-runs them.
// The result is therefore the reference's result for every frame.
#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <limits>
#include <mutex>

#include "exact_common.cuh"
#include "kernels.h"
#include "pdl.cuh"
#include "tc_path.h"
#include "tc_ptx.cuh"

namespace vfr {
namespace {

constexpr int kTileM = 128;  // frames per tile: TMEM lanes
constexpr int kTileN = 256;  // rows per MMA / accumulator
constexpr int kTileK = 64;   // fp16 elements per 128-byte swizzled row
// Candidates kept per frame per candidate list (in registers).  A list whose
// K-th best lies close to the frame's 8th-best distance leaves the frame
// uncertified (and re-run exactly), so the size follows how many of a
// frame's neighbours one list can hold: short flat work items (at most
// kShortItemTiles tiles) keep 8, long flat items and IVF lists (and the coarse
// centroid lists) keep 16.  Fewer kept keys mean fewer insertions in the
// epilogue.
constexpr int kShortKeep = 8;
constexpr int kIvfKeep = 16;
constexpr int kItemKeep = kIvfKeep;  // largest list size (workspace sizing)
constexpr int kShortItemTiles = 12;  // c2's 11-tile items: 8-entry lists certify every frame
constexpr int kRerank = 64;     // candidates re-ranked exactly per frame (more on distance ties)
constexpr int kRerankMax = 128;
constexpr int kMaxSegments = 256;
constexpr int kEpiWarps = 8;     // two per TMEM lane quarter, each on half of a tile's columns
constexpr int kHalves = 2;       // candidate lists per (work item, frame)
constexpr int kThreadsTC = 64 + 32 * kEpiWarps;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr uint32_t kBBytes = kTileN * kTileK * 2;
constexpr uint32_t kNormBytes = kEpiWarps * 2 * (kTileN / kHalves) * sizeof(float);  // per warp, double buffered
constexpr int kSmallBlock = 32;  // frame blocks up to this size use the spread layout
constexpr int kPairMinFrames = 4096;  // with VFR_PAIR=1, launches from this size use CTA pairs when their items are long

// Shared-memory layouts of cand_kernel.  The MMA is always M = 128: query
// row m of the A tile feeds TMEM lane m, and an epilogue warp can read only
// the 32 lanes of its quarter (warp % 4), all four of whose warps run on
// one SM sub-partition.
//
// kFullLayout: 128 query rows per tile, 4 stages of (A 16 KB, B 32 KB).
//
// kSpreadLayout (blocks of at most 32 frames): an M = 64 MMA whose A rows
// 0-7, 16-23, 32-39 and 48-55 hold the frames (four TMA boxes of 8 rows);
// those rows land on TMEM lanes 0-7, 32-39, 64-71 and 96-103, so all four
// lane quarters, and all eight epilogue warps on four sub-partitions, share
// the per-tile filtering that otherwise falls on two warps of one.  The 1 KB
// A blocks of two stages interleave in one 8 KB pack (stage s at s KB,
// quarter q at +2q KB); the MMA's other A rows read whatever lies there
// (their TMEM lanes are never read).  Six stages: three packs, the row-norm
// buffers, and six 32 KB B tiles, 192 KB of database tiles in flight per SM.
enum { kFullLayout = 0, kSpreadLayout = 1, kPairLayout = 2 };
template <int kLayout>
struct Pipe;
template <>
struct Pipe<kFullLayout> {
    static constexpr int kM = kTileM;
    static constexpr int kStages = 4;
    static constexpr int kBlocks = 1;            // A boxes per stage
    static constexpr int kBlockRows = kTileM;    // rows per A box
    static constexpr int kRowsPerQuarter = 32;   // real A rows per TMEM lane quarter
    static constexpr uint32_t kTx = kTileM * kTileK * 2 + kBBytes;
    __host__ __device__ static constexpr uint32_t a_off(int s) { return s * (16384u + kBBytes); }
    __host__ __device__ static constexpr uint32_t a_block_off(int s, int) { return a_off(s); }
    __host__ __device__ static constexpr uint32_t b_off(int s) { return a_off(s) + 16384u; }
    __host__ __device__ static constexpr uint32_t norm_off(int ew) { return kStages * (16384u + kBBytes) + ew * 1024u; }
    static constexpr uint32_t kBarOff = kStages * (16384u + kBBytes) + kNormBytes;
    static constexpr size_t kSmem = 1024 + kBarOff + 256;
};
template <>
struct Pipe<kSpreadLayout> {
    // M = 64: the MMA's 64 A rows land on TMEM lanes 0-15, 32-47, 64-79 and
    // 96-111 (16 per lane quarter), so frames at A rows 0-7, 16-23, 32-39 and
    // 48-55 reach lanes 0-7, 32-39, 64-71 and 96-103, as the epilogue reads
    // them; half the MMA work of M = 128 for the same 32 frames.
    static constexpr int kM = 64;
    static constexpr int kStages = 6;
    static constexpr int kBlocks = 4;
    static constexpr int kBlockRows = 8;
    static constexpr int kRowsPerQuarter = 8;
    static constexpr uint32_t kTx = 4 * 1024 + kBBytes;
    // the 1 KB A blocks of two stages interleave in an 8 KB pack (stage s at
    // s KB, quarter q at +2q KB); three packs, then the row-norm buffers
    __host__ __device__ static constexpr uint32_t a_off(int s) { return (s / 2) * 8192u + (s % 2) * 1024u; }
    __host__ __device__ static constexpr uint32_t a_block_off(int s, int q) { return a_off(s) + q * 2048u; }
    __host__ __device__ static constexpr uint32_t b_off(int s) { return 32768u + s * kBBytes; }
    __host__ __device__ static constexpr uint32_t norm_off(int ew) { return 24576u + ew * 1024u; }
    static constexpr uint32_t kBarOff = 32768u + kStages * kBBytes;
    static constexpr size_t kSmem = 1024 + kBarOff + 256;
};
// kPairLayout (large flat launches): a cluster of two CTAs runs one M = 256,
// N = 256 MMA (cta_group::2).  CTA r holds the 128 frames of its query tile
// (A) and database rows [128 r, 128 r + 128) of each tile (B, half of N) at
// the same offsets as the other CTA, and its TMEM receives its frames' 128 x
// 256 block of D, so the epilogue is the full layout's.  Per stage and CTA:
// A 16 KB + B 16 KB, six stages (twice the full layout's bytes in flight per
// MMA, a third less L2 traffic per FLOP).
template <>
struct Pipe<kPairLayout> {
    static constexpr int kM = 2 * kTileM;  // the pair's MMA
    static constexpr int kStages = 6;
    static constexpr int kBlocks = 1;
    static constexpr int kBlockRows = kTileM;
    static constexpr int kRowsPerQuarter = 32;
    static constexpr uint32_t kBHalf = kBBytes / 2;
    static constexpr uint32_t kTx = 2 * (kTileM * kTileK * 2 + kBHalf);  // both CTAs' loads of a stage
    __host__ __device__ static constexpr uint32_t a_off(int s) { return s * (16384u + kBHalf); }
    __host__ __device__ static constexpr uint32_t a_block_off(int s, int) { return a_off(s); }
    __host__ __device__ static constexpr uint32_t b_off(int s) { return a_off(s) + 16384u; }
    __host__ __device__ static constexpr uint32_t norm_off(int ew) { return kStages * (16384u + kBHalf) + ew * 1024u; }
    static constexpr uint32_t kBarOff = kStages * (16384u + kBHalf) + kNormBytes;
    static constexpr size_t kSmem = 1024 + kBarOff + 256;
};
static_assert(Pipe<kPairLayout>::kSmem <= 232448, "cand_kernel shared memory (pair layout)");
static_assert((Pipe<kSpreadLayout>::kStages + 1) / 2 * 8192u <= 24576u, "A packs below the norm buffers");
static_assert(Pipe<kFullLayout>::kSmem <= 232448 && Pipe<kSpreadLayout>::kSmem <= 232448, "cand_kernel shared memory");
static_assert(kNormBytes == kEpiWarps * 1024, "one 1 KB row-norm double buffer per epilogue warp");
constexpr uint32_t kTmemCols = 512;  // two 128 x 256 fp32 accumulators
// Per-frame bound words of a flat call: [0] the shared filter bound, [8, 16)
// the group slots (one 32-byte aligned pair of 16-byte loads)
constexpr int kBoundWords = 16;
constexpr int kBoundSlotWord = 8;
constexpr int kBoundSlots = 8;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint32_t kFormatF16 = 0;

struct CandArgs {
    int frames;  // rows of the query matrix (padding rows past it are skipped)
    int n_qtiles;
    int segments;
    int tiles_per_seg;
    int ksteps;
    int64_t n;
    int64_t seg_rows;
    const float *row_norms;
    float coef;  // -2 / s^2
    // flat: keys [frame][lists][K] and thresholds [frame][thr_stride], list =
    // seg * kHalves + half, so a frame's candidates are one contiguous block;
    // IVF fine stage: keys [half][K][pair], counts and thresholds [half][pair]
    unsigned long long *out_keys;
    int *out_count;  // IVF only
    float *out_thr;
    int lists;       // flat: candidate lists per frame (segments * kHalves)
    int thr_stride;  // flat: lists rounded up to a multiple of 4 (16-byte rows)
    DeviceCounters *counters;
    // IVF fine stage only: work items (list, frame tile within the list's
    // pairs) from a device table; A rows are the (frame, probe) pairs of the
    // list in list order, B rows the list's rows.
    const int2 *items;
    const int *item_count;
    const int32_t *list_offsets;  // database row offsets [nlist + 1]
    const int32_t *list_start;    // pair offsets [nlist + 1] (lists in size order, not id order)
    const int32_t *list_count;    // pairs per list [nlist]
    int pair_stride;              // output stride: pairs capacity
    int pair_layout;              // flat, kPairLayout: items are (query-tile pair, segment)
    // Per-frame bound words shared by every CTA (null: off; flat, and the
    // IVF fine stage): kBoundWords per frame, total-order bits of approximate
    // distances d~, +inf at call start.  Word 0: a list whose 8 best so far
    // have d~ <= u publishes u + 2e + slack, a d~ no row of the frame's exact
    // top 8 reaches or ties.  Words 8-15: group slots, the smallest best d~
    // of the lists in each group (disjoint rows).  Every CTA may drop rows
    // above the bounds; a list's reported threshold is then min(its K-th
    // best, the bounds it used), which keeps the certificate.
    unsigned int *gbound;
    const float4 *qstats;          // (||q||^2, ||q^||, ||q - q^||) per frame
    const int32_t *pair_frame;     // IVF fine stage: the frame of each A row (pair)
    float max_norm, max_hat, max_residual, acc_rel, norm_rel, exact_rel;
};

// One work item: A rows [a_row0, a_row0 + a_rows) against database rows
// [b_row0, b_end), in `tiles` tiles of kTileN rows.
struct Item {
    int a_row0;
    int a_rows;
    int64_t b_row0;
    int64_t b_end;
    int tiles;
    int seg;  // flat only
};

template <bool kIvf>
__device__ __forceinline__ int item_total(const CandArgs &a) {
    if constexpr (kIvf) return *a.item_count;
    else return a.segments * (a.pair_layout ? (a.n_qtiles + 1) / 2 : a.n_qtiles);
}

// IVF items come largest first (the item table follows the lists in
// descending size); CTA g takes items g, g + G, ... of a "snake" order that
// reverses every other round of G, so each CTA's load evens out.
template <bool kIvf>
__device__ __forceinline__ Item item_at(const CandArgs &a, int item, int total, int rank = 0) {
    Item it{};
    if constexpr (kIvf) {
        const int g = static_cast<int>(gridDim.x);
        const int round = item / g, pos = item - round * g;
        const int in_round = min(g, total - round * g);
        const int2 e = a.items[(round & 1) ? round * g + (in_round - 1 - pos) : item];
        it.a_row0 = a.list_start[e.x] + e.y * kTileM;
        it.a_rows = min(kTileM, a.list_start[e.x] + a.list_count[e.x] - it.a_row0);
        it.b_row0 = a.list_offsets[e.x];
        it.b_end = a.list_offsets[e.x + 1];
        it.seg = e.x;  // the list (its group slot in the frames' bound words)
    } else {
        // pair layout: CTA `rank` of the pair takes query tile 2 p + rank
        // (the second tile of an odd count is padding: no frames)
        const int per_seg = a.pair_layout ? (a.n_qtiles + 1) / 2 : a.n_qtiles;
        const int qtile = a.pair_layout ? 2 * (item % per_seg) + rank : item % per_seg;
        it.seg = item / per_seg;
        it.a_row0 = qtile * kTileM;
        it.a_rows = max(0, min(kTileM, a.frames - it.a_row0));
        it.b_row0 = it.seg * a.seg_rows;
        it.b_end = min(it.b_row0 + a.seg_rows, a.n);
    }
    it.tiles = static_cast<int>((it.b_end - it.b_row0 + kTileN - 1) / kTileN);
    return it;
}

// Sorted ascending list of the kItemKeep smallest approximate distances seen
// (with their rows), in registers.  Insertion is a fixed compare-exchange
// chain, so the lanes of a warp that insert in the same step share it.  Ties
// between equal approximate distances may resolve either way: only "every
// dropped row has d~ >= the threshold" matters to the exact stage.
template <int kItemKeep>
struct TopList {
    float dist[kItemKeep];
    uint32_t row[kItemKeep];
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int i = 0; i < kItemKeep; ++i) {
            dist[i] = __int_as_float(0x7f800000);
            row[i] = 0;
        }
    }
    // Replaces the list with the kItemKeep smallest of (list U chunk): sorts
    // the 16 chunk values with a bitonic network, takes the elementwise
    // minimum of the list and the chunk's kItemKeep smallest reversed (a
    // bitonic sequence holding the kItemKeep smallest of both), and cleans it.
    // Cheaper than one insertion per value once many values of the chunk pass
    // the threshold.
    __device__ __forceinline__ void merge16(float (&cd)[16], uint32_t (&cr)[16]) {
        static_assert(kItemKeep <= 16 && (kItemKeep & (kItemKeep - 1)) == 0, "power of two up to 16");
#pragma unroll
        for (int k = 2; k <= 16; k <<= 1) {
#pragma unroll
            for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int l = i ^ j;
                    if (l > i) {
                        const bool asc = (i & k) == 0;
                        const bool swap = asc ? (cd[l] < cd[i]) : (cd[i] < cd[l]);
                        const float a0 = cd[i], a1 = cd[l];
                        const uint32_t b0 = cr[i], b1 = cr[l];
                        cd[i] = swap ? a1 : a0;
                        cd[l] = swap ? a0 : a1;
                        cr[i] = swap ? b1 : b0;
                        cr[l] = swap ? b0 : b1;
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kItemKeep; ++i) {
            const bool take = cd[kItemKeep - 1 - i] < dist[i];
            dist[i] = take ? cd[kItemKeep - 1 - i] : dist[i];
            row[i] = take ? cr[kItemKeep - 1 - i] : row[i];
        }
#pragma unroll
        for (int j = kItemKeep / 2; j > 0; j >>= 1) {
#pragma unroll
            for (int i = 0; i < kItemKeep; ++i) {
                const int l = i ^ j;
                if (l > i) {
                    const bool swap = dist[l] < dist[i];
                    const float a0 = dist[i], a1 = dist[l];
                    const uint32_t b0 = row[i], b1 = row[l];
                    dist[i] = swap ? a1 : a0;
                    dist[l] = swap ? a0 : a1;
                    row[i] = swap ? b1 : b0;
                    row[l] = swap ? b0 : b1;
                }
            }
        }
    }
    __device__ __forceinline__ void insert(float dd, uint32_t r) {
        dist[kItemKeep - 1] = dd;
        row[kItemKeep - 1] = r;
#pragma unroll
        for (int i = kItemKeep - 1; i > 0; --i) {
            const bool swap = dist[i] < dist[i - 1];
            const float lo = swap ? dist[i] : dist[i - 1], hi = swap ? dist[i - 1] : dist[i];
            const uint32_t rl = swap ? row[i] : row[i - 1], rh = swap ? row[i - 1] : row[i];
            dist[i - 1] = lo;
            dist[i] = hi;
            row[i - 1] = rl;
            row[i] = rh;
        }
    }
};

// The frame's exactness certificate: every dropped candidate has an
// approximate distance >= bound; qs = (||q||^2, ||q^||, ||q - q^||); the
// database bounds are max ||x||, max ||x^||, max ||x - x^||.  True when no
// dropped candidate can reach (or tie) the `rank`-th exact distance dk.
// The bound e on |(d~ + ||q||^2) - true distance| for an approximate key
// distance d~ of this frame (the certificate's error model).
__device__ __forceinline__ float approx_error(float4 qs, float max_norm, float max_hat, float max_residual,
                                              float acc_rel, float norm_rel) {
    return 2.f * (qs.y * max_residual + qs.z * max_norm) + 2.f * acc_rel * qs.y * max_hat +
           norm_rel * (max_norm * max_norm + qs.x) + 6e-8f * (max_norm * max_norm + 2.f * qs.y * max_hat);
}

// A list's own filter bound from its 8th best approximate distance u (the
// frame's qe = ||q||^2 + e and 2e): the 8 rows at or below u have exact
// distances within (u + qe)(1 + exact_rel), so no row whose d~ exceeds
// u + 2e + slack reaches or ties the frame's exact 8th best (+inf while the
// list holds fewer than 8).
__device__ __forceinline__ float own_bound(float u, float qe, float two_e, float exact_rel) {
    return u + two_e + (8.f * exact_rel * fabsf(u + qe) + 1e-6f * (fabsf(u) + fabsf(qe)) + 1e-30f);
}

// A frame's bound from its bound words (kBoundWords layout): the smaller of
// the shared word and the own bound of the group slots' maximum.
__device__ __forceinline__ float frame_bound(const unsigned int *w, float qe, float two_e, float exact_rel) {
    const uint4 s0 = __ldcg(reinterpret_cast<const uint4 *>(w + kBoundSlotWord));
    const uint4 s1 = __ldcg(reinterpret_cast<const uint4 *>(w + kBoundSlotWord + 4));
    // total-order bits: the largest word is the largest value
    const uint32_t umax = max(max(max(s0.x, s0.y), max(s0.z, s0.w)), max(max(s1.x, s1.y), max(s1.z, s1.w)));
    return fminf(from_total_order_bits(__ldcg(w)), own_bound(from_total_order_bits(umax), qe, two_e, exact_rel));
}

// Four consecutive row norms.  Flat segments start on tile boundaries, so the
// address is 16-byte aligned; IVF lists start anywhere.
template <bool kIvf>
__device__ __forceinline__ float4 load_norms4(const float *p) {
    if constexpr (kIvf) return make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
    else return __ldg(reinterpret_cast<const float4 *>(p));
}

template <bool kIvf, int K, int kLayout = kFullLayout>
__global__ void __launch_bounds__(kThreadsTC, 1)
    cand_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_x, CandArgs a) {
    using P = Pipe<kLayout>;
    constexpr int kStages = P::kStages;
    constexpr bool kPair = kLayout == kPairLayout;
    static_assert(!kIvf || kLayout == kFullLayout, "IVF work items use the full layout");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + P::kBarOff);
    uint64_t *full = bars;
    uint64_t *empty = bars + kStages;
    uint64_t *acc_full = bars + 2 * kStages;
    uint64_t *acc_empty = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    launch_dependents();
    // the IVF work-item table comes from the kernels before this one; the
    // flat producer waits for the query tiles only (below)
    if constexpr (kIvf) grid_dependency_wait();
    const int items = item_total<kIvf>(a);
    // pair layout: the cluster is the unit of work; CTA rank 0 (the leader)
    // issues the MMA and owns the stage barriers both CTAs' loads complete
    const int rank = kPair ? static_cast<int>(tc::cluster_rank()) : 0;
    const int first_item = kPair ? static_cast<int>(tc::cluster_id()) : static_cast<int>(blockIdx.x);
    const int item_step = kPair ? static_cast<int>(tc::cluster_count()) : static_cast<int>(gridDim.x);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&acc_full[b], 1);
            tc::mbar_init(&acc_empty[b], kPair ? 2 * kEpiWarps : kEpiWarps);
        }
        *abort_flag = 0;
        tc::fence_mbarrier_init();
    }
    if (warp == 0 && lane == 0) {
        tc::tma_prefetch(&tmap_q);
        tc::tma_prefetch(&tmap_x);
    }
    if (warp == 1) {
        if constexpr (kPair) {
            tc::tmem_alloc_pair(tmem_slot, kTmemCols);
            tc::tmem_relinquish_pair();
        } else {
            tc::tmem_alloc(tmem_slot, kTmemCols);
            tc::tmem_relinquish();
        }
    }
    tc::tc_fence_before();
    if constexpr (kPair) tc::cluster_sync();  // the leader's barriers exist before the other CTA's loads
    else __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&]() {
        *abort_flag = 1;
        if (a.counters) atomicAdd(&a.counters->timeouts, 1ull);
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            // Flat: the database tiles of the first stages do not depend on
            // the query preparation, so they are requested before waiting
            // for it; those stages then only add their query tile.
            // pair layout: this CTA's database rows are its half of each
            // tile; every load completes on the leader's stage barrier,
            // whose expected bytes (both CTAs' loads) the leader sets
            const int32_t b_half = kPair ? rank * (kTileN / 2) : 0;
            auto stage_bar = [&](int st) -> uint32_t {
                return kPair ? tc::map_to_rank(&full[st], 0) : tc::smem_u32(&full[st]);
            };
            auto load = [&](void *dst, const CUtensorMap *map, int st, int32_t x, int32_t y) {
                if constexpr (kPair) tc::tma_load_2d_pair(dst, map, stage_bar(st), x, y);
                else tc::tma_load_2d(dst, map, &full[st], x, y);
            };
            int early = 0;
            if constexpr (!kIvf) {
                if (first_item < items) {
                    const Item it0 = item_at<kIvf>(a, first_item, items, rank);
                    early = min(kStages, it0.tiles * a.ksteps);
                    for (int s = 0; s < early; ++s) {
                        const int t = s / a.ksteps, k = s % a.ksteps;
                        if (rank == 0) tc::mbar_arrive_expect_tx(&full[s], P::kTx);
                        load(smem + P::b_off(s), &tmap_x, s, k * kTileK,
                             static_cast<int32_t>(it0.b_row0 + t * kTileN) + b_half);
                    }
                }
                grid_dependency_wait();
            }
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            for (int item = first_item; item < items && !*abort_flag; item += item_step) {
                const Item it = item_at<kIvf>(a, item, items, rank);
                for (int t = 0; t < it.tiles && !*abort_flag; ++t) {
                    for (int k = 0; k < a.ksteps; ++k, ++issued) {
                        if (!tc::mbar_wait(&empty[stage], phase ^ 1, kWaitLimitNs)) {
                            fail();
                            break;
                        }
                        if (issued >= early) {  // else the database tile is already requested
                            if (rank == 0) tc::mbar_arrive_expect_tx(&full[stage], P::kTx);
                            load(smem + P::b_off(stage), &tmap_x, stage, k * kTileK,
                                 static_cast<int32_t>(it.b_row0 + t * kTileN) + b_half);
                        }
#pragma unroll
                        for (int qb = 0; qb < P::kBlocks; ++qb)
                            load(smem + P::a_block_off(stage, qb), &tmap_q, stage, k * kTileK,
                                 it.a_row0 + qb * P::kBlockRows);
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            // let every issued copy land before the CTA can exit
            for (int s = 0; s < kStages; ++s) {
                if (!tc::mbar_wait(&empty[stage], phase ^ 1, kWaitLimitNs)) break;
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
        // Lanes 1-31 wait here for the producer lane, so the warp reaches
        // the CTA barrier below converged: lanes left parked at that barrier
        // for the whole kernel resumed microseconds after it released.
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (one thread; the pair's leader)
            const uint32_t idesc = tc::idesc_f16(P::kM, kTileN, kFormatF16);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t acc_count = 0;
            for (int item = first_item; item < items && !*abort_flag; item += item_step) {
                const Item it = item_at<kIvf>(a, item, items, rank);
                for (int t = 0; t < it.tiles && !*abort_flag; ++t) {
                    const uint32_t b = acc_count & 1;
                    if (!tc::mbar_wait(&acc_empty[b], ((acc_count >> 1) & 1) ^ 1, kWaitLimitNs)) {
                        fail();
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t d_tmem = tmem + b * kTileN;
                    bool ok = true;
                    for (int k = 0; k < a.ksteps; ++k) {
                        if (!tc::mbar_wait(&full[stage], phase, kWaitLimitNs)) {
                            fail();
                            ok = false;
                            break;
                        }
                        tc::tc_fence_after();
                        const uint32_t sa = tc::smem_u32(smem + P::a_off(stage));
                        const uint32_t sb = tc::smem_u32(smem + P::b_off(stage));
#pragma unroll
                        for (int kk = 0; kk < kTileK / 16; ++kk) {
                            if constexpr (kPair)
                                tc::mma_f16_pair(d_tmem, tc::smem_desc_sw128(sa + kk * 32),
                                                 tc::smem_desc_sw128(sb + kk * 32), idesc, (k | kk) != 0);
                            else
                                tc::mma_f16(d_tmem, tc::smem_desc_sw128(sa + kk * 32),
                                            tc::smem_desc_sw128(sb + kk * 32), idesc, (k | kk) != 0);
                        }
                        if constexpr (kPair) tc::mma_commit_pair(&empty[stage]);  // both CTAs' stage
                        else tc::mma_commit(&empty[stage]);
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    if constexpr (kPair) tc::mma_commit_pair(&acc_full[b]);  // both CTAs' epilogues
                    else tc::mma_commit(&acc_full[b]);
                    ++acc_count;
                }
            }
        }
        __syncwarp();  // converged at the CTA barrier, as the producer warp
    } else {
        // ---------------- epilogue: one thread per frame of the tile; the two
        // warps of a TMEM lane quarter split each tile's columns in halves.
        // The frames' statistics and bound words come from the preparation
        // kernel: wait for it (flat; the IVF kernel waited at its start).
        if constexpr (!kIvf) grid_dependency_wait();
        const int ew = warp - 2;
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        const int half = ew >> 2;
        constexpr int kHalfCols = kTileN / kHalves;
        // this lane's frame in the tile: lanes past the layout's rows per
        // quarter hold no frame (spread layout)
        const int r = quarter * P::kRowsPerQuarter + lane;
        const bool lane_real = lane < P::kRowsPerQuarter;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        uint32_t acc_count = 0;
        const float inf = __int_as_float(0x7f800000);
        // pair layout: the accumulator is the leader's to reuse; both CTAs'
        // epilogue warps release it on the leader's barrier
        auto release_acc = [&](uint32_t buf) {
            if (kPair && rank != 0) tc::mbar_arrive_cluster(tc::map_to_rank(&acc_empty[buf], 0));
            else tc::mbar_arrive(&acc_empty[buf]);
        };
        for (int item = first_item; item < items && !*abort_flag; item += item_step) {
            const Item it = item_at<kIvf>(a, item, items, rank);
            const int64_t row0 = it.b_row0;
            const int tiles = it.tiles;
            TopList<K> top;
            top.init();
            bool aborted = false;
            // The frame's bound words (flat, when enabled; kBoundWords per
            // frame): word 0 is the shared filter bound, the minimum of every
            // list's published own bound; words 8-15 are group slots, slot j
            // the smallest best d~ of the lists whose index is j mod 8.  Rows
            // of different slots come from disjoint lists, so the 8 slots name
            // 8 distinct rows and their maximum bounds the frame's 8th best as
            // a list's own 8th best does.  Both are read at every tile start
            // and published after every tile that improved them.  The list's
            // own bound (its 8th best u plus 2e and rounding slack, a d~ no
            // row of the frame's exact top 8 reaches) filters at once.
            unsigned int *gp = nullptr;
            float g = inf, qe = 0.f, two_e = 0.f, published = inf, own = inf, best_published = inf;
            const int slot = (it.seg * kHalves + half) & (kBoundSlots - 1);
            {
                if (a.gbound != nullptr && lane_real && r < it.a_rows) {
                    const long long fr = kIvf ? static_cast<long long>(a.pair_frame[it.a_row0 + r])
                                              : static_cast<long long>(it.a_row0) + r;
                    const float4 qs = a.qstats[fr];
                    const float e = approx_error(qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel, a.norm_rel);
                    gp = a.gbound + fr * kBoundWords;
                    qe = qs.x + e;
                    two_e = 2.f * e;
                }
            }
            // This warp's copy of the row norms, one tile ahead: lane l holds
            // norms [4l, 4l+4) of the next tile's half in registers until the
            // current tile is done, then stores them into the other buffer.
            float *nbuf = reinterpret_cast<float *>(smem + P::norm_off(ew));
            {
                reinterpret_cast<float4 *>(nbuf)[lane] = load_norms4<kIvf>(a.row_norms + row0 + half * kHalfCols + lane * 4);
                __syncwarp();
            }
            for (int t = 0; t < tiles; ++t) {
                const uint32_t b = acc_count & 1;
                const uint32_t tile_row = static_cast<uint32_t>(row0 + static_cast<int64_t>(t) * kTileN);
                float4 pre0 = make_float4(0.f, 0.f, 0.f, 0.f);
                if (t + 1 < tiles) pre0 = load_norms4<kIvf>(a.row_norms + tile_row + kTileN + half * kHalfCols + lane * 4);
                if (gp != nullptr) g = frame_bound(gp, qe, two_e, a.exact_rel);
                // every lane polls; the outcome is made warp-uniform before the
                // .sync.aligned TMEM loads
                const bool ready = tc::mbar_wait(&acc_full[b], (acc_count >> 1) & 1, kWaitLimitNs);
                if (!__all_sync(kFullMask, ready)) {
                    if (lane == 0) fail();
                    aborted = true;
                    break;
                }
                tc::tc_fence_after();
                if (quarter * P::kRowsPerQuarter >= it.a_rows) {
                    // every TMEM lane of this warp is a padding row of a partial
                    // frame tile: release the accumulator without reading it
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) release_acc(b);
                    ++acc_count;
                    continue;
                }
                // Segments start on tile boundaries and rows past n carry +inf
                // norms, so every column of the tile can be filtered as is.
                const float *cur_norms = nbuf + (t & 1) * kHalfCols;
                const uint32_t tcol = tmem + lane_addr + b * kTileN + half * kHalfCols;
                const uint32_t col_row = tile_row + half * kHalfCols;
                float v[2][16];
                __syncwarp();
                tc::tmem_ld16(tcol, v[0]);
#pragma unroll 2
                for (int c = 0; c < kHalfCols / 16; ++c) {
                    const int cur = c & 1;
                    if (c + 1 < kHalfCols / 16) {
                        __syncwarp();
                        tc::tmem_ld16_nowait(tcol + (c + 1) * 16, v[cur ^ 1]);
                    }
                    // filter against the threshold at chunk start: the chunk's
                    // minimum first, and the survivor mask only when some lane
                    // of the warp has a survivor (in steady state most chunks
                    // have none, and the vote is warp-uniform)
                    float dd[16];
                    uint32_t mask = 0;
                    const float thr = fminf(fminf(top.dist[K - 1], g), own);
                    // IVF: rows past the list's end belong to the next list
                    const int64_t lim = kIvf ? it.b_end - (static_cast<int64_t>(col_row) + c * 16) : 16;
#pragma unroll
                    for (int e4 = 0; e4 < 4; ++e4) {
                        const float4 nn = reinterpret_cast<const float4 *>(cur_norms + c * 16)[e4];
                        const float nv[4] = {nn.x, nn.y, nn.z, nn.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int e = e4 * 4 + u;
                            dd[e] = fmaf(a.coef, v[cur][e], nv[u]);
                            if constexpr (kIvf) dd[e] = e < lim ? dd[e] : inf;
                        }
                    }
                    float lo8[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) lo8[e] = fminf(dd[e], dd[e + 8]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) lo8[e] = fminf(lo8[e], lo8[e + 4]);
                    const float cmin = fminf(fminf(lo8[0], lo8[2]), fminf(lo8[1], lo8[3]));
                    // lanes with no frame hold no distances (spread layout)
                    const bool survive = __any_sync(kFullMask, lane_real && cmin < thr);  // warp-uniform
                    if (survive) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) mask |= (dd[e] < thr ? 1u : 0u) << e;
                        if (!lane_real) mask = 0u;
                    }
                    // many survivors (the start of an item): one bulk merge for
                    // the warp; otherwise insert the few survivors one by one
                    // (re-checked, the threshold drops as they go in)
                    if (survive && __reduce_max_sync(kFullMask, static_cast<unsigned>(__popc(mask))) >= 6u) {
                        uint32_t cr[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) cr[e] = col_row + c * 16 + e;
                        top.merge16(dd, cr);
                        if (gp != nullptr) own = own_bound(top.dist[7], qe, two_e, a.exact_rel);
                        mask = 0;
                    }
                    while (mask) {
                        const int e = __ffs(mask) - 1;
                        mask &= mask - 1;
                        float x = dd[0];
#pragma unroll
                        for (int i = 1; i < 16; ++i) x = e == i ? dd[i] : x;
                        if (x < fminf(top.dist[K - 1], own)) {
                            top.insert(x, col_row + c * 16 + e);
                            if (gp != nullptr) own = own_bound(top.dist[7], qe, two_e, a.exact_rel);
                        }
                    }

                    if (c + 1 < kHalfCols / 16) tc::tmem_wait_ld(v[cur ^ 1]);
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(b);
                ++acc_count;
                if (gp != nullptr && top.dist[7] < published) {
                    published = top.dist[7];
                    atomicMin(gp, total_order_bits(own));
                }
                if (gp != nullptr && top.dist[0] < best_published) {
                    best_published = top.dist[0];
                    atomicMin(gp + kBoundSlotWord + slot, total_order_bits(best_published));
                }
                if (t + 1 < tiles) {
                    reinterpret_cast<float4 *>(nbuf + ((t + 1) & 1) * kHalfCols)[lane] = pre0;
                    __syncwarp();
                }
            }
            if (aborted) break;
            int cnt = 0;
#pragma unroll
            for (int i = 0; i < K; ++i) cnt += top.dist[i] < inf;
            if constexpr (kIvf) {
                if (r < it.a_rows) {
                    const size_t pos = static_cast<size_t>(it.a_row0) + r;
                    const size_t stride = static_cast<size_t>(a.pair_stride);
#pragma unroll
                    for (int i = 0; i < K; ++i)
                        if (i < cnt) a.out_keys[(half * K + i) * stride + pos] = make_key(top.dist[i], top.row[i]);
                    a.out_count[half * stride + pos] = cnt;
                    // as flat lists: min(K-th best, the last shared bound read, own bound)
                    a.out_thr[half * stride + pos] = fminf(fminf(cnt == K ? top.dist[K - 1] : inf, g), own);
                }
            } else if (lane_real && r < it.a_rows) {
                // every slot is written (kEmptyKey past cnt), so the merge
                // copies a frame's block without reading counts
                const size_t frame = static_cast<size_t>(it.a_row0) + r;
                const int list = it.seg * kHalves + half;
                ulonglong2 *dk = reinterpret_cast<ulonglong2 *>(a.out_keys + (frame * a.lists + list) * K);
#pragma unroll
                for (int i = 0; i < K; i += 2)
                    dk[i / 2] = make_ulonglong2(i < cnt ? make_key(top.dist[i], top.row[i]) : kEmptyKey,
                                                i + 1 < cnt ? make_key(top.dist[i + 1], top.row[i + 1]) : kEmptyKey);
                // rows this list dropped have d~ >= min(its K-th best, the
                // smallest shared bound it filtered with (the last one read),
                // its own final bound); all three only ever decrease
                a.out_thr[frame * a.thr_stride + list] = fminf(fminf(cnt == K ? top.dist[K - 1] : inf, g), own);
            }
        }
    }
    tc::tc_fence_before();
    if constexpr (kPair) tc::cluster_sync();  // neither CTA leaves while the other may use its memory
    else __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        if constexpr (kPair) tc::tmem_dealloc_pair(tmem, kTmemCols);
        else tc::tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------- queries
__global__ void prep_queries_kernel(const float *__restrict__ q, __half *__restrict__ qh, float4 *__restrict__ stats,
                                    long long frames, int d, int d_pad, float scale, int32_t *zero,
                                    unsigned int *gbound) {
    launch_dependents();  // the candidate kernel may start its prologue and database loads now
    if (blockIdx.x == 0 && threadIdx.x == 0 && zero) *zero = 0;  // the call's fallback frame count
    const long long f = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (f >= frames) return;
    const float inv = 1.0f / scale;  // exact: scale is a power of two
    float qn2 = 0.f, hat2 = 0.f, res2 = 0.f;
#pragma unroll 8
    for (int k = lane; k < d_pad; k += 32) {
        float v = k < d ? q[f * d + k] : 0.f;
        float sv = fminf(fmaxf(v * scale, -65504.f), 65504.f);
        __half h = __float2half_rn(sv);
        qh[f * d_pad + k] = h;
        float back = __half2float(h) * inv;
        float res = v - back;
        qn2 = fmaf(v, v, qn2);
        hat2 = fmaf(back, back, hat2);
        res2 = fmaf(res, res, res2);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        qn2 += __shfl_xor_sync(kFullMask, qn2, s);
        hat2 += __shfl_xor_sync(kFullMask, hat2, s);
        res2 += __shfl_xor_sync(kFullMask, res2, s);
    }
    if (lane == 0) {
        stats[f] = make_float4(qn2, sqrtf(hat2) * 1.00001f, sqrtf(res2) * 1.00001f, 0.f);
    }
    if (gbound && lane < kBoundWords)
        gbound[f * kBoundWords + lane] = total_order_bits(__int_as_float(0x7f800000));
}

// ---------------------------------------------------------------- merge
struct MergeArgs {
    int keep;  // keys per candidate list (kShortKeep or kIvfKeep)
    int d;
    int lists;       // candidate lists per frame
    int thr_stride;  // thresholds per frame row (lists rounded up to 4)
    int sort_size;   // key slots per frame: lists * keep rounded up to 32
    const unsigned long long *keys;  // [frame][lists][keep]
    const float *thr;                // [frame][thr_stride]
    const float4 *qstats;
    const float *queries;
    float *out;
    const float *index_rate;
    int mode;
    int k;
    float *dist_out;
    int64_t *label_out;
    int64_t label_base;
    const float *vectors;
    const int32_t *ids;
    float max_norm, max_hat, max_residual;
    float acc_rel;     // bound on the relative fp32 accumulation error of a dot product
    float norm_rel;    // bound on the relative error of an fp32 squared norm
    float exact_rel;   // bound on the relative error of the exact fp32 distance
    int32_t *fallback_list;
    int32_t *fallback_count;
    DeviceCounters *counters;
    int stage_rows;  // re-rank rows staged in shared memory per chunk (0: read them from global memory)
    float *raw_out;  // optional: the frames before the blend (RetrievalProtection::save_raw)
    const unsigned int *gbound;  // flat: the call's per-frame bound words (kBoundWords each), or null
};

constexpr int kMergeThreads = 256;     // per frame, when many frames share the GPU
constexpr int kMergeThreadsMax = 512;  // per frame, when a launch has few frames


// Shared state of select_rerank (one per CTA, in shared memory).
struct SelectState {
    unsigned int hist[2][256];  // radix passes alternate between the two
    uint32_t bin, below_bin, in_bin;
    uint32_t dropped_min;
    int count;
    float red_f[kMergeThreadsMax / 32];
    int red_i[kMergeThreadsMax / 32];
    uint32_t red_lo[kMergeThreadsMax / 32], red_hi[kMergeThreadsMax / 32];
    float all_f;
    int all_i;
    uint32_t all_lo, all_hi;
};

// The real keys among a CTA's key slots: how many, and the smallest and
// largest distance bits; plus the block-wide min of each thread's `tmin`.
struct KeyStats {
    int total;
    uint32_t lo, hi;
    float tmin;
};

// Block-wide KeyStats over keys[0 .. slots) (in shared memory); every thread
// of the CTA calls it and gets the result.  Its barrier also publishes the
// shared-memory writes made before the call.
template <int kT>
__device__ KeyStats key_stats(const unsigned long long *keys, int slots, float tmin, SelectState &st) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    KeyStats ks{0, 0xffffffffu, 0u, tmin};
    for (int i = tid; i < 256; i += kT) st.hist[0][i] = 0u;  // select_rerank's first pass
    for (int i = tid; i < slots; i += kT) {
        const unsigned long long key = keys[i];
        if (key != kEmptyKey) {
            const uint32_t b = static_cast<uint32_t>(key >> 32);
            ks.lo = min(ks.lo, b);
            ks.hi = max(ks.hi, b);
            ++ks.total;
        }
    }
    ks.total = __reduce_add_sync(kFullMask, ks.total);
    ks.lo = __reduce_min_sync(kFullMask, ks.lo);
    ks.hi = __reduce_max_sync(kFullMask, ks.hi);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) ks.tmin = fminf(ks.tmin, __shfl_xor_sync(kFullMask, ks.tmin, s));
    if (lane == 0) {
        st.red_i[warp] = ks.total;
        st.red_lo[warp] = ks.lo;
        st.red_hi[warp] = ks.hi;
        st.red_f[warp] = ks.tmin;
    }
    __syncthreads();
    if (warp == 0) {  // combines the warps' partials, then every thread reads the result
        const bool have = lane < kT / 32;
        int t = have ? st.red_i[lane] : 0;
        uint32_t l = have ? st.red_lo[lane] : 0xffffffffu, h = have ? st.red_hi[lane] : 0u;
        float f = have ? st.red_f[lane] : __int_as_float(0x7f800000);
        t = __reduce_add_sync(kFullMask, t);
        l = __reduce_min_sync(kFullMask, l);
        h = __reduce_max_sync(kFullMask, h);
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) f = fminf(f, __shfl_xor_sync(kFullMask, f, s));
        if (lane == 0) {
            st.all_i = t;
            st.all_lo = l;
            st.all_hi = h;
            st.all_f = f;
        }
    }
    __syncthreads();
    return KeyStats{st.all_i, st.all_lo, st.all_hi, st.all_f};
}

// Keys kept for the exact re-rank when a radix pass can stop early: the pass
// stops once the keys at or below the bin holding the kRerank-th smallest
// distance number at most this many (or fewer, as the caller asks: the rows
// its shared memory can stage at once).
constexpr int kRerankStop = 80;

constexpr int kWideBins = 4096;  // bins of the optional 12-bit first pass

// Chooses the keys to re-rank among keys[0 .. slots) (ks from key_stats; the
// slots past the real keys hold kEmptyKey; slots a multiple of 32) without
// sorting them.  A radix select over the distance bits below the real keys'
// common prefix finds the digit bin holding the kRerank-th smallest distance
// (a first 12-bit digit when the caller lends a `wide` histogram of
// kWideBins cleared bins, then 8-bit digits); it refines that bin only while
// the keys at or below it number more than rerank_stop.  Every key at or
// below the final bin is kept (kRerank to rerank_stop keys, or up to
// kRerankMax when distances tie in every bit, with `too_many` reporting an
// overflow past kRerankMax).  Every dropped key has a larger approximate
// distance than every kept one; `bound` is the smallest dropped distance
// (+inf when nothing is dropped).  Histogram updates are aggregated per warp
// (match_any), so a crowded digit costs one shared atomic per warp.
// Returns the number of keys written to sel_keys.  Called by every thread of
// the CTA.

template <int kT>
__device__ int select_rerank(const unsigned long long *keys, int slots, const KeyStats &ks,
                             unsigned long long *sel_keys, SelectState &st, float &bound, bool &too_many,
                             unsigned int *wide = nullptr, int rerank_stop = kRerankStop) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int total = ks.total;
    const uint32_t lo = ks.lo, hi = ks.hi;
    const uint32_t stop = static_cast<uint32_t>(rerank_stop);
    uint32_t limit = 0xffffffffu;  // keep every real key whose distance bits are <= limit
    if (total > kRerank) {
        if (lo == hi) {
            limit = lo;  // every real key has the same distance
        } else {
            int top = 31 - __clz(lo ^ hi);               // highest bit in which the keys differ
            uint32_t mask_bits = ~((2u << top) - 1u);    // the common prefix (0 when top == 31)
            uint32_t prefix = lo & mask_bits;
            uint32_t rank = kRerank, below = 0;          // 1-based rank inside the prefix group
            bool done = false;
            if (wide != nullptr) {
                // One 12-bit pass (kWideBins bins, cleared by the caller;
                // every real key shares the prefix here), usually enough on
                // its own.  Thread t owns bins [t * kPerLane, +kPerLane).
                constexpr int kPerLane = kWideBins / kT;
                const int shift = top > 11 ? top - 11 : 0;
                const uint32_t digits = (2u << (top - shift)) - 1u;
                for (int i = tid; i < slots; i += kT) {
                    const unsigned long long key = keys[i];
                    const bool in = key != kEmptyKey;
                    const uint32_t digit = in ? (static_cast<uint32_t>(key >> 32) >> shift) & digits : 0xffffffffu;
                    const unsigned peers = __match_any_sync(kFullMask, digit);
                    if (in && lane == __ffs(peers) - 1) atomicAdd(&wide[digit], __popc(peers));
                }
                __syncthreads();
                uint32_t c[kPerLane], sum = 0;
#pragma unroll
                for (int k = 0; k < kPerLane; ++k) {
                    c[k] = wide[tid * kPerLane + k];
                    sum += c[k];
                }
                uint32_t incl = sum;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t up = __shfl_up_sync(kFullMask, incl, off);
                    if (lane >= off) incl += up;
                }
                if (lane == 31) st.red_i[warp] = static_cast<int>(incl);
                __syncthreads();
                uint32_t before = 0;
                for (int w = 0; w < warp; ++w) before += static_cast<uint32_t>(st.red_i[w]);
                if (tid == kT - 1 && before + incl < rank) {  // cannot happen: `total` counts the real keys
                    st.bin = digits;
                    st.below_bin = 0u;
                    st.in_bin = kRerankMax + 1u;
                }
                uint32_t acc = before + incl - sum;
                if (acc < rank && rank <= before + incl) {
                    for (int k = 0; k < kPerLane; ++k) {
                        if (acc + c[k] >= rank) {
                            st.bin = static_cast<uint32_t>(tid * kPerLane + k);
                            st.below_bin = acc;
                            st.in_bin = c[k];
                            break;
                        }
                        acc += c[k];
                    }
                }
                __syncthreads();
                const uint32_t bin = st.bin, acc_b = st.below_bin, cnt = st.in_bin;
                if (below + acc_b + cnt <= stop || shift == 0) {
                    limit = prefix | (bin << shift) | ((1u << shift) - 1u);
                    done = true;
                } else {
                    below += acc_b;
                    rank -= acc_b;
                    prefix |= bin << shift;
                    mask_bits |= digits << shift;
                    top = shift - 1;
                }
            }
            int pass = 0;
            while (!done) {
                const int shift = top > 7 ? top - 7 : 0;
                const uint32_t digits = (2u << (top - shift)) - 1u;
                unsigned int *hist = st.hist[pass & 1];  // cleared before this pass
                for (int i = tid; i < slots; i += kT) {
                    const unsigned long long key = keys[i];
                    const uint32_t b = static_cast<uint32_t>(key >> 32);
                    const bool in = key != kEmptyKey && (b & mask_bits) == prefix;
                    const uint32_t digit = in ? (b >> shift) & digits : 0xffffffffu;
                    const unsigned peers = __match_any_sync(kFullMask, digit);
                    if (in && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
                }
                __syncthreads();
                if (warp == 0) {
                    uint32_t c[8], sum = 0;
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        c[k] = hist[lane * 8 + k];
                        sum += c[k];
                    }
                    uint32_t incl = sum;
#pragma unroll
                    for (int off = 1; off < 32; off <<= 1) {
                        const uint32_t up = __shfl_up_sync(kFullMask, incl, off);
                        if (lane >= off) incl += up;
                    }
                    uint32_t acc = incl - sum;
                    if (lane == 31 && incl < rank) {  // cannot happen: `total` counts the real keys
                        st.bin = digits;
                        st.below_bin = 0u;
                        st.in_bin = kRerankMax + 1u;
                    }
                    if (acc < rank && rank <= incl) {
                        for (int k = 0; k < 8; ++k) {
                            if (acc + c[k] >= rank) {
                                st.bin = static_cast<uint32_t>(lane * 8 + k);
                                st.below_bin = acc;
                                st.in_bin = c[k];
                                break;
                            }
                            acc += c[k];
                        }
                    }
                } else {
                    // meanwhile the other warps clear the next pass's histogram
                    for (int i = tid - 32; i < 256; i += kT - 32) st.hist[(pass + 1) & 1][i] = 0u;
                }
                __syncthreads();
                const uint32_t bin = st.bin, acc = st.below_bin, cnt = st.in_bin;
                if (below + acc + cnt <= stop || shift == 0) {
                    limit = prefix | (bin << shift) | ((1u << shift) - 1u);
                    break;
                }
                below += acc;
                rank -= acc;
                prefix |= bin << shift;
                mask_bits |= digits << shift;
                top = shift - 1;
                ++pass;
            }
        }
    }
    if (tid == 0) {
        st.count = 0;
        st.dropped_min = 0xffffffffu;
    }
    __syncthreads();
    uint32_t dropped = 0xffffffffu;
    for (int i = tid; i < slots; i += kT) {
        const unsigned long long key = keys[i];
        if (key == kEmptyKey) continue;
        const uint32_t b = static_cast<uint32_t>(key >> 32);
        if (b <= limit) {
            const int pos = atomicAdd(&st.count, 1);
            if (pos < kRerankMax) sel_keys[pos] = key;
        } else {
            dropped = min(dropped, b);
        }
    }
    dropped = __reduce_min_sync(kFullMask, dropped);
    if (lane == 0 && dropped != 0xffffffffu) atomicMin(&st.dropped_min, dropped);
    __syncthreads();
    const int selected = st.count;
    too_many = selected > kRerankMax;
    bound = st.dropped_min != 0xffffffffu ? from_total_order_bits(st.dropped_min) : __int_as_float(0x7f800000);
    return selected < kRerankMax ? selected : kRerankMax;
}

// Reduces the octets' sorted top-8 lists (octet_best[kOct][8], kOct 32 or
// 64) to the CTA's top-8 keys in best[0..8); warp 0 does the work (with 64
// lists, lane l first merges lists l and l + 32), then the CTA syncs.
template <int kOct>
__device__ __forceinline__ void merge_octet_lists(const unsigned long long *octet_best, unsigned long long *best) {
    static_assert(kOct == 32 || kOct == 64, "octet lists per CTA");
    const int lane = threadIdx.x & 31;
    if ((threadIdx.x >> 5) == 0) {
        unsigned long long own[8];
        if constexpr (kOct == 32) {
#pragma unroll
            for (int i = 0; i < 8; ++i) own[i] = octet_best[lane * 8 + i];
        } else {
            // the 8 smallest of two sorted lists, in order
            const unsigned long long *x = octet_best + lane * 8, *y = octet_best + (lane + 32) * 8;
            int ix = 0, iy = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const unsigned long long vx = x[ix], vy = y[iy];
                const bool take_x = vx <= vy;
                own[i] = take_x ? vx : vy;
                ix += take_x;
                iy += !take_x;
            }
        }
        int head = 0;
        for (int i = 0; i < 8; ++i) {
            unsigned long long mine = kEmptyKey;
#pragma unroll
            for (int h = 0; h < 8; ++h) mine = h == head ? own[h] : mine;
            unsigned long long mn = mine;
#pragma unroll
            for (int s = 16; s > 0; s >>= 1) {
                unsigned long long o = __shfl_xor_sync(kFullMask, mn, s);
                mn = o < mn ? o : mn;
            }
            if (mine == mn && mn != kEmptyKey) ++head;
            if (lane == 0) best[i] = mn;
        }
    }
    __syncthreads();
}

__device__ __forceinline__ bool certify(float bound, float dk, float4 qs, float max_norm, float max_hat,
                                        float max_residual, float acc_rel, float norm_rel, float exact_rel) {
    if (!(bound < __int_as_float(0x7f800000)) && bound == bound) return true;  // nothing was dropped
    const float e = approx_error(qs, max_norm, max_hat, max_residual, acc_rel, norm_rel);
    const float lower = bound + qs.x - e;
    return lower > dk * (1.f + 4.f * exact_rel) + 1e-30f;
}

// Shared scratch of narrow_rerank.
struct NarrowState {
    unsigned long long keys[kRerankMax];
    int count;
    float upper;
};

// Drops from sel_keys[0 .. m) the candidates that cannot reach the frame's
// `rank`-th exact distance, so their rows are never fetched: with U the
// rank-th smallest upper bound d~ + ||q||^2 + e among them, a candidate
// whose lower bound d~ + ||q||^2 - e exceeds U (1 + 4 exact_rel) has an
// exact distance (reference order, relative error within exact_rel) above
// at least `rank` of the others, so it is neither in nor tied with the
// top `rank`.  The certificate over the candidates the selection dropped is
// unchanged.  Compacts sel_keys (order not kept); returns the count.  Called
// by every thread.
template <int kT>
__device__ int narrow_rerank(unsigned long long *sel_keys, int m, int rank, float qsx, float e, float exact_rel,
                             NarrowState &ns) {
    if (m <= rank) return m;
    const int tid = threadIdx.x;
    if (tid == 0) ns.count = 0;
    for (int c = tid; c < m; c += kT) {
        const unsigned long long key = sel_keys[c];
        int rk = 0;
        for (int i = 0; i < m; ++i) rk += sel_keys[i] < key;
        if (rk == rank - 1) ns.upper = key_dist(key);
    }
    __syncthreads();
    const float limit = (ns.upper + qsx + e) * (1.f + 4.f * exact_rel) + 1e-30f;
    for (int c = tid; c < m; c += kT) {
        const unsigned long long key = sel_keys[c];
        if (!(key_dist(key) + qsx - e > limit)) ns.keys[atomicAdd(&ns.count, 1)] = key;
    }
    __syncthreads();
    const int kept = ns.count;
    for (int c = tid; c < kept; c += kT) sel_keys[c] = ns.keys[c];
    __syncthreads();
    return kept;
}

// Exact distances of staged rows [0, rows) (stage rows of `stride` floats;
// sel_keys / exact_keys indexed from c0): octet o takes rows o, o + kOct, ...
// up to N rows.  Called by every thread; +inf and NaN distances become
// kEmptyKey (they never enter a top-8 list in the reference).
template <int N, int kOct>
__device__ __forceinline__ void stage_distances(const float *q, const float *stage, int stride, int rows, int c0,
                                                int d, int octet, int j, int lane, const unsigned long long *sel_keys,
                                                unsigned long long *exact_keys) {
    const float *xs[N];
#pragma unroll
    for (int kk = 0; kk < N; ++kk) {
        const int c = octet + kOct * kk;
        xs[kk] = stage + (c < rows ? c : 0) * stride;
    }
    float dist[N];
    octet_l2n<N, false>(q, xs, d, j, lane & ~7, kFullMask, dist);
#pragma unroll
    for (int kk = 0; kk < N; ++kk) {
        const int c = octet + kOct * kk;
        if (j == 0 && c < rows)
            exact_keys[c0 + c] = dist[kk] < __int_as_float(0x7f800000) ? make_key(dist[kk], key_pos(sel_keys[c0 + c]))
                                                                       : kEmptyKey;
    }
}

// Shared-memory row stride of the staged re-rank rows, in floats: 8 floats
// of padding put the 4 rows a warp reads at once on different banks.
__host__ __device__ constexpr int stage_stride(int d) { return d + 8; }

// Dynamic shared memory of merge_kernel: thresholds, the query row, then one
// region that holds the key slots and (with a stage) the 12-bit radix
// histogram while the re-rank set is chosen, and the staged rows after.
struct MergeSmem {
    size_t thr, q, keys, wide, stage, total;
};
__host__ __device__ inline MergeSmem merge_smem(int sort_size, int thr_stride, int d, int stage_rows) {
    MergeSmem m{};
    m.thr = 0;
    m.q = static_cast<size_t>(thr_stride) * 4;  // thr_stride is a multiple of 4
    m.keys = m.q + static_cast<size_t>((d + 3) & ~3) * 4;
    m.wide = m.keys + ((static_cast<size_t>(sort_size) * 8 + 255) & ~size_t(255));
    m.stage = m.keys;
    const size_t select_end = stage_rows > 0 ? m.wide + kWideBins * 4 : m.wide;
    const size_t stage_end = m.stage + static_cast<size_t>(stage_rows) * stage_stride(d) * 4;
    m.total = select_end > stage_end ? select_end : stage_end;
    return m;
}

template <int kT>
__global__ void __launch_bounds__(kT, kT == kMergeThreads ? 3 : 1) merge_kernel(MergeArgs a) {
    constexpr int kOct = kT / 8;           // octets: 8 threads per exact distance
    constexpr int kPerOctet = 64 / kOct;   // rows per octet per pass of 64 rows
    extern __shared__ __align__(16) uint8_t msm[];
    const MergeSmem lay = merge_smem(a.sort_size, a.thr_stride, a.d, a.stage_rows);
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(msm + lay.keys);
    float *thr = reinterpret_cast<float *>(msm + lay.thr);
    float *q = reinterpret_cast<float *>(msm + lay.q);
    float *stage = reinterpret_cast<float *>(msm + lay.stage);
    unsigned int *wide = a.stage_rows > 0 ? reinterpret_cast<unsigned int *>(msm + lay.wide) : nullptr;
    __shared__ unsigned long long exact_keys[kRerankMax];  // (exact distance, row) per re-ranked key
    __shared__ unsigned long long best[8];
    __shared__ int certified_s;
    __shared__ SelectState sel;
    __shared__ unsigned long long sel_keys[kRerankMax];
    __shared__ NarrowState narrow;
    __shared__ double weights[8];
    __shared__ int best_slot[8];
    __shared__ __align__(8) uint64_t gather_bar;
    __shared__ __align__(8) uint64_t stage_bar;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, octet = tid >> 3, j = tid & 7;
    const long long frame = blockIdx.x;
    const int d = a.d;
    const float *src = a.queries + frame * d;
    float *dst = a.out + frame * d;
    const float inf = __int_as_float(0x7f800000);
    const int real_slots = a.lists * a.keep;

    // the exact kernel behind launches once every CTA of this grid has
    // started (so it takes no SM slot a merge CTA still needs) and waits for
    // this grid's completion before it reads anything: its launch latency
    // overlaps the merge
    launch_dependents();
    if (tid == 0) {
        tc::mbar_init(&gather_bar, 1);
        tc::mbar_init(&stage_bar, 1);
        tc::fence_mbarrier_init();
    }
    if (tid < 8) best[tid] = kEmptyKey;
    if (wide)
        for (int i = tid; i < kWideBins; i += kT) wide[i] = 0u;
    // the caller's inputs first, while the candidate kernel may still run
    const float ratio = a.mode == kModeBlend ? load_ratio(a.index_rate) : 1.f;
    float *raw_row = a.raw_out ? a.raw_out + frame * d : nullptr;
    for (int i = tid; i < d; i += kT) {
        const float v = src[i];
        q[i] = v;
        if (raw_row) raw_row[i] = v;
    }
    for (int i = real_slots + tid; i < a.sort_size; i += kT) keys[i] = kEmptyKey;
    grid_dependency_wait();
    // the certifying thread's query stats, early (prepared two kernels back)
    const float4 qstat = tid == 32 ? a.qstats[frame] : make_float4(0.f, 0.f, 0.f, 0.f);
    // then the frame's candidate block (keys, thresholds): two bulk copies.
    // Warp 0 alone polls the barriers (a thread parked in a barrier poll can
    // resume microseconds after the phase completes); the CTA barrier that
    // follows releases the rest at once.
    bool landed = true;
    if (warp == 0) {
        if (lane == 0) {
            const uint32_t kbytes = static_cast<uint32_t>(real_slots) * 8;
            const uint32_t tbytes = static_cast<uint32_t>(a.thr_stride) * 4;
            tc::mbar_arrive_expect_tx(&gather_bar, kbytes + tbytes);
            tc::bulk_load(keys, a.keys + static_cast<size_t>(frame) * real_slots, kbytes, &gather_bar);
            tc::bulk_load(thr, a.thr + static_cast<size_t>(frame) * a.thr_stride, tbytes, &gather_bar);
        }
        __syncwarp();
        landed = tc::mbar_wait(&gather_bar, 0, kWaitLimitNs);
    }
    if (__syncthreads_or(!landed)) {
        // the copy never completed: give it one more bounded wait before the
        // shared memory is released, and hand the frame to the exact re-run
        if (warp == 0) tc::mbar_wait(&gather_bar, 0, kWaitLimitNs);
        if (tid == 0) {
            if (a.counters) atomicAdd(&a.counters->timeouts, 1ull);
            const int pos = atomicAdd(a.fallback_count, 1);
            a.fallback_list[pos] = static_cast<int32_t>(frame);
        }
        return;
    }
    if (a.mode == kModeBlend && !(ratio > 0.f)) {
        if (dst != src)
            for (int i = tid; i < d; i += kT) dst[i] = q[i];
        return;
    }
    float tmin = inf;
    for (int s = tid; s < a.lists; s += kT) tmin = fminf(tmin, thr[s]);
    const KeyStats ks = key_stats<kT>(keys, a.sort_size, tmin, sel);
    float cut;
    bool too_many_ties;
    const int stop = a.stage_rows >= kRerank ? min(kRerankStop, a.stage_rows) : kRerankStop;
    int m = select_rerank<kT>(keys, a.sort_size, ks, sel_keys, sel, cut, too_many_ties, wide, stop);
    const float t_final = fminf(ks.tmin, cut);
    {
        const float4 qs = a.qstats[frame];
        m = narrow_rerank<kT>(sel_keys, m, 8, qs.x,
                              approx_error(qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel, a.norm_rel),
                              a.exact_rel, narrow);
    }

    // exact re-rank in the reference order (flat scan position == row): one
    // octet per distance, each written to exact_keys; +inf and NaN distances
    // never enter a top-8 list in the reference, so they become kEmptyKey
    if (a.stage_rows > 0) {
        // the chunk's rows arrive by bulk copies into shared memory, all in
        // flight at once, then the octets read them from there
        const int stride = stage_stride(d);
        uint32_t phase = 0;
        for (int c0 = 0; c0 < m; c0 += a.stage_rows) {
            const int rows_n = min(a.stage_rows, m - c0);
            bool arrived = true;
            if (warp == 0) {
                // the stage reuses the key slots and histogram that the
                // threads have just read and updated
                tc::fence_proxy_async_smem();
                if (lane == 0) tc::mbar_arrive_expect_tx(&stage_bar, static_cast<uint32_t>(rows_n * d * 4));
                __syncwarp();
                for (int i = lane; i < rows_n; i += 32)
                    tc::bulk_load(stage + i * stride, a.vectors + static_cast<size_t>(key_pos(sel_keys[c0 + i])) * d,
                                  static_cast<uint32_t>(d * 4), &stage_bar);
                arrived = tc::mbar_wait(&stage_bar, phase, kWaitLimitNs);
            }
            phase ^= 1u;
            if (__syncthreads_or(!arrived)) {
                // a copy that never completed: let the copies in flight land
                // (bounded) before the CTA's shared memory is released, and
                // hand the frame to the exact re-run
                if (warp == 0) tc::mbar_wait(&stage_bar, phase ^ 1u, kWaitLimitNs);
                if (tid == 0) {
                    if (a.counters) atomicAdd(&a.counters->timeouts, 1ull);
                    const int pos = atomicAdd(a.fallback_count, 1);
                    a.fallback_list[pos] = static_cast<int32_t>(frame);
                }
                return;
            }
            // warp-uniform trip counts: every octet takes part in the
            // shuffles; an octet takes two rows when the chunk has more rows
            // than octets (one pass, the query loads shared)
            if (rows_n <= kOct)
                stage_distances<1, kOct>(q, stage, stride, rows_n, c0, d, octet, j, lane, sel_keys, exact_keys);
            else
                for (int cb = 0; cb < rows_n; cb += 2 * kOct)
                    stage_distances<2, kOct>(q, stage + cb * stride, stride, rows_n - cb, c0 + cb, d, octet, j, lane,
                                             sel_keys, exact_keys);
            __syncthreads();  // the next chunk overwrites the stage; exact_keys are complete
        }
    } else {
        for (int c0 = 0; c0 < m; c0 += 64) {
            uint32_t rows[kPerOctet];
            const float *xs[kPerOctet];
#pragma unroll
            for (int kk = 0; kk < kPerOctet; ++kk) {
                const int c = c0 + octet + kOct * kk;
                rows[kk] = key_pos(sel_keys[c < m ? c : 0]);
                xs[kk] = a.vectors + static_cast<size_t>(rows[kk]) * d;
            }
            float dist[kPerOctet];
            octet_l2n<kPerOctet>(q, xs, d, j, lane & ~7, kFullMask, dist);
#pragma unroll
            for (int kk = 0; kk < kPerOctet; ++kk) {
                const int c = c0 + octet + kOct * kk;
                if (j == 0 && c < m) exact_keys[c] = dist[kk] < inf ? make_key(dist[kk], rows[kk]) : kEmptyKey;
            }
        }
        __syncthreads();
    }
    // the frame's top 8: each re-ranked key's rank is the number of smaller
    // keys (keys are distinct: one row each)
    for (int c = tid; c < m; c += kT) {
        const unsigned long long key = exact_keys[c];
        if (key == kEmptyKey) continue;
        int rank = 0;
        for (int i = 0; i < m; ++i) rank += exact_keys[i] < key;
        if (rank < 8) {
            best[rank] = key;
            best_slot[rank] = c;
        }
    }
    __syncthreads();
    int count = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) count += best[i] != kEmptyKey;
    // in parallel: the certificate (thread 32) and the neighbour weights
    // (threads 0-7, one each)
    const bool staged_all = a.stage_rows > 0 && m <= a.stage_rows;
    if (tid == 32) {
        const float d8 = count == 8 ? key_dist(best[7]) : inf;
        const bool ok = !too_many_ties && certify(t_final, d8, qstat, a.max_norm, a.max_hat, a.max_residual,
                                                  a.acc_rel, a.norm_rel, a.exact_rel);
        certified_s = ok ? 1 : 0;
    }
    if (tid < 8) weights[tid] = tid < count ? reference_weight(key_dist(best[tid])) : 0.0;
    __syncthreads();
    if (certified_s == 0) {
        if (tid == 0) {
            const int pos = atomicAdd(a.fallback_count, 1);
            a.fallback_list[pos] = static_cast<int32_t>(frame);
        }
        return;
    }
    if (tid == 0 && a.counters) atomicAdd(&a.counters->candidate_frames, 1ull);
    if (a.mode == kModeSearch) {
        if (tid < a.k) {
            const bool have = tid < count;
            a.dist_out[frame * a.k + tid] = have ? key_dist(best[tid]) : inf;
            a.label_out[frame * a.k + tid] =
                have ? static_cast<int64_t>(a.ids[key_pos(best[tid])]) + a.label_base : -1;
        }
        return;
    }
    if (count == 0) {
        if (tid == 0 && a.counters) atomicAdd(&a.counters->empty_frames, 1ull);
        if (dst != src)
            for (int i = tid; i < d; i += kT) dst[i] = q[i];
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
    if (staged_all) {
        const float *vrow[8];
        const int stride = stage_stride(d);
#pragma unroll
        for (int kq = 0; kq < 8; ++kq) vrow[kq] = stage + (kq < count ? best_slot[kq] : 0) * stride;
        for (int i = tid; i < d; i += kT) {
            float v[8];
#pragma unroll
            for (int kq = 0; kq < 8; ++kq) v[kq] = vrow[kq][i];
            dst[i] = reference_blend_element<kT == kMergeThreadsMax>(q[i], v, w, sum, count, ratio);
        }
    } else {
        uint32_t rows[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rows[i] = key_pos(best[i]);
        for (int i = tid; i < d; i += kT) {
            float v[8];
#pragma unroll
            for (int kq = 0; kq < 8; ++kq)
                v[kq] = kq < count ? __ldg(a.vectors + static_cast<size_t>(rows[kq]) * d + i) : 0.f;
            dst[i] = reference_blend_element(q[i], v, w, sum, count, ratio);
        }
    }
}

// ---------------------------------------------------------------- merge (small launches)
//
// merge_small_kernel: merge_kernel's job for launches of at most two frames
// per SM (realtime blocks), where each CTA's chain of dependent steps sets
// the time.  The re-rank set comes from one proof instead of a radix
// selection and a narrowing pass: U = the 8th smallest approximate distance
// among all the frame's candidate keys (found exactly by warp-level
// extraction), and a key is re-ranked unless its lower bound d~ + ||q||^2 - e
// exceeds (U + ||q||^2 + e) (1 + 4 exact_rel) -- the test narrow_rerank
// applies, which shows such a row can neither enter nor tie the exact top 8.
// The rows a candidate stage never kept are covered by the list thresholds
// (the certificate, as in merge_kernel).  The thread that finds a kept key
// issues the bulk copy of its row into the stage at once, so the row fetches
// overlap the rest of the filter pass.

// 64-bit minimum over the warp.
__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long v) {
    const uint32_t hi = __reduce_min_sync(kFullMask, static_cast<uint32_t>(v >> 32));
    const uint32_t lo =
        __reduce_min_sync(kFullMask, static_cast<uint32_t>(v >> 32) == hi ? static_cast<uint32_t>(v) : 0xffffffffu);
    return (static_cast<unsigned long long>(hi) << 32) | lo;
}

// The 8 smallest of keys[lane], keys[lane + 32], ... below `count`
// (kEmptyKey entries never count; the other keys are distinct), ascending
// and padded with kEmptyKey; every lane of the warp gets them.
__device__ __noinline__ void warp_smallest8(const unsigned long long *keys, int count,
                                            unsigned long long (&out)[8]) {
    const int lane = threadIdx.x & 31;
    unsigned long long prev = 0;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        unsigned long long mn = kEmptyKey;
        for (int i = lane; i < count; i += 32) {
            const unsigned long long k = keys[i];
            if ((r == 0 || k > prev) && k < mn) mn = k;
        }
        mn = warp_min_u64(mn);
        out[r] = mn;
        prev = mn;
    }
}

// Compare-exchange of two keys (ascending).
__device__ __forceinline__ void key_cx(unsigned long long &a, unsigned long long &b) {
    const unsigned long long lo = a < b ? a : b, hi = a < b ? b : a;
    a = lo;
    b = hi;
}

// warp_smallest8 for a warp whose lanes hold at most 8 keys each: the keys
// go to registers once, each lane sorts its 8 (a 19-exchange network), and
// the warp merges the 32 sorted lists, one warp minimum per output key.
__device__ __noinline__ void warp_smallest8_reg(const unsigned long long *keys, int count,
                                                unsigned long long (&out)[8]) {
    const int lane = threadIdx.x & 31;
    unsigned long long v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int i = lane + 32 * e;
        v[e] = i < count ? keys[i] : kEmptyKey;
    }
    // Batcher's odd-even merge network for 8 inputs
    key_cx(v[0], v[1]); key_cx(v[2], v[3]); key_cx(v[4], v[5]); key_cx(v[6], v[7]);
    key_cx(v[0], v[2]); key_cx(v[1], v[3]); key_cx(v[4], v[6]); key_cx(v[5], v[7]);
    key_cx(v[1], v[2]); key_cx(v[5], v[6]);
    key_cx(v[0], v[4]); key_cx(v[1], v[5]); key_cx(v[2], v[6]); key_cx(v[3], v[7]);
    key_cx(v[2], v[4]); key_cx(v[3], v[5]);
    key_cx(v[1], v[2]); key_cx(v[3], v[4]); key_cx(v[5], v[6]);
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const unsigned long long mn = warp_min_u64(v[0]);
        out[r] = mn;
        if (v[0] == mn && mn != kEmptyKey) {  // the owner pops its head (keys are distinct)
#pragma unroll
            for (int e = 0; e < 7; ++e) v[e] = v[e + 1];
            v[7] = kEmptyKey;
        }
    }
}

// Dynamic shared memory of merge_small_kernel: thresholds, query row, key
// slots, then the stage (its own region, so copies land while keys are read).
struct SmallSmem {
    size_t thr, q, keys, stage, total;
};
__host__ __device__ inline SmallSmem small_smem(int sort_size, int thr_stride, int d, int stage_rows) {
    SmallSmem m{};
    m.thr = 0;
    m.q = static_cast<size_t>(thr_stride) * 4;
    m.keys = (m.q + static_cast<size_t>((d + 3) & ~3) * 4 + 15) & ~size_t(15);
    m.stage = (m.keys + static_cast<size_t>(sort_size) * 8 + 15) & ~size_t(15);
    m.total = m.stage + static_cast<size_t>(stage_rows) * stage_stride(d) * 4;
    return m;
}

// Out-of-line pieces of merge_small_kernel's rare paths (a frame handed to
// the exact re-run, a timed-out copy, search output, rows beyond the stage):
// that kernel runs each instruction about once per launch, so its time
// follows its code size, and these stay out of the common path's lines.
__device__ __noinline__ void hand_to_rerun(const MergeArgs &a, long long frame, bool timed_out) {
    if (timed_out && a.counters) atomicAdd(&a.counters->timeouts, 1ull);
    const int pos = atomicAdd(a.fallback_count, 1);
    a.fallback_list[pos] = static_cast<int32_t>(frame);
}

__device__ __noinline__ void write_search(const MergeArgs &a, long long frame, const unsigned long long *best,
                                          int count) {
    const int t = threadIdx.x;
    if (t < a.k) {
        const bool have = t < count;
        a.dist_out[frame * a.k + t] = have ? key_dist(best[t]) : __int_as_float(0x7f800000);
        a.label_out[frame * a.k + t] = have ? static_cast<int64_t>(a.ids[key_pos(best[t])]) + a.label_base : -1;
    }
}

// Exact distances of re-rank keys [c0, m) read from global memory (the
// kept rows the stage could not hold), one octet per row.
template <int kOct>
__device__ __noinline__ void global_distances(const MergeArgs &a, const float *q, int c0, int m,
                                              const unsigned long long *sel_keys, unsigned long long *exact_keys) {
    const int tid = threadIdx.x, lane = tid & 31, octet = tid >> 3, j = tid & 7;
    for (; c0 < m; c0 += kOct) {
        const int c = c0 + octet;
        const uint32_t row = key_pos(sel_keys[c < m ? c : c0]);
        const float *xs[1] = {a.vectors + static_cast<size_t>(row) * a.d};
        float dist[1];
        octet_l2n<1>(q, xs, a.d, j, lane & ~7, kFullMask, dist);
        if (j == 0 && c < m) exact_keys[c] = dist[0] < __int_as_float(0x7f800000) ? make_key(dist[0], row) : kEmptyKey;
    }
}

constexpr int kSmallStageMin = 16;  // fewer stage rows than this: merge_kernel instead
constexpr int kSmallStageMax = 64;

template <int kT>
__global__ void __launch_bounds__(kT, kT == kMergeThreadsMax ? 1 : 2) merge_small_kernel(MergeArgs a) {
    constexpr int kOct = kT / 8;
    constexpr int kWarps = kT / 32;
    extern __shared__ __align__(16) uint8_t msm[];
    const SmallSmem lay = small_smem(a.sort_size, a.thr_stride, a.d, a.stage_rows);
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(msm + lay.keys);
    float *thr = reinterpret_cast<float *>(msm + lay.thr);
    float *q = reinterpret_cast<float *>(msm + lay.q);
    float *stage = reinterpret_cast<float *>(msm + lay.stage);
    __shared__ unsigned long long exact_keys[kRerankMax];
    __shared__ unsigned long long sel_keys[kRerankMax];
    __shared__ unsigned long long best[8];
    __shared__ int best_slot[8];
    __shared__ double weights[8];
    __shared__ unsigned long long warp_top[kWarps * 8];
    __shared__ float warp_tmin[kWarps];
    __shared__ unsigned long long u8_s;
    __shared__ float tmin_s;
    __shared__ int count_s, bound_count_s, certified_s;
    __shared__ __align__(8) uint64_t gather_bar;
    __shared__ __align__(8) uint64_t stage_bar;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, octet = tid >> 3, j = tid & 7;
    const long long frame = blockIdx.x;
    const int d = a.d;
    const float *src = a.queries + frame * d;
    float *dst = a.out + frame * d;
    const float inf = __int_as_float(0x7f800000);
    const int real_slots = a.lists * a.keep;
    const int stride = stage_stride(d);
    launch_dependents();  // as in merge_kernel: the exact kernel's launch overlaps this one

    if (tid == 0) {
        tc::mbar_init(&gather_bar, 1);
        tc::mbar_init(&stage_bar, 1);
        tc::fence_mbarrier_init();
        count_s = 0;
        bound_count_s = 0;
    }
    if (tid < 8) best[tid] = kEmptyKey;
    // the caller's inputs first, while the candidate kernel may still run
    const float ratio = a.mode == kModeBlend ? load_ratio(a.index_rate) : 1.f;
    float *raw_row = a.raw_out ? a.raw_out + frame * d : nullptr;
    for (int i = tid; i < d; i += kT) {
        const float v = src[i];
        q[i] = v;
        if (raw_row) raw_row[i] = v;
    }
    for (int i = real_slots + tid; i < a.sort_size; i += kT) keys[i] = kEmptyKey;
    grid_dependency_wait();
    const float4 qs = a.qstats[frame];
    bool landed = true;
    if (warp == 0) {
        if (lane == 0) {
            const uint32_t kbytes = static_cast<uint32_t>(real_slots) * 8;
            const uint32_t tbytes = static_cast<uint32_t>(a.thr_stride) * 4;
            tc::mbar_arrive_expect_tx(&gather_bar, kbytes + tbytes);
            tc::bulk_load(keys, a.keys + static_cast<size_t>(frame) * real_slots, kbytes, &gather_bar);
            tc::bulk_load(thr, a.thr + static_cast<size_t>(frame) * a.thr_stride, tbytes, &gather_bar);
        }
        __syncwarp();
        landed = tc::mbar_wait(&gather_bar, 0, kWaitLimitNs);
    }
    if (__syncthreads_or(!landed)) {
        if (warp == 0) tc::mbar_wait(&gather_bar, 0, kWaitLimitNs);
        if (tid == 0) hand_to_rerun(a, frame, true);
        return;
    }
    if (a.mode == kModeBlend && !(ratio > 0.f)) {
        if (dst != src)
            for (int i = tid; i < d; i += kT) dst[i] = q[i];
        return;
    }
    // The re-rank set is every key whose lower bound d~ + ||q||^2 - e does
    // not exceed `limit`.  First choice: the candidate stage's final frame
    // bound G (no row above it reaches or ties the exact top 8), when at most
    // a stage's worth of keys lie at or below it; else the narrowing limit
    // from U, the 8th smallest key (per warp, the 8 smallest of its slice of
    // the key slots, then warp 0 reduces them).
    const float e = approx_error(qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel, a.norm_rel);
    {
        float tmin = inf;
        for (int s = tid; s < a.lists; s += kT) tmin = fminf(tmin, thr[s]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tmin = fminf(tmin, __shfl_xor_sync(kFullMask, tmin, o));
        if (lane == 0) warp_tmin[warp] = tmin;
    }
    float limit = inf;
    bool by_bound = false;
    // (the 512-thread form: its stage holds up to 64 rows; with the 256-thread
    // form's 32 the bound's set often does not fit, and the count is wasted)
    if (kT == kMergeThreadsMax && a.gbound != nullptr) {
        limit = frame_bound(a.gbound + frame * kBoundWords, qs.x + e, 2.f * e, a.exact_rel) + qs.x - e;
        int n = 0;
        for (int i = tid; i < a.sort_size; i += kT) {
            const unsigned long long k = keys[i];
            n += k != kEmptyKey && !(key_dist(k) + qs.x - e > limit);
        }
        if (n) atomicAdd(&bound_count_s, n);
        __syncthreads();
        by_bound = bound_count_s <= a.stage_rows;  // CTA-uniform
        if (tid == 0) {
            float t = inf;
            for (int w = 0; w < kWarps; ++w) t = fminf(t, warp_tmin[w]);
            tmin_s = t;
        }
    }
    if (!by_bound) {
        const int chunk = (a.sort_size + kWarps - 1) / kWarps;
        const int lo = warp * chunk;
        const int n = max(0, min(chunk, a.sort_size - lo));
        unsigned long long top[8];
        if (chunk <= 256)  // warp-uniform
            warp_smallest8_reg(keys + lo, n, top);
        else
            warp_smallest8(keys + lo, n, top);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < 8; ++r) warp_top[warp * 8 + r] = top[r];
        }
        __syncthreads();
        if (warp == 0) {
            static_assert(kWarps * 8 <= 256, "one register list per lane");
            warp_smallest8_reg(warp_top, kWarps * 8, top);
            float tmin = lane < kWarps ? warp_tmin[lane] : inf;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) tmin = fminf(tmin, __shfl_xor_sync(kFullMask, tmin, o));
            if (lane == 0) {
                u8_s = top[7];
                tmin_s = tmin;
            }
        }
        __syncthreads();
        const unsigned long long u8 = u8_s;
        limit = u8 == kEmptyKey ? inf : (key_dist(u8) + qs.x + e) * (1.f + 4.f * a.exact_rel) + 1e-30f;
    }
    for (int base = 0; base < a.sort_size; base += kT) {  // sort_size and kT are multiples of 32
        const int i = base + tid;
        const unsigned long long k = i < a.sort_size ? keys[i] : kEmptyKey;
        const bool keep = k != kEmptyKey && !(key_dist(k) + qs.x - e > limit);
        const unsigned ball = __ballot_sync(kFullMask, keep);
        if (ball == 0u) continue;
        int first = 0;
        if (lane == 0) first = atomicAdd(&count_s, __popc(ball));
        first = __shfl_sync(kFullMask, first, 0);
        if (keep) {
            const int pos = first + __popc(ball & ((1u << lane) - 1u));
            if (pos < kRerankMax) sel_keys[pos] = k;
            if (pos < a.stage_rows) {
                tc::mbar_expect_tx(&stage_bar, static_cast<uint32_t>(d) * 4);
                tc::bulk_load(stage + pos * stride, a.vectors + static_cast<size_t>(key_pos(k)) * d,
                              static_cast<uint32_t>(d) * 4, &stage_bar);
            }
        }
    }
    __syncthreads();  // the count is final and every expect_tx precedes the arrival below
    const int total = count_s;
    const bool too_many = total > kRerankMax;
    const int m = min(total, kRerankMax);
    const int staged = min(m, a.stage_rows);
    bool arrived = true;
    if (warp == 0) {
        if (lane == 0) tc::mbar_arrive(&stage_bar);
        __syncwarp();
        arrived = tc::mbar_wait(&stage_bar, 0, kWaitLimitNs);
    }
    if (__syncthreads_or(!arrived)) {
        // a copy never completed: let the copies in flight land (bounded)
        // before the shared memory is released, and hand the frame on
        if (warp == 0) tc::mbar_wait(&stage_bar, 0, kWaitLimitNs);
        if (tid == 0) hand_to_rerun(a, frame, true);
        return;
    }
    // exact distances in the reference order: staged rows from shared
    // memory, any others from global memory (flat scan position == row)
    // (a warp whose four octets have no staged row skips the pass: the
    // chains are long and issue-bound, so idle octets would slow the rest)
    // (stage_rows never exceeds the octets: the host caps it at kOct)
    if (warp * 4 < staged)
        stage_distances<1, kOct>(q, stage, stride, staged, 0, d, octet, j, lane, sel_keys, exact_keys);
    if (staged < m) global_distances<kOct>(a, q, staged, m, sel_keys, exact_keys);
    __syncthreads();
    // the frame's top 8 by rank counting (keys are distinct: one row each)
    for (int c = tid; c < m; c += kT) {
        const unsigned long long key = exact_keys[c];
        if (key == kEmptyKey) continue;
        int rank = 0;
        for (int i = 0; i < m; ++i) rank += exact_keys[i] < key;
        if (rank < 8) {
            best[rank] = key;
            best_slot[rank] = c;
        }
    }
    __syncthreads();
    int count = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) count += best[i] != kEmptyKey;
    if (tid == 32) {
        const float d8 = count == 8 ? key_dist(best[7]) : inf;
        const bool ok = !too_many && certify(tmin_s, d8, qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel,
                                             a.norm_rel, a.exact_rel);
        certified_s = ok ? 1 : 0;
    }
    if (tid < 8) weights[tid] = tid < count ? reference_weight(key_dist(best[tid])) : 0.0;
    __syncthreads();
    if (certified_s == 0) {
        if (tid == 0) hand_to_rerun(a, frame, false);
        return;
    }
    if (tid == 0 && a.counters) atomicAdd(&a.counters->candidate_frames, 1ull);
    if (a.mode == kModeSearch) {
        if (warp == 0) write_search(a, frame, best, count);
        return;
    }
    if (count == 0) {
        if (tid == 0 && a.counters) atomicAdd(&a.counters->empty_frames, 1ull);
        if (dst != src)
            for (int i = tid; i < d; i += kT) dst[i] = q[i];
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
    // each neighbour's row: in the stage, or in global memory when it was
    // kept beyond the stage (generic loads read either)
    const float *vrow[8];
#pragma unroll
    for (int kq = 0; kq < 8; ++kq) {
        const int slot = kq < count ? best_slot[kq] : 0;
        vrow[kq] = slot < staged ? stage + slot * stride
                                 : a.vectors + static_cast<size_t>(key_pos(best[kq])) * d;
    }
    for (int i = tid; i < d; i += kT) {
        float v[8];
#pragma unroll
        for (int kq = 0; kq < 8; ++kq) v[kq] = kq < count ? vrow[kq][i] : 0.f;
        dst[i] = reference_blend_element<true>(q[i], v, w, sum, count, ratio);
    }
}

// ---------------------------------------------------------------- flat merge, one warp per frame
//
// merge_warp_kernel: the flat merge of launches with more than two frames
// per SM, one warp per frame and no CTA-wide barrier (8 frames per CTA).
// The frame's candidate block (lists x keep keys; each list ascending,
// kEmptyKey past its count) is read from global memory (L2: the candidate
// kernel has just written it), once to find U, the 8th smallest key (each
// lane keeps the 8 smallest of its slots in registers, then a warp merge),
// and once to collect every key whose lower bound d~ + ||q||^2 - e does not
// exceed (U + ||q||^2 + e)(1 + 4 exact_rel) -- the rows that may still
// enter the exact top 8.  Octets compute their exact distances two rows at
// a time in the reference's order (the flat scan position is the row), a
// warp merge gives the top 8, and the lists' thresholds certify the rows the
// candidate stage dropped, as in merge_kernel.
constexpr int kMergeWarps = 8;
constexpr int kMergeBatch = 8;  // key loads in flight per lane

__global__ void __launch_bounds__(32 * kMergeWarps, 3) merge_warp_kernel(MergeArgs a, long long frames) {
    extern __shared__ __align__(16) float mwq[];  // [kMergeWarps][d rounded up to 4] frame rows
    __shared__ unsigned long long sel[kMergeWarps][kRerankMax];
    __shared__ unsigned long long ex[kMergeWarps][kRerankMax];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, octet = lane >> 3, j = lane & 7;
    const long long frame = static_cast<long long>(blockIdx.x) * kMergeWarps + w;
    launch_dependents();  // as in merge_kernel: the exact kernel's launch overlaps this one
    if (frame >= frames) return;
    const int d = a.d;
    float *q = mwq + static_cast<size_t>(w) * ((d + 3) & ~3);
    const float *src = a.queries + frame * d;
    float *dst = a.out + frame * d;
    const float inf = __int_as_float(0x7f800000);
    // the caller's inputs first, while the candidate kernel may still run
    const float ratio = a.mode == kModeBlend ? load_ratio(a.index_rate) : 1.f;
    float *raw_row = a.raw_out ? a.raw_out + frame * d : nullptr;
    for (int i = lane; i < d; i += 32) {
        const float v = src[i];
        q[i] = v;
        if (raw_row) raw_row[i] = v;
    }
    __syncwarp();
    grid_dependency_wait();
    if (a.mode == kModeBlend && !(ratio > 0.f)) {
        if (dst != src)
            for (int i = lane; i < d; i += 32) dst[i] = q[i];
        return;
    }
    const int slots = a.lists * a.keep;
    const unsigned long long *fk = a.keys + static_cast<size_t>(frame) * slots;
    float tmin = inf;
    for (int l = lane; l < a.lists; l += 32) tmin = fminf(tmin, __ldcg(a.thr + frame * a.thr_stride + l));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tmin = fminf(tmin, __shfl_xor_sync(kFullMask, tmin, o));
    // U: each lane's 8 smallest slots (sorted insertion), then 8 warp pops.
    // The slots are read kMergeBatch at a time, all loads of a batch issued
    // before any is used (the key block sits in L2: one round trip a batch).
    unsigned long long v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = kEmptyKey;
    for (int base = 0; base < slots; base += 32 * kMergeBatch) {
        unsigned long long kb[kMergeBatch];
#pragma unroll
        for (int t = 0; t < kMergeBatch; ++t) {
            const int i = base + 32 * t + lane;
            kb[t] = i < slots ? __ldcg(fk + i) : kEmptyKey;
        }
#pragma unroll
        for (int t = 0; t < kMergeBatch; ++t) {
            if (kb[t] < v[7]) {
                v[7] = kb[t];
#pragma unroll
                for (int e = 6; e >= 0; --e) key_cx(v[e], v[e + 1]);
            }
        }
    }
    unsigned long long u8 = kEmptyKey;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const unsigned long long mn = warp_min_u64(v[0]);
        u8 = mn;
        if (v[0] == mn && mn != kEmptyKey) {
#pragma unroll
            for (int e = 0; e < 7; ++e) v[e] = v[e + 1];
            v[7] = kEmptyKey;
        }
    }
    const float4 qs = a.qstats[frame];
    const float e = approx_error(qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel, a.norm_rel);
    const float limit = u8 == kEmptyKey ? inf : (key_dist(u8) + qs.x + e) * (1.f + 4.f * a.exact_rel) + 1e-30f;
    // the re-rank set, in slot order (batched loads, as above)
    int total = 0;
    for (int base = 0; base < slots; base += 32 * kMergeBatch) {
        unsigned long long kb[kMergeBatch];
#pragma unroll
        for (int t = 0; t < kMergeBatch; ++t) {
            const int i = base + 32 * t + lane;
            kb[t] = i < slots ? __ldcg(fk + i) : kEmptyKey;
        }
#pragma unroll
        for (int t = 0; t < kMergeBatch; ++t) {
            const bool kept = kb[t] != kEmptyKey && !(key_dist(kb[t]) + qs.x - e > limit);
            const unsigned ball = __ballot_sync(kFullMask, kept);
            if (kept) {
                const int pos = total + __popc(ball & ((1u << lane) - 1u));
                if (pos < kRerankMax) sel[w][pos] = kb[t];
            }
            total += __popc(ball);
        }
    }
    const int m = min(total, kRerankMax);
    __syncwarp();
    for (int c0 = 0; c0 < m; c0 += 8) {
        uint32_t rows[2];
        const float *xs[2];
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int c = c0 + octet + 4 * kk;
            rows[kk] = key_pos(sel[w][c < m ? c : c0]);
            xs[kk] = a.vectors + static_cast<size_t>(rows[kk]) * d;
        }
        float dist[2];
        octet_l2n<2>(q, xs, d, j, lane & ~7, kFullMask, dist);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int c = c0 + octet + 4 * kk;
            if (j == 0 && c < m) ex[w][c] = dist[kk] < inf ? make_key(dist[kk], rows[kk]) : kEmptyKey;
        }
    }
    __syncwarp();
    // the exact top 8 (m <= 128: four keys a lane, sorted, then 8 pops)
    unsigned long long best[8];
    {
        unsigned long long t[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) t[s] = lane + 32 * s < m ? ex[w][lane + 32 * s] : kEmptyKey;
        key_cx(t[0], t[1]); key_cx(t[2], t[3]); key_cx(t[0], t[2]); key_cx(t[1], t[3]); key_cx(t[1], t[2]);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const unsigned long long mn = warp_min_u64(t[0]);
            best[r] = mn;
            if (t[0] == mn && mn != kEmptyKey) {
                t[0] = t[1];
                t[1] = t[2];
                t[2] = t[3];
                t[3] = kEmptyKey;
            }
        }
    }
    int count = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) count += best[i] != kEmptyKey;
    const float d8 = count == 8 ? key_dist(best[7]) : inf;
    if (total > kRerankMax || !certify(tmin, d8, qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel, a.norm_rel,
                                       a.exact_rel)) {
        if (lane == 0) a.fallback_list[atomicAdd(a.fallback_count, 1)] = static_cast<int32_t>(frame);
        return;
    }
    if (lane == 0 && a.counters) atomicAdd(&a.counters->candidate_frames, 1ull);
    unsigned long long mine = kEmptyKey;
#pragma unroll
    for (int i = 0; i < 8; ++i) mine = lane == i ? best[i] : mine;
    if (a.mode == kModeSearch) {
        if (lane < a.k) {
            const bool have = lane < count;
            a.dist_out[frame * a.k + lane] = have ? key_dist(mine) : inf;
            a.label_out[frame * a.k + lane] = have ? static_cast<int64_t>(a.ids[key_pos(mine)]) + a.label_base : -1;
        }
        return;
    }
    if (count == 0) {
        if (lane == 0 && a.counters) atomicAdd(&a.counters->empty_frames, 1ull);
        if (dst != src)
            for (int i = lane; i < d; i += 32) dst[i] = q[i];
        return;
    }
    const double wk = lane < count ? reference_weight(key_dist(mine)) : 0.0;
    double wv[8];
    const float *vr[8];
    double wsum = -0.0;  // the reference's order: S = w0 + w1 + ... (zeros past count)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        wv[k] = __shfl_sync(kFullMask, wk, k);
        const uint32_t rk = key_pos(__shfl_sync(kFullMask, mine, k));
        vr[k] = a.vectors + static_cast<size_t>(k < count ? rk : 0u) * d;
        wsum = __dadd_rn(wsum, wv[k]);
    }
    const WeightDivisor sum = weight_divisor(wsum);
    if ((d & 3) == 0 && ((reinterpret_cast<uintptr_t>(a.vectors) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        // four elements per lane and step: one 16-byte load per neighbour
        // row, a quarter of the dependent row round trips; each element's
        // arithmetic (and so its result) is the scalar loop's
        for (int i4 = lane; i4 < (d >> 2); i4 += 32) {
            float4 r4[8];
#pragma unroll
            for (int k = 0; k < 8; ++k)
                r4[k] = k < count ? __ldg(reinterpret_cast<const float4 *>(vr[k]) + i4) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 q4 = reinterpret_cast<const float4 *>(q)[i4];
            float x[8];
            float4 o;
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = r4[k].x;
            o.x = reference_blend_element<false>(q4.x, x, wv, sum, count, ratio);
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = r4[k].y;
            o.y = reference_blend_element<false>(q4.y, x, wv, sum, count, ratio);
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = r4[k].z;
            o.z = reference_blend_element<false>(q4.z, x, wv, sum, count, ratio);
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = r4[k].w;
            o.w = reference_blend_element<false>(q4.w, x, wv, sum, count, ratio);
            reinterpret_cast<float4 *>(dst)[i4] = o;
        }
        return;
    }
    for (int i = lane; i < d; i += 32) {
        float x[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = k < count ? __ldg(vr[k] + i) : 0.f;
        dst[i] = reference_blend_element<true>(q[i], x, wv, sum, count, ratio);
    }
}

// ---------------------------------------------------------------- index build
__global__ void max_abs_kernel(const float *__restrict__ x, size_t count, unsigned int *out) {
    float m = 0.f;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float v = fabsf(x[i]);
        m = v > m ? v : m;  // NaN never enters (the parser rejects non-finite values)
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, s));
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// One warp per row: fp16 shadow, fp32 squared norm, and the maxima of the
// row norm, the fp16 row's norm and the rounding residual norm.
__global__ void build_rows_kernel(const float *__restrict__ x, __half *__restrict__ xh, float *__restrict__ norms,
                                  int64_t n, int d, int d_pad, float scale, unsigned int *maxima) {
    const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const float inv = 1.0f / scale;
    float n2 = 0.f, hat2 = 0.f, res2 = 0.f;
    for (int k = lane; k < d_pad; k += 32) {
        float v = k < d ? x[row * d + k] : 0.f;
        __half h = __float2half_rn(v * scale);
        xh[row * d_pad + k] = h;
        float back = __half2float(h) * inv;
        float res = v - back;
        n2 = fmaf(v, v, n2);
        hat2 = fmaf(back, back, hat2);
        res2 = fmaf(res, res, res2);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        n2 += __shfl_xor_sync(kFullMask, n2, s);
        hat2 += __shfl_xor_sync(kFullMask, hat2, s);
        res2 += __shfl_xor_sync(kFullMask, res2, s);
    }
    if (lane == 0) {
        norms[row] = n2;
        atomicMax(&maxima[0], __float_as_uint(sqrtf(n2)));
        atomicMax(&maxima[1], __float_as_uint(sqrtf(hat2)));
        atomicMax(&maxima[2], __float_as_uint(sqrtf(res2)));
    }
}

__global__ void fill_kernel(float *p, size_t count, float value) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        p[i] = value;
}

// ---------------------------------------------------------------- host helpers
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    require(fn != nullptr, "cuTensorMapEncodeTiled is unavailable");
    return fn;
}

// 2-D fp16 tensor map over a row-major [rows][cols] matrix, box [box_rows][64],
// 128-byte swizzle; out-of-range rows read as zero.
void encode_rows(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
    require(reinterpret_cast<uintptr_t>(base) % 16 == 0 && (cols * 2) % 16 == 0, "tensor map alignment");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileK), box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult rc = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    require(rc == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed");
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Plan {
    int n_qtiles, segments, tiles_per_seg;
};

// Launches merge_kernel over `frames` frames.  When the launch has at most
// two frames per SM, each CTA's latency sets the time, so the re-rank rows
// are staged in shared memory by bulk copies (64 or 32 rows per chunk, as
// the opt-in shared memory allows; rows of d % 4 == 0 floats, 16-byte
// aligned); larger launches keep many CTAs per SM and read the rows from
// global memory.
void launch_merge(VfrIndex *ix, MergeArgs &ma, size_t frames, cudaStream_t stream) {
    ma.stage_rows = 0;
    const bool few = ix->d % 4 == 0 && reinterpret_cast<uintptr_t>(ix->vectors) % 16 == 0 &&
                     frames <= static_cast<size_t>(ix->sm_count) * 2;
    if (few && ix->small_merge) {
        // merge_small_kernel, with as many stage rows as fit (at least
        // kSmallStageMin): 512 threads (one CTA per SM) when every frame
        // has an SM of its own, else 256 threads and half the shared
        // memory each, so two CTAs per SM take the launch in one wave
        const bool one_wave = frames <= static_cast<size_t>(ix->sm_count);
        const int max_rows = one_wave ? kSmallStageMax : kMergeThreads / 8;
        // two CTAs: half the SM's shared memory each, less the per-CTA
        // reservation and static arrays (4 KB covers both)
        const size_t budget = one_wave ? static_cast<size_t>(ix->merge_smem_max)
                                       : static_cast<size_t>(ix->merge_smem_max) / 2 - 4096;
        for (int rows = max_rows; rows >= kSmallStageMin; --rows) {
            const size_t need = small_smem(ma.sort_size, ma.thr_stride, ix->d, rows).total;
            if (need <= budget) {
                ma.stage_rows = rows;
                if (one_wave)
                    cuda_check(launch_pdl(merge_small_kernel<kMergeThreadsMax>, dim3(static_cast<unsigned>(frames)),
                                          dim3(kMergeThreadsMax), need, stream, ma));
                else
                    cuda_check(launch_pdl(merge_small_kernel<kMergeThreads>, dim3(static_cast<unsigned>(frames)),
                                          dim3(kMergeThreads), need, stream, ma));
                return;
            }
        }
    }
    if (!few && ix->small_merge) {
        // many frames: one warp per frame
        const size_t smem = static_cast<size_t>(kMergeWarps) * ((ix->d + 3) & ~3) * sizeof(float);
        cuda_check(launch_pdl(merge_warp_kernel, dim3(static_cast<unsigned>((frames + kMergeWarps - 1) / kMergeWarps)),
                              dim3(32 * kMergeWarps), smem, stream, ma, static_cast<long long>(frames)));
        return;
    }
    if (few) {
        // as many rows as fit, up to kRerankStop (the usual re-rank set); at
        // least 32, else the rows stay in global memory
        for (int rows = kRerankStop; rows >= 32; --rows)
            if (merge_smem(ma.sort_size, ma.thr_stride, ix->d, rows).total <=
                static_cast<size_t>(ix->merge_smem_max)) {
                ma.stage_rows = rows;
                break;
            }
    }
    const size_t smem = merge_smem(ma.sort_size, ma.thr_stride, ix->d, ma.stage_rows).total;
    require(smem <= static_cast<size_t>(ix->merge_smem_max), "candidate lists exceed the merge's shared memory");
    if (ma.stage_rows > 0)
        cuda_check(launch_pdl(merge_kernel<kMergeThreadsMax>, dim3(static_cast<unsigned>(frames)),
                              dim3(kMergeThreadsMax), smem, stream, ma));
    else
        cuda_check(launch_pdl(merge_kernel<kMergeThreads>, dim3(static_cast<unsigned>(frames)), dim3(kMergeThreads),
                              smem, stream, ma));
}

// Launches the flat candidate kernel behind prep_queries_kernel (it starts
// loading database tiles before the query tiles exist); the candidate list
// size follows the work-item length.
void launch_cand_flat(const Plan &p, int grid, const void *q16, int d_pad, const CUtensorMap &tmap_x,
                      const CandArgs &ca, cudaStream_t stream) {
    const bool small = ca.frames <= kSmallBlock;
    CUtensorMap tmap_q;
    encode_rows(&tmap_q, q16, d_pad, ca.frames,
                small ? Pipe<kSpreadLayout>::kBlockRows : Pipe<kFullLayout>::kBlockRows);
    const bool short_items = p.tiles_per_seg <= kShortItemTiles;
    auto kernel = small ? (short_items ? cand_kernel<false, kShortKeep, kSpreadLayout>
                                       : cand_kernel<false, kIvfKeep, kSpreadLayout>)
                        : (short_items ? cand_kernel<false, kShortKeep> : cand_kernel<false, kIvfKeep>);
    const size_t smem = small ? Pipe<kSpreadLayout>::kSmem : Pipe<kFullLayout>::kSmem;
    cuda_check(launch_pdl(kernel, dim3(grid), dim3(kThreadsTC), smem, stream, tmap_q, tmap_x, ca));
}

// Launches the CTA-pair candidate kernel (clusters of two CTAs, cta_group::2
// MMA) behind prep_queries_kernel; `tmap_x_half` boxes 128 database rows.
void launch_cand_pair(int clusters, const void *q16, int d_pad, const CUtensorMap &tmap_x_half, const CandArgs &ca,
                      cudaStream_t stream) {
    CUtensorMap tmap_q;
    encode_rows(&tmap_q, q16, d_pad, ca.frames, Pipe<kPairLayout>::kBlockRows);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters));
    cfg.blockDim = dim3(kThreadsTC);
    cfg.dynamicSmemBytes = Pipe<kPairLayout>::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cuda_check(cudaLaunchKernelEx(&cfg, cand_kernel<false, kIvfKeep, kPairLayout>, tmap_q, tmap_x_half, ca));
}

// The shared filter bound of a flat call: per-frame bounds, the frames'
// stats and the index's certificate constants.
void set_shared_bound(CandArgs &ca, const VfrIndex *ix, unsigned int *gbound, const float4 *qstats) {
    ca.gbound = gbound;
    ca.qstats = qstats;
    ca.max_norm = ix->max_row_norm;
    ca.max_hat = ix->max_row_hat;
    ca.max_residual = ix->max_row_residual;
    ca.acc_rel = static_cast<float>(ix->d_pad) * std::ldexp(1.0f, -22);
    ca.norm_rel = static_cast<float>(ix->d_pad) * std::ldexp(1.0f, -23);
    ca.exact_rel = static_cast<float>(ix->d / 8 + 9) * std::ldexp(1.0f, -24);
}

Plan make_plan(size_t frames, int64_t n, int sms) {
    Plan p{};
    p.n_qtiles = static_cast<int>((frames + kTileM - 1) / kTileM);
    const int64_t ntiles = (n + kTileN - 1) / kTileN;
    const int64_t cap = std::max<int64_t>(static_cast<int64_t>(p.n_qtiles) * 16, static_cast<int64_t>(sms) * 8);
    double best = 1e300;
    p.segments = 1;
    p.tiles_per_seg = static_cast<int>(ntiles);
    for (int64_t s = 1; s <= std::min<int64_t>(kMaxSegments, ntiles); ++s) {
        const int64_t tps = (ntiles + s - 1) / s;
        const int64_t seg = (ntiles + tps - 1) / tps;
        if (seg * p.n_qtiles > cap) break;
        const int64_t waves = (seg * p.n_qtiles + sms - 1) / sms;
        // each item restarts its per-frame top list (a burst of insertions
        // worth ~2 tiles of epilogue work) and adds keys to the merge
        const double cost = static_cast<double>(waves * (tps + 2)) + 0.02 * static_cast<double>(seg);
        if (cost < best - 1e-9) {
            best = cost;
            p.segments = static_cast<int>(seg);
            p.tiles_per_seg = static_cast<int>(tps);
        }
    }
    return p;
}

// make_plan for the CTA-pair layout: work items are (query-tile pair,
// segment) and `clusters` pairs run at once; the candidate lists per frame
// (segments x kHalves) stay within the same workspace bound.
Plan make_plan_pair(size_t frames, int64_t n, int sms, int clusters) {
    Plan p{};
    p.n_qtiles = static_cast<int>((frames + kTileM - 1) / kTileM);
    const int64_t pairs = (p.n_qtiles + 1) / 2;
    const int64_t ntiles = (n + kTileN - 1) / kTileN;
    const int64_t cap = std::max<int64_t>(static_cast<int64_t>(p.n_qtiles) * 16, static_cast<int64_t>(sms) * 8);
    double best = 1e300;
    p.segments = 1;
    p.tiles_per_seg = static_cast<int>(ntiles);
    for (int64_t s = 1; s <= std::min<int64_t>(kMaxSegments, ntiles); ++s) {
        const int64_t tps = (ntiles + s - 1) / s;
        const int64_t seg = (ntiles + tps - 1) / tps;
        if (seg * p.n_qtiles > cap) break;
        const int64_t waves = (seg * pairs + clusters - 1) / clusters;
        const double cost = static_cast<double>(waves * (tps + 2)) + 0.02 * static_cast<double>(seg);
        if (cost < best - 1e-9) {
            best = cost;
            p.segments = static_cast<int>(seg);
            p.tiles_per_seg = static_cast<int>(tps);
        }
    }
    return p;
}

// Records a flat call's plan in the index (reported by diagnostics).
void note_plan(VfrIndex *ix, const Plan &p, size_t frames) {
    ix->last_keep = p.tiles_per_seg <= kShortItemTiles ? kShortKeep : kIvfKeep;
    ix->last_segments = p.segments;
    ix->last_tiles_per_seg = p.tiles_per_seg;
    ix->last_layout = frames <= static_cast<size_t>(kSmallBlock) ? kSpreadLayout : kFullLayout;
}

int64_t items_cap(size_t frames, int sms) {
    const int64_t qt = static_cast<int64_t>((frames + kTileM - 1) / kTileM);
    return std::max<int64_t>(qt * 16, static_cast<int64_t>(sms) * 8);
}

struct WsLayout {
    size_t q16, qstats, keys, thr, flist, fcount, gbound, total;
};

WsLayout ws_layout(size_t frames, int d_pad, int sms) {
    WsLayout l{};
    const size_t fr = (frames + kTileM - 1) / kTileM * kTileM;
    const size_t items = static_cast<size_t>(items_cap(frames, sms)) * kHalves;  // candidate lists
    size_t off = 0;
    l.q16 = off;
    off = align256(off + fr * d_pad * sizeof(__half));
    l.qstats = off;
    off = align256(off + fr * sizeof(float4));
    // frame-major candidate blocks: frames x lists <= items x 128 entries;
    // each threshold row is padded to a multiple of 4
    l.keys = off;
    off = align256(off + items * kItemKeep * kTileM * sizeof(unsigned long long));
    l.thr = off;
    off = align256(off + (items * kTileM + fr * 4) * sizeof(float));
    l.flist = off;
    off = align256(off + fr * sizeof(int32_t));
    l.fcount = off;
    off = align256(off + 16);
    l.gbound = off;
    off = align256(off + fr * kBoundWords * sizeof(unsigned int));
    l.total = off;
    return l;
}

// ================================================================ IVF-Flat
//
// Coarse stage: cand_kernel<false> over the fp16 centroid shadow gives each
// frame candidate lists of centroids; coarse_select_warp_kernel (one warp
// per frame; coarse_select_kernel, one CTA per frame, when a frame has more
// than 32 candidate lists) re-ranks them with
// exact fp32 distances in the reference order, keeps the first nprobe by
// (distance total order, list id) -- crates/vocal-cpu/src/retrieval.rs:45-51 --
// and certifies that no dropped centroid could enter them.  Fine stage: the
// (frame, probe) pairs are bucketed by list, their fp16 frames gathered into
// list order, cand_kernel<true> scans each list's rows for its pairs, and
// ivf_merge_warp_kernel re-ranks per frame with the scan position (probe
// rank, storage row) as the tie order -- :52-64 -- then certifies and blends.
// Frames left uncertified by either stage are re-run by the exact engine.

constexpr int kIvfMaxProbe = 8;

struct CoarseArgs {
    int d;
    int nlist;
    int nprobe;
    int lists;       // coarse candidate lists per frame
    int thr_stride;  // thresholds per frame row
    int slots;       // lists * kItemKeep rounded up to 32
    const unsigned long long *keys;  // [frame][lists][kItemKeep]
    const float *thr;                // [frame][thr_stride]
    const float4 *qstats;
    const float *queries;
    float *out;
    const float *index_rate;
    int mode;
    const float *centroids;  // fp32 [nlist][d]
    float max_norm, max_hat, max_residual, acc_rel, norm_rel, exact_rel;  // centroid bounds
    int32_t *probes;      // [frames][nprobe] list ids, coarse rank order
    int32_t *probe_ok;    // [frames] 1 when the fine stage handles the frame
    int32_t *list_count;  // [nlist] pairs per list (atomic)
    int32_t *fallback_list;
    int32_t *fallback_count;
};

__global__ void __launch_bounds__(kMergeThreads) coarse_select_kernel(CoarseArgs a) {
    extern __shared__ __align__(16) uint8_t csm[];
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(csm);
    float *q = reinterpret_cast<float *>(csm + static_cast<size_t>(a.slots) * 8);
    __shared__ SelectState sel;
    __shared__ unsigned long long sel_keys[kRerankMax];
    __shared__ unsigned long long exact_keys[kRerankMax];
    __shared__ unsigned long long top_keys[kIvfMaxProbe];
    __shared__ int ok_s;
    const int tid = threadIdx.x, lane = tid & 31, octet = tid >> 3, j = tid & 7;
    const long long frame = blockIdx.x;
    const int d = a.d, P = a.nprobe;
    const float *src = a.queries + frame * d;
    const float inf = __int_as_float(0x7f800000);
    if (a.mode == kModeBlend && !(load_ratio(a.index_rate) > 0.f)) {
        // r <= 0: the frame is left as is (copied when out of place)
        float *dst = a.out + frame * d;
        if (dst != src)
            for (int i = tid; i < d; i += kMergeThreads) dst[i] = src[i];
        if (tid == 0) a.probe_ok[frame] = 0;
        return;
    }
    for (int i = tid; i < d; i += kMergeThreads) q[i] = src[i];
    // the frame's contiguous candidate block (slots past a list's count hold kEmptyKey)
    float tmin = inf;
    for (int s = tid; s < a.lists; s += kMergeThreads) tmin = fminf(tmin, a.thr[frame * a.thr_stride + s]);
    const int real_slots = a.lists * kItemKeep;
    const unsigned long long *fk = a.keys + static_cast<size_t>(frame) * real_slots;
#pragma unroll 4
    for (int i = tid; i < a.slots; i += kMergeThreads) keys[i] = i < real_slots ? fk[i] : kEmptyKey;
    const KeyStats ks = key_stats<kMergeThreads>(keys, a.slots, tmin, sel);
    float cut;
    bool too_many;
    int m = select_rerank<kMergeThreads>(keys, a.slots, ks, sel_keys, sel, cut, too_many);
    const float bound = fminf(ks.tmin, cut);
    const float4 qs = a.qstats[frame];
    // exact centroid distances (no narrowing: the centroid rows come from
    // L2, so the extra pass costs more than it saves); every centroid takes part, as in the
    // reference's sort (no +inf filter here)
    for (int c0 = 0; c0 < m; c0 += 64) {
        uint32_t lists[2];
        const float *xs[2];
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int c = c0 + octet + 32 * kk;
            lists[kk] = key_pos(sel_keys[c < m ? c : 0]);
            xs[kk] = a.centroids + static_cast<size_t>(lists[kk]) * d;
        }
        float dist[2];
        octet_l2n<2>(q, xs, d, j, lane & ~7, kFullMask, dist);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int c = c0 + octet + 32 * kk;
            if (c < m && j == 0) exact_keys[c] = make_key(dist[kk], lists[kk]);
        }
    }
    __syncthreads();
    // rank selection of the first P keys (keys are distinct: list ids are)
    for (int c = tid; c < m; c += kMergeThreads) {
        const unsigned long long kc = exact_keys[c];
        int rank = 0;
        for (int i = 0; i < m; ++i) rank += exact_keys[i] < kc;
        if (rank < P) top_keys[rank] = kc;
    }
    __syncthreads();
    if (tid == 0) {
        bool ok = !too_many && m >= P;
        if (ok) {
            const float dp = key_dist(top_keys[P - 1]);
            ok = certify(bound, dp, qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel, a.norm_rel, a.exact_rel);
        }
        ok_s = ok;
        a.probe_ok[frame] = ok ? 1 : 0;
        if (!ok) {
            const int pos = atomicAdd(a.fallback_count, 1);
            a.fallback_list[pos] = static_cast<int32_t>(frame);
        }
    }
    __syncthreads();
    if (ok_s && tid < P) {
        const int32_t list = static_cast<int32_t>(key_pos(top_keys[tid]));
        a.probes[frame * P + tid] = list;
        atomicAdd(&a.list_count[list], 1);
    }
}

// One CTA of 1024 threads: pair offsets per list (exclusive scan of
// list_count), reset of the scatter cursors, and the fine-stage work items
// (list, frame tile within the list's pairs).
__global__ void __launch_bounds__(1024) bucket_scan_kernel(const int32_t *__restrict__ list_count,
                                                           const int32_t *__restrict__ order, int nlist,
                                                           int32_t *__restrict__ list_start,
                                                           int32_t *__restrict__ list_cursor, int2 *__restrict__ items,
                                                           int *__restrict__ item_count) {
    __shared__ int warp_pairs[32], warp_items[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (nlist + 1023) / 1024;
    const int l0 = min(nlist, tid * per), l1 = min(nlist, l0 + per);
    int pairs = 0, tiles = 0;
    for (int o = l0; o < l1; ++o) {
        const int c = list_count[order[o]];
        pairs += c;
        tiles += (c + kTileM - 1) / kTileM;
    }
    int ip = pairs, it = tiles;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int up = __shfl_up_sync(kFullMask, ip, off), ut = __shfl_up_sync(kFullMask, it, off);
        if (lane >= off) {
            ip += up;
            it += ut;
        }
    }
    if (lane == 31) {
        warp_pairs[warp] = ip;
        warp_items[warp] = it;
    }
    __syncthreads();
    if (warp == 0) {
        int wp = warp_pairs[lane], wi = warp_items[lane];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int up = __shfl_up_sync(kFullMask, wp, off), ut = __shfl_up_sync(kFullMask, wi, off);
            if (lane >= off) {
                wp += up;
                wi += ut;
            }
        }
        warp_pairs[lane] = wp;
        warp_items[lane] = wi;
    }
    __syncthreads();
    int pbase = ip - pairs + (warp > 0 ? warp_pairs[warp - 1] : 0);
    int ibase = it - tiles + (warp > 0 ? warp_items[warp - 1] : 0);
    for (int o = l0; o < l1; ++o) {
        const int l = order[o];
        const int c = list_count[l];
        list_start[l] = pbase;
        list_cursor[l] = 0;
        const int nt = (c + kTileM - 1) / kTileM;
        for (int t = 0; t < nt; ++t) items[ibase + t] = make_int2(l, t);
        pbase += c;
        ibase += nt;
    }
    if (tid == 1023) {
        list_start[nlist] = warp_pairs[31];
        *item_count = warp_items[31];
    }
}

__global__ void bucket_scatter_kernel(const int32_t *__restrict__ probes, const int32_t *__restrict__ probe_ok,
                                      long long frames, int P, const int32_t *__restrict__ list_start,
                                      int32_t *__restrict__ list_cursor, int32_t *__restrict__ pair_frame,
                                      int32_t *__restrict__ pair_slot) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= frames * P) return;
    const long long f = i / P;
    if (!probe_ok[f]) return;
    const int32_t list = probes[i];
    const int32_t pos = list_start[list] + atomicAdd(&list_cursor[list], 1);
    pair_frame[pos] = static_cast<int32_t>(f);
    pair_slot[i] = pos;
}

// One warp per pair: its frame's fp16 row into list order.
__global__ void gather_pairs_kernel(const __half *__restrict__ q16, int d_pad, const int32_t *__restrict__ pair_frame,
                                    const int32_t *__restrict__ pair_total, __half *__restrict__ qp,
                                    long long max_pairs) {
    const long long pos = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (pos >= max_pairs || pos >= *pair_total) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(q16 + static_cast<size_t>(pair_frame[pos]) * d_pad);
    uint4 *dst = reinterpret_cast<uint4 *>(qp + static_cast<size_t>(pos) * d_pad);
    for (int i = lane; i < d_pad / 8; i += 32) dst[i] = src[i];
}

struct IvfMergeArgs {
    long long frames;
    int d;
    int nprobe;
    int pair_stride;
    const int32_t *probes;
    const int32_t *probe_ok;
    const int32_t *pair_slot;
    const int32_t *offsets;
    const unsigned long long *keys;  // [kHalves * kItemKeep][pair_stride]
    const int *counts;               // [kHalves][pair_stride]
    const float *thr;
    const float4 *qstats;
    const float *queries;
    float *out;
    const float *index_rate;
    int mode;
    int k;
    float *dist_out;
    int64_t *label_out;
    int64_t label_base;
    const float *vectors;
    const int32_t *ids;
    float max_norm, max_hat, max_residual, acc_rel, norm_rel, exact_rel;
    int32_t *fallback_list;
    int32_t *fallback_count;
    RerunHint *hints;  // [kSplitFrames] or null: what the exact re-run needs to rescan
    DeviceCounters *counters;
};

// ---------------------------------------------------------------- IVF merge, one warp per frame
//
// ivf_merge_warp_kernel: one warp per frame and no CTA-wide barrier, so a
// launch of many frames keeps a few dozen frames in flight per SM (a CTA per
// frame with CTA-wide selection passes kept three).  Per frame: lane 2p + h loads the
// candidate list (probe p, column half h; at most 16 keys, ascending) into
// its warp's shared slots; U = the 8th smallest key of all lists (a warp
// merge of the list heads); the re-rank set is every key whose lower bound
// d~ + ||q||^2 - e does not exceed (U + ||q||^2 + e)(1 + 4 exact_rel) (the
// narrowing test: a dropped row can neither enter nor tie the exact top 8;
// rows the candidate stage never kept are covered by the lists' thresholds
// in the certificate); the four octets compute the kept rows' exact
// distances in the reference order, keyed by scan position (probe rank,
// storage row); the top 8 by a warp merge; certificate; search output or
// blend.
constexpr int kIvfWarps = 8;

__global__ void __launch_bounds__(32 * kIvfWarps, 3) ivf_merge_warp_kernel(IvfMergeArgs a) {
    extern __shared__ __align__(16) float ivq[];  // [kIvfWarps][dq] frame rows
    __shared__ unsigned long long lists[kIvfWarps][kIvfMaxProbe * kHalves * kItemKeep];
    __shared__ unsigned long long sel[kIvfWarps][kRerankMax];
    __shared__ unsigned long long ex[kIvfWarps][kRerankMax];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, octet = lane >> 3, j = lane & 7;
    const long long frame = static_cast<long long>(blockIdx.x) * kIvfWarps + w;
    launch_dependents();  // as in merge_kernel: the exact kernel's launch overlaps this one
    if (frame >= a.frames || !a.probe_ok[frame]) return;  // r <= 0 (handled) or exact re-run
    const int d = a.d, P = a.nprobe;
    const int dq = (d + 3) & ~3;
    float *q = ivq + static_cast<size_t>(w) * dq;
    unsigned long long *lk = lists[w];
    const size_t stride = static_cast<size_t>(a.pair_stride);
    const float *src = a.queries + frame * d;
    float *dst = a.out + frame * d;
    const float inf = __int_as_float(0x7f800000);
    const float ratio = a.mode == kModeBlend ? load_ratio(a.index_rate) : 1.f;
    for (int i = lane; i < d; i += 32) q[i] = src[i];
    // probe p's list on lane p: start, end and scan-position base
    int32_t pstart = 0, pend = 0;
    if (lane < P) {
        const int32_t list = a.probes[frame * P + lane];
        pstart = a.offsets[list];
        pend = a.offsets[list + 1];
    }
    uint32_t incl = lane < P ? static_cast<uint32_t>(pend - pstart) : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t up = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += up;
    }
    const uint32_t pbase = incl - (lane < P ? static_cast<uint32_t>(pend - pstart) : 0u);
    // candidate list (probe lane / 2, half lane % 2) into the warp's slots
    const int L = P * kHalves;
    int cnt = 0;
    float thr = inf;
    if (lane < L) {
        const int p = lane / kHalves, h = lane % kHalves;
        const size_t pos = static_cast<size_t>(a.pair_slot[frame * P + p]);
        cnt = a.counts[h * stride + pos];
        thr = a.thr[h * stride + pos];
        // all of the list's loads in flight at once, beside the count's (the
        // keys of one pair are kItemKeep strided words apart; every slot of
        // the [half][K][pair] array exists, those past the count are unused)
        unsigned long long kv[kItemKeep];
#pragma unroll
        for (int i = 0; i < kItemKeep; ++i) kv[i] = __ldg(a.keys + (h * kItemKeep + i) * stride + pos);
#pragma unroll
        for (int i = 0; i < kItemKeep; ++i)
            if (i < cnt) lk[lane * kItemKeep + i] = kv[i];
    }
    float tmin = thr;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tmin = fminf(tmin, __shfl_xor_sync(kFullMask, tmin, o));
    __syncwarp();
    // U: the 8th smallest key of all lists
    unsigned long long u8 = kEmptyKey;
    {
        int head = 0;
#pragma unroll 1
        for (int r = 0; r < 8; ++r) {
            const unsigned long long c = head < cnt ? lk[lane * kItemKeep + head] : kEmptyKey;
            const unsigned long long m = warp_min_u64(c);
            if (c == m && m != kEmptyKey) ++head;
            u8 = m;
        }
    }
    const float4 qs = a.qstats[frame];
    const float e = approx_error(qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel, a.norm_rel);
    const float limit = u8 == kEmptyKey ? inf : (key_dist(u8) + qs.x + e) * (1.f + 4.f * a.exact_rel) + 1e-30f;
    // the re-rank set, compacted into sel (each lane scans one list)
    int kept = 0;
    for (int i = 0; i < cnt; ++i) kept += !(key_dist(lk[lane * kItemKeep + i]) + qs.x - e > limit);
    uint32_t kincl = static_cast<uint32_t>(kept);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t up = __shfl_up_sync(kFullMask, kincl, o);
        if (lane >= o) kincl += up;
    }
    const int total = __shfl_sync(kFullMask, static_cast<int>(kincl), 31);
    {
        int at = static_cast<int>(kincl) - kept;
        for (int i = 0; i < cnt; ++i) {
            const unsigned long long k = lk[lane * kItemKeep + i];
            if (!(key_dist(k) + qs.x - e > limit)) {
                if (at < kRerankMax) sel[w][at] = k;
                ++at;
            }
        }
    }
    const bool too_many = total > kRerankMax;
    const int m = min(total, kRerankMax);
    __syncwarp();
    // exact distances, two rows per octet per round, keyed by scan position
    for (int c0 = 0; c0 < m; c0 += 8) {
        uint32_t rows[2];
        const float *xs[2];
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int c = c0 + octet + 4 * kk;
            rows[kk] = key_pos(sel[w][c < m ? c : c0]);
            xs[kk] = a.vectors + static_cast<size_t>(rows[kk]) * d;
        }
        float dist[2];
        octet_l2n<2>(q, xs, d, j, lane & ~7, kFullMask, dist);
        uint32_t sp[2] = {0u, 0u};
        for (int pr = 0; pr < P; ++pr) {  // the probe holding each row (lists are disjoint row ranges)
            const int32_t s = __shfl_sync(kFullMask, pstart, pr), t = __shfl_sync(kFullMask, pend, pr);
            const uint32_t b = __shfl_sync(kFullMask, pbase, pr);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
                if (static_cast<int32_t>(rows[kk]) >= s && static_cast<int32_t>(rows[kk]) < t)
                    sp[kk] = b + (rows[kk] - static_cast<uint32_t>(s));
        }
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int c = c0 + octet + 4 * kk;
            if (j == 0 && c < m) ex[w][c] = dist[kk] < inf ? make_key(dist[kk], sp[kk]) : kEmptyKey;
        }
    }
    __syncwarp();
    // the exact top 8: per lane the keys lane, lane + 32, ... (sorted), then 8 warp minima
    unsigned long long best[8];
    {
        unsigned long long v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) v[t] = lane + 32 * t < m ? ex[w][lane + 32 * t] : kEmptyKey;
        key_cx(v[0], v[1]); key_cx(v[2], v[3]); key_cx(v[0], v[2]); key_cx(v[1], v[3]); key_cx(v[1], v[2]);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const unsigned long long mn = warp_min_u64(v[0]);
            best[r] = mn;
            if (v[0] == mn && mn != kEmptyKey) {
                v[0] = v[1];
                v[1] = v[2];
                v[2] = v[3];
                v[3] = kEmptyKey;
            }
        }
    }
    int count = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) count += best[i] != kEmptyKey;
    const float d8 = count == 8 ? key_dist(best[7]) : inf;
    const bool ok = !too_many && certify(tmin, d8, qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel,
                                         a.norm_rel, a.exact_rel);
    if (!ok) {
        int pos = 0;
        if (lane == 0) {
            pos = atomicAdd(a.fallback_count, 1);
            a.fallback_list[pos] = static_cast<int32_t>(frame);
        }
        pos = __shfl_sync(kFullMask, pos, 0);
        if (a.hints != nullptr && pos < kSplitFrames) {
            // The probes the re-run must rescan: those with a list whose
            // threshold cannot certify d8 (every probe when the re-rank set
            // overflowed or holds fewer than 8 rows).  A list that certifies
            // d8 dropped only rows that can neither reach nor tie the frame's
            // exact 8th best (d8 bounds it from above); rows outside the
            // re-rank set are beaten by the 8 rows at or below U.  So the
            // other probes contribute at most their re-ranked rows, of which
            // the exact top 8 is handed over.
            uint32_t scan_mask = ~0u;
            if (!too_many && count == 8) {
                const bool fails = lane < L && !certify(thr, d8, qs, a.max_norm, a.max_hat, a.max_residual,
                                                        a.acc_rel, a.norm_rel, a.exact_rel);
                const uint32_t fb = __ballot_sync(kFullMask, fails);
                scan_mask = 0u;
                for (int p = 0; p < P; ++p)
                    if ((fb >> (p * kHalves)) & ((1u << kHalves) - 1u)) scan_mask |= 1u << p;
                if (scan_mask == 0u) scan_mask = ~0u;
            }
            unsigned long long v[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const unsigned long long key = lane + 32 * t < m ? ex[w][lane + 32 * t] : kEmptyKey;
                const uint32_t spos = key_pos(key);
                bool rescanned = true;
                for (int pr = 0; pr < P; ++pr) {
                    const int32_t s = __shfl_sync(kFullMask, pstart, pr), t2 = __shfl_sync(kFullMask, pend, pr);
                    const uint32_t b = __shfl_sync(kFullMask, pbase, pr);
                    if (spos >= b && spos < b + static_cast<uint32_t>(t2 - s)) rescanned = (scan_mask >> pr) & 1u;
                }
                v[t] = key != kEmptyKey && !rescanned ? key : kEmptyKey;
            }
            key_cx(v[0], v[1]); key_cx(v[2], v[3]); key_cx(v[0], v[2]); key_cx(v[1], v[3]); key_cx(v[1], v[2]);
            RerunHint *h = a.hints + pos;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const unsigned long long mn = warp_min_u64(v[0]);
                if (lane == 0) h->keys[r] = mn;
                if (v[0] == mn && mn != kEmptyKey) {
                    v[0] = v[1];
                    v[1] = v[2];
                    v[2] = v[3];
                    v[3] = kEmptyKey;
                }
            }
            if (lane == 0) {
                h->scan_mask = scan_mask;
                h->frame = static_cast<int32_t>(frame);
            }
        }
        return;
    }
    if (lane == 0 && a.counters) atomicAdd(&a.counters->candidate_frames, 1ull);
    // lane k < 8: its neighbour's storage row (scan position -> probe -> row)
    unsigned long long mine = kEmptyKey;
#pragma unroll
    for (int i = 0; i < 8; ++i) mine = lane == i ? best[i] : mine;
    int32_t row = -1;
    {
        const uint32_t spos = key_pos(mine);
        for (int pr = 0; pr < P; ++pr) {
            const int32_t s = __shfl_sync(kFullMask, pstart, pr), t = __shfl_sync(kFullMask, pend, pr);
            const uint32_t b = __shfl_sync(kFullMask, pbase, pr);
            if (mine != kEmptyKey && spos >= b && spos < b + static_cast<uint32_t>(t - s))
                row = s + static_cast<int32_t>(spos - b);
        }
    }
    if (a.mode == kModeSearch) {
        if (lane < a.k) {
            const bool have = lane < count;
            a.dist_out[frame * a.k + lane] = have ? key_dist(mine) : inf;
            a.label_out[frame * a.k + lane] = have ? static_cast<int64_t>(a.ids[row]) + a.label_base : -1;
        }
        return;
    }
    if (count == 0) {
        if (lane == 0 && a.counters) atomicAdd(&a.counters->empty_frames, 1ull);
        if (dst != src)
            for (int i = lane; i < d; i += 32) dst[i] = q[i];
        return;
    }
    const double wk = lane < count ? reference_weight(key_dist(mine)) : 0.0;
    double wv[8];
    const float *vr[8];
    double wsum = -0.0;  // the reference's order: S = w0 + w1 + ... (zeros past count)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        wv[k] = __shfl_sync(kFullMask, wk, k);
        const int32_t rk = __shfl_sync(kFullMask, row, k);
        vr[k] = a.vectors + static_cast<size_t>(rk >= 0 ? rk : 0) * d;
        wsum = __dadd_rn(wsum, wv[k]);
    }
    const WeightDivisor sum = weight_divisor(wsum);
    if ((d & 3) == 0 && ((reinterpret_cast<uintptr_t>(a.vectors) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        // four elements per lane and step: one 16-byte load per neighbour
        // row, a quarter of the dependent row round trips; each element's
        // arithmetic (and so its result) is the scalar loop's
        for (int i4 = lane; i4 < (d >> 2); i4 += 32) {
            float4 r4[8];
#pragma unroll
            for (int k = 0; k < 8; ++k)
                r4[k] = k < count ? __ldg(reinterpret_cast<const float4 *>(vr[k]) + i4) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 q4 = reinterpret_cast<const float4 *>(q)[i4];
            float v[8];
            float4 o;
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = r4[k].x;
            o.x = reference_blend_element<false>(q4.x, v, wv, sum, count, ratio);
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = r4[k].y;
            o.y = reference_blend_element<false>(q4.y, v, wv, sum, count, ratio);
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = r4[k].z;
            o.z = reference_blend_element<false>(q4.z, v, wv, sum, count, ratio);
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = r4[k].w;
            o.w = reference_blend_element<false>(q4.w, v, wv, sum, count, ratio);
            reinterpret_cast<float4 *>(dst)[i4] = o;
        }
        return;
    }
    for (int i = lane; i < d; i += 32) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = k < count ? __ldg(vr[k] + i) : 0.f;
        dst[i] = reference_blend_element<true>(q[i], v, wv, sum, count, ratio);
    }
}

// coarse_select_warp_kernel: coarse_select_kernel's result with one warp per
// frame, for launches whose frames have at most 32 coarse candidate lists
// (one per lane; at most 16 keys each, ascending).  U = the nprobe-th
// smallest key; every key whose lower bound can reach (U + ||q||^2 + e)(1 +
// 4 exact_rel) is re-ranked with the exact centroid distance in the
// reference order; the first nprobe by (distance total order, list id) --
// crates/vocal-cpu/src/retrieval.rs:45-51 -- are certified against the
// lists' thresholds, then recorded and counted per list.
__global__ void __launch_bounds__(32 * kIvfWarps) coarse_select_warp_kernel(CoarseArgs a, long long frames) {
    extern __shared__ __align__(16) float cq[];  // [kIvfWarps][dq]
    __shared__ unsigned long long lists[kIvfWarps][32 * kItemKeep];
    __shared__ unsigned long long sel[kIvfWarps][kRerankMax];
    __shared__ unsigned long long ex[kIvfWarps][kRerankMax];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, octet = lane >> 3, j = lane & 7;
    const long long frame = static_cast<long long>(blockIdx.x) * kIvfWarps + w;
    if (frame >= frames) return;
    const int d = a.d, P = a.nprobe;
    const float *src = a.queries + frame * d;
    const float inf = __int_as_float(0x7f800000);
    if (a.mode == kModeBlend && !(load_ratio(a.index_rate) > 0.f)) {
        // r <= 0: the frame is left as is (copied when out of place)
        float *dst = a.out + frame * d;
        if (dst != src)
            for (int i = lane; i < d; i += 32) dst[i] = src[i];
        if (lane == 0) a.probe_ok[frame] = 0;
        return;
    }
    float *q = cq + static_cast<size_t>(w) * ((d + 3) & ~3);
    unsigned long long *lk = lists[w];
    for (int i = lane; i < d; i += 32) q[i] = src[i];
    const unsigned long long *fk = a.keys + static_cast<size_t>(frame) * a.lists * kItemKeep;
    int cnt = 0;
    float thr = inf;
    if (lane < a.lists) {
        thr = a.thr[frame * a.thr_stride + lane];
        // the list's 16 keys (slots past its count hold kEmptyKey): every
        // load in flight before the first store
        ulonglong2 kv[kItemKeep / 2];
#pragma unroll
        for (int i = 0; i < kItemKeep / 2; ++i) kv[i] = __ldg(reinterpret_cast<const ulonglong2 *>(fk + lane * kItemKeep) + i);
#pragma unroll
        for (int i = 0; i < kItemKeep / 2; ++i) {
            lk[lane * kItemKeep + 2 * i] = kv[i].x;
            lk[lane * kItemKeep + 2 * i + 1] = kv[i].y;
            cnt += (kv[i].x != kEmptyKey) + (kv[i].y != kEmptyKey);
        }
    }
    float tmin = thr;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tmin = fminf(tmin, __shfl_xor_sync(kFullMask, tmin, o));
    __syncwarp();
    unsigned long long up = kEmptyKey;  // the P-th smallest approximate key
    {
        int head = 0;
#pragma unroll 1
        for (int r = 0; r < P; ++r) {
            const unsigned long long c = head < cnt ? lk[lane * kItemKeep + head] : kEmptyKey;
            const unsigned long long m = warp_min_u64(c);
            if (c == m && m != kEmptyKey) ++head;
            up = m;
        }
    }
    const float4 qs = a.qstats[frame];
    const float e = approx_error(qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel, a.norm_rel);
    const float limit = up == kEmptyKey ? inf : (key_dist(up) + qs.x + e) * (1.f + 4.f * a.exact_rel) + 1e-30f;
    int kept = 0;
    for (int i = 0; i < cnt; ++i) kept += !(key_dist(lk[lane * kItemKeep + i]) + qs.x - e > limit);
    uint32_t kincl = static_cast<uint32_t>(kept);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(kFullMask, kincl, o);
        if (lane >= o) kincl += u;
    }
    const int total = __shfl_sync(kFullMask, static_cast<int>(kincl), 31);
    {
        int at = static_cast<int>(kincl) - kept;
        for (int i = 0; i < cnt; ++i) {
            const unsigned long long k = lk[lane * kItemKeep + i];
            if (!(key_dist(k) + qs.x - e > limit)) {
                if (at < kRerankMax) sel[w][at] = k;
                ++at;
            }
        }
    }
    const bool too_many = total > kRerankMax;
    const int m = min(total, kRerankMax);
    __syncwarp();
    // exact centroid distances (every centroid takes part, as in the
    // reference's sort: no +inf filter here)
    for (int c0 = 0; c0 < m; c0 += 8) {
        uint32_t ls[2];
        const float *xs[2];
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int c = c0 + octet + 4 * kk;
            ls[kk] = key_pos(sel[w][c < m ? c : c0]);
            xs[kk] = a.centroids + static_cast<size_t>(ls[kk]) * d;
        }
        float dist[2];
        octet_l2n<2>(q, xs, d, j, lane & ~7, kFullMask, dist);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int c = c0 + octet + 4 * kk;
            if (j == 0 && c < m) ex[w][c] = make_key(dist[kk], ls[kk]);
        }
    }
    __syncwarp();
    // the first P exact keys: per lane keys lane, lane + 32, ... (sorted), P warp minima
    unsigned long long top = kEmptyKey, pth = kEmptyKey;
    {
        unsigned long long v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) v[t] = lane + 32 * t < m ? ex[w][lane + 32 * t] : kEmptyKey;
        key_cx(v[0], v[1]); key_cx(v[2], v[3]); key_cx(v[0], v[2]); key_cx(v[1], v[3]); key_cx(v[1], v[2]);
#pragma unroll 1
        for (int r = 0; r < P; ++r) {
            const unsigned long long mn = warp_min_u64(v[0]);
            if (lane == r) top = mn;
            pth = mn;
            if (v[0] == mn && mn != kEmptyKey) {
                v[0] = v[1];
                v[1] = v[2];
                v[2] = v[3];
                v[3] = kEmptyKey;
            }
        }
    }
    bool ok = !too_many && m >= P && pth != kEmptyKey;
    if (ok)
        ok = certify(tmin, key_dist(pth), qs, a.max_norm, a.max_hat, a.max_residual, a.acc_rel, a.norm_rel,
                     a.exact_rel);
    if (lane == 0) {
        a.probe_ok[frame] = ok ? 1 : 0;
        if (!ok) {
            const int pos = atomicAdd(a.fallback_count, 1);
            a.fallback_list[pos] = static_cast<int32_t>(frame);
        }
    }
    if (ok && lane < P) {
        const int32_t list = static_cast<int32_t>(key_pos(top));
        a.probes[frame * P + lane] = list;
        atomicAdd(&a.list_count[list], 1);
    }
}

struct IvfWs {
    size_t q16, qstats, ckeys, cthr, probes, probe_ok, list_count, list_cursor, list_start, items, item_count,
        pair_frame, pair_slot, qp, fkeys, fcounts, fthr, flist, fcount, gbound, total;
};

IvfWs ivf_ws_layout(size_t frames, int d_pad, int nlist, int nprobe, int sms) {
    IvfWs l{};
    const size_t fr = (frames + kTileM - 1) / kTileM * kTileM;
    const size_t clists = static_cast<size_t>(items_cap(frames, sms)) * kHalves;
    const size_t pairs = frames * static_cast<size_t>(nprobe);
    const size_t max_items = (pairs + kTileM - 1) / kTileM + static_cast<size_t>(nlist);
    size_t off = 0;
    auto take = [&](size_t &field, size_t bytes) {
        field = off;
        off = align256(off + bytes);
    };
    take(l.q16, fr * d_pad * sizeof(__half));
    take(l.qstats, fr * sizeof(float4));
    take(l.ckeys, clists * kItemKeep * kTileM * sizeof(unsigned long long));
    take(l.cthr, (clists * kTileM + fr * 4) * sizeof(float));
    take(l.probes, pairs * sizeof(int32_t));
    take(l.probe_ok, fr * sizeof(int32_t));
    take(l.list_count, static_cast<size_t>(nlist) * sizeof(int32_t));
    take(l.list_cursor, static_cast<size_t>(nlist) * sizeof(int32_t));
    take(l.list_start, static_cast<size_t>(nlist + 1) * sizeof(int32_t));
    take(l.items, max_items * sizeof(int2));
    take(l.item_count, 16);
    take(l.pair_frame, pairs * sizeof(int32_t));
    take(l.pair_slot, pairs * sizeof(int32_t));
    take(l.qp, pairs * d_pad * sizeof(__half));
    take(l.fkeys, static_cast<size_t>(kHalves) * kItemKeep * pairs * sizeof(unsigned long long));
    take(l.fcounts, kHalves * pairs * sizeof(int));
    take(l.fthr, kHalves * pairs * sizeof(float));
    take(l.flist, fr * sizeof(int32_t));
    take(l.fcount, 16);
    take(l.gbound, fr * kBoundWords * sizeof(unsigned int));
    l.total = off;
    return l;
}

}  // namespace

namespace {

// fp16 shadow + squared norms + bounds of `rows` fp32 rows into `xh`/`norms`
// (already allocated, rows_pad rows); returns {max ||x||, max ||x^||, max ||x - x^||}.
void build_shadow(const float *x, int64_t rows, int64_t rows_pad, int d, int d_pad, float scale, __half *xh,
                  float *norms, float out[3]) {
    cuda_check(cudaMemset(xh, 0, static_cast<size_t>(rows_pad) * d_pad * sizeof(__half)));
    unsigned int *maxima = nullptr;
    cuda_check(cudaMalloc(reinterpret_cast<void **>(&maxima), 4 * sizeof(unsigned int)));
    cuda_check(cudaMemset(maxima, 0, 4 * sizeof(unsigned int)));
    fill_kernel<<<64, 256>>>(norms + rows, static_cast<size_t>(rows_pad - rows), std::numeric_limits<float>::infinity());
    build_rows_kernel<<<static_cast<unsigned>((rows * 32 + 255) / 256), 256>>>(x, xh, norms, rows, d, d_pad, scale,
                                                                             maxima);
    cudaError_t rc = cudaGetLastError();
    unsigned int m[3] = {0, 0, 0};
    if (rc == cudaSuccess) rc = cudaMemcpy(m, maxima, sizeof(m), cudaMemcpyDeviceToHost);
    cudaFree(maxima);
    cuda_check(rc);
    std::memcpy(out, m, sizeof(m));
    out[0] *= 1.0001f;
    out[1] *= 1.0001f;
    out[2] = out[2] * 1.0001f + 1e-30f;
}


}  // namespace

float max_abs(const float *x, size_t count) {
    unsigned int *m = nullptr;
    cuda_check(cudaMalloc(reinterpret_cast<void **>(&m), sizeof(unsigned int)));
    cuda_check(cudaMemset(m, 0, sizeof(unsigned int)));
    max_abs_kernel<<<1024, 256>>>(x, count, m);
    cudaError_t rc = cudaGetLastError();
    unsigned int bits = 0;
    if (rc == cudaSuccess) rc = cudaMemcpy(&bits, m, 4, cudaMemcpyDeviceToHost);
    cudaFree(m);
    cuda_check(rc);
    float v;
    std::memcpy(&v, &bits, 4);
    return v;
}

void build_tc(VfrIndex *ix) {
    const bool ivf = ix->nlist > 1;
    if (ivf && ix->nprobe > kIvfMaxProbe) return;  // wide probes use the exact engine
    int dev = 0;
    cuda_check(cudaGetDevice(&dev));
    cuda_check(cudaDeviceGetAttribute(&ix->sm_count, cudaDevAttrMultiProcessorCount, dev));
    ix->d_pad = (ix->d + kTileK - 1) / kTileK * kTileK;
    // IVF lists start anywhere, so a list's last tile can reach 255 rows past n
    ix->n_pad = (ix->n + kTileN - 1) / kTileN * kTileN + (ivf ? kTileN : 0);
    cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->vectors_h),
                          static_cast<size_t>(ix->n_pad) * ix->d_pad * sizeof(__half)),
               "cudaMalloc fp16 shadow");
    cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->row_norms), ix->n_pad * sizeof(float)), "cudaMalloc norms");
    // power-of-two scale keeping |s x| within [1, 8192] where possible, so
    // frames up to 8x the database's magnitude still fit fp16
    float maxabs = max_abs(ix->vectors, static_cast<size_t>(ix->n) * ix->d);
    if (ivf) maxabs = std::max(maxabs, max_abs(ix->centroids, static_cast<size_t>(ix->nlist) * ix->d));
    int e = 0;
    if (maxabs > 0.f) {
        const int ex = static_cast<int>(std::floor(std::log2(maxabs)));
        if (ex > 13) e = 13 - ex;
        if (ex < 0) e = -ex;
    }
    ix->tc_scale = std::ldexp(1.0f, e);
    float m[3];
    build_shadow(ix->vectors, ix->n, ix->n_pad, ix->d, ix->d_pad, ix->tc_scale, ix->vectors_h, ix->row_norms, m);
    ix->max_row_norm = m[0];
    ix->max_row_hat = m[1];
    ix->max_row_residual = m[2];
    bool finite = std::isfinite(ix->max_row_norm) && std::isfinite(ix->max_row_hat);
    if (ivf && finite) {
        ix->nlist_pad = (ix->nlist + kTileN - 1) / kTileN * kTileN;
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->centroids_h),
                              static_cast<size_t>(ix->nlist_pad) * ix->d_pad * sizeof(__half)));
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->centroid_norms), ix->nlist_pad * sizeof(float)));
        build_shadow(ix->centroids, ix->nlist, ix->nlist_pad, ix->d, ix->d_pad, ix->tc_scale, ix->centroids_h,
                     ix->centroid_norms, m);
        ix->max_cent_norm = m[0];
        ix->max_cent_hat = m[1];
        ix->max_cent_residual = m[2];
        finite = std::isfinite(ix->max_cent_norm) && std::isfinite(ix->max_cent_hat);
    }
    if (!finite) {
        // squared norms overflow fp32: the candidate bounds are meaningless,
        // so this index stays on the exact engine
        release_tc(ix);
        return;
    }
    encode_rows(&ix->tmap_vectors, ix->vectors_h, ix->d_pad, ix->n_pad, kTileN);
    encode_rows(&ix->tmap_vectors_half, ix->vectors_h, ix->d_pad, ix->n_pad, kTileN / 2);
    if (ivf) {
        encode_rows(&ix->tmap_centroids, ix->centroids_h, ix->d_pad, ix->nlist_pad, kTileN);
        // lists by descending size (ties by id): the fine stage's item table
        // follows this order, largest work first
        std::vector<int32_t> order(static_cast<size_t>(ix->nlist));
        for (int32_t l = 0; l < ix->nlist; ++l) order[l] = l;
        const std::vector<int32_t> &off = ix->host_offsets;
        std::stable_sort(order.begin(), order.end(),
                         [&](int32_t x, int32_t y) { return off[x + 1] - off[x] > off[y + 1] - off[y]; });
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->list_order), order.size() * sizeof(int32_t)));
        cuda_check(cudaMemcpy(ix->list_order, order.data(), order.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
    }
    constexpr int kBig = static_cast<int>(Pipe<kFullLayout>::kSmem), kSmall = static_cast<int>(Pipe<kSpreadLayout>::kSmem);
    cuda_check(cudaFuncSetAttribute(cand_kernel<false, kShortKeep>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBig));
    cuda_check(cudaFuncSetAttribute(cand_kernel<false, kIvfKeep>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBig));
    cuda_check(cudaFuncSetAttribute(cand_kernel<true, kIvfKeep>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBig));
    cuda_check(cudaFuncSetAttribute(cand_kernel<false, kShortKeep, kSpreadLayout>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kSmall));
    cuda_check(cudaFuncSetAttribute(cand_kernel<false, kIvfKeep, kSpreadLayout>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kSmall));
    ix->pair_clusters = 0;
    if (!ivf) {
        // CTA pairs (clusters of two) that can be resident at once
        constexpr int kPairSmem = static_cast<int>(Pipe<kPairLayout>::kSmem);
        cuda_check(cudaFuncSetAttribute(cand_kernel<false, kIvfKeep, kPairLayout>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmem));
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(static_cast<unsigned>(2 * (ix->sm_count / 2)));
        cfg.blockDim = dim3(kThreadsTC);
        cfg.dynamicSmemBytes = kPairSmem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        // opt-in (VFR_PAIR=1): measured on c5 it runs at the one-CTA
        // layout's rate per clock, so the one-CTA layout stays the default
        const char *env = std::getenv("VFR_PAIR");
        if (env && env[0] == '1') {
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, cand_kernel<false, kIvfKeep, kPairLayout>, &cfg) ==
                cudaSuccess)
                ix->pair_clusters = clusters;
            cudaGetLastError();  // a device without the query keeps the one-CTA layouts
        }
    }
    {
        int optin = 0;
        cuda_check(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ix->device));
        cudaFuncAttributes fa{}, fb{}, fc{}, fd{};
        cuda_check(cudaFuncGetAttributes(&fa, merge_kernel<kMergeThreads>));
        cuda_check(cudaFuncGetAttributes(&fb, merge_kernel<kMergeThreadsMax>));
        cuda_check(cudaFuncGetAttributes(&fc, merge_small_kernel<kMergeThreadsMax>));
        cuda_check(cudaFuncGetAttributes(&fd, merge_small_kernel<kMergeThreads>));
        ix->merge_smem_max = optin - static_cast<int>(std::max(
                                         {fa.sharedSizeBytes, fb.sharedSizeBytes, fc.sharedSizeBytes, fd.sharedSizeBytes}));
        cuda_check(cudaFuncSetAttribute(merge_kernel<kMergeThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        ix->merge_smem_max));
        cuda_check(cudaFuncSetAttribute(merge_kernel<kMergeThreadsMax>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        ix->merge_smem_max));
        cuda_check(cudaFuncSetAttribute(merge_small_kernel<kMergeThreadsMax>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, ix->merge_smem_max));
        cuda_check(cudaFuncSetAttribute(merge_small_kernel<kMergeThreads>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, ix->merge_smem_max));
        // merge_warp_kernel: one frame row per warp (d <= 4096: at most
        // 128 KB beside its 16 KB of static key arrays)
        cuda_check(cudaFuncSetAttribute(merge_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kMergeWarps * ((ix->d + 3) & ~3) * static_cast<int>(sizeof(float))));
    }
    cuda_check(cudaFuncSetAttribute(coarse_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
    if (ivf) {
        // the warp-per-frame kernels: one frame row per warp in dynamic
        // shared memory, beside their static per-warp key arrays
        const int rows = kIvfWarps * ((ix->d + 3) & ~3) * static_cast<int>(sizeof(float));
        cuda_check(cudaFuncSetAttribute(ivf_merge_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, rows));
        cuda_check(cudaFuncSetAttribute(coarse_select_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, rows));
    }
    {
        const char *env = std::getenv("VFR_SMALL_MERGE");
        ix->small_merge = !(env && env[0] == '0');
    }
    cuda_check(cudaDeviceSynchronize());
    ix->have_tc = true;
}

void release_tc(VfrIndex *ix) noexcept {
    if (!ix->shared) {
        if (ix->vectors_h) cudaFree(ix->vectors_h);
        if (ix->row_norms) cudaFree(ix->row_norms);
        if (ix->centroids_h) cudaFree(ix->centroids_h);
        if (ix->centroid_norms) cudaFree(ix->centroid_norms);
        if (ix->list_order) cudaFree(ix->list_order);
    }
    ix->list_order = nullptr;
    ix->centroids_h = nullptr;
    ix->centroid_norms = nullptr;
    if (ix->ws.base) cudaFree(ix->ws.base);
    ix->vectors_h = nullptr;
    ix->row_norms = nullptr;
    ix->ws = Workspace{};
    ix->have_tc = false;
}

void reserve_tc(VfrIndex *ix, size_t frames) {
    if (!ix->have_tc || frames <= ix->ws.frames) return;
    const size_t bytes = ix->nlist > 1
                             ? ivf_ws_layout(frames, ix->d_pad, ix->nlist, ix->nprobe, ix->sm_count).total
                             : ws_layout(frames, ix->d_pad, ix->sm_count).total;
    void *p = nullptr;
    cuda_check(cudaMalloc(&p, bytes), "cudaMalloc retrieval workspace");
    if (ix->ws.base) {
        cuda_check(cudaDeviceSynchronize());
        cudaFree(ix->ws.base);
    }
    ix->ws.base = p;
    ix->ws.bytes = bytes;
    ix->ws.frames = frames;
}

bool use_tc(const VfrIndex *ix, size_t frames) {
    if (!ix->have_tc || ix->engine == VFR_ENGINE_EXACT) return false;
    if (ix->engine == VFR_ENGINE_TENSOR) return true;
    // AUTO: tiny databases are cheaper on the exact engine alone
    return ix->n >= 2048 && frames >= 1;
}

namespace {

// IVF-Flat: coarse candidates + certified probe selection, bucketing of the
// (frame, probe) pairs by list, per-list candidates, exact merge, and the
// exact engine for uncertified frames.  Workspace from ivf_ws_layout.
void run_ivf(VfrIndex *ix, const float *queries, float *out, const float *rate, int mode, int k, float *dist_out,
             int64_t *label_out, size_t frames, cudaStream_t stream) {
    const int P = ix->nprobe;
    const IvfWs l = ivf_ws_layout(ix->ws.frames, ix->d_pad, ix->nlist, P, ix->sm_count);
    uint8_t *ws = static_cast<uint8_t *>(ix->ws.base);
    __half *q16 = reinterpret_cast<__half *>(ws + l.q16);
    float4 *qstats = reinterpret_cast<float4 *>(ws + l.qstats);
    auto *ckeys = reinterpret_cast<unsigned long long *>(ws + l.ckeys);
    float *cthr = reinterpret_cast<float *>(ws + l.cthr);
    int32_t *probes = reinterpret_cast<int32_t *>(ws + l.probes);
    int32_t *probe_ok = reinterpret_cast<int32_t *>(ws + l.probe_ok);
    int32_t *list_count = reinterpret_cast<int32_t *>(ws + l.list_count);
    int32_t *list_cursor = reinterpret_cast<int32_t *>(ws + l.list_cursor);
    int32_t *list_start = reinterpret_cast<int32_t *>(ws + l.list_start);
    int2 *items = reinterpret_cast<int2 *>(ws + l.items);
    int *item_count = reinterpret_cast<int *>(ws + l.item_count);
    int32_t *pair_frame = reinterpret_cast<int32_t *>(ws + l.pair_frame);
    int32_t *pair_slot = reinterpret_cast<int32_t *>(ws + l.pair_slot);
    __half *qp = reinterpret_cast<__half *>(ws + l.qp);
    auto *fkeys = reinterpret_cast<unsigned long long *>(ws + l.fkeys);
    int *fcounts = reinterpret_cast<int *>(ws + l.fcounts);
    float *fthr = reinterpret_cast<float *>(ws + l.fthr);
    int32_t *flist = reinterpret_cast<int32_t *>(ws + l.flist);
    int32_t *fcount = reinterpret_cast<int32_t *>(ws + l.fcount);
    unsigned int *gbound = reinterpret_cast<unsigned int *>(ws + l.gbound);
    const size_t pair_cap = ix->ws.frames * static_cast<size_t>(P);
    const float coef = -2.0f / (ix->tc_scale * ix->tc_scale);
    const float acc_rel = static_cast<float>(ix->d_pad) * std::ldexp(1.0f, -22);
    const float norm_rel = static_cast<float>(ix->d_pad) * std::ldexp(1.0f, -23);
    const float exact_rel = static_cast<float>(ix->d / 8 + 9) * std::ldexp(1.0f, -24);

    // 1. frames -> fp16
    const long long lanes = static_cast<long long>(frames) * 32;
    ix->prof.begin(kProfPrep, stream);
    prep_queries_kernel<<<static_cast<unsigned>((lanes + 255) / 256), 256, 0, stream>>>(
        queries, q16, qstats, static_cast<long long>(frames), ix->d, ix->d_pad, ix->tc_scale, fcount, gbound);
    cuda_check(cudaGetLastError());
    ix->prof.end(stream);
    cuda_check(cudaMemsetAsync(list_count, 0, static_cast<size_t>(ix->nlist) * sizeof(int32_t), stream));

    // 2. coarse candidates over the centroids
    const Plan pc = make_plan(frames, ix->nlist, ix->sm_count);
    ix->last_keep = kIvfKeep;
    ix->last_segments = pc.segments;
    ix->last_tiles_per_seg = pc.tiles_per_seg;
    ix->last_layout = kFullLayout;
    CUtensorMap tmap_q;
    encode_rows(&tmap_q, q16, ix->d_pad, frames, kTileM);
    CandArgs ca{};
    ca.frames = static_cast<int>(frames);
    ca.n_qtiles = pc.n_qtiles;
    ca.segments = pc.segments;
    ca.tiles_per_seg = pc.tiles_per_seg;
    ca.ksteps = ix->d_pad / kTileK;
    ca.n = ix->nlist;
    ca.seg_rows = static_cast<int64_t>(pc.tiles_per_seg) * kTileN;
    ca.row_norms = ix->centroid_norms;
    ca.coef = coef;
    ca.out_keys = ckeys;
    ca.out_thr = cthr;
    ca.lists = pc.segments * kHalves;
    ca.thr_stride = (ca.lists + 3) & ~3;
    ca.counters = ix->counters;
    ix->prof.begin(kProfCand, stream);
    cand_kernel<false, kIvfKeep><<<std::min(pc.segments * pc.n_qtiles, ix->sm_count), kThreadsTC, Pipe<kFullLayout>::kSmem, stream>>>(
        tmap_q, ix->tmap_centroids, ca);
    cuda_check(cudaGetLastError());
    ix->prof.end(stream);

    // 3. certified probe lists
    CoarseArgs cs{};
    cs.d = ix->d;
    cs.nlist = ix->nlist;
    cs.nprobe = P;
    cs.lists = ca.lists;
    cs.thr_stride = ca.thr_stride;
    cs.slots = (cs.lists * kItemKeep + 31) / 32 * 32;
    cs.keys = ckeys;
    cs.thr = cthr;
    cs.qstats = qstats;
    cs.queries = queries;
    cs.out = out;
    cs.index_rate = rate;
    cs.mode = mode;
    cs.centroids = ix->centroids;
    cs.max_norm = ix->max_cent_norm;
    cs.max_hat = ix->max_cent_hat;
    cs.max_residual = ix->max_cent_residual;
    cs.acc_rel = acc_rel;
    cs.norm_rel = norm_rel;
    cs.exact_rel = exact_rel;
    cs.probes = probes;
    cs.probe_ok = probe_ok;
    cs.list_count = list_count;
    cs.fallback_list = flist;
    cs.fallback_count = fcount;
    ix->prof.begin(kProfMerge, stream);
    if (cs.lists <= 32)
        coarse_select_warp_kernel<<<static_cast<unsigned>((frames + kIvfWarps - 1) / kIvfWarps), 32 * kIvfWarps,
                                    static_cast<size_t>(kIvfWarps) * ((ix->d + 3) & ~3) * 4, stream>>>(
            cs, static_cast<long long>(frames));
    else
        coarse_select_kernel<<<static_cast<unsigned>(frames), kMergeThreads,
                               static_cast<size_t>(cs.slots) * 8 + static_cast<size_t>(ix->d) * 4, stream>>>(cs);
    cuda_check(cudaGetLastError());
    // 4. pairs bucketed by list, frames gathered into list order
    bucket_scan_kernel<<<1, 1024, 0, stream>>>(list_count, ix->list_order, ix->nlist, list_start, list_cursor, items,
                                                item_count);
    cuda_check(cudaGetLastError());
    const long long npairs = static_cast<long long>(frames) * P;
    bucket_scatter_kernel<<<static_cast<unsigned>((npairs + 255) / 256), 256, 0, stream>>>(
        probes, probe_ok, static_cast<long long>(frames), P, list_start, list_cursor, pair_frame, pair_slot);
    cuda_check(cudaGetLastError());
    gather_pairs_kernel<<<static_cast<unsigned>((npairs * 32 + 255) / 256), 256, 0, stream>>>(
        q16, ix->d_pad, pair_frame, list_start + ix->nlist, qp, npairs);
    cuda_check(cudaGetLastError());
    ix->prof.end(stream);

    // 5. per-list candidates
    CUtensorMap tmap_qp;
    encode_rows(&tmap_qp, qp, ix->d_pad, pair_cap, kTileM);
    CandArgs cf{};
    cf.ksteps = ix->d_pad / kTileK;
    cf.n = ix->n;
    cf.row_norms = ix->row_norms;
    cf.coef = coef;
    cf.out_keys = fkeys;
    cf.out_count = fcounts;
    cf.out_thr = fthr;
    cf.counters = ix->counters;
    cf.items = items;
    cf.item_count = item_count;
    cf.list_offsets = ix->offsets;
    cf.list_start = list_start;
    cf.list_count = list_count;
    cf.pair_stride = static_cast<int>(pair_cap);
    cf.pair_frame = pair_frame;
    set_shared_bound(cf, ix, gbound, qstats);
    ix->prof.begin(kProfCand, stream);
    cand_kernel<true, kIvfKeep><<<ix->sm_count, kThreadsTC, Pipe<kFullLayout>::kSmem, stream>>>(tmap_qp, ix->tmap_vectors, cf);
    cuda_check(cudaGetLastError());
    ix->prof.end(stream);

    // 6. exact merge, certificate, blend / search output
    IvfMergeArgs im{};
    im.d = ix->d;
    im.nprobe = P;
    im.pair_stride = static_cast<int>(pair_cap);
    im.probes = probes;
    im.probe_ok = probe_ok;
    im.pair_slot = pair_slot;
    im.offsets = ix->offsets;
    im.keys = fkeys;
    im.counts = fcounts;
    im.thr = fthr;
    im.qstats = qstats;
    im.queries = queries;
    im.out = out;
    im.index_rate = rate;
    im.mode = mode;
    im.k = k;
    im.dist_out = dist_out;
    im.label_out = label_out;
    im.label_base = ix->label_base;
    im.vectors = ix->vectors;
    im.ids = ix->ids;
    im.max_norm = ix->max_row_norm;
    im.max_hat = ix->max_row_hat;
    im.max_residual = ix->max_row_residual;
    im.acc_rel = acc_rel;
    im.norm_rel = norm_rel;
    im.exact_rel = exact_rel;
    im.fallback_list = flist;
    im.hints = ix->rerun_hints;
    im.fallback_count = fcount;
    im.counters = ix->counters;
    im.frames = static_cast<long long>(frames);
    ix->prof.begin(kProfMerge, stream);
    ivf_merge_warp_kernel<<<static_cast<unsigned>((frames + kIvfWarps - 1) / kIvfWarps), 32 * kIvfWarps,
                            static_cast<size_t>(kIvfWarps) * ((ix->d + 3) & ~3) * 4, stream>>>(im);
    cuda_check(cudaGetLastError());
    ix->prof.end(stream);

    // 7. frames either certificate left open: exact re-run
    ExactArgs ea{};
    ea.d = ix->d;
    ea.nlist = ix->nlist;
    ea.nprobe = ix->nprobe;
    ea.centroids = ix->centroids;
    ea.offsets = ix->offsets;
    ea.vectors = ix->vectors;
    ea.ids = ix->ids;
    ea.queries = queries;
    ea.out = out;
    ea.index_rate = rate;
    ea.mode = mode;
    ea.k = k;
    ea.dist_out = dist_out;
    ea.label_out = label_out;
    ea.label_base = ix->label_base;
    ea.counters = ix->counters;
    ea.frame_list = flist;
    ea.frame_count = fcount;
    ea.split_keys = ix->split_keys;
    ea.split_done = ix->split_done;
    ea.probes = probes;
    ea.probe_ok = probe_ok;
    ea.hints = ix->rerun_hints;
    ix->prof.begin(kProfExact, stream);
    launch_exact(ea, static_cast<long long>(frames), stream, true);
    ix->prof.end(stream);
}

}  // namespace

void run_tc(VfrIndex *ix, const float *queries, float *out, const float *rate, int mode, int k, float *dist_out,
            int64_t *label_out, size_t frames, cudaStream_t stream, float *raw) {
    if (frames > ix->ws.frames) {
        cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
        cuda_check(cudaStreamIsCapturing(stream, &st));
        require(st == cudaStreamCaptureStatusNone,
                "retrieval workspace too small for this frame count during stream capture; call "
                "vfr_retrieval_reserve first");
        reserve_tc(ix, frames);
    }
    if (ix->nlist > 1) {
        if (raw)
            cuda_check(cudaMemcpyAsync(raw, queries, frames * static_cast<size_t>(ix->d) * sizeof(float),
                                       cudaMemcpyDeviceToDevice, stream));
        run_ivf(ix, queries, out, rate, mode, k, dist_out, label_out, frames, stream);
        return;
    }
    const WsLayout l = ws_layout(ix->ws.frames, ix->d_pad, ix->sm_count);
    uint8_t *ws = static_cast<uint8_t *>(ix->ws.base);
    __half *q16 = reinterpret_cast<__half *>(ws + l.q16);
    float4 *qstats = reinterpret_cast<float4 *>(ws + l.qstats);
    auto *keys = reinterpret_cast<unsigned long long *>(ws + l.keys);
    float *thr = reinterpret_cast<float *>(ws + l.thr);
    int32_t *flist = reinterpret_cast<int32_t *>(ws + l.flist);
    int32_t *fcount = reinterpret_cast<int32_t *>(ws + l.fcount);
    unsigned int *gbound = reinterpret_cast<unsigned int *>(ws + l.gbound);

    Plan p = make_plan(frames, ix->n, ix->sm_count);
    // large launches with long work items run on CTA pairs
    bool pair = false;
    if (ix->pair_clusters > 0 && frames >= static_cast<size_t>(kPairMinFrames)) {
        const Plan pp = make_plan_pair(frames, ix->n, ix->sm_count, ix->pair_clusters);
        if (pp.tiles_per_seg > kShortItemTiles) {
            p = pp;
            pair = true;
        }
    }
    const long long lanes = static_cast<long long>(frames) * 32;
    ix->prof.begin(kProfPrep, stream);
    prep_queries_kernel<<<static_cast<unsigned>((lanes + 255) / 256), 256, 0, stream>>>(
        queries, q16, qstats, static_cast<long long>(frames), ix->d, ix->d_pad, ix->tc_scale, fcount, gbound);
    cuda_check(cudaGetLastError());
    ix->prof.end(stream);

    CandArgs ca{};
    ca.frames = static_cast<int>(frames);
    ca.n_qtiles = p.n_qtiles;
    ca.segments = p.segments;
    ca.tiles_per_seg = p.tiles_per_seg;
    ca.ksteps = ix->d_pad / kTileK;
    ca.n = ix->n;
    ca.seg_rows = static_cast<int64_t>(p.tiles_per_seg) * kTileN;
    ca.row_norms = ix->row_norms;
    ca.coef = -2.0f / (ix->tc_scale * ix->tc_scale);
    ca.out_keys = keys;
    ca.out_thr = thr;
    ca.lists = p.segments * kHalves;
    ca.thr_stride = (ca.lists + 3) & ~3;
    ca.counters = ix->counters;
    set_shared_bound(ca, ix, gbound, qstats);
    ca.pair_layout = pair ? 1 : 0;
    note_plan(ix, p, frames);
    if (pair) ix->last_layout = kPairLayout;
    ix->prof.begin(kProfCand, stream);
    if (pair) {
        const int items = p.segments * ((p.n_qtiles + 1) / 2);
        launch_cand_pair(std::min(items, ix->pair_clusters), q16, ix->d_pad, ix->tmap_vectors_half, ca, stream);
    } else {
        const int items = p.segments * p.n_qtiles;
        launch_cand_flat(p, std::min(items, ix->sm_count), q16, ix->d_pad, ix->tmap_vectors, ca, stream);
    }
    ix->prof.end(stream);

    MergeArgs ma{};
    ma.d = ix->d;
    ma.lists = ca.lists;
    ma.thr_stride = ca.thr_stride;
    ma.keep = p.tiles_per_seg <= kShortItemTiles ? kShortKeep : kIvfKeep;
    ma.sort_size = (ma.lists * ma.keep + 31) / 32 * 32;  // key slots per frame
    ma.keys = keys;
    ma.thr = thr;
    ma.qstats = qstats;
    ma.queries = queries;
    ma.out = out;
    ma.index_rate = rate;
    ma.mode = mode;
    ma.k = k;
    ma.dist_out = dist_out;
    ma.label_out = label_out;
    ma.label_base = ix->label_base;
    ma.vectors = ix->vectors;
    ma.ids = ix->ids;
    ma.max_norm = ix->max_row_norm;
    ma.max_hat = ix->max_row_hat;
    ma.max_residual = ix->max_row_residual;
    ma.acc_rel = static_cast<float>(ix->d_pad) * std::ldexp(1.0f, -22);
    ma.norm_rel = static_cast<float>(ix->d_pad) * std::ldexp(1.0f, -23);
    ma.exact_rel = static_cast<float>(ix->d / 8 + 9) * std::ldexp(1.0f, -24);
    ma.fallback_list = flist;
    ma.raw_out = raw;
    ma.fallback_count = fcount;
    ma.counters = ix->counters;
    ma.gbound = gbound;
    ix->prof.begin(kProfMerge, stream);
    launch_merge(ix, ma, frames, stream);
    ix->prof.end(stream);

    // frames the certificate could not settle: exact re-run
    ExactArgs ea{};
    ea.d = ix->d;
    ea.nlist = ix->nlist;
    ea.nprobe = ix->nprobe;
    ea.centroids = ix->centroids;
    ea.offsets = ix->offsets;
    ea.vectors = ix->vectors;
    ea.ids = ix->ids;
    ea.queries = queries;
    ea.out = out;
    ea.index_rate = rate;
    ea.mode = mode;
    ea.k = k;
    ea.dist_out = dist_out;
    ea.label_out = label_out;
    ea.label_base = ix->label_base;
    ea.counters = ix->counters;
    ea.frame_list = flist;
    ea.frame_count = fcount;
    ea.split_keys = ix->split_keys;
    ea.split_done = ix->split_done;
    ix->prof.begin(kProfExact, stream);
    launch_exact(ea, static_cast<long long>(frames), stream, true);
    ix->prof.end(stream);
}

// ---------------------------------------------------------------- no-allocation blend
//
// vfr_retrieval_blend_noalloc: the tensor-core blend of vocal_faiss_gpu_blend
// for callers that must not allocate device memory during a call -- for
// example a realtime audio callback, where cudaMalloc/cudaFree can
// synchronise the device and take driver locks (an unbounded stall inside a
// hard deadline), or a host whose device memory budget is fixed up front.
// Its working memory is the file-scope array below, sized for at most
// kNoAllocMaxFrames frames of width <= kNoAllocMaxWidth (5.3 MiB, held by
// every GPU that loads the library until the process exits).  The array's
// device address is looked up once per device (cudaGetSymbolAddress) on the
// first call made on that device, so that first call should come before any
// stream capture.  All calls share the array and it keeps the last call's
// contents (each call overwrites what it reads and clears its fallback
// counter), so calls whose kernels overlap on the GPU -- on different streams,
// or on several indexes of one device -- race and must be serialised by the
// caller.
namespace {

constexpr size_t kNoAllocMaxFrames = 256;
constexpr int kNoAllocMaxWidth = 1024;  // d_pad limit: covers RVC v1 (256) and v2 (768)
constexpr int kNoAllocMaxItems = 148;   // work items; each writes kHalves candidate lists
constexpr size_t kNoAllocQ16 = 0;
constexpr size_t kNoAllocQStats = kNoAllocQ16 + kNoAllocMaxFrames * kNoAllocMaxWidth * sizeof(__half);
constexpr size_t kNoAllocKeys = kNoAllocQStats + kNoAllocMaxFrames * sizeof(float4);
constexpr size_t kNoAllocLists = static_cast<size_t>(kNoAllocMaxItems) * kHalves;
constexpr size_t kNoAllocThr = kNoAllocKeys + kNoAllocLists * kItemKeep * kTileM * sizeof(unsigned long long);
constexpr size_t kNoAllocList = kNoAllocThr + (kNoAllocLists * kTileM + kNoAllocMaxFrames * 4) * sizeof(float);
constexpr size_t kNoAllocCount = kNoAllocList + kNoAllocMaxFrames * sizeof(int32_t);
constexpr size_t kNoAllocBound = kNoAllocCount + 256;
constexpr size_t kNoAllocBytes = kNoAllocBound + kNoAllocMaxFrames * kBoundWords * sizeof(unsigned int);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kNoAllocMaxDevices = 64;
std::once_flag g_noalloc_once[kNoAllocMaxDevices];
void *g_noalloc_addr[kNoAllocMaxDevices];
cudaError_t g_noalloc_status[kNoAllocMaxDevices];

// Host-side address of the scratch array on `device` (which is current).
void *noalloc_scratch(int device) {
    require(device >= 0 && device < kNoAllocMaxDevices, "device ordinal out of range for the no-allocation path");
    std::call_once(g_noalloc_once[device], [device] {
        g_noalloc_status[device] = cudaGetSymbolAddress(&g_noalloc_addr[device], g_noalloc_scratch);
    });
    cuda_check(g_noalloc_status[device], "cudaGetSymbolAddress(no-allocation scratch)");
    return g_noalloc_addr[device];
}

// make_plan restricted to kNoAllocMaxItems work items.
Plan make_plan_noalloc(size_t frames, int64_t n, int sms) {
    Plan p{};
    p.n_qtiles = static_cast<int>((frames + kTileM - 1) / kTileM);
    const int64_t ntiles = (n + kTileN - 1) / kTileN;
    double best = 1e300;
    p.segments = 0;
    for (int64_t s = 1; s <= std::min<int64_t>(kMaxSegments, ntiles); ++s) {
        const int64_t tps = (ntiles + s - 1) / s;
        const int64_t seg = (ntiles + tps - 1) / tps;
        if (seg * p.n_qtiles > kNoAllocMaxItems) break;
        const int64_t waves = (seg * p.n_qtiles + sms - 1) / sms;
        const double cost = static_cast<double>(waves * (tps + 2)) + 0.02 * static_cast<double>(seg);
        if (cost < best - 1e-9) {
            best = cost;
            p.segments = static_cast<int>(seg);
            p.tiles_per_seg = static_cast<int>(tps);
        }
    }
    return p;
}

}  // namespace

void run_tc_noalloc(VfrIndex *ix, float *features, const float *rate, size_t frames, cudaStream_t stream) {
    uint8_t *ws = static_cast<uint8_t *>(noalloc_scratch(ix->device));
    __half *q16 = reinterpret_cast<__half *>(ws + kNoAllocQ16);
    float4 *qstats = reinterpret_cast<float4 *>(ws + kNoAllocQStats);
    auto *keys = reinterpret_cast<unsigned long long *>(ws + kNoAllocKeys);
    float *thr = reinterpret_cast<float *>(ws + kNoAllocThr);
    int32_t *flist = reinterpret_cast<int32_t *>(ws + kNoAllocList);
    int32_t *fcount = reinterpret_cast<int32_t *>(ws + kNoAllocCount);
    unsigned int *gbound = reinterpret_cast<unsigned int *>(ws + kNoAllocBound);

    const Plan p = make_plan_noalloc(frames, ix->n, ix->sm_count);
    require(p.segments > 0, "no-allocation scratch cannot hold this plan");
    const long long lanes = static_cast<long long>(frames) * 32;
    prep_queries_kernel<<<static_cast<unsigned>((lanes + 255) / 256), 256, 0, stream>>>(
        features, q16, qstats, static_cast<long long>(frames), ix->d, ix->d_pad, ix->tc_scale, fcount, gbound);
    cuda_check(cudaGetLastError());

    CandArgs ca{};
    ca.frames = static_cast<int>(frames);
    ca.n_qtiles = p.n_qtiles;
    ca.segments = p.segments;
    ca.tiles_per_seg = p.tiles_per_seg;
    ca.ksteps = ix->d_pad / kTileK;
    ca.n = ix->n;
    ca.seg_rows = static_cast<int64_t>(p.tiles_per_seg) * kTileN;
    ca.row_norms = ix->row_norms;
    ca.coef = -2.0f / (ix->tc_scale * ix->tc_scale);
    ca.out_keys = keys;
    ca.out_thr = thr;
    ca.lists = p.segments * kHalves;
    ca.thr_stride = (ca.lists + 3) & ~3;
    ca.counters = ix->counters;
    set_shared_bound(ca, ix, gbound, qstats);
    const int items = p.segments * p.n_qtiles;
    note_plan(ix, p, frames);
    launch_cand_flat(p, std::min(items, ix->sm_count), q16, ix->d_pad, ix->tmap_vectors, ca, stream);

    MergeArgs ma{};
    ma.d = ix->d;
    ma.lists = ca.lists;
    ma.thr_stride = ca.thr_stride;
    ma.keep = p.tiles_per_seg <= kShortItemTiles ? kShortKeep : kIvfKeep;
    ma.sort_size = (ma.lists * ma.keep + 31) / 32 * 32;  // key slots per frame
    ma.keys = keys;
    ma.thr = thr;
    ma.qstats = qstats;
    ma.queries = features;
    ma.out = features;
    ma.index_rate = rate;
    ma.mode = kModeBlend;
    ma.k = 8;
    ma.label_base = ix->label_base;
    ma.vectors = ix->vectors;
    ma.ids = ix->ids;
    ma.max_norm = ix->max_row_norm;
    ma.max_hat = ix->max_row_hat;
    ma.max_residual = ix->max_row_residual;
    ma.acc_rel = static_cast<float>(ix->d_pad) * std::ldexp(1.0f, -22);
    ma.norm_rel = static_cast<float>(ix->d_pad) * std::ldexp(1.0f, -23);
    ma.exact_rel = static_cast<float>(ix->d / 8 + 9) * std::ldexp(1.0f, -24);
    ma.fallback_list = flist;
    ma.fallback_count = fcount;
    ma.counters = ix->counters;
    ma.gbound = gbound;
    launch_merge(ix, ma, frames, stream);

    ExactArgs ea{};
    ea.d = ix->d;
    ea.nlist = ix->nlist;
    ea.nprobe = ix->nprobe;
    ea.centroids = ix->centroids;
    ea.offsets = ix->offsets;
    ea.vectors = ix->vectors;
    ea.ids = ix->ids;
    ea.queries = features;
    ea.out = features;
    ea.index_rate = rate;
    ea.mode = kModeBlend;
    ea.k = 8;
    ea.label_base = ix->label_base;
    ea.counters = ix->counters;
    ea.frame_list = flist;
    ea.frame_count = fcount;
    ea.split_keys = ix->split_keys;
    ea.split_done = ix->split_done;
    launch_exact(ea, static_cast<long long>(frames), stream, true);
    cuda_check(cudaGetLastError());
}

}  // namespace vfr

extern "C" int vfr_retrieval_blend_noalloc(VfrIndex *index, float *features, size_t frames, int32_t width,
                                           const float *index_rate, VfrStream *stream, char **error) {
    return vfr::guarded(error, [&] {
        vfr::require(index && features && frames > 0 && index_rate, "invalid FAISS GPU blend arguments");
        vfr::require(width == index->d, "FAISS feature width mismatch");
        vfr::require(stream && stream->stream, "invalid FAISS CUDA stream");
        vfr::require(index->have_tc && index->nlist == 1,
                     "no-allocation blend needs the tensor-core layout (flat index, tensor or auto engine)");
        vfr::require(frames <= vfr::kNoAllocMaxFrames,
                     "no-allocation blend takes at most 256 frames per call");
        vfr::require(index->d_pad <= vfr::kNoAllocMaxWidth, "no-allocation blend takes feature widths up to 1024");
        int previous = 0;
        vfr::cuda_check(cudaGetDevice(&previous));
        if (previous != index->device) vfr::cuda_check(cudaSetDevice(index->device));
        try {
            vfr::run_tc_noalloc(index, features, index_rate, frames, static_cast<cudaStream_t>(stream->stream));
        } catch (...) {
            if (previous != index->device) cudaSetDevice(previous);
            throw;
        }
        if (previous != index->device) vfr::cuda_check(cudaSetDevice(previous));
    });
}
