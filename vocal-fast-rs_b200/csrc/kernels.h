// Kernel launch interface between the C ABI (abi.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vfr {

constexpr int kTopK = 8;       // kTopK, crates/vocal-tensorrt/native/retrieval_kernels.cuh:8
constexpr int kMaxProbe = 32;  // kMaxProbe, retrieval_kernels.cuh:7

// Device diagnostic counters written by the kernels (one block per index).
struct DeviceCounters {
    unsigned long long empty_frames;      // frames whose probed lists held no row
    unsigned long long fallback_frames;   // frames re-run by the exact scan
    unsigned long long timeouts;          // bounded waits that gave up
    unsigned long long candidate_frames;  // frames served by the tensor-core path
    unsigned long long rerun_rows;        // rows the exact re-runs scanned
};

enum { kModeBlend = 0, kModeSearch = 1 };

// Exact SIMT engine (exact_kernels.cu).
struct ExactArgs {
    int d;
    int nlist;
    int nprobe;
    const float *centroids;
    const int32_t *offsets;
    const float *vectors;
    const int32_t *ids;
    const float *queries;
    float *out;  // may alias queries
    const float *index_rate;
    int mode;
    int k;
    float *dist_out;
    int64_t *label_out;
    int64_t label_base;
    DeviceCounters *counters;
    const int32_t *frame_list;   // optional: frames to process (device)
    const int32_t *frame_count;  // with frame_list: its length (device)
    // optional, with frame_list: scratch that lets up to kSplitFrames listed
    // frames share the grid ([kSplitFrames][kExactSplitGrid][8] keys and
    // kSplitFrames counters, zero between calls)
    unsigned long long *split_keys;
    int32_t *split_done;
    // optional (IVF): the coarse stage's lists per frame ([frame][nprobe], in
    // coarse order) and whether they are set; reused instead of recomputed
    const int32_t *probes;
    const int32_t *probe_ok;
    // optional (IVF, with split scratch): the fine stage's hints for the
    // first kSplitFrames listed frames (RerunHint, below); null = full scans
    struct RerunHint *hints;
};
constexpr int kSplitFrames = 64;       // listed frames that share the grid
constexpr int kExactSplitGrid = 1184;  // CTAs of a frame-list launch at most
constexpr size_t kSplitKeyBytes = static_cast<size_t>(kSplitFrames) * kExactSplitGrid * 8 * 8;
// What the IVF merge hands the exact re-run about a frame it could not
// certify (entry i of the hint array belongs to entry i of the frame list):
// bit p of scan_mask marks probe p (coarse order) whose candidate lists
// could not certify the frame, and keys[] holds the exact top 8 (distance,
// scan position) of the re-ranked rows of the other probes.  Rows of those
// other probes outside keys[] cannot enter the frame's exact top 8 (their
// lists' thresholds or the narrowing limit exclude them), so the re-run
// scans only the marked probes and merges keys[] in.  frame = -1 when the
// entry holds nothing; the re-run clears it after use.
struct RerunHint {
    unsigned long long keys[8];
    int32_t frame;
    uint32_t scan_mask;
};
// frames: the frame count, or with a frame list the largest possible length.
// after_kernel: launched behind another kernel of the same call, which it may
// overlap until its own dependency wait (programmatic dependent launch).
void launch_exact(const ExactArgs &args, long long frames, cudaStream_t stream, bool after_kernel = false);

// Unvoiced-frame protection (protect_kernels.cu).
void launch_protect(float *features, const float *raw, const float *pitchf, const float *ratio, const float *protect,
                    int frames, int hubert_frames, int width, cudaStream_t stream);

// RVC frontend after the blend, with the protection fused (protect_kernels.cu).
int frontend_frames(int hubert_frames, int f0_frames);
void launch_frontend(const float *hubert, const float *raw, const float *f0, const float *ratio,
                     const float *protect, int hubert_frames, int f0_frames, int width, float *feats, float *pitchf,
                     int32_t *pitch, cudaStream_t stream);

// The generic engine's linear 2x frontend with its protection and coarse
// pitch (protect_kernels.cu).
void launch_engine_frontend(const float *blended, const float *raw, const float *hz, float protect, int frames,
                            int hz_frames, int width, float *out, int32_t *coarse, cudaStream_t stream);

// Index of the first non-finite value of x[0 .. count) (all ones when none);
// synchronous, on the legacy stream of the current device (ingest_kernels.cu).
unsigned long long first_nonfinite(const float *x, unsigned long long count, int sm_count);

// IVF trainer (training_kernels.cu): out[r] = x[rows[r]]; fixed-point
// centroid sums (sums[labels[r]][c] += rint(x[r][c] * scale)); means
// (sum / count * inv_scale, 0 for empty clusters); int64 -> int32 labels.
void launch_gather_rows(const float *x, const int64_t *rows, long long count, int d, float *out,
                        cudaStream_t stream);
void launch_fixed_sums(const float *x, const int64_t *labels, long long rows, int d, double scale,
                       unsigned long long *sums, cudaStream_t stream);
void launch_means(const unsigned long long *sums, const long long *counts, int k, int d, double inv_scale,
                  float *centroids, cudaStream_t stream);
void launch_narrow_labels(const int64_t *wide, long long n, int32_t *out, cudaStream_t stream);

// Sharded helpers (shard_kernels.cu).
void launch_merge_topk(const float *dist, const int64_t *labels, int shards, long long frames, float *out_dist,
                       int64_t *out_labels, cudaStream_t stream);
void launch_gather_owned(const float *vectors, const int32_t *row_of_id, int64_t n, int64_t label_base, int d,
                         const int64_t *labels, long long frames, float *out, cudaStream_t stream);
void launch_blend_gathered(const float *queries, float *out, const float *dist, const float *neighbours,
                           long long frames, int d, const float *index_rate, cudaStream_t stream);
void launch_blend_gathered_rows(const float *queries, float *out, const float *dist, const float *rows_buf,
                                const int32_t *slot_rows, long long rows, long long frames, int d,
                                const float *index_rate, cudaStream_t stream);

}  // namespace vfr
