// Tensor-core engine: fp16 shadow of the database, tcgen05/TMEM distance GEMM
// with fused per-frame candidate selection, exact fp32 re-rank and blend.
#pragma once

#include "vfr_common.h"

namespace vfr {

void build_tc(VfrIndex *ix);                 // derived layout, at create time
void release_tc(VfrIndex *ix) noexcept;      // frees what build_tc/reserve_tc made
void reserve_tc(VfrIndex *ix, size_t frames);  // workspace for `frames` frames
bool use_tc(const VfrIndex *ix, size_t frames);
float max_abs(const float *x, size_t count);  // max |x[i]| (synchronous)
// raw (blend only, may be null): receives the frames as they were before the
// blend; the flat path writes it from the merge kernel's own load.
void run_tc(VfrIndex *ix, const float *queries, float *out, const float *rate, int mode, int k, float *dist_out,
            int64_t *label_out, size_t frames, cudaStream_t stream, float *raw = nullptr);

// In-place tensor-core blend using the library's static scratch array
// instead of the index workspace (vfr_retrieval_blend_noalloc).
void run_tc_noalloc(VfrIndex *ix, float *features, const float *rate, size_t frames, cudaStream_t stream);

}  // namespace vfr
