// Unvoiced-frame protection, the step after the retrieval blend in the
// reference's realtime pipeline (crates/vocal-tensorrt/native/
// retrieval_protection.cu:4-16, called from crates/vocal-tensorrt/src/
// pipeline.rs:1858-1870 after the frontend's 2x interpolation).  For frames
// whose pitch is not positive, the blended, interpolated features are mixed
// back toward the raw HuBERT features saved before the blend:
//   f = f * p + raw[min(frame / 2, hubert_frames - 1)] * (1 - p)
// skipped entirely when index_rate <= 0 or p >= 0.5 (both read from device
// memory, so a captured graph follows updates; NaN passes both tests, as in
// the reference).  Each operation is rounded on its own (no contraction into
// fused multiply-adds), which the oracle restates.
//
// HBM-bound elementwise work: frames x width x 8 bytes of features plus the
// raw rows; one float4 per thread when the width allows, grid-strided.
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace vfr {
namespace {

__device__ __forceinline__ float protect_value(float f, float r, float p) {
    return __fadd_rn(__fmul_rn(f, p), __fmul_rn(r, __fsub_rn(1.0f, p)));
}

// width % 4 == 0: thread i handles features [4i, 4i + 4) of one frame.
__global__ void protect_vec4_kernel(float4 *__restrict__ features, const float4 *__restrict__ raw,
                                    const float *__restrict__ pitchf, const float *__restrict__ ratio,
                                    const float *__restrict__ protect, long long quads, int quads_per_frame,
                                    int hubert_frames) {
    const float r = *ratio, p = *protect;
    if (r <= 0.0f || p >= 0.5f) return;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < quads;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long frame = i / quads_per_frame;
        if (pitchf[frame] > 0.0f) continue;
        const long long row = frame / 2 < hubert_frames - 1 ? frame / 2 : hubert_frames - 1;
        const float4 f = features[i];
        const float4 x = __ldg(raw + row * quads_per_frame + (i - frame * quads_per_frame));
        features[i] = make_float4(protect_value(f.x, x.x, p), protect_value(f.y, x.y, p),
                                  protect_value(f.z, x.z, p), protect_value(f.w, x.w, p));
    }
}

__global__ void protect_scalar_kernel(float *__restrict__ features, const float *__restrict__ raw,
                                      const float *__restrict__ pitchf, const float *__restrict__ ratio,
                                      const float *__restrict__ protect, long long elements, int width,
                                      int hubert_frames) {
    const float r = *ratio, p = *protect;
    if (r <= 0.0f || p >= 0.5f) return;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < elements;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long frame = i / width;
        if (pitchf[frame] > 0.0f) continue;
        const long long row = frame / 2 < hubert_frames - 1 ? frame / 2 : hubert_frames - 1;
        features[i] = protect_value(features[i], __ldg(raw + row * width + (i - frame * width)), p);
    }
}

}  // namespace

void launch_protect(float *features, const float *raw, const float *pitchf, const float *ratio, const float *protect,
                    int frames, int hubert_frames, int width, int sm_count, cudaStream_t stream) {
    const long long elements = static_cast<long long>(frames) * width;
    const bool vec = width % 4 == 0 && reinterpret_cast<uintptr_t>(features) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(raw) % 16 == 0;
    const long long items = vec ? elements / 4 : elements;
    const long long blocks_needed = (items + 255) / 256;
    const int grid = static_cast<int>(blocks_needed < sm_count * 8LL ? blocks_needed : sm_count * 8LL);
    if (vec)
        protect_vec4_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<float4 *>(features),
                                                       reinterpret_cast<const float4 *>(raw), pitchf, ratio,
                                                       protect, items, width / 4, hubert_frames);
    else
        protect_scalar_kernel<<<grid, 256, 0, stream>>>(features, raw, pitchf, ratio, protect, elements, width,
                                                         hubert_frames);
}

}  // namespace vfr
