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
// raw rows; one CTA per frame, float4 lanes when the width allows.
#include <cmath>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace vfr {
namespace {

__device__ __forceinline__ float protect_value(float f, float r, float p) {
    return __fadd_rn(__fmul_rn(f, p), __fmul_rn(r, __fsub_rn(1.0f, p)));
}

// One CTA per interpolated frame: a voiced frame's CTA returns at once, an
// unvoiced one mixes its width features toward the raw row (float4 lanes when
// kVec: width % 4 == 0 and both rows 16-byte aligned).
template <bool kVec>
__global__ void protect_rows_kernel(float *__restrict__ features, const float *__restrict__ raw,
                                    const float *__restrict__ pitchf, const float *__restrict__ ratio,
                                    const float *__restrict__ protect, int width, int hubert_frames) {
    const float r = *ratio, p = *protect;
    const int frame = blockIdx.x;
    if (r <= 0.0f || p >= 0.5f || pitchf[frame] > 0.0f) return;
    const int row = frame / 2 < hubert_frames - 1 ? frame / 2 : hubert_frames - 1;
    float *out = features + static_cast<long long>(frame) * width;
    const float *src = raw + static_cast<long long>(row) * width;
    if (kVec) {
        float4 *o4 = reinterpret_cast<float4 *>(out);
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        for (int c = threadIdx.x; c < width / 4; c += blockDim.x) {
            const float4 f = o4[c], x = __ldg(s4 + c);
            o4[c] = make_float4(protect_value(f.x, x.x, p), protect_value(f.y, x.y, p), protect_value(f.z, x.z, p),
                                protect_value(f.w, x.w, p));
        }
    } else {
        for (int c = threadIdx.x; c < width; c += blockDim.x) out[c] = protect_value(out[c], __ldg(src + c), p);
    }
}

// threads per frame CTA: the row's lanes rounded up to a warp, at most 256
int row_threads(int lanes) {
    const int t = (lanes + 31) / 32 * 32;
    return t < 256 ? t : 256;
}

bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

void launch_protect(float *features, const float *raw, const float *pitchf, const float *ratio, const float *protect,
                    int frames, int hubert_frames, int width, cudaStream_t stream) {
    const bool vec = width % 4 == 0 && aligned16(features) && aligned16(raw);
    if (vec)
        protect_rows_kernel<true><<<frames, row_threads(width / 4), 0, stream>>>(features, raw, pitchf, ratio,
                                                                                  protect, width, hubert_frames);
    else
        protect_rows_kernel<false><<<frames, row_threads(width), 0, stream>>>(features, raw, pitchf, ratio, protect,
                                                                               width, hubert_frames);
}

}  // namespace vfr

// ---------------------------------------------------------------- frontend
// The RVC frontend after the blend (crates/vocal-tensorrt/native/
// frontend.cpp:36-75, a TensorRT graph in the reference): the last HuBERT
// frame is appended, the frames are interpolated 2x (nearest, asymmetric:
// output frame t reads input frame t / 2) and cropped to
// target = min(2 (hubert_frames + 1), f0_frames); pitchf is f0 cropped the
// same way and pitch its coarse mel bin, round(clamp((1127 ln(1 + f0 / 700)
// - mel_min) * 254 / (mel_max - mel_min) + 1, 1, 255)).  Output frame t thus
// reads HuBERT row min(t / 2, hubert_frames - 1), the row the protection
// (above) mixes back toward, so both run in one pass: when raw is given,
// unvoiced frames get f * p + raw[row] * (1 - p) under the same ratio and
// amount conditions.
namespace vfr {
namespace {

// One CTA per output frame t: copies HuBERT row min(t / 2, hubert_frames - 1)
// (mixed toward the raw row when protecting and the frame is unvoiced) and,
// from thread 0, pitchf[t] and pitch[t].
template <bool kVec>
__global__ void frontend_kernel(const float *__restrict__ hubert, const float *__restrict__ raw,
                                const float *__restrict__ f0, const float *__restrict__ ratio,
                                const float *__restrict__ protect, int hubert_frames, int width, float mel_min,
                                float mel_scale, float *__restrict__ feats, float *__restrict__ pitchf,
                                int32_t *__restrict__ pitch) {
    const int t = blockIdx.x;
    const int row = t / 2 < hubert_frames - 1 ? t / 2 : hubert_frames - 1;
    const float f = f0[t];
    const bool protecting = raw != nullptr && !(*ratio <= 0.0f || *protect >= 0.5f) && !(f > 0.0f);
    const float p = protecting ? *protect : 0.0f;
    const float *src = hubert + static_cast<long long>(row) * width;
    const float *rsrc = protecting ? raw + static_cast<long long>(row) * width : nullptr;
    float *out = feats + static_cast<long long>(t) * width;
    if (kVec) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        const float4 *r4 = reinterpret_cast<const float4 *>(rsrc);
        float4 *o4 = reinterpret_cast<float4 *>(out);
        for (int c = threadIdx.x; c < width / 4; c += blockDim.x) {
            float4 v = __ldg(s4 + c);
            if (protecting) {
                const float4 x = __ldg(r4 + c);
                v = make_float4(protect_value(v.x, x.x, p), protect_value(v.y, x.y, p), protect_value(v.z, x.z, p),
                                protect_value(v.w, x.w, p));
            }
            o4[c] = v;
        }
    } else {
        for (int c = threadIdx.x; c < width; c += blockDim.x) {
            const float v = __ldg(src + c);
            out[c] = protecting ? protect_value(v, __ldg(rsrc + c), p) : v;
        }
    }
    if (threadIdx.x == 0) {
        pitchf[t] = f;
        // the graph's order: ((f * (1/700)) + 1) -> log -> * 1127, then
        // (mel - mel_min) * mel_scale + 1 (constants from the host, as the
        // graph's are); NaN and the clamp's low side both give 1
        const float mel = __fmul_rn(logf(__fadd_rn(__fmul_rn(f, 1.0f / 700.0f), 1.0f)), 1127.0f);
        float coarse = __fadd_rn(__fmul_rn(__fsub_rn(mel, mel_min), mel_scale), 1.0f);
        coarse = fminf(fmaxf(coarse, 1.0f), 255.0f);
        pitch[t] = static_cast<int32_t>(rintf(coarse));
    }
}

}  // namespace

int frontend_frames(int hubert_frames, int f0_frames) {
    const long long interp = 2LL * (hubert_frames + 1);
    return static_cast<int>(interp < f0_frames ? interp : f0_frames);
}

void launch_frontend(const float *hubert, const float *raw, const float *f0, const float *ratio,
                     const float *protect, int hubert_frames, int f0_frames, int width, float *feats, float *pitchf,
                     int32_t *pitch, cudaStream_t stream) {
    const int target = frontend_frames(hubert_frames, f0_frames);
    // frontend.cpp:66-67, computed on the host in f32 like the graph's constants
    const float mel_min = 1127.0f * std::log1p(50.0f / 700.0f);
    const float mel_max = 1127.0f * std::log1p(1100.0f / 700.0f);
    const float mel_scale = 254.0f / (mel_max - mel_min);
    const bool vec = width % 4 == 0 && aligned16(hubert) && aligned16(feats) && (raw == nullptr || aligned16(raw));
    if (vec)
        frontend_kernel<true><<<target, row_threads(width / 4), 0, stream>>>(
            hubert, raw, f0, ratio, protect, hubert_frames, width, mel_min, mel_scale, feats, pitchf, pitch);
    else
        frontend_kernel<false><<<target, row_threads(width), 0, stream>>>(
            hubert, raw, f0, ratio, protect, hubert_frames, width, mel_min, mel_scale, feats, pitchf, pitch);
}

}  // namespace vfr

// ------------------------------------------------------- engine frontend
// The generic engine's frontend (crates/vocal-engine/src/pipeline.rs): the
// blended features are interpolated 2x linearly (75-96: output frame t reads
// source t / 2, left = floor, right = min(left + 1, frames - 1), weight 0 or
// 0.5, a (1 - w) + b w), the features saved before the blend are
// interpolated the same way and, when protect < 0.5, every frame below
// min(2 frames, pitch frames) becomes f v + before (1 - v) with v = 1 for
// pitch > 0 and protect otherwise (312-333); the coarse pitch of those frames
// is f0_to_coarse (625-633: 1 at or below 0 Hz, Rust's f32 ln, division by
// 700 and by the mel span, rounding half away from zero, 0 for NaN through
// the saturating cast).  Every operation is rounded on its own, as in the
// Rust source.
namespace vfr {
namespace {

__device__ __forceinline__ float lerp_half(float a, float b, float w) {
    return __fadd_rn(__fmul_rn(a, __fsub_rn(1.0f, w)), __fmul_rn(b, w));
}

__device__ __forceinline__ float engine_protect(float f, float before, float v) {
    return __fadd_rn(__fmul_rn(f, v), __fmul_rn(before, __fsub_rn(1.0f, v)));
}

// One CTA per output frame (2 frames of them); four columns per lane when kVec.
template <bool kVec>
__global__ void engine_frontend_kernel(const float *__restrict__ blended, const float *__restrict__ raw,
                                       const float *__restrict__ hz, float protect, int frames, int pitch_frames,
                                       int width, float mel_min, float mel_span, float *__restrict__ out,
                                       int32_t *__restrict__ coarse) {
    const int t = blockIdx.x;
    const int left = t >> 1;
    const int right = left + 1 < frames ? left + 1 : frames - 1;
    const float w = (t & 1) ? 0.5f : 0.0f;
    const bool mixing = raw != nullptr && t < pitch_frames;
    const float v = mixing ? (hz[t] > 0.0f ? 1.0f : protect) : 1.0f;
    const long long lo = static_cast<long long>(left) * width, hi = static_cast<long long>(right) * width;
    float *o = out + static_cast<long long>(t) * width;
    if (kVec) {
        for (int c = threadIdx.x; c < width / 4; c += blockDim.x) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(blended + lo) + c);
            const float4 b = __ldg(reinterpret_cast<const float4 *>(blended + hi) + c);
            float4 f = make_float4(lerp_half(a.x, b.x, w), lerp_half(a.y, b.y, w), lerp_half(a.z, b.z, w),
                                   lerp_half(a.w, b.w, w));
            if (mixing) {
                const float4 ra = __ldg(reinterpret_cast<const float4 *>(raw + lo) + c);
                const float4 rb = __ldg(reinterpret_cast<const float4 *>(raw + hi) + c);
                f = make_float4(engine_protect(f.x, lerp_half(ra.x, rb.x, w), v),
                                engine_protect(f.y, lerp_half(ra.y, rb.y, w), v),
                                engine_protect(f.z, lerp_half(ra.z, rb.z, w), v),
                                engine_protect(f.w, lerp_half(ra.w, rb.w, w), v));
            }
            reinterpret_cast<float4 *>(o)[c] = f;
        }
    } else {
        for (int c = threadIdx.x; c < width; c += blockDim.x) {
            float f = lerp_half(__ldg(blended + lo + c), __ldg(blended + hi + c), w);
            if (mixing) f = engine_protect(f, lerp_half(__ldg(raw + lo + c), __ldg(raw + hi + c), w), v);
            o[c] = f;
        }
    }
    if (threadIdx.x == 0 && coarse != nullptr && t < pitch_frames) {
        const float f0 = hz[t];
        int32_t bin = 1;
        if (!(f0 <= 0.0f)) {
            const float mel = __fmul_rn(1127.0f, logf(__fadd_rn(1.0f, __fdiv_rn(f0, 700.0f))));
            const float x = __fadd_rn(__fdiv_rn(__fmul_rn(__fsub_rn(mel, mel_min), 254.0f), mel_span), 1.0f);
            const float r = roundf(x);  // half away from zero, as Rust's f32::round
            // Rust's clamp keeps NaN and `as i32` maps NaN to 0
            bin = r != r ? 0 : static_cast<int32_t>(fminf(fmaxf(r, 1.0f), 255.0f));
        }
        coarse[t] = bin;
    }
}

}  // namespace

void launch_engine_frontend(const float *blended, const float *raw, const float *hz, float protect, int frames,
                            int hz_frames, int width, float *out, int32_t *coarse, cudaStream_t stream) {
    const int out_frames = 2 * frames;
    const int pitch_frames = hz == nullptr ? 0 : (hz_frames < out_frames ? hz_frames : out_frames);
    // pipeline.rs:313: the pre-blend features take part only when protect < 0.5
    const float *mix = (hz != nullptr && protect < 0.5f) ? raw : nullptr;
    // pipeline.rs:629-630, f32 on the host like the Rust constants
    const float mel_min = 1127.0f * std::log(1.0f + 50.0f / 700.0f);
    const float mel_max = 1127.0f * std::log(1.0f + 1100.0f / 700.0f);
    const float mel_span = mel_max - mel_min;
    const bool vec = width % 4 == 0 && aligned16(blended) && aligned16(out) && (mix == nullptr || aligned16(mix));
    if (vec)
        engine_frontend_kernel<true><<<out_frames, row_threads(width / 4), 0, stream>>>(
            blended, mix, hz, protect, frames, pitch_frames, width, mel_min, mel_span, out, coarse);
    else
        engine_frontend_kernel<false><<<out_frames, row_threads(width), 0, stream>>>(
            blended, mix, hz, protect, frames, pitch_frames, width, mel_min, mel_span, out, coarse);
}

}  // namespace vfr
