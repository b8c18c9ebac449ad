// Device primitives shared by the exact (SIMT) and tensor-core paths.
//
// Exactness contract: distances, neighbour order and blended features equal
// the reference CPU retrieval (crates/vocal-cpu/src/retrieval.rs:5-83)
// bit-for-bit.  Every floating-point operation below therefore uses an
// explicit round-to-nearest intrinsic so nvcc cannot contract mul+add into
// FMA, and every reduction follows the reference's order:
//   * avx2_l2 (retrieval.rs:10-26): eight lane accumulators, lane j summing
//     (a_i - b_i)^2 for i = j (mod 8), i < 8*floor(d/8), in increasing i,
//     starting at +0.0; the lanes folded 0..7 starting at -0.0 (Rust's float
//     Sum); plus the tail folded the same way (scalar_l2, :5-7);
//   * weights (:69-73): w = 1 / (max(d, 1e-12f) as f64)^2, S = sum of the 8
//     slots (unfilled slots are 0) from -0.0;
//   * blend (:74-81): r_j = sum_k ((x_kj as f64) * w_k / S) from -0.0, to f32,
//     q_j = q_j * (1 - r) + r_j * r in f32.
#pragma once

#include <cstdint>

namespace vfr {

constexpr unsigned kFullMask = 0xffffffffu;
constexpr unsigned long long kEmptyKey = ~0ull;

// f32 -> u32 whose unsigned order is f32::total_cmp order.
__device__ __forceinline__ uint32_t total_order_bits(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_total_order_bits(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}
// Neighbour key: distance in total order, then scan position (probe rank
// major, storage row minor) -- the order in which the reference's insertion
// top-8 keeps the earlier-scanned row on a distance tie.
__device__ __forceinline__ unsigned long long make_key(float dist, uint32_t scan_pos) {
    return (static_cast<unsigned long long>(total_order_bits(dist)) << 32) | scan_pos;
}
__device__ __forceinline__ float key_dist(unsigned long long key) {
    return from_total_order_bits(static_cast<uint32_t>(key >> 32));
}
__device__ __forceinline__ uint32_t key_pos(unsigned long long key) { return static_cast<uint32_t>(key); }

// Sorted ascending top-8 of keys held in registers by each thread.
struct Top8 {
    unsigned long long k[8];
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int i = 0; i < 8; ++i) k[i] = kEmptyKey;
    }
    __device__ __forceinline__ void insert(unsigned long long key) {
        if (key >= k[7]) return;
        k[7] = key;
#pragma unroll
        for (int i = 7; i > 0; --i) {
            if (k[i] < k[i - 1]) {
                unsigned long long t = k[i];
                k[i] = k[i - 1];
                k[i - 1] = t;
            }
        }
    }
};

// Squared L2 distance between q (shared memory) and x (global), computed by
// the 8 threads of an "octet" (lanes 8o..8o+7 of a warp), in the AVX2 order.
// All 8 threads return the same value.  `mask` covers the calling lanes.
__device__ __forceinline__ float octet_l2(const float *__restrict__ q, const float *__restrict__ x, int d, int j,
                                          int octet_base, unsigned mask) {
    const int d8 = d & ~7;
    float acc = 0.0f;  // _mm256_setzero_ps
    // unrolled so several independent row loads are in flight; the
    // accumulation order per lane is unchanged
#pragma unroll 16
    for (int i = j; i < d8; i += 8) {
        float t = __fsub_rn(q[i], __ldg(x + i));
        acc = __fadd_rn(acc, __fmul_rn(t, t));
    }
    float s = -0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) s = __fadd_rn(s, __shfl_sync(mask, acc, octet_base + l));
    float tail = -0.0f;
    for (int i = d8; i < d; ++i) {
        float t = __fsub_rn(q[i], __ldg(x + i));
        tail = __fadd_rn(tail, __fmul_rn(t, t));
    }
    return __fadd_rn(s, tail);
}

// octet_l2 for N rows at once: N independent accumulation chains per lane
// (each in the reference order), so N times as many row loads are in flight.
// out[k] is the distance to x[k]; all 8 threads get the same values.  Rows
// in global memory go through the read-only cache (kGlobal); kGlobal = false
// reads rows staged in shared memory.
template <int N, bool kGlobal = true>
__device__ __forceinline__ void octet_l2n(const float *__restrict__ q, const float *const (&x)[N], int d, int j,
                                          int octet_base, unsigned mask, float (&out)[N]) {
    const int d8 = d & ~7;
    float acc[N];
#pragma unroll
    for (int k = 0; k < N; ++k) acc[k] = 0.0f;
    // Each unrolled body issues all its row loads before the dependent adds,
    // so the number of serialised memory round trips is d/8 / unroll: deep
    // for the few-row re-ranks (random rows, latency bound), shallower for
    // the 4-row scans (register bound) and for rows in shared memory.
    constexpr int kUnroll = !kGlobal ? 8 : N <= 2 ? 16 : 4;
#pragma unroll kUnroll
    for (int i = j; i < d8; i += 8) {
        const float qi = q[i];
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const float t = __fsub_rn(qi, kGlobal ? __ldg(x[k] + i) : x[k][i]);
            acc[k] = __fadd_rn(acc[k], __fmul_rn(t, t));
        }
    }
#pragma unroll
    for (int k = 0; k < N; ++k) {
        float s = -0.0f;
#pragma unroll
        for (int l = 0; l < 8; ++l) s = __fadd_rn(s, __shfl_sync(mask, acc[k], octet_base + l));
        float tail = -0.0f;
        for (int i = d8; i < d; ++i) {
            const float t = __fsub_rn(q[i], kGlobal ? __ldg(x[k] + i) : x[k][i]);
            tail = __fadd_rn(tail, __fmul_rn(t, t));
        }
        out[k] = __fadd_rn(s, tail);
    }
}

// The reference's f64 weight of one neighbour at squared distance `dist`.
__device__ __forceinline__ double reference_weight(float dist) {
    const float s = fmaxf(dist, 1e-12f);  // f32::max: NaN yields the other operand
    const double sd = static_cast<double>(s);
    return __ddiv_rn(1.0, __dmul_rn(sd, sd));
}

// The reference's f64 weights for `count` neighbours; returns S.
__device__ __forceinline__ double reference_weights(const float *dist, int count, double *w) {
    double sum = -0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const double wk = k < count ? reference_weight(dist[k]) : 0.0;
        w[k] = wk;
        sum = __dadd_rn(sum, wk);
    }
    return sum;
}

// Division by one frame's weight sum S, correctly rounded like the
// reference's f64 `/`, for the frame's 8 x d quotients t / S.  With
// y = RN(1/S) computed once, Markstein's FMA refinement (P. W. Markstein,
// IBM J. Res. Develop. 34(1), 1990, the correction step of IA-64 division):
// q0 = RN(t y); q1 = RN(q0 + RN(t - S q0) y) is within one ulp of t/S; then
// r = t - S q1 is exact and RN(q1 + r y) = RN(t/S), y being within half an
// ulp of 1/S.  The argument needs no overflow or underflow on the way, which
// S in [2^-500, 2^500] and |t| in [2^-400, 2^400] guarantee; t == +-0 gives
// t * y (exact, sign kept), other operands the divide instruction sequence.
// tests/division_check.c checks the same operations against t / S.
struct WeightDivisor {
    double s, y;
    bool fast;
};
__device__ __forceinline__ WeightDivisor weight_divisor(double s) {
    WeightDivisor d;
    d.s = s;
    d.fast = s >= 0x1p-500 && s <= 0x1p500;
    d.y = d.fast ? __drcp_rn(s) : 0.0;
    return d;
}
// Markstein's quotient, valid for the operands `markstein_ok` admits.
__device__ __forceinline__ double markstein_quotient(double t, const WeightDivisor &d) {
    const double q0 = __dmul_rn(t, d.y);
    const double r0 = __fma_rn(-d.s, q0, t);
    const double q1 = __fma_rn(r0, d.y, q0);
    const double r1 = __fma_rn(-d.s, q1, t);
    const double q = __fma_rn(r1, d.y, q1);
    return t == 0.0 ? q0 : q;
}
__device__ __forceinline__ bool markstein_ok(double t, const WeightDivisor &d) {
    const double at = fabs(t);
    return d.fast && (at == 0.0 || (at >= 0x1p-400 && at <= 0x1p400));
}

// t / S through the divide instruction sequence, out of line: the operands
// Markstein's quotient does not admit are rare, and keeping the sequence out
// of the unrolled blend keeps latency-bound kernels' code small.
static __device__ __noinline__ double slow_quotient(double t, double s) { return __ddiv_rn(t, s); }

// One output element of the blend: retrieved from the gathered neighbour
// values v[k] (k < count), then q*(1-r) + retrieved*r; the quotients are
// summed in the reference's order.  kSideBySide computes the 8 quotients as
// independent chains (latency-bound callers with registers to spare; a
// quotient outside Markstein's domain sends the element through the divide
// instruction sequence); otherwise one quotient at a time.
template <bool kSideBySide = false>
__device__ __forceinline__ float reference_blend_element(float q, const float *v, const double *w,
                                                         const WeightDivisor &sum, int count, float ratio) {
    double acc = -0.0;
    if constexpr (kSideBySide) {
        double t[8], quo[8];
        bool ok = true;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            t[k] = __dmul_rn(static_cast<double>(v[k]), w[k]);
            quo[k] = markstein_quotient(t[k], sum);
            ok = ok && (k >= count || markstein_ok(t[k], sum));
        }
        if (!ok) {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (k < count) quo[k] = slow_quotient(t[k], sum.s);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (k < count) acc = __dadd_rn(acc, quo[k]);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (k < count) {
                const double t = __dmul_rn(static_cast<double>(v[k]), w[k]);
                acc = __dadd_rn(acc, markstein_ok(t, sum) ? markstein_quotient(t, sum) : __ddiv_rn(t, sum.s));
            }
        }
    }
    float retrieved = __double2float_rn(acc);
    return __fadd_rn(__fmul_rn(q, __fsub_rn(1.0f, ratio)), __fmul_rn(retrieved, ratio));
}

// index_rate as the reference CUDA kernels read it (retrieval_block.cuh:30-31):
// clamped to [0, 1]; NaN reads as 0.
__device__ __forceinline__ float load_ratio(const float *index_rate) {
    return fminf(fmaxf(*index_rate, 0.0f), 1.0f);
}

}  // namespace vfr
