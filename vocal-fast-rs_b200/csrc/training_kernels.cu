// Device kernels of the IVF trainer: row gathers, the fixed-point centroid
// sums and the means.
//
// Centroid sums are taken in 64-bit fixed point (each coordinate rounded to
// a multiple of 2^-s chosen so no sum can overflow), so the atomic additions
// commute and the means do not depend on the order in which rows arrive:
// the CPU restatement reproduces them bit for bit.
#include <cstdint>

#include "kernels.h"

namespace vfr {
namespace {

// One CTA per output row: out[r] = x[rows[r]].
__global__ void gather_rows_kernel(const float *__restrict__ x, const int64_t *__restrict__ rows, int d,
                                   float *__restrict__ out) {
    const long long r = blockIdx.x;
    const float *src = x + rows[r] * static_cast<long long>(d);
    float *dst = out + r * static_cast<long long>(d);
    for (int c = threadIdx.x; c < d; c += blockDim.x) dst[c] = __ldg(src + c);
}

// One CTA per training row: sums[label][c] += rint(x[c] * scale).
__global__ void fixed_sum_kernel(const float *__restrict__ x, const int64_t *__restrict__ labels, int d,
                                 double scale, unsigned long long *__restrict__ sums) {
    const long long r = blockIdx.x;
    const long long label = labels[r];
    const float *src = x + r * static_cast<long long>(d);
    unsigned long long *dst = sums + label * d;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const long long q = __double2ll_rn(__dmul_rn(static_cast<double>(__ldg(src + c)), scale));
        atomicAdd(dst + c, static_cast<unsigned long long>(q));
    }
}

// centroid[j][c] = sum / count * 2^-s for a non-empty cluster, 0 otherwise.
__global__ void means_kernel(const unsigned long long *__restrict__ sums, const long long *__restrict__ counts,
                             int k, int d, double inv_scale, float *__restrict__ centroids) {
    const long long total = static_cast<long long>(k) * d;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long count = counts[i / d];
        float v = 0.0f;
        if (count > 0) {
            const double sum = __ll2double_rn(static_cast<long long>(sums[i]));
            v = __double2float_rn(__dmul_rn(__ddiv_rn(sum, __ll2double_rn(count)), inv_scale));
        }
        centroids[i] = v;
    }
}

__global__ void narrow_labels_kernel(const int64_t *__restrict__ wide, long long n, int32_t *__restrict__ out) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = static_cast<int32_t>(wide[i]);
}

}  // namespace

void launch_gather_rows(const float *x, const int64_t *rows, long long count, int d, float *out,
                        cudaStream_t stream) {
    if (count <= 0) return;
    gather_rows_kernel<<<static_cast<unsigned>(count), 128, 0, stream>>>(x, rows, d, out);
}

void launch_fixed_sums(const float *x, const int64_t *labels, long long rows, int d, double scale,
                       unsigned long long *sums, cudaStream_t stream) {
    if (rows <= 0) return;
    fixed_sum_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(x, labels, d, scale, sums);
}

void launch_means(const unsigned long long *sums, const long long *counts, int k, int d, double inv_scale,
                  float *centroids, cudaStream_t stream) {
    const long long total = static_cast<long long>(k) * d;
    const long long blocks = (total + 255) / 256;
    means_kernel<<<static_cast<unsigned>(blocks < 4096 ? blocks : 4096), 256, 0, stream>>>(sums, counts, k, d,
                                                                                           inv_scale, centroids);
}

void launch_narrow_labels(const int64_t *wide, long long n, int32_t *out, cudaStream_t stream) {
    if (n <= 0) return;
    const long long blocks = (n + 255) / 256;
    narrow_labels_kernel<<<static_cast<unsigned>(blocks < 4096 ? blocks : 4096), 256, 0, stream>>>(wide, n, out);
}

}  // namespace vfr
