// Device half of the index ingest: the reference's parse rejects non-finite
// rows (crates/vocal-model/src/retrieval.rs:226-240, Reader::floats); when
// the rows go straight from the image to HBM the check runs here, over the
// uploaded rows, at HBM speed, and reports the first offending element so
// the host can rank it against the other payload faults by file position.
#include <cstdint>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace vfr {
namespace {

__device__ __forceinline__ bool nonfinite(float v) {
    return (__float_as_uint(v) & 0x7f800000u) == 0x7f800000u;
}

__global__ void first_nonfinite_kernel(const float *__restrict__ x, unsigned long long count,
                                       unsigned long long *__restrict__ first) {
    unsigned long long found = ~0ull;
    const unsigned long long quads = count / 4;
    const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    const unsigned long long tid = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    for (unsigned long long i = tid; i < quads; i += stride) {
        const float4 v = __ldg(x4 + i);
        if (nonfinite(v.x) || nonfinite(v.y) || nonfinite(v.z) || nonfinite(v.w)) {
            const unsigned long long e =
                4 * i + (nonfinite(v.x) ? 0 : nonfinite(v.y) ? 1 : nonfinite(v.z) ? 2 : 3);
            found = e < found ? e : found;
        }
    }
    for (unsigned long long e = quads * 4 + tid; e < count; e += stride)
        if (nonfinite(__ldg(x + e))) found = e < found ? e : found;
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_down_sync(0xffffffffu, found, o);
        found = other < found ? other : found;
    }
    if ((threadIdx.x & 31) == 0 && found != ~0ull) atomicMin(first, found);
}

}  // namespace

unsigned long long first_nonfinite(const float *x, unsigned long long count, int sm_count) {
    unsigned long long *d_first = nullptr;
    unsigned long long first = ~0ull;
    cudaError_t rc = cudaMalloc(reinterpret_cast<void **>(&d_first), sizeof(first));
    if (rc == cudaSuccess) rc = cudaMemcpy(d_first, &first, sizeof(first), cudaMemcpyHostToDevice);
    if (rc == cudaSuccess && count > 0) {
        const unsigned long long blocks = (count / 4 + 255) / 256 + 1;
        const int grid = static_cast<int>(blocks < sm_count * 8ull ? blocks : sm_count * 8ull);
        first_nonfinite_kernel<<<grid, 256>>>(x, count, d_first);
        rc = cudaGetLastError();
    }
    if (rc == cudaSuccess) rc = cudaMemcpy(&first, d_first, sizeof(first), cudaMemcpyDeviceToHost);
    if (d_first) cudaFree(d_first);
    if (rc != cudaSuccess) throw std::runtime_error(std::string("row check: ") + cudaGetErrorString(rc));
    return first;
}

}  // namespace vfr
