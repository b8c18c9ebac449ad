// Self-test of the bounded wait that every mbarrier wait in the library's
// kernels uses (tc::mbar_wait): a single thread waits on a barrier whose
// phase completes only when `arrive` is set, with the caller's time limit.
// With arrive = 0 nothing ever completes the phase, the wait gives up after
// the limit, and the kernel reports that instead of spinning on: the way a
// kernel of this library unwinds when a copy it waits for never lands.
#include <cstdint>

#include "tc_ptx.cuh"
#include "vfr_common.h"

namespace vfr {
namespace {

__global__ void bounded_wait_kernel(uint64_t limit_ns, int arrive, int32_t *timed_out, uint64_t *elapsed_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    tc::mbar_init(&bar, 1);
    tc::fence_mbarrier_init();
    if (arrive) tc::mbar_arrive(&bar);
    const uint64_t t0 = tc::global_timer_ns();
    const bool ok = tc::mbar_wait(&bar, 0, limit_ns);
    *elapsed_ns = tc::global_timer_ns() - t0;
    *timed_out = ok ? 0 : 1;
}

}  // namespace
}  // namespace vfr

extern "C" int vfr_selftest_bounded_wait(uint64_t limit_ns, int32_t arrive, int32_t *timed_out, uint64_t *elapsed_ns,
                                         char **error) {
    return vfr::guarded(error, [&] {
        vfr::require(timed_out && elapsed_ns, "invalid self-test arguments");
        vfr::require(limit_ns > 0 && limit_ns <= 2000000000ull, "wait limit must be in (0, 2 s]");
        int32_t *d_flag = nullptr;
        uint64_t *d_ns = nullptr;
        vfr::cuda_check(cudaMalloc(reinterpret_cast<void **>(&d_flag), sizeof(int32_t)));
        cudaError_t rc = cudaMalloc(reinterpret_cast<void **>(&d_ns), sizeof(uint64_t));
        if (rc == cudaSuccess) {
            vfr::bounded_wait_kernel<<<1, 32>>>(limit_ns, arrive, d_flag, d_ns);
            rc = cudaGetLastError();
        }
        if (rc == cudaSuccess) rc = cudaMemcpy(timed_out, d_flag, sizeof(int32_t), cudaMemcpyDeviceToHost);
        if (rc == cudaSuccess) rc = cudaMemcpy(elapsed_ns, d_ns, sizeof(uint64_t), cudaMemcpyDeviceToHost);
        cudaFree(d_flag);
        if (d_ns) cudaFree(d_ns);
        vfr::cuda_check(rc, "bounded-wait self-test");
    });
}
