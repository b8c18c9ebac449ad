// Event-pair kernel timing for benchmarks (vfr_retrieval_profile).
#include "vfr_common.h"

namespace vfr {

cudaEvent_t Profiler::next(cudaStream_t s) {
    if (used == pool.size()) {
        cudaEvent_t e;
        cuda_check(cudaEventCreate(&e));
        pool.push_back(e);
    }
    cudaEvent_t e = pool[used++];
    cuda_check(cudaEventRecord(e, s));
    return e;
}

void Profiler::begin(int kernel, cudaStream_t s) {
    if (!enabled) return;
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &st) != cudaSuccess || st != cudaStreamCaptureStatusNone) return;
    marks.emplace_back(kernel, used);
    next(s);
}

void Profiler::end(cudaStream_t s) {
    if (!enabled || marks.empty() || marks.back().second + 1 != used) return;
    next(s);
}

Profiler::~Profiler() {
    for (cudaEvent_t e : pool) cudaEventDestroy(e);
}

}  // namespace vfr
