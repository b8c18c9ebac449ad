#include "tc_path.h"

namespace vfr {
void build_tc(VfrIndex *) {}
void release_tc(VfrIndex *) noexcept {}
void reserve_tc(VfrIndex *, size_t) {}
bool use_tc(const VfrIndex *, size_t) { return false; }
void run_tc(VfrIndex *, const float *, float *, const float *, int, int, float *, int64_t *, size_t, cudaStream_t) {
    throw std::runtime_error("tensor-core engine not built");
}
}  // namespace vfr
