// Shared host-side definitions of libvfr_retrieval: error convention, the
// device index object and its layout in HBM.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/vfr_retrieval.h"
#include "kernels.h"

namespace vfr {

// Error convention of the reference bridge (crates/vocal-tensorrt/native/
// bridge.h:24-32): exceptions become rc 1 + malloc'd message, anything else 2.
char *make_error(const char *message) noexcept;

inline void require(bool ok, const std::string &message) {
    if (!ok) throw std::runtime_error(message);
}
inline void cuda_check(cudaError_t rc, const char *what = nullptr) {
    if (rc != cudaSuccess) {
        std::string m = cudaGetErrorString(rc);
        if (what) m = std::string(what) + ": " + m;
        throw std::runtime_error(m);
    }
}
template <class F>
int guarded(char **error, F &&f) noexcept {
    try {
        f();
        return 0;
    } catch (const std::exception &e) {
        if (error) *error = make_error(e.what());
        return 1;
    } catch (...) {
        return 2;
    }
}

// Host parsed index (normalised RetrievalIndex arrays).
struct HostIndex {
    int32_t d = 0;
    int32_t nlist = 0;
    int32_t nprobe = 0;
    int64_t n = 0;
    std::vector<float> centroids;
    std::vector<int32_t> offsets;
    std::vector<float> vectors;
    std::vector<int32_t> ids;
};

HostIndex parse_faiss(const uint8_t *bytes, size_t length);
bool find_vfrm_faiss(const uint8_t *image, size_t length, size_t *offset, size_t *size);

// Workspace of the tensor-core path, sized for `frames` frames.
struct Workspace {
    size_t frames = 0;
    void *base = nullptr;
    size_t bytes = 0;
};

}  // namespace vfr

// Device-resident index.  Field order is private to this library.
struct VfrIndex {
    int device = 0;
    int32_t d = 0;
    int32_t nlist = 0;
    int32_t nprobe = 0;
    int64_t n = 0;
    int64_t label_base = 0;
    int32_t engine = VFR_ENGINE_AUTO;
    int32_t candidates = 64;
    // The reference's four arrays (retrieval.cu:9-18), fp32 / i32.
    float *centroids = nullptr;  // [nlist][d]
    int32_t *offsets = nullptr;  // [nlist+1]
    float *vectors = nullptr;    // [n][d] inverted-list order
    int32_t *ids = nullptr;      // [n] FAISS labels
    int32_t *row_of_id = nullptr;  // [n] inverse permutation of ids
    vfr::DeviceCounters *counters = nullptr;
    std::vector<int32_t> host_offsets;  // list bounds, for host-side dispatch
    // Tensor-core layout (built when the engine uses tensor cores).
    __nv_bfloat16 *vectors_bf16 = nullptr;    // [n_pad][d_pad] K-major, zero padded
    __nv_bfloat16 *centroids_bf16 = nullptr;  // [nlist_pad][d_pad]
    float *row_norms = nullptr;               // [n_pad] ||x||^2 (fp32 of the fp32 row), +inf on padding
    float *centroid_norms = nullptr;          // [nlist_pad]
    int32_t d_pad = 0;                        // d rounded up to 64
    int64_t n_pad = 0;                        // n rounded up to 256
    int32_t nlist_pad = 0;
    float max_row_norm = 0.f;       // max ||x||
    float max_row_residual = 0.f;   // max ||x - bf16(x)||
    float max_centroid_norm = 0.f;
    float max_centroid_residual = 0.f;
    alignas(64) CUtensorMap tmap_vectors;    // bf16 rows, box [256][64]
    alignas(64) CUtensorMap tmap_centroids;  // bf16 centroids, box [256][64]
    bool have_tc = false;
    vfr::Workspace ws;
};

struct VfrHostIndex {
    vfr::HostIndex h;
};
