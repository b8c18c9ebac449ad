// Shared host-side definitions of libvfr_retrieval: error convention, the
// device index object and its layout in HBM.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "vfr_retrieval.h"  // include/, on the compiler search path
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

// Where a FAISS image keeps each part of the index (byte positions in the
// image); centroids are copied (and checked) during the walk.
struct FaissLayout {
    static constexpr size_t kImplicitIds = ~size_t(0);  // IxF2: ids are 0..n-1
    static constexpr size_t kNoFault = ~size_t(0);
    struct List {
        size_t vec_pos;  // size * d little-endian f32
        size_t id_pos;   // size little-endian u64 ids (kImplicitIds for IxF2)
        uint64_t size;
    };
    int32_t d = 0;
    int32_t nlist = 0;
    int32_t nprobe = 0;
    int64_t n = 0;
    std::vector<float> centroids;
    std::vector<int32_t> offsets;
    std::vector<List> lists;  // file order = row order
    bool trailing = false;    // IxF2 bytes after the rows
    // byte position in the image of row element `element` (row-major, list order)
    size_t row_position(uint64_t element) const;
};

FaissLayout faiss_layout(const uint8_t *bytes, size_t length);
// ids in row order; returns the position of the first duplicate or
// out-of-range id (kNoFault when they form a permutation of 0..n-1).
size_t scan_ids(const FaissLayout &layout, const uint8_t *bytes, std::vector<int32_t> &ids);
// Throws the payload error that comes first in the file, then the IxF2
// trailing-data error; returns when there is none.
void raise_first_fault(const FaissLayout &layout, size_t nonfinite_pos, size_t bad_id_pos);
HostIndex parse_faiss(const uint8_t *bytes, size_t length);
bool find_vfrm_faiss(const uint8_t *image, size_t length, size_t *offset, size_t *size);

// Workspace of the tensor-core path, sized for `frames` frames.
// Event-pair timing of library kernels (bench instrumentation).
struct Profiler {
    bool enabled = false;
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
    std::vector<std::pair<int, size_t>> marks;  // (kernel id, start event index)
    cudaEvent_t next(cudaStream_t s);
    void begin(int kernel, cudaStream_t s);
    void end(cudaStream_t s);
    ~Profiler();
};
enum { kProfPrep = 0, kProfCand = 1, kProfMerge = 2, kProfExact = 3, kProfCount = 4 };

struct Workspace {
    size_t frames = 0;
    void *base = nullptr;
    size_t bytes = 0;
};

}  // namespace vfr

namespace vfr {
struct SharedRows;
}

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
    // Tensor-core layout (built when the engine uses tensor cores): an fp16
    // shadow of the rows scaled by a power of two, K-major with rows padded
    // to 256 and width to 64, and per-row fp32 squared norms.
    __half *vectors_h = nullptr;   // [n_pad][d_pad], zero padded
    float *row_norms = nullptr;    // [n_pad] ||x||^2, +inf on padding rows
    int32_t d_pad = 0;
    int64_t n_pad = 0;
    float tc_scale = 1.f;          // power of two applied before fp16 rounding
    // Bounds used by the exactness certificate (host copies, rounded up).
    float max_row_norm = 0.f;      // max ||x||
    float max_row_hat = 0.f;       // max ||fp16(s x) / s||
    float max_row_residual = 0.f;  // max ||x - fp16(s x) / s||
    int sm_count = 148;
    int merge_smem_max = 96 * 1024;  // dynamic shared memory merge_kernel may use (set by build_tc)
    // Small launches (at most two frames per SM) use merge_small_kernel;
    // VFR_SMALL_MERGE=0 in the environment at index creation selects
    // merge_kernel for them instead (comparison runs).
    bool small_merge = true;
    // IVF: the same layout for the coarse centroids (nlist_pad rows).
    __half *centroids_h = nullptr;
    float *centroid_norms = nullptr;
    int32_t nlist_pad = 0;
    float max_cent_norm = 0.f, max_cent_hat = 0.f, max_cent_residual = 0.f;
    int32_t *list_order = nullptr;  // [nlist] list ids by descending size (IVF fine-stage order)
    alignas(64) CUtensorMap tmap_centroids;
    alignas(64) CUtensorMap tmap_vectors;  // fp16 rows, box [256 rows][64]
    alignas(64) CUtensorMap tmap_vectors_half;  // fp16 rows, box [128 rows][64] (CTA-pair tiles)
    int pair_clusters = 0;  // CTA pairs that fit at once (0: no pair layout)
    bool have_tc = false;
    vfr::Workspace ws;
    vfr::Profiler prof;
    // Set when the device arrays above (rows, ids, lists, shadow, norms) are
    // shared with other handles loaded from the same content; they are then
    // freed with the last handle, not by this one.
    std::shared_ptr<vfr::SharedRows> shared;
    // Re-run scratch of the exact kernel, per handle: lets a few uncertified
    // frames share its grid (ExactArgs::split_keys / split_done).
    unsigned long long *split_keys = nullptr;
    int32_t *split_done = nullptr;
    vfr::RerunHint *rerun_hints = nullptr;  // [kSplitFrames], frame = -1 between calls
    // 2-D exact engine (exact2d.cu) for small IVF batches: the most rows a
    // frame's probed lists can hold, and its scratch.
    int64_t max_probed_rows = 0;
    // Engine that served the last call (diagnostics): 0 none yet, 1 exact
    // (one CTA per frame), 2 tensor cores, 3 the 2-D exact engine.
    int32_t last_engine = 0;
    void *x2_ws = nullptr;
    size_t x2_bytes = 0;
    // Plan of the last tensor-core call on the host (diagnostics): candidate
    // list size per (work item, frame), database segments, tiles per
    // segment, and the A-tile layout (0 full, 1 spread, -1 no call yet).
    int32_t last_keep = 0, last_segments = 0, last_tiles_per_seg = 0, last_layout = -1;
};

namespace vfr {
// Device arrays and derived layout of an index loaded with
// VFR_SHARE_STORAGE; `proto` holds no workspace, counters or events.
struct SharedRows {
    VfrIndex proto;
    ~SharedRows();
};
}  // namespace vfr

struct VfrHostIndex {
    vfr::HostIndex h;
};
