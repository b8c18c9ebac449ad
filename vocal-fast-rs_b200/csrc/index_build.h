// Index construction shared by the C ABI, the ingest and the IVF trainer:
// option checks, handles, the derived layout and an internal search.
#pragma once

#include "vfr_common.h"

namespace vfr {

// Makes the index's device current for the duration of a call.
class DeviceGuard {
public:
    explicit DeviceGuard(int device) {
        cuda_check(cudaGetDevice(&previous_));
        if (previous_ != device) cuda_check(cudaSetDevice(device));
        device_ = device;
    }
    ~DeviceGuard() {
        if (previous_ != device_) cudaSetDevice(previous_);
    }
    DeviceGuard(const DeviceGuard &) = delete;
    DeviceGuard &operator=(const DeviceGuard &) = delete;

private:
    int previous_ = 0;
    int device_ = 0;
};

void free_index(VfrIndex *ix) noexcept;
// retrieval.cu:42-59 checks, with the same messages.
void validate_arrays(int32_t d, int32_t nlist, int32_t nprobe, size_t n, const float *centroids,
                     size_t centroid_count, const int32_t *offsets, size_t offset_count, const float *vectors,
                     size_t vector_value_count, const int32_t *ids, size_t id_count);
VfrOptions resolve_options(const VfrOptions *opt);
// inverse[ids[r]] = r when ids is a permutation of 0..n-1 (returns false otherwise)
bool inverse_ids(const int32_t *ids, size_t n, std::vector<int32_t> &inverse);
// A handle with its scalar fields set and no device arrays yet.
VfrIndex *new_handle(int32_t d, int32_t nlist, int32_t nprobe, size_t n, const int32_t *offsets,
                     const VfrOptions &o);
// Counters, the tensor-core layout and the workspace reservation.
void finish_index(VfrIndex *ix, const VfrOptions &o);
// The k (1..8) nearest rows of each query, as vfr_retrieval_search.
void search_rows(VfrIndex *ix, const float *queries, size_t frames, int k, float *dist, int64_t *labels,
                 cudaStream_t stream);


// IVF trainer (training.cpp).  kmeans: centroids [k][d] (device) from x
// [n][d] (device); objective [niter] (host, may be null).  ivf_assign: exact
// nearest centroid of each row, ties to the lower one.  ivf_build: a device
// index with every row in the list of its nearest centroid.  ivf_write: FAISS
// IndexIVFFlat bytes from host arrays; returns the size (writes only when
// capacity suffices).
void kmeans(const float *x, int64_t n, int32_t d, int32_t k, int32_t niter, int32_t max_points_per_centroid,
            uint64_t seed, float *centroids, double *objective, cudaStream_t stream);
void ivf_assign(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, int32_t *lists, float *dist,
                cudaStream_t stream);
VfrIndex *ivf_build(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, int32_t nprobe,
                    const VfrOptions *opt);
size_t ivf_write(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, const int32_t *lists,
                 int32_t nprobe, uint8_t *out, size_t capacity);

}  // namespace vfr
