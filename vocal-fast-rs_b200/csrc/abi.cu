// C ABI of libvfr_retrieval.so (declared in include/vfr_retrieval.h).
//
// Index ownership, validation and dispatch.  The validation and the drop-in
// entry points follow crates/vocal-tensorrt/native/retrieval.cu:34-128 (same
// limits and messages); the error convention follows
// crates/vocal-tensorrt/native/bridge.h:24-32.
#include <algorithm>
#include <cmath>
#include <functional>
#include <cstdio>
#include <map>
#include <memory>
#include <mutex>
#include <string>

#include "exact2d.h"
#include "index_build.h"
#include "ingest.h"
#include "kernels.h"
#include "tc_path.h"
#include "vfr_common.h"

namespace vfr {

char *make_error(const char *message) noexcept {
    if (!message) message = "native retrieval error";
    size_t bytes = std::strlen(message) + 1;
    auto *result = static_cast<char *>(std::malloc(bytes));
    if (result) std::memcpy(result, message, bytes);
    return result;
}

SharedRows::~SharedRows() {
    int previous = 0;
    cudaGetDevice(&previous);
    cudaSetDevice(proto.device);
    for (void *p : {static_cast<void *>(proto.centroids), static_cast<void *>(proto.offsets),
                    static_cast<void *>(proto.vectors), static_cast<void *>(proto.ids),
                    static_cast<void *>(proto.row_of_id), static_cast<void *>(proto.vectors_h),
                    static_cast<void *>(proto.row_norms), static_cast<void *>(proto.centroids_h),
                    static_cast<void *>(proto.centroid_norms), static_cast<void *>(proto.list_order)})
        if (p) cudaFree(p);
    cudaSetDevice(previous);
}

void free_index(VfrIndex *ix) noexcept {
    if (!ix) return;
    int previous = 0;
    cudaGetDevice(&previous);
    cudaSetDevice(ix->device);
    release_tc(ix);
    if (!ix->shared)
        for (void *p : {static_cast<void *>(ix->centroids), static_cast<void *>(ix->offsets),
                        static_cast<void *>(ix->vectors), static_cast<void *>(ix->ids),
                        static_cast<void *>(ix->row_of_id)})
            if (p) cudaFree(p);
    if (ix->counters) cudaFree(ix->counters);
    if (ix->x2_ws) cudaFree(ix->x2_ws);
    if (ix->split_keys) cudaFree(ix->split_keys);
    if (ix->split_done) cudaFree(ix->split_done);
    if (ix->rerun_hints) cudaFree(ix->rerun_hints);
    ix->shared.reset();
    cudaSetDevice(previous);
    delete ix;
}

template <class T>
void alloc_copy(T **dst, const T *src, size_t count) {
    cuda_check(cudaMalloc(reinterpret_cast<void **>(dst), std::max<size_t>(count, 1) * sizeof(T)), "cudaMalloc");
    if (count) cuda_check(cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice), "cudaMemcpy");
}

// retrieval.cu:42-59 checks, with the same messages.
void validate_arrays(int32_t d, int32_t nlist, int32_t nprobe, size_t n, const float *centroids,
                     size_t centroid_count, const int32_t *offsets, size_t offset_count, const float *vectors,
                     size_t vector_value_count, const int32_t *ids, size_t id_count) {
    require(d > 0 && d <= 4096, "invalid FAISS GPU index dimension");
    require(nlist > 0 && nprobe > 0 && nprobe <= nlist && nprobe <= kMaxProbe, "invalid FAISS GPU IVF configuration");
    require(n > 0 && n <= static_cast<size_t>(INT32_MAX), "invalid FAISS GPU vector count");
    require(centroids && centroid_count == static_cast<size_t>(nlist) * d, "invalid FAISS centroid payload");
    require(offsets && offset_count == static_cast<size_t>(nlist) + 1, "invalid FAISS list offsets");
    require(vectors && vector_value_count == n * static_cast<size_t>(d), "invalid FAISS vector payload");
    require(ids && id_count == n, "invalid FAISS id payload");
    require(offsets[0] == 0 && offsets[nlist] == static_cast<int32_t>(n), "FAISS list offsets do not cover vectors");
    for (int32_t i = 0; i < nlist; ++i) require(offsets[i] <= offsets[i + 1], "FAISS list offsets are not monotonic");
}

VfrOptions resolve_options(const VfrOptions *opt) {
    VfrOptions o{};
    o.struct_size = sizeof(VfrOptions);
    if (opt) {
        require(opt->struct_size >= static_cast<int32_t>(offsetof(VfrOptions, max_frames) + sizeof(int64_t)),
                "VfrOptions.struct_size too small");
        o = *opt;
    }
    require(o.engine >= VFR_ENGINE_AUTO && o.engine <= VFR_ENGINE_TENSOR, "invalid retrieval engine");
    if (o.candidates == 0) o.candidates = 64;
    require(o.candidates >= 16 && o.candidates <= 128 && o.candidates % 16 == 0,
            "candidate width must be a multiple of 16 in 16..128");
    require(o.label_base >= 0 && o.max_frames >= 0, "invalid label base or frame reservation");
    require((o.flags & ~VFR_SHARE_STORAGE) == 0, "unknown retrieval option flags");
    return o;
}

// The inverse map used by vfr_gather_owned, when ids form a permutation of
// 0..n-1 (the reference parser guarantees it; the raw ABI, like
// retrieval.cu, accepts any ids).
bool inverse_ids(const int32_t *ids, size_t n, std::vector<int32_t> &inverse) {
    inverse.assign(n, -1);
    for (size_t r = 0; r < n; ++r) {
        if (ids[r] < 0 || static_cast<size_t>(ids[r]) >= n || inverse[ids[r]] >= 0) return false;
        inverse[ids[r]] = static_cast<int32_t>(r);
    }
    return true;
}

VfrIndex *new_handle(int32_t d, int32_t nlist, int32_t nprobe, size_t n, const int32_t *offsets,
                     const VfrOptions &o) {
    auto *ix = new VfrIndex{};
    ix->d = d;
    ix->nlist = nlist;
    ix->nprobe = nprobe;
    ix->n = static_cast<int64_t>(n);
    ix->label_base = o.label_base;
    ix->engine = o.engine;
    ix->candidates = o.candidates;
    ix->host_offsets.assign(offsets, offsets + nlist + 1);
    try {
        cuda_check(cudaGetDevice(&ix->device));
    } catch (...) {
        delete ix;
        throw;
    }
    return ix;
}

// The most rows one frame's probed lists can hold: the nprobe largest lists.
int64_t max_probed_rows(const std::vector<int32_t> &offsets, int nprobe) {
    std::vector<int64_t> sizes;
    for (size_t l = 0; l + 1 < offsets.size(); ++l) sizes.push_back(offsets[l + 1] - offsets[l]);
    const size_t p = std::min(sizes.size(), static_cast<size_t>(std::max(nprobe, 1)));
    std::partial_sort(sizes.begin(), sizes.begin() + p, sizes.end(), std::greater<int64_t>());
    int64_t total = 0;
    for (size_t i = 0; i < p; ++i) total += sizes[i];
    return total;
}

// Bytes of exact row and centroid reads above which a small IVF batch goes
// to the tensor-core path instead of the 2-D exact engine.
constexpr double kExact2dBytes = 400e6;

size_t exact2d_frame_limit(const VfrIndex *ix) {
    if (ix->nlist <= 1 || ix->engine != VFR_ENGINE_AUTO || ix->d > exact2d_max_width()) return 0;
    const double per_frame = static_cast<double>(ix->nlist + ix->max_probed_rows) * ix->d * 4.0;
    return static_cast<size_t>(std::min(65535.0, std::floor(kExact2dBytes / per_frame)));
}

bool use_exact2d(const VfrIndex *ix, size_t frames) { return frames <= exact2d_frame_limit(ix); }

void reserve_exact2d(VfrIndex *ix, size_t frames) {
    const size_t f = std::min(frames, exact2d_frame_limit(ix));
    if (f == 0) return;
    const size_t bytes = exact2d_layout(f, ix->nlist, ix->nprobe, ix->max_probed_rows).total;
    if (bytes <= ix->x2_bytes) return;
    void *p = nullptr;
    cuda_check(cudaMalloc(&p, bytes), "cudaMalloc exact2d scratch");
    if (ix->x2_ws) {
        cuda_check(cudaDeviceSynchronize());
        cudaFree(ix->x2_ws);
    }
    ix->x2_ws = p;
    ix->x2_bytes = bytes;
}

// Counters, the tensor-core layout and the workspace reservation.
void finish_index(VfrIndex *ix, const VfrOptions &o) {
    cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->counters), sizeof(DeviceCounters)));
    cuda_check(cudaMemset(ix->counters, 0, sizeof(DeviceCounters)));
    ix->max_probed_rows = max_probed_rows(ix->host_offsets, ix->nprobe);
    if (!ix->shared && ix->engine != VFR_ENGINE_EXACT) build_tc(ix);
    if (o.max_frames > 0) {
        reserve_tc(ix, static_cast<size_t>(o.max_frames));
        reserve_exact2d(ix, static_cast<size_t>(o.max_frames));
    }
    cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->split_keys), kSplitKeyBytes), "cudaMalloc re-run scratch");
    cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->split_done), kSplitFrames * sizeof(int32_t)));
    cuda_check(cudaMemset(ix->split_done, 0, kSplitFrames * sizeof(int32_t)));
    cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->rerun_hints), kSplitFrames * sizeof(RerunHint)));
    cuda_check(cudaMemset(ix->rerun_hints, 0xff, kSplitFrames * sizeof(RerunHint)));  // frame = -1
    cuda_check(cudaDeviceSynchronize());
}

VfrIndex *create_index(int32_t d, int32_t nlist, int32_t nprobe, size_t n, const float *centroids,
                       size_t centroid_count, const int32_t *offsets, size_t offset_count, const float *vectors,
                       size_t vector_value_count, const int32_t *ids, size_t id_count, const VfrOptions *opt) {
    validate_arrays(d, nlist, nprobe, n, centroids, centroid_count, offsets, offset_count, vectors,
                    vector_value_count, ids, id_count);
    const VfrOptions o = resolve_options(opt);
    std::vector<int32_t> inverse;
    const bool permutation = inverse_ids(ids, n, inverse);
    VfrIndex *ix = new_handle(d, nlist, nprobe, n, offsets, o);
    try {
        alloc_copy(&ix->centroids, centroids, centroid_count);
        alloc_copy(&ix->offsets, offsets, offset_count);
        alloc_copy(&ix->vectors, vectors, vector_value_count);
        alloc_copy(&ix->ids, ids, id_count);
        if (permutation) alloc_copy(&ix->row_of_id, inverse.data(), n);
        finish_index(ix, o);
    } catch (...) {
        free_index(ix);
        throw;
    }
    return ix;
}

// ---- device ingest of FAISS bytes ---------------------------------------

struct ShareKey {
    ContentHash hash;
    size_t length;
    int device;
    bool tensor;
    bool operator<(const ShareKey &k) const {
        if (!(hash == k.hash)) return hash < k.hash;
        if (length != k.length) return length < k.length;
        if (device != k.device) return device < k.device;
        return tensor < k.tensor;
    }
};

std::mutex share_lock;
std::map<ShareKey, std::weak_ptr<SharedRows>> &share_table() {
    static auto *table = new std::map<ShareKey, std::weak_ptr<SharedRows>>();
    return *table;
}

VfrIndex *handle_from_shared(const std::shared_ptr<SharedRows> &rows, const VfrOptions &o) {
    auto *ix = new VfrIndex(rows->proto);
    ix->shared = rows;
    ix->label_base = o.label_base;
    ix->engine = o.engine;
    ix->candidates = o.candidates;
    try {
        DeviceGuard guard(ix->device);
        finish_index(ix, o);
    } catch (...) {
        free_index(ix);
        throw;
    }
    return ix;
}

// Turns a freshly loaded handle into the first holder of shared rows.
void publish_shared(VfrIndex *ix, const ShareKey &key) {
    auto rows = std::make_shared<SharedRows>();
    rows->proto = *ix;
    rows->proto.counters = nullptr;
    rows->proto.split_keys = nullptr;
    rows->proto.split_done = nullptr;
    rows->proto.rerun_hints = nullptr;
    rows->proto.ws = Workspace{};
    rows->proto.prof.pool.clear();
    rows->proto.prof.marks.clear();
    rows->proto.prof.used = 0;
    ix->shared = rows;
    std::lock_guard<std::mutex> g(share_lock);
    share_table()[key] = rows;
}

// RetrievalIndex::from_faiss + GpuRetrievalIndex::new in one pass
// (crates/vocal-model/src/retrieval.rs:62-193, crates/vocal-tensorrt/src/
// retrieval.rs:27-60): the structure is walked on the host, the rows go from
// the image to HBM through staged_upload without a host copy, the finite
// check runs on the device, and the error raised is the one the reference
// parser raises first.
VfrIndex *load_index(const uint8_t *bytes, size_t length, int32_t feature_dims, const VfrOptions *opt) {
    const VfrOptions o = resolve_options(opt);
    const bool share = (o.flags & VFR_SHARE_STORAGE) != 0;
    ShareKey key{};
    if (share) {
        require(bytes != nullptr || length == 0, "null FAISS byte buffer");
        key.hash = content_hash(bytes, length);
        key.length = length;
        cuda_check(cudaGetDevice(&key.device));
        key.tensor = o.engine != VFR_ENGINE_EXACT;
        std::shared_ptr<SharedRows> rows;
        {
            std::lock_guard<std::mutex> g(share_lock);
            auto it = share_table().find(key);
            if (it != share_table().end() && !(rows = it->second.lock())) share_table().erase(it);
        }
        if (rows) {
            if (feature_dims > 0 && rows->proto.d != feature_dims)
                throw std::runtime_error("RVC retrieval index: index feature width does not match the voice model");
            return handle_from_shared(rows, o);
        }
    }
    FaissLayout L = faiss_layout(bytes, length);
    std::vector<int32_t> ids;
    const size_t bad_id = scan_ids(L, bytes, ids);
    if (bad_id != FaissLayout::kNoFault) {
        // error path: a non-finite row before the bad id wins, as in the reference
        size_t nonfinite = FaissLayout::kNoFault;
        for (const auto &list : L.lists) {
            if (list.vec_pos > bad_id || nonfinite != FaissLayout::kNoFault) break;
            for (uint64_t i = 0; i < list.size * static_cast<uint64_t>(L.d); ++i) {
                float v;
                std::memcpy(&v, bytes + list.vec_pos + 4 * i, 4);
                if (!std::isfinite(v)) {
                    nonfinite = list.vec_pos + 4 * i;
                    break;
                }
            }
        }
        raise_first_fault(L, nonfinite, bad_id);
    }
    const size_t n = static_cast<size_t>(L.n);
    const size_t values = n * static_cast<size_t>(L.d);
    std::vector<int32_t> inverse;
    const bool permutation = inverse_ids(ids.data(), n, inverse);
    VfrIndex *ix = new_handle(L.d, L.nlist, L.nprobe, n, L.offsets.data(), o);
    try {
        alloc_copy(&ix->centroids, L.centroids.data(), L.centroids.size());
        alloc_copy(&ix->offsets, L.offsets.data(), L.offsets.size());
        alloc_copy(&ix->ids, ids.data(), n);
        if (permutation) alloc_copy(&ix->row_of_id, inverse.data(), n);
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->vectors), values * sizeof(float)), "cudaMalloc rows");
        std::vector<UploadSpan> spans;
        size_t at = 0;
        for (const auto &list : L.lists) {
            const size_t b = static_cast<size_t>(list.size) * L.d * sizeof(float);
            if (b) spans.push_back({bytes + list.vec_pos, b, at});
            at += b;
        }
        staged_upload(ix->vectors, spans, ix->device);
        const unsigned long long first = first_nonfinite(ix->vectors, values, ix->sm_count);
        raise_first_fault(L, first == ~0ull ? FaissLayout::kNoFault : L.row_position(first), FaissLayout::kNoFault);
        if (feature_dims > 0 && L.d != feature_dims)
            throw std::runtime_error("RVC retrieval index: index feature width does not match the voice model");
        validate_arrays(L.d, L.nlist, L.nprobe, n, L.centroids.data(), L.centroids.size(), L.offsets.data(),
                        L.offsets.size(), ix->vectors, values, ids.data(), n);
        finish_index(ix, o);
        if (share) publish_shared(ix, key);
    } catch (...) {
        free_index(ix);
        throw;
    }
    return ix;
}

cudaStream_t stream_of(VfrStream *stream) {
    require(stream && stream->stream, "invalid FAISS CUDA stream");
    return static_cast<cudaStream_t>(stream->stream);
}

ExactArgs exact_args(VfrIndex *ix, const float *queries, float *out, const float *rate, int mode) {
    ExactArgs a{};
    a.d = ix->d;
    a.nlist = ix->nlist;
    a.nprobe = ix->nprobe;
    a.centroids = ix->centroids;
    a.offsets = ix->offsets;
    a.vectors = ix->vectors;
    a.ids = ix->ids;
    a.queries = queries;
    a.out = out;
    a.index_rate = rate;
    a.mode = mode;
    a.label_base = ix->label_base;
    a.counters = ix->counters;
    return a;
}

// The 2-D exact engine's call: scratch grown outside stream capture.
void run_exact2d(VfrIndex *ix, const ExactArgs &a, size_t frames, cudaStream_t s) {
    const Exact2dLayout l = exact2d_layout(frames, ix->nlist, ix->nprobe, ix->max_probed_rows);
    if (l.total > ix->x2_bytes) {
        cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
        cuda_check(cudaStreamIsCapturing(s, &st));
        require(st == cudaStreamCaptureStatusNone,
                "retrieval workspace too small for this frame count during stream capture; call "
                "vfr_retrieval_reserve first");
        reserve_exact2d(ix, frames);
    }
    ix->last_engine = 3;
    ix->prof.begin(kProfExact, s);
    launch_exact2d(a, ix->x2_ws, l, static_cast<long long>(frames), s);
    ix->prof.end(s);
}

void search_rows(VfrIndex *ix, const float *queries, size_t frames, int k, float *dist, int64_t *labels,
                 cudaStream_t s) {
    if (use_exact2d(ix, frames)) {
        ExactArgs a = exact_args(ix, queries, nullptr, nullptr, kModeSearch);
        a.k = k;
        a.dist_out = dist;
        a.label_out = labels;
        run_exact2d(ix, a, frames, s);
    } else if (ix->have_tc && use_tc(ix, frames)) {
        ix->last_engine = 2;
        run_tc(ix, queries, nullptr, nullptr, kModeSearch, k, dist, labels, frames, s);
    } else {
        ix->last_engine = 1;
        ExactArgs a = exact_args(ix, queries, nullptr, nullptr, kModeSearch);
        a.k = k;
        a.dist_out = dist;
        a.label_out = labels;
        launch_exact(a, static_cast<long long>(frames), s);
    }
    cuda_check(cudaGetLastError());
}

void blend_impl(VfrIndex *ix, const float *queries, float *out, size_t frames, int32_t width, const float *rate,
                VfrStream *stream, float *raw = nullptr) {
    require(ix && queries && out && frames > 0 && rate, "invalid FAISS GPU blend arguments");
    require(frames <= static_cast<size_t>(INT32_MAX), "FAISS frame count exceeds CUDA grid limit");
    require(width == ix->d, "FAISS feature width mismatch");
    cudaStream_t s = stream_of(stream);
    DeviceGuard guard(ix->device);
    if (raw) {
        const size_t bytes = frames * static_cast<size_t>(width) * sizeof(float);
        const auto *r = reinterpret_cast<const uint8_t *>(raw), *q = reinterpret_cast<const uint8_t *>(queries);
        require(r + bytes <= q || q + bytes <= r, "raw feature buffer overlaps the features");
    }
    if (use_exact2d(ix, frames)) {
        if (raw)
            cuda_check(cudaMemcpyAsync(raw, queries, frames * static_cast<size_t>(width) * sizeof(float),
                                       cudaMemcpyDeviceToDevice, s));
        run_exact2d(ix, exact_args(ix, queries, out, rate, kModeBlend), frames, s);
    } else if (ix->have_tc && use_tc(ix, frames)) {
        ix->last_engine = 2;
        run_tc(ix, queries, out, rate, kModeBlend, 8, nullptr, nullptr, frames, s, raw);
    } else {
        ix->last_engine = 1;
        if (raw)
            cuda_check(cudaMemcpyAsync(raw, queries, frames * static_cast<size_t>(width) * sizeof(float),
                                       cudaMemcpyDeviceToDevice, s));
        ix->prof.begin(kProfExact, s);
        launch_exact(exact_args(ix, queries, out, rate, kModeBlend), static_cast<long long>(frames), s);
        ix->prof.end(s);
    }
    cuda_check(cudaGetLastError());
}

}  // namespace vfr

using vfr::guarded;
using vfr::require;
using vfr::cuda_check;

extern "C" int vocal_faiss_gpu_create(int32_t dimensions, int32_t nlist, int32_t nprobe, size_t vector_count,
                                      const float *centroids, size_t centroid_count, const int32_t *offsets,
                                      size_t offset_count, const float *vectors, size_t vector_value_count,
                                      const int32_t *ids, size_t id_count, VfrIndex **out, char **error) {
    return guarded(error, [&] {
        require(out, "null FAISS GPU index output");
        *out = nullptr;
        *out = vfr::create_index(dimensions, nlist, nprobe, vector_count, centroids, centroid_count, offsets,
                                 offset_count, vectors, vector_value_count, ids, id_count, nullptr);
    });
}

extern "C" int vfr_retrieval_create(int32_t dimensions, int32_t nlist, int32_t nprobe, size_t vector_count,
                                    const float *centroids, size_t centroid_count, const int32_t *offsets,
                                    size_t offset_count, const float *vectors, size_t vector_value_count,
                                    const int32_t *ids, size_t id_count, const VfrOptions *options,
                                    VfrIndex **out, char **error) {
    return guarded(error, [&] {
        require(out, "null FAISS GPU index output");
        *out = nullptr;
        *out = vfr::create_index(dimensions, nlist, nprobe, vector_count, centroids, centroid_count, offsets,
                                 offset_count, vectors, vector_value_count, ids, id_count, options);
    });
}

extern "C" void vocal_faiss_gpu_destroy(VfrIndex *index) { vfr::free_index(index); }

extern "C" int vocal_faiss_gpu_blend(VfrIndex *index, float *features, size_t frames, int32_t width,
                                     const float *index_rate, VfrStream *stream, char **error) {
    return guarded(error, [&] { vfr::blend_impl(index, features, features, frames, width, index_rate, stream); });
}

extern "C" int vfr_retrieval_blend_from(VfrIndex *index, const float *queries, float *out, size_t frames,
                                        int32_t width, const float *index_rate, VfrStream *stream, char **error) {
    return guarded(error, [&] { vfr::blend_impl(index, queries, out, frames, width, index_rate, stream); });
}

extern "C" int vfr_retrieval_blend_save_raw(VfrIndex *index, float *features, float *raw, size_t frames,
                                            int32_t width, const float *index_rate, VfrStream *stream,
                                            char **error) {
    return guarded(error, [&] {
        require(raw != nullptr, "null raw feature buffer");
        vfr::blend_impl(index, features, features, frames, width, index_rate, stream, raw);
    });
}

extern "C" int vfr_rvc_frontend(const float *hubert, const float *raw, const float *f0, const float *ratio,
                                const float *protect, int32_t hubert_frames, int32_t f0_frames, int32_t width,
                                float *feats, float *pitchf, int32_t *pitch, int32_t *out_frames, VfrStream *stream,
                                char **error) {
    return guarded(error, [&] {
        require(hubert && f0 && feats && pitchf && pitch && stream, "null RVC frontend binding");
        require(!raw || (ratio && protect), "null retrieval protection binding");
        require(hubert_frames > 0 && f0_frames > 0 && width > 0 && hubert_frames < INT32_MAX / 2 - 1 &&
                    f0_frames <= INT32_MAX / width,
                "invalid RVC frontend dimensions");
        const int target = vfr::frontend_frames(hubert_frames, f0_frames);
        if (out_frames) *out_frames = target;
        vfr::launch_frontend(hubert, raw, f0, ratio, protect, hubert_frames, f0_frames, width, feats, pitchf, pitch,
                             static_cast<cudaStream_t>(stream->stream));
        cuda_check(cudaGetLastError());
    });
}

extern "C" int vfr_engine_frontend(const float *blended, const float *raw, const float *hz, float protect,
                                   int32_t frames, int32_t hz_frames, int32_t width, float *out, int32_t *coarse,
                                   VfrStream *stream, char **error) {
    return guarded(error, [&] {
        require(blended && out && stream && (!hz || hz_frames <= 0 || coarse), "null engine frontend binding");
        require(std::isfinite(protect) && protect >= 0.0f && protect <= 1.0f, "protect must be finite and in [0,1]");
        // 2 frames <= 2^24 keeps t / 2.0 exact in f32, as the Rust source computes it
        require(frames > 0 && width > 0 && frames <= (1 << 23) && 2LL * frames * width <= INT32_MAX &&
                    (!hz || hz_frames >= 0),
                "invalid engine frontend dimensions");
        vfr::launch_engine_frontend(blended, raw, hz, protect, frames, hz ? hz_frames : 0, width, out, coarse,
                                    static_cast<cudaStream_t>(stream->stream));
        cuda_check(cudaGetLastError());
    });
}

extern "C" int vocal_retrieval_protect(float *features, const float *raw, const float *pitchf, const float *ratio,
                                       const float *protect, int32_t frames, int32_t hubert_frames, int32_t width,
                                       VfrStream *stream, char **error) {
    return guarded(error, [&] {
        require(features && raw && pitchf && ratio && protect && stream, "null retrieval protection binding");
        require(frames > 0 && hubert_frames > 0 && width > 0 && frames <= INT32_MAX / width,
                "invalid retrieval protection dimensions");
        vfr::launch_protect(features, raw, pitchf, ratio, protect, frames, hubert_frames, width,
                            static_cast<cudaStream_t>(stream->stream));
        cuda_check(cudaGetLastError());
    });
}

extern "C" int vfr_retrieval_search(VfrIndex *index, const float *queries, size_t frames, int32_t width, int32_t k,
                                    float *distances, int64_t *labels, VfrStream *stream, char **error) {
    return guarded(error, [&] {
        require(index && queries && distances && labels && frames > 0, "invalid FAISS GPU search arguments");
        require(frames <= static_cast<size_t>(INT32_MAX), "FAISS frame count exceeds CUDA grid limit");
        require(width == index->d, "FAISS feature width mismatch");
        require(k >= 1 && k <= vfr::kTopK, "search k must be in 1..8");
        cudaStream_t s = vfr::stream_of(stream);
        vfr::DeviceGuard guard(index->device);
        vfr::search_rows(index, queries, frames, k, distances, labels, s);
    });
}

extern "C" int vfr_retrieval_reserve(VfrIndex *index, size_t max_frames, char **error) {
    return guarded(error, [&] {
        require(index, "null index");
        require(max_frames <= static_cast<size_t>(INT32_MAX), "FAISS frame count exceeds CUDA grid limit");
        vfr::DeviceGuard guard(index->device);
        if (index->have_tc) vfr::reserve_tc(index, max_frames);
        vfr::reserve_exact2d(index, max_frames);
    });
}

extern "C" size_t vfr_retrieval_diagnostics(VfrIndex *index, char *json, size_t length) {
    if (!index) return 0;
    vfr::DeviceCounters c{};
    int previous = 0;
    cudaGetDevice(&previous);
    cudaSetDevice(index->device);
    cudaDeviceSynchronize();
    cudaMemcpy(&c, index->counters, sizeof(c), cudaMemcpyDeviceToHost);
    cudaSetDevice(previous);
    const char *engine = index->engine == VFR_ENGINE_EXACT ? "exact" : index->engine == VFR_ENGINE_TENSOR ? "tensor"
                                                                                                          : "auto";
    char buf[1024];
    int m = std::snprintf(buf, sizeof(buf),
                          "{\"engine\":\"%s\",\"tensor_cores\":%s,\"candidates\":%d,\"dimensions\":%d,\"nlist\":%d,"
                          "\"nprobe\":%d,\"vectors\":%lld,\"label_base\":%lld,\"device\":%d,\"workspace_frames\":%zu,"
                          "\"workspace_bytes\":%zu,\"empty_frames\":%llu,\"fallback_frames\":%llu,"
                          "\"candidate_frames\":%llu,\"rerun_rows\":%llu,\"timeouts\":%llu,\"max_row_norm\":%.9g,"
                          "\"max_row_residual\":%.9g,\"shared_handles\":%ld,\"last_plan\":{\"keep\":%d,"
                          "\"segments\":%d,\"tiles_per_segment\":%d,\"layout\":\"%s\"},\"last_engine\":\"%s\"}",
                          engine, index->have_tc ? "true" : "false", index->candidates, index->d, index->nlist,
                          index->nprobe, static_cast<long long>(index->n), static_cast<long long>(index->label_base),
                          index->device, index->ws.frames, index->ws.bytes, c.empty_frames, c.fallback_frames,
                          c.candidate_frames, c.rerun_rows, c.timeouts, index->max_row_norm, index->max_row_residual,
                          static_cast<long>(index->shared ? index->shared.use_count() : 0), index->last_keep,
                          index->last_segments, index->last_tiles_per_seg,
                          index->last_layout < 0 ? "none" : index->last_layout == 0 ? "full" : index->last_layout == 1 ? "spread" : "pair",
                          index->last_engine == 1   ? "exact"
                          : index->last_engine == 2 ? "tensor"
                          : index->last_engine == 3 ? "exact2d"
                                                    : "none");
    size_t need = m > 0 ? static_cast<size_t>(m) : 0;
    if (json && length) {
        size_t w = std::min(need, length - 1);
        std::memcpy(json, buf, w);
        json[w] = 0;
    }
    return need;
}

extern "C" size_t vfr_retrieval_profile(VfrIndex *index, int32_t enable, char *json, size_t length) {
    if (!index) return 0;
    auto &p = index->prof;
    static const char *names[vfr::kProfCount] = {"prep_queries", "cand_kernel", "merge_kernel", "exact_kernel"};
    double ms[vfr::kProfCount] = {0, 0, 0, 0};
    long long launches[vfr::kProfCount] = {0, 0, 0, 0};
    for (auto &m : p.marks) {
        if (m.second + 1 >= p.used) continue;
        float t = 0.f;
        cudaEventSynchronize(p.pool[m.second + 1]);
        if (cudaEventElapsedTime(&t, p.pool[m.second], p.pool[m.second + 1]) == cudaSuccess) {
            ms[m.first] += t;
            launches[m.first] += 1;
        }
    }
    std::string out = "{";
    for (int k = 0; k < vfr::kProfCount; ++k) {
        char buf[160];
        std::snprintf(buf, sizeof(buf), "%s\"%s\":{\"launches\":%lld,\"ms\":%.6f}", k ? "," : "", names[k],
                      launches[k], ms[k]);
        out += buf;
    }
    out += "}";
    p.marks.clear();
    p.used = 0;
    p.enabled = enable != 0;
    if (json && length) {
        size_t w = std::min(out.size(), length - 1);
        std::memcpy(json, out.data(), w);
        json[w] = 0;
    }
    return out.size();
}

extern "C" void vfr_free_error(char *message) { std::free(message); }

// ---- host index (parse / VFRM / upload) -----------------------------------

extern "C" int vfr_index_parse_faiss(const uint8_t *bytes, size_t length, VfrHostIndex **out, char **error) {
    return guarded(error, [&] {
        require(out, "null index output");
        *out = nullptr;
        auto *h = new VfrHostIndex{};
        try {
            h->h = vfr::parse_faiss(bytes, length);
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
}

extern "C" int vfr_index_from_vfrm(const uint8_t *image, size_t length, int32_t feature_dims, VfrHostIndex **out,
                                   char **error) {
    return guarded(error, [&] {
        require(out && image, "null VFRM input or output");
        *out = nullptr;
        size_t off = 0, size = 0;
        if (!vfr::find_vfrm_faiss(image, length, &off, &size)) return;
        auto *h = new VfrHostIndex{};
        try {
            h->h = vfr::parse_faiss(image + off, size);
            if (feature_dims > 0 && h->h.d != feature_dims)
                throw std::runtime_error("RVC retrieval index: index feature width does not match the voice model");
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
}

extern "C" void vfr_index_free(VfrHostIndex *index) { delete index; }

extern "C" void vfr_index_info(const VfrHostIndex *index, int32_t *dimensions, int32_t *nlist, int32_t *nprobe,
                               int64_t *vector_count) {
    if (!index) return;
    if (dimensions) *dimensions = index->h.d;
    if (nlist) *nlist = index->h.nlist;
    if (nprobe) *nprobe = index->h.nprobe;
    if (vector_count) *vector_count = index->h.n;
}
extern "C" const float *vfr_index_centroids(const VfrHostIndex *index) { return index ? index->h.centroids.data() : nullptr; }
extern "C" const int32_t *vfr_index_offsets(const VfrHostIndex *index) { return index ? index->h.offsets.data() : nullptr; }
extern "C" const float *vfr_index_vectors(const VfrHostIndex *index) { return index ? index->h.vectors.data() : nullptr; }
extern "C" const int32_t *vfr_index_ids(const VfrHostIndex *index) { return index ? index->h.ids.data() : nullptr; }

extern "C" int vfr_index_upload(const VfrHostIndex *index, VfrIndex **out, char **error) {
    return guarded(error, [&] {
        require(index && out, "null index or output");
        require(index->h.n > 0, "retrieval index has no vectors");
        const auto &h = index->h;
        *out = nullptr;
        *out = vfr::create_index(h.d, h.nlist, h.nprobe, static_cast<size_t>(h.n), h.centroids.data(),
                                 h.centroids.size(), h.offsets.data(), h.offsets.size(), h.vectors.data(),
                                 h.vectors.size(), h.ids.data(), h.ids.size(), nullptr);
    });
}

extern "C" int vfr_index_load(const uint8_t *bytes, size_t length, const VfrOptions *options, VfrIndex **out,
                              char **error) {
    return guarded(error, [&] {
        require(out, "null FAISS GPU index output");
        *out = nullptr;
        *out = vfr::load_index(bytes, length, 0, options);
    });
}

extern "C" int vfr_index_load_vfrm(const uint8_t *image, size_t length, int32_t feature_dims,
                                   const VfrOptions *options, VfrIndex **out, char **error) {
    return guarded(error, [&] {
        require(out && image, "null VFRM input or output");
        *out = nullptr;
        size_t off = 0, size = 0;
        if (!vfr::find_vfrm_faiss(image, length, &off, &size)) return;
        *out = vfr::load_index(image + off, size, feature_dims, options);
    });
}

extern "C" int vfr_index_load_file(const char *path, int32_t feature_dims, const VfrOptions *options, VfrIndex **out,
                                   char **error) {
    return guarded(error, [&] {
        require(out && path, "null index path or output");
        *out = nullptr;
        vfr::MappedFile file(path);
        static const uint8_t vfrm[4] = {'V', 'F', 'R', 'M'};
        if (file.size >= 4 && std::memcmp(file.data, vfrm, 4) == 0) {
            size_t off = 0, size = 0;
            if (!vfr::find_vfrm_faiss(file.data, file.size, &off, &size)) return;
            *out = vfr::load_index(file.data + off, size, feature_dims, options);
        } else {
            *out = vfr::load_index(file.data, file.size, feature_dims, options);
        }
    });
}

extern "C" int vfr_index_content_hash(const uint8_t *bytes, size_t length, uint64_t *hash, char **error) {
    return guarded(error, [&] {
        require(hash && (bytes || length == 0), "null hash input or output");
        const vfr::ContentHash h = vfr::content_hash(bytes, length);
        hash[0] = h.lo;
        hash[1] = h.hi;
    });
}

// ---- IVF training --------------------------------------------------------

extern "C" int vfr_kmeans(const float *x, int64_t n, int32_t d, int32_t k, int32_t niter,
                          int32_t max_points_per_centroid, uint64_t seed, float *centroids, double *objective,
                          VfrStream *stream, char **error) {
    return guarded(error, [&] {
        cudaStream_t s = vfr::stream_of(stream);
        vfr::kmeans(x, n, d, k, niter, max_points_per_centroid, seed, centroids, objective, s);
    });
}

extern "C" int vfr_ivf_assign(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d,
                              int32_t *lists, float *distances, VfrStream *stream, char **error) {
    return guarded(error, [&] {
        cudaStream_t s = vfr::stream_of(stream);
        vfr::ivf_assign(centroids, k, x, n, d, lists, distances, s);
    });
}

extern "C" int vfr_ivf_build(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, int32_t nprobe,
                             const VfrOptions *options, VfrIndex **out, char **error) {
    return guarded(error, [&] {
        require(out, "null FAISS GPU index output");
        *out = nullptr;
        *out = vfr::ivf_build(centroids, k, x, n, d, nprobe, options);
    });
}

extern "C" int vfr_ivf_write(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d,
                             const int32_t *lists, int32_t nprobe, uint8_t *out, size_t capacity, size_t *size,
                             char **error) {
    return guarded(error, [&] {
        require(size, "null size output");
        *size = vfr::ivf_write(centroids, k, x, n, d, lists, nprobe, out, capacity);
    });
}

// ---- sharded building blocks ----------------------------------------------

extern "C" int vfr_merge_topk(const float *dist, const int64_t *labels, int32_t shards, size_t frames,
                              float *out_dist, int64_t *out_labels, VfrStream *stream, char **error) {
    return guarded(error, [&] {
        require(dist && labels && out_dist && out_labels, "invalid merge arguments");
        require(shards >= 1 && shards <= 64, "shard count must be in 1..64");
        require(frames <= static_cast<size_t>(INT32_MAX), "frame count exceeds CUDA grid limit");
        vfr::launch_merge_topk(dist, labels, shards, static_cast<long long>(frames), out_dist, out_labels,
                               vfr::stream_of(stream));
        vfr::cuda_check(cudaGetLastError());
    });
}

extern "C" int vfr_gather_owned(VfrIndex *index, const int64_t *labels, size_t frames, float *out, VfrStream *stream,
                                char **error) {
    return guarded(error, [&] {
        require(index && labels && out, "invalid gather arguments");
        require(index->row_of_id, "index ids are not a permutation of 0..n");
        require(frames <= static_cast<size_t>(INT32_MAX) / 8, "frame count exceeds CUDA grid limit");
        vfr::DeviceGuard guard(index->device);
        vfr::launch_gather_owned(index->vectors, index->row_of_id, index->n, index->label_base, index->d, labels,
                                 static_cast<long long>(frames), out, vfr::stream_of(stream));
        vfr::cuda_check(cudaGetLastError());
    });
}

extern "C" int vfr_blend_gathered(const float *queries, float *out, const float *dist, const float *neighbours,
                                  size_t frames, int32_t width, const float *index_rate, VfrStream *stream,
                                  char **error) {
    return guarded(error, [&] {
        require(queries && out && dist && neighbours && index_rate, "invalid blend arguments");
        require(width > 0 && width <= 4096, "invalid feature width");
        require(frames <= static_cast<size_t>(INT32_MAX), "frame count exceeds CUDA grid limit");
        vfr::launch_blend_gathered(queries, out, dist, neighbours, static_cast<long long>(frames), width, index_rate,
                                   vfr::stream_of(stream));
        vfr::cuda_check(cudaGetLastError());
    });
}

extern "C" int vfr_blend_gathered_rows(const float *queries, float *out, const float *dist, const float *rows,
                                       size_t row_count, const int32_t *slot_rows, size_t frames, int32_t width,
                                       const float *index_rate, VfrStream *stream, char **error) {
    return guarded(error, [&] {
        require(queries && out && dist && slot_rows && index_rate && (rows || row_count == 0),
                "invalid blend arguments");
        require(width > 0 && width <= 4096, "invalid feature width");
        require(frames <= static_cast<size_t>(INT32_MAX), "frame count exceeds CUDA grid limit");
        require(row_count <= static_cast<size_t>(INT32_MAX), "gathered row count exceeds the slot index range");
        vfr::launch_blend_gathered_rows(queries, out, dist, rows, slot_rows, static_cast<long long>(row_count),
                                        static_cast<long long>(frames), width, index_rate, vfr::stream_of(stream));
        vfr::cuda_check(cudaGetLastError());
    });
}
