// Single-process multi-GPU retrieval: one handle over several devices of a
// node, for a C or Rust caller that drives its GPUs from one process (the
// torch.distributed host in vfr/sharded.py covers one process per GPU).
//
// Row sharding (flat indexes): shard s holds rows [first_s, first_{s+1}) as
// an index on devices[s] whose labels are global rows.  A call records an
// event on the caller's stream (devices[0], the home device), and on every
// shard's own stream copies the frames over NVLink (peer copy; none for a
// shard on the home device), searches the shard and writes its exact top 8
// straight into the home device's gather buffer (plain stores to peer
// memory).  The home stream waits for every shard, merges the lists by
// (distance, global row) -- the single-index scan order -- and then either
// maps the rows to the caller's FAISS ids (search) or blends each frame with
// its winners' fp32 rows read from the shards that own them (plain loads over
// NVLink, the peer blend kernel).  The results equal one index's bit for bit.
//
// Query sharding: every device holds a replica; shard s blends (or searches)
// the frames [s F / G, (s + 1) F / G) and copies its share back to the home
// device.
//
// No collective library is involved: within one process the devices' memory
// is directly addressable once peer access is enabled, so copies and loads
// over NVLink replace the all-gather and the exchange.  No bulk or tensor
// copy ever reads another GPU's memory (the candidate kernel's TMA reads only
// its own device's rows and frames).
#include <algorithm>
#include <memory>
#include <mutex>
#include <vector>

#include "exact_common.cuh"
#include "index_build.h"
#include "peer_table.h"
#include "vfr_common.h"

struct VfrShardedIndex {
    int mode = VFR_SHARD_ROWS;
    int d = 0;
    int home = 0;
    std::vector<int> devices;
    std::vector<VfrIndex *> parts;
    std::vector<int64_t> first;  // rows: the first global row of each shard (and n at the end)
    int32_t *ids = nullptr;      // rows: the caller's FAISS id of every global row, on the home device
    vfr::PeerTable table{};      // rows: each shard's fp32 rows as the home device addresses them
    std::vector<cudaStream_t> streams;
    std::vector<cudaEvent_t> done;
    cudaEvent_t start = nullptr;
    size_t cap = 0;  // frames the scratch below holds
    float *dist_all = nullptr;    // rows: [shards][cap][8] on the home device
    int64_t *labels_all = nullptr;
    float *dist = nullptr;        // rows: merged [cap][8]
    int64_t *labels = nullptr;
    std::vector<float *> q_local;    // per shard not on the home device: its frames (rows: all; queries: its share)
    std::vector<float *> out_local;  // queries: per shard not on the home device, its share's output
    std::vector<float *> sdist;      // queries: per shard not on the home device, its share's distances
    std::vector<int64_t *> slabels;
    std::mutex lock;
};

namespace vfr {
namespace {

__global__ void ids_from_rows_kernel(const float *__restrict__ dist, const int64_t *__restrict__ rows,
                                     const int32_t *__restrict__ ids, long long frames, int k,
                                     float *__restrict__ out_dist, int64_t *__restrict__ out_labels) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= frames * k) return;
    const long long f = i / k;
    const int j = static_cast<int>(i - f * k);
    const int64_t row = rows[f * 8 + j];
    out_dist[i] = dist[f * 8 + j];
    out_labels[i] = row < 0 ? -1 : static_cast<int64_t>(ids[row]);
}

void call_ok(int rc, char *err, const char *what) {
    if (rc == 0) return;
    std::string m = std::string(what) + ": " + (err ? err : "error");
    if (err) vfr_free_error(err);
    throw std::runtime_error(m);
}

template <class T>
void device_alloc(T **p, size_t count) {
    cuda_check(cudaMalloc(reinterpret_cast<void **>(p), std::max<size_t>(count, 1) * sizeof(T)), "cudaMalloc");
}

void free_scratch(VfrShardedIndex *h) noexcept {
    auto release = [](int device, void *p) {
        if (!p) return;
        cudaSetDevice(device);
        cudaFree(p);
    };
    release(h->home, h->dist_all);
    release(h->home, h->labels_all);
    release(h->home, h->dist);
    release(h->home, h->labels);
    h->dist_all = h->dist = nullptr;
    h->labels_all = h->labels = nullptr;
    for (size_t s = 0; s < h->parts.size(); ++s) {
        if (s < h->q_local.size()) release(h->devices[s], h->q_local[s]);
        if (s < h->out_local.size()) release(h->devices[s], h->out_local[s]);
        if (s < h->sdist.size()) release(h->devices[s], h->sdist[s]);
        if (s < h->slabels.size()) release(h->devices[s], h->slabels[s]);
    }
    std::fill(h->q_local.begin(), h->q_local.end(), nullptr);
    std::fill(h->out_local.begin(), h->out_local.end(), nullptr);
    std::fill(h->sdist.begin(), h->sdist.end(), nullptr);
    std::fill(h->slabels.begin(), h->slabels.end(), nullptr);
    h->cap = 0;
}

void destroy(VfrShardedIndex *h) noexcept {
    if (!h) return;
    int previous = 0;
    cudaGetDevice(&previous);
    for (size_t s = 0; s < h->streams.size(); ++s) {
        cudaSetDevice(h->devices[s]);
        if (h->streams[s]) cudaStreamSynchronize(h->streams[s]);
    }
    free_scratch(h);
    for (size_t s = 0; s < h->parts.size(); ++s) {
        cudaSetDevice(h->devices[s]);
        if (h->done[s]) cudaEventDestroy(h->done[s]);
        if (h->streams[s]) cudaStreamDestroy(h->streams[s]);
        vocal_faiss_gpu_destroy(h->parts[s]);
    }
    cudaSetDevice(h->home);
    if (h->start) cudaEventDestroy(h->start);
    if (h->ids) cudaFree(h->ids);
    cudaSetDevice(previous);
    delete h;
}

// Frames of shard s in query mode.
void share(const VfrShardedIndex *h, size_t frames, size_t s, size_t &a, size_t &b) {
    const size_t g = h->parts.size();
    a = frames * s / g;
    b = frames * (s + 1) / g;
}

// Scratch for `frames` frames; grows only outside stream capture.
void reserve(VfrShardedIndex *h, size_t frames, cudaStream_t hs) {
    if (frames <= h->cap) return;
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    cuda_check(cudaStreamIsCapturing(hs, &st));
    require(st == cudaStreamCaptureStatusNone,
            "sharded index scratch too small during stream capture (set VfrOptions.max_frames)");
    for (size_t s = 0; s < h->streams.size(); ++s) {
        DeviceGuard g(h->devices[s]);
        cuda_check(cudaStreamSynchronize(h->streams[s]));
    }
    {
        DeviceGuard g(h->home);
        cuda_check(cudaStreamSynchronize(hs));
    }
    free_scratch(h);
    const size_t g = h->parts.size();
    const size_t d = static_cast<size_t>(h->d);
    if (h->mode == VFR_SHARD_ROWS) {
        DeviceGuard guard(h->home);
        device_alloc(&h->dist_all, g * frames * 8);
        device_alloc(&h->labels_all, g * frames * 8);
        device_alloc(&h->dist, frames * 8);
        device_alloc(&h->labels, frames * 8);
    }
    for (size_t s = 0; s < g; ++s) {
        if (h->devices[s] == h->home) continue;
        DeviceGuard guard(h->devices[s]);
        // rows: every frame; queries: at most ceil(frames / g) + 1 (any smaller call's share fits)
        const size_t m = h->mode == VFR_SHARD_ROWS ? frames : (frames + g - 1) / g + 1;
        device_alloc(&h->q_local[s], m * d);
        if (h->mode == VFR_SHARD_QUERIES) {
            device_alloc(&h->out_local[s], m * d);
            device_alloc(&h->sdist[s], m * 8);
            device_alloc(&h->slabels[s], m * 8);
        }
    }
    h->cap = frames;
}

// Row mode: every shard's exact top 8 (global rows) into the home gather
// buffer, then the merge on the home stream.
void row_topk(VfrShardedIndex *h, const float *queries, size_t frames, cudaStream_t hs) {
    const size_t g = h->parts.size();
    const size_t bytes = frames * static_cast<size_t>(h->d) * sizeof(float);
    {
        DeviceGuard guard(h->home);
        cuda_check(cudaEventRecord(h->start, hs));
    }
    for (size_t s = 0; s < g; ++s) {
        DeviceGuard guard(h->devices[s]);
        cudaStream_t ss = h->streams[s];
        cuda_check(cudaStreamWaitEvent(ss, h->start, 0));
        const float *qs = queries;
        if (h->devices[s] != h->home) {
            cuda_check(cudaMemcpyPeerAsync(h->q_local[s], h->devices[s], queries, h->home, bytes, ss));
            qs = h->q_local[s];
        }
        VfrStream vs{ss};
        char *err = nullptr;
        call_ok(vfr_retrieval_search(h->parts[s], qs, frames, h->d, 8, h->dist_all + s * frames * 8,
                                     h->labels_all + s * frames * 8, &vs, &err),
                err, "shard search");
        cuda_check(cudaEventRecord(h->done[s], ss));
    }
    DeviceGuard guard(h->home);
    for (size_t s = 0; s < g; ++s) cuda_check(cudaStreamWaitEvent(hs, h->done[s], 0));
    launch_merge_topk(h->dist_all, h->labels_all, static_cast<int>(g), static_cast<long long>(frames), h->dist,
                      h->labels, hs);
    cuda_check(cudaGetLastError());
}

// Query mode: shard s runs `run(part, queries, out_or_null, dist, labels, frames, stream)` on its share.
template <class F>
void query_shares(VfrShardedIndex *h, const float *queries, float *out, float *dist, int64_t *labels, int k,
                  size_t frames, cudaStream_t hs, F &&run) {
    const size_t g = h->parts.size();
    const size_t d = static_cast<size_t>(h->d);
    {
        DeviceGuard guard(h->home);
        cuda_check(cudaEventRecord(h->start, hs));
    }
    for (size_t s = 0; s < g; ++s) {
        size_t a = 0, b = 0;
        share(h, frames, s, a, b);
        DeviceGuard guard(h->devices[s]);
        cudaStream_t ss = h->streams[s];
        cuda_check(cudaStreamWaitEvent(ss, h->start, 0));
        if (b > a) {
            const size_t m = b - a;
            const float *qs = queries + a * d;
            float *os = out ? out + a * d : nullptr;
            float *ds = dist ? dist + a * k : nullptr;
            int64_t *ls = labels ? labels + a * k : nullptr;
            const bool remote = h->devices[s] != h->home;
            if (remote) {
                cuda_check(cudaMemcpyPeerAsync(h->q_local[s], h->devices[s], qs, h->home, m * d * sizeof(float), ss));
                qs = h->q_local[s];
                if (os) os = h->out_local[s];
                if (ds) ds = h->sdist[s];
                if (ls) ls = h->slabels[s];
            }
            run(h->parts[s], qs, os, ds, ls, m, ss);
            if (remote) {
                if (out)
                    cuda_check(cudaMemcpyPeerAsync(out + a * d, h->home, os, h->devices[s], m * d * sizeof(float), ss));
                if (dist)
                    cuda_check(cudaMemcpyPeerAsync(dist + a * k, h->home, ds, h->devices[s], m * k * sizeof(float), ss));
                if (labels)
                    cuda_check(cudaMemcpyPeerAsync(labels + a * k, h->home, ls, h->devices[s],
                                                   m * k * sizeof(int64_t), ss));
            }
        }
        cuda_check(cudaEventRecord(h->done[s], ss));
    }
    DeviceGuard guard(h->home);
    for (size_t s = 0; s < g; ++s) cuda_check(cudaStreamWaitEvent(hs, h->done[s], 0));
}

cudaStream_t home_stream(VfrShardedIndex *h, VfrStream *stream) {
    require(stream && stream->stream, "invalid FAISS CUDA stream");
    (void)h;
    return static_cast<cudaStream_t>(stream->stream);
}

void enable_peer(int from, int to) {
    if (from == to) return;
    int can = 0;
    cuda_check(cudaDeviceCanAccessPeer(&can, from, to));
    require(can == 1, "sharded index: device " + std::to_string(from) + " cannot access device " +
                          std::to_string(to) + " (peer access)");
    DeviceGuard guard(from);
    const cudaError_t rc = cudaDeviceEnablePeerAccess(to, 0);
    if (rc == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();  // clear the sticky-free status of an already enabled pair
        return;
    }
    cuda_check(rc, "cudaDeviceEnablePeerAccess");
}

}  // namespace
}  // namespace vfr

using vfr::guarded;
using vfr::require;

extern "C" int vfr_retrieval_create_sharded(int32_t device_count, const int32_t *devices, int32_t mode,
                                            int32_t dimensions, int32_t nlist, int32_t nprobe, size_t vector_count,
                                            const float *centroids, size_t centroid_count, const int32_t *offsets,
                                            size_t offset_count, const float *vectors, size_t vector_value_count,
                                            const int32_t *ids, size_t id_count, const VfrOptions *options,
                                            VfrShardedIndex **out, char **error) {
    return guarded(error, [&] {
        require(out, "null sharded index output");
        *out = nullptr;
        require(devices && device_count >= 1 && device_count <= vfr::kMaxPeerShards,
                "sharded index: device count must be in 1..64");
        require(mode == VFR_SHARD_ROWS || mode == VFR_SHARD_QUERIES, "sharded index: unknown shard mode");
        require(dimensions > 0 && vector_count > 0, "invalid FAISS GPU index dimensions");
        require(vectors && vector_value_count == vector_count * static_cast<size_t>(dimensions),
                "FAISS vector array length does not match the index");
        require(ids && id_count == vector_count, "FAISS id array length does not match the index");
        if (mode == VFR_SHARD_ROWS) {
            require(nlist == 1, "row sharding needs a flat index (nlist 1)");
            require(vector_count >= static_cast<size_t>(device_count), "row sharding: fewer rows than shards");
        }
        int ndev = 0;
        vfr::cuda_check(cudaGetDeviceCount(&ndev));
        for (int s = 0; s < device_count; ++s)
            require(devices[s] >= 0 && devices[s] < ndev, "sharded index: device ordinal out of range");
        auto h = std::unique_ptr<VfrShardedIndex, void (*)(VfrShardedIndex *)>(new VfrShardedIndex(), vfr::destroy);
        h->mode = mode;
        h->d = dimensions;
        h->home = devices[0];
        h->devices.assign(devices, devices + device_count);
        const size_t g = static_cast<size_t>(device_count);
        h->parts.assign(g, nullptr);
        h->streams.assign(g, nullptr);
        h->done.assign(g, nullptr);
        h->q_local.assign(g, nullptr);
        h->out_local.assign(g, nullptr);
        h->sdist.assign(g, nullptr);
        h->slabels.assign(g, nullptr);
        for (int s = 1; s < device_count; ++s) {
            vfr::enable_peer(h->home, devices[s]);
            vfr::enable_peer(devices[s], h->home);
        }
        VfrOptions o{};
        if (options) {
            require(options->struct_size >= static_cast<int32_t>(sizeof(int32_t)), "invalid VfrOptions.struct_size");
            std::memcpy(&o, options, std::min<size_t>(sizeof(o), static_cast<size_t>(options->struct_size)));
        }
        o.struct_size = sizeof(VfrOptions);
        const size_t d = static_cast<size_t>(dimensions);
        if (mode == VFR_SHARD_ROWS) {
            h->first.resize(g + 1);
            for (size_t s = 0; s <= g; ++s) h->first[s] = static_cast<int64_t>(vector_count * s / g);
            std::vector<int32_t> local_ids;
            for (size_t s = 0; s < g; ++s) {
                vfr::DeviceGuard guard(devices[s]);
                const size_t rows = static_cast<size_t>(h->first[s + 1] - h->first[s]);
                local_ids.resize(rows);
                for (size_t r = 0; r < rows; ++r) local_ids[r] = static_cast<int32_t>(r);
                const int32_t off[2] = {0, static_cast<int32_t>(rows)};
                VfrOptions so = o;
                so.label_base = h->first[s];
                char *err = nullptr;
                vfr::call_ok(vfr_retrieval_create(dimensions, 1, 1, rows, centroids, centroid_count, off, 2,
                                                  vectors + static_cast<size_t>(h->first[s]) * d, rows * d,
                                                  local_ids.data(), rows, &so, &h->parts[s], &err),
                             err, "shard create");
            }
            vfr::DeviceGuard guard(h->home);
            vfr::device_alloc(&h->ids, vector_count);
            vfr::cuda_check(cudaMemcpy(h->ids, ids, vector_count * sizeof(int32_t), cudaMemcpyHostToDevice));
            h->table.shards = device_count;
            h->table.d = dimensions;
            for (size_t s = 0; s < g; ++s) {
                h->table.rows[s] = h->parts[s]->vectors;
                h->table.row_of_id[s] = nullptr;  // shard labels are global rows
                h->table.bounds[s] = h->first[s];
            }
            h->table.bounds[g] = h->first[g];
        } else {
            for (size_t s = 0; s < g; ++s) {
                vfr::DeviceGuard guard(devices[s]);
                char *err = nullptr;
                vfr::call_ok(vfr_retrieval_create(dimensions, nlist, nprobe, vector_count, centroids, centroid_count,
                                                  offsets, offset_count, vectors, vector_value_count, ids, id_count,
                                                  &o, &h->parts[s], &err),
                             err, "replica create");
            }
        }
        for (size_t s = 0; s < g; ++s) {
            vfr::DeviceGuard guard(devices[s]);
            vfr::cuda_check(cudaStreamCreateWithFlags(&h->streams[s], cudaStreamNonBlocking));
            vfr::cuda_check(cudaEventCreateWithFlags(&h->done[s], cudaEventDisableTiming));
        }
        {
            vfr::DeviceGuard guard(h->home);
            vfr::cuda_check(cudaEventCreateWithFlags(&h->start, cudaEventDisableTiming));
        }
        if (o.max_frames > 0) {
            vfr::DeviceGuard guard(h->home);
            vfr::reserve(h.get(), static_cast<size_t>(o.max_frames), static_cast<cudaStream_t>(nullptr));
        }
        *out = h.release();
    });
}

extern "C" void vfr_retrieval_destroy_sharded(VfrShardedIndex *index) { vfr::destroy(index); }

extern "C" int vfr_retrieval_search_sharded(VfrShardedIndex *index, const float *queries, size_t frames,
                                            int32_t width, int32_t k, float *distances, int64_t *labels,
                                            VfrStream *stream, char **error) {
    return guarded(error, [&] {
        require(index && queries && distances && labels, "invalid FAISS GPU search arguments");
        require(width == index->d, "FAISS feature width mismatch");
        require(k >= 1 && k <= 8, "search k must be in 1..8");
        require(frames <= static_cast<size_t>(INT32_MAX) / 8, "FAISS frame count exceeds CUDA grid limit");
        if (frames == 0) return;
        std::lock_guard<std::mutex> hold(index->lock);
        cudaStream_t hs = vfr::home_stream(index, stream);
        vfr::reserve(index, frames, hs);
        if (index->mode == VFR_SHARD_ROWS) {
            vfr::row_topk(index, queries, frames, hs);
            vfr::DeviceGuard guard(index->home);
            const long long total = static_cast<long long>(frames) * k;
            vfr::ids_from_rows_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, hs>>>(
                index->dist, index->labels, index->ids, static_cast<long long>(frames), k, distances, labels);
            vfr::cuda_check(cudaGetLastError());
        } else {
            vfr::query_shares(index, queries, nullptr, distances, labels, k, frames, hs,
                              [&](VfrIndex *part, const float *q, float *, float *dd, int64_t *ll, size_t m,
                                  cudaStream_t ss) {
                                  VfrStream vs{ss};
                                  char *err = nullptr;
                                  vfr::call_ok(vfr_retrieval_search(part, q, m, index->d, k, dd, ll, &vs, &err), err,
                                               "replica search");
                              });
        }
    });
}

extern "C" int vfr_retrieval_blend_sharded(VfrShardedIndex *index, const float *queries, float *out, size_t frames,
                                           int32_t width, const float *index_rate, VfrStream *stream,
                                           char **error) {
    return guarded(error, [&] {
        require(index && queries && out && index_rate, "invalid FAISS GPU blend arguments");
        require(width == index->d, "FAISS feature width mismatch");
        require(frames <= static_cast<size_t>(INT32_MAX) / 8, "FAISS frame count exceeds CUDA grid limit");
        if (frames == 0) return;
        std::lock_guard<std::mutex> hold(index->lock);
        cudaStream_t hs = vfr::home_stream(index, stream);
        vfr::reserve(index, frames, hs);
        if (index->mode == VFR_SHARD_ROWS) {
            vfr::row_topk(index, queries, frames, hs);
            vfr::DeviceGuard guard(index->home);
            vfr::launch_blend_peer(index->table, queries, out, index->dist, index->labels,
                                   static_cast<long long>(frames), index_rate, hs);
        } else {
            vfr::query_shares(index, queries, out, nullptr, nullptr, 8, frames, hs,
                              [&](VfrIndex *part, const float *q, float *o, float *, int64_t *, size_t m,
                                  cudaStream_t ss) {
                                  VfrStream vs{ss};
                                  char *err = nullptr;
                                  vfr::call_ok(vfr_retrieval_blend_from(part, q, o, m, index->d, index_rate, &vs,
                                                                        &err),
                                               err, "replica blend");
                              });
        }
    });
}
