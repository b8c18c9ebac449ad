/*
 * vfr_retrieval.h -- C ABI of libvfr_retrieval.so, the B200 (sm_100a)
 * feature-retrieval library.
 *
 * The hot path is the per-frame k=8 squared-L2 nearest-neighbour search of
 * HuBERT/ContentVec features against a FAISS Flat / IVF-Flat retrieval index,
 * followed by the inverse-square-distance weighted gather-blend at index_rate.
 *
 * Conventions, mirrored from the reference bridge
 * (crates/vocal-tensorrt/native/bridge.h:21-32):
 *   - every fallible call returns 0 on success, 1 on a failure whose message
 *     is stored in *error (if error != NULL), 2 on an unknown failure;
 *   - *error is allocated with malloc and released with vfr_free_error (plain
 *     free() compatible, like vocal_trt_free_error, bridge.h:23);
 *   - device pointers are plain CUDA device addresses on the index's device;
 *     calls are asynchronous and ordered on the given stream; the blend and
 *     search entry points perform no allocation, host synchronisation or
 *     host<->device copy once the index's workspace covers the frame count
 *     (see vfr_retrieval_reserve).
 *
 * Results are those of the reference's CPU retrieval
 * (crates/vocal-cpu/src/retrieval.rs:27-83): exact fp32 squared distances in
 * its AVX2 summation order, top-8 with scan-order tie-breaking, f64 weights
 * 1/max(d,1e-12)^2, f32 blend q*(1-r) + retrieved*r.  Where the reference CPU
 * and CUDA paths differ, this library follows the CUDA path: a frame whose
 * probed lists are all empty keeps its query (the CPU path returns an error),
 * and index_rate is clamped to [0,1] with r <= 0 leaving features untouched.
 */
#ifndef VFR_RETRIEVAL_H
#define VFR_RETRIEVAL_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VFR_API __attribute__((visibility("default")))
#else
#define VFR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque device-resident index (role of vocal::RetrievalGpuIndex,
 * crates/vocal-tensorrt/native/bridge.h:64-67). */
typedef struct VfrIndex VfrIndex;

/* Parsed host-side index: the normalised arrays of the reference's
 * RetrievalIndex (crates/vocal-model/src/retrieval.rs:6-14). */
typedef struct VfrHostIndex VfrHostIndex;

/* Stream handle with the layout of vocal::Stream
 * (crates/vocal-tensorrt/native/bridge.h:54): one cudaStream_t. */
typedef struct VfrStream {
    void *stream;
} VfrStream;

/* ------------------------------------------------------------------------ */
/* Drop-in entry points: same names, argument meaning and error behaviour as */
/* crates/vocal-tensorrt/native/bridge.h:241-251 (Rust externs at           */
/* crates/vocal-tensorrt/src/ffi.rs:174-199).                               */
/* ------------------------------------------------------------------------ */

/* Replaces vocal_faiss_gpu_create (crates/vocal-tensorrt/native/retrieval.cu:34-90).
 * Validates the normalised arrays (d in 1..4096, 0 < nprobe <= min(nlist, 32),
 * 0 < n <= INT32_MAX, payload sizes, monotone offsets covering n), copies them
 * to the current CUDA device and builds the derived device layout (fp16
 * shadow, row norms, tensor-map descriptors). */
VFR_API int vocal_faiss_gpu_create(int32_t dimensions, int32_t nlist, int32_t nprobe, size_t vector_count,
                           const float *centroids, size_t centroid_count, const int32_t *offsets,
                           size_t offset_count, const float *vectors, size_t vector_value_count,
                           const int32_t *ids, size_t id_count, VfrIndex **out, char **error);

/* Replaces vocal_faiss_gpu_destroy (crates/vocal-tensorrt/native/retrieval.cu:92-94). */
VFR_API void vocal_faiss_gpu_destroy(VfrIndex *index);

/* Replaces vocal_faiss_gpu_blend (crates/vocal-tensorrt/native/retrieval.cu:96-128).
 * features: device f32 [frames][width], blended in place.  index_rate: device
 * f32 scalar, read by the kernels (a captured CUDA graph sees updates). */
VFR_API int vocal_faiss_gpu_blend(VfrIndex *index, float *features, size_t frames, int32_t width,
                          const float *index_rate, VfrStream *stream, char **error);

/* Frees an error string (bridge.h:23, vocal_trt_free_error). */
VFR_API void vfr_free_error(char *message);

/* Replaces vocal_retrieval_protect (crates/vocal-tensorrt/native/
 * retrieval_protection.cu:18-33; Rust binding crates/vocal-tensorrt/src/
 * ffi.rs:405-416): after the frontend's 2x interpolation, every frame f with
 * pitchf[f] <= 0 (or NaN) becomes features * p + raw[min(f / 2,
 * hubert_frames - 1)] * (1 - p), p = *protect; nothing changes when
 * *ratio <= 0 or *protect >= 0.5.  features: device f32 [frames][width];
 * raw: device f32 [hubert_frames][width] (the features saved before the
 * blend); pitchf: device f32 [frames]; ratio, protect: device scalars.  Same
 * checks and messages as the reference; stream->stream may be the default
 * stream. */
VFR_API int vocal_retrieval_protect(float *features, const float *raw, const float *pitchf, const float *ratio,
                                    const float *protect, int32_t frames, int32_t hubert_frames, int32_t width,
                                    VfrStream *stream, char **error);

/* ------------------------------------------------------------------------ */
/* Index loading (restates crates/vocal-model/src/retrieval.rs:45-268)      */
/* ------------------------------------------------------------------------ */

/* RetrievalIndex::from_faiss (retrieval.rs:62-193): bounded reader of
 * little-endian FAISS IxF2 / IwFl (L2, Flat quantizer, ArrayInvertedLists). */
VFR_API int vfr_index_parse_faiss(const uint8_t *bytes, size_t length, VfrHostIndex **out, char **error);

/* RetrievalIndex::from_package (retrieval.rs:45-57): finds the U8 tensor
 * aux.retrieval.faiss in a VFRM v1 image (crates/vocal-model/src/inspection.rs:
 * 70-178) and parses it.  *out is NULL (return 0) when the tensor is absent.
 * feature_dims > 0 additionally requires d == feature_dims (768 v2, 256 v1). */
VFR_API int vfr_index_from_vfrm(const uint8_t *image, size_t length, int32_t feature_dims, VfrHostIndex **out,
                        char **error);

VFR_API void vfr_index_free(VfrHostIndex *index);

/* Accessors (retrieval.rs:16-43).  Array pointers stay valid until free. */
VFR_API void vfr_index_info(const VfrHostIndex *index, int32_t *dimensions, int32_t *nlist, int32_t *nprobe,
                    int64_t *vector_count);
VFR_API const float *vfr_index_centroids(const VfrHostIndex *index);
VFR_API const int32_t *vfr_index_offsets(const VfrHostIndex *index);
VFR_API const float *vfr_index_vectors(const VfrHostIndex *index);
VFR_API const int32_t *vfr_index_ids(const VfrHostIndex *index);

/* GpuRetrievalIndex::new (crates/vocal-tensorrt/src/retrieval.rs:30-87):
 * uploads a parsed index (same checks as vocal_faiss_gpu_create). */
VFR_API int vfr_index_upload(const VfrHostIndex *index, VfrIndex **out, char **error);

/* ------------------------------------------------------------------------ */
/* Extended entry points                                                    */
/* ------------------------------------------------------------------------ */

/* Search engine selection. */
enum {
    VFR_ENGINE_AUTO = 0,   /* tensor-core candidates + exact re-rank, exact fallback */
    VFR_ENGINE_EXACT = 1,  /* SIMT exact scan only (no tensor cores) */
    VFR_ENGINE_TENSOR = 2  /* tensor-core candidates + exact re-rank */
};

/* VfrOptions.flags */
enum {
    /* Loaders only: handles loaded from identical FAISS bytes on one device
     * (same engine class) share one copy of the device arrays; each handle
     * keeps its own workspace and counters.  "Identical" is decided by the
     * 128-bit content hash (vfr_index_content_hash) and the byte length,
     * without comparing the bytes: two different images collide by accident
     * with probability about 2^-128, but the hash is not collision-resistant
     * against crafted inputs, so enable sharing only for index files the
     * caller trusts (its own voices), not for files supplied by others. */
    VFR_SHARE_STORAGE = 1
};

typedef struct VfrOptions {
    int32_t struct_size;   /* sizeof(VfrOptions) */
    int32_t engine;        /* VFR_ENGINE_* */
    int32_t candidates;    /* re-rank width per frame (16..128, multiple of 16); 0 = 64 */
    int32_t flags;         /* VFR_SHARE_STORAGE, loaders only; 0 = none */
    int64_t label_base;    /* added to every returned label (row-sharded shards) */
    int64_t max_frames;    /* workspace pre-size; 0 = grow on demand (outside capture) */
} VfrOptions;

/* vocal_faiss_gpu_create with options (NULL = defaults). */
VFR_API int vfr_retrieval_create(int32_t dimensions, int32_t nlist, int32_t nprobe, size_t vector_count,
                         const float *centroids, size_t centroid_count, const int32_t *offsets,
                         size_t offset_count, const float *vectors, size_t vector_value_count,
                         const int32_t *ids, size_t id_count, const VfrOptions *options, VfrIndex **out,
                         char **error);

/* Device ingest: RetrievalIndex::from_faiss + GpuRetrievalIndex::new in one
 * call (crates/vocal-model/src/retrieval.rs:45-193, crates/vocal-tensorrt/
 * src/retrieval.rs:27-60) without the host copy of the rows: the FAISS
 * structure is checked on the host with the parser's checks and messages,
 * the rows go straight from `bytes` to device memory through pinned staging
 * buffers on several host threads, and the finite check runs on the device;
 * the error reported is the one the reference parser reports first.  options
 * may be NULL; with VFR_SHARE_STORAGE, handles loaded from identical bytes
 * on the same device share the device arrays. */
VFR_API int vfr_index_load(const uint8_t *bytes, size_t length, const VfrOptions *options, VfrIndex **out,
                           char **error);
/* The same from a VFRM image's aux.retrieval.faiss tensor; *out stays NULL
 * (rc 0) when the image has none; feature_dims > 0 must match the index
 * width (retrieval.rs:45-57). */
VFR_API int vfr_index_load_vfrm(const uint8_t *image, size_t length, int32_t feature_dims,
                                const VfrOptions *options, VfrIndex **out, char **error);
/* The same from a file (a FAISS .index, or a VFRM package recognised by its
 * magic), mapped read-only: the page cache is the only host copy. */
VFR_API int vfr_index_load_file(const char *path, int32_t feature_dims, const VfrOptions *options, VfrIndex **out,
                                char **error);

/* The 128-bit content hash VFR_SHARE_STORAGE keys shared storage by
 * (hash[0], hash[1]); the same bytes give the same hash on every host and
 * thread count.  Host memory only; usable without a GPU. */
VFR_API int vfr_index_content_hash(const uint8_t *bytes, size_t length, uint64_t *hash, char **error);

/* IVF training (the offline FAISS step the reference runs with
 * IndexIVFFlat::train/add; recipe in crates/vocal-directml/tests/fixtures/
 * README.md and scripts/benchmark-retrieval.py:56-65), on the device.
 * vfr_kmeans: k centroids [k][d] (device) from x [n][d] (device, finite):
 * at most k * max_points_per_centroid rows sampled (0 = all), k of them as the
 * first centroids, niter Lloyd iterations (exact nearest centroid; means in
 * 64-bit fixed point) with empty clusters re-seeded by splitting; objective
 * (host [niter], may be NULL) receives each iteration's sum of distances.
 * Deterministic for a given seed.  Synchronous. */
VFR_API int vfr_kmeans(const float *x, int64_t n, int32_t d, int32_t k, int32_t niter, int32_t max_points_per_centroid,
                       uint64_t seed, float *centroids, double *objective, VfrStream *stream, char **error);
/* lists[r] (device i32 [n]) = the nearest of the k centroids to row r, ties to
 * the lower one; distances (device f32 [n], may be NULL) its squared L2. */
VFR_API int vfr_ivf_assign(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, int32_t *lists,
                           float *distances, VfrStream *stream, char **error);
/* IndexIVFFlat::add into a device index directly: every row of x (device) in
 * the list of its nearest centroid (device), lists in input order, labels the
 * input row numbers. */
VFR_API int vfr_ivf_build(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, int32_t nprobe,
                          const VfrOptions *options, VfrIndex **out, char **error);
/* FAISS IndexIVFFlat bytes (IwFl, Flat-L2 quantizer, ArrayInvertedLists) from
 * host arrays: *size receives the byte count; out is written when capacity
 * suffices (pass NULL to query the size). */
VFR_API int vfr_ivf_write(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d,
                          const int32_t *lists, int32_t nprobe, uint8_t *out, size_t capacity, size_t *size,
                          char **error);

/* Sizes the per-index workspace for up to max_frames frames per call, so that
 * later calls allocate nothing (required before CUDA graph capture). */
VFR_API int vfr_retrieval_reserve(VfrIndex *index, size_t max_frames, char **error);

/* Search without blend: per frame the k (1..8) nearest rows as exact squared
 * distances (ascending, ties in scan order) and FAISS labels (ids[] +
 * label_base).  Missing results: +inf / -1.  All pointers are device memory. */
VFR_API int vfr_retrieval_search(VfrIndex *index, const float *queries, size_t frames, int32_t width, int32_t k,
                         float *distances, int64_t *labels, VfrStream *stream, char **error);

/* Out-of-place blend: reads queries, writes out (may alias queries). */
VFR_API int vfr_retrieval_blend_from(VfrIndex *index, const float *queries, float *out, size_t frames, int32_t width,
                             const float *index_rate, VfrStream *stream, char **error);

/* The RVC frontend after the blend with the protection fused in, replacing
 * the TensorRT frontend graph (crates/vocal-tensorrt/native/frontend.cpp:
 * 36-75) and the vocal_retrieval_protect pass after it
 * (crates/vocal-tensorrt/src/pipeline.rs:1826-1828): the last HuBERT frame
 * is appended, the frames are interpolated 2x (nearest: output frame t reads
 * frame t / 2) and cropped to target = min(2 (hubert_frames + 1), f0_frames)
 * frames; pitchf = f0[0 .. target) and pitch = the coarse mel bin
 * round(clamp((1127 ln(1 + f0/700) - mel_min) * 254 / (mel_max - mel_min)
 * + 1, 1, 255)).  When raw is not null the unvoiced frames (f0 <= 0) are
 * protected as vocal_retrieval_protect does, under the same ratio and
 * protect device scalars.  hubert, raw: device f32 [hubert_frames][width];
 * f0: device f32 [f0_frames]; feats: device f32 [target][width]; pitchf:
 * device f32 [target]; pitch: device i32 [target]; *out_frames (host, may
 * be null) receives target. */
VFR_API int vfr_rvc_frontend(const float *hubert, const float *raw, const float *f0, const float *ratio,
                             const float *protect, int32_t hubert_frames, int32_t f0_frames, int32_t width,
                             float *feats, float *pitchf, int32_t *pitch, int32_t *out_frames, VfrStream *stream,
                             char **error);

/* The generic engine's frontend after its index blend, replacing
 * FeatureMatrix::interpolate_2x and the protection loop of RvcPipeline::run
 * (crates/vocal-engine/src/pipeline.rs:75-96 and 312-333): out[2 frames]
 * is the linear 2x interpolation of blended (output frame t mixes frames
 * floor(t/2) and min(floor(t/2) + 1, frames - 1) at weight 0 or 0.5); when
 * hz and raw are given and protect < 0.5, each frame t < min(2 frames,
 * hz_frames) becomes f v + before (1 - v), before the same interpolation of
 * raw and v = 1 if hz[t] > 0 else protect; coarse[t] = f0_to_coarse(hz[t])
 * (pipeline.rs:625-633) for the same frames when hz is given.  blended, raw:
 * device f32 [frames][width]; hz: device f32 [hz_frames] or null; out:
 * device f32 [2 frames][width]; coarse: device i32 [min(2 frames,
 * hz_frames)] (required with hz and hz_frames > 0).  protect: finite, in [0, 1];
 * 2 frames <= 2^24. */
VFR_API int vfr_engine_frontend(const float *blended, const float *raw, const float *hz, float protect, int32_t frames,
                                int32_t hz_frames, int32_t width, float *out, int32_t *coarse, VfrStream *stream,
                                char **error);

/* vocal_faiss_gpu_blend with RetrievalProtection::save_raw fused in
 * (crates/vocal-tensorrt/src/pipeline.rs:1842-1853,
 * crates/vocal-tensorrt/src/retrieval/protection.rs:47-55): raw (device f32
 * [frames][width], not overlapping features) receives the features as they
 * are before the blend, then features are blended in place.  On the flat
 * tensor-core path the merge kernel writes raw from its own load of each
 * frame, so the separate device copy of the reference disappears. */
VFR_API int vfr_retrieval_blend_save_raw(VfrIndex *index, float *features, float *raw, size_t frames,
                                         int32_t width, const float *index_rate, VfrStream *stream, char **error);

/* JSON diagnostics (engine, candidate width, empty-frame count, fallback
 * count, rows the exact re-runs scanned, layout).  Returns the length needed (excluding NUL); writes at most
 * length bytes including NUL.  Synchronises the index's device. */
VFR_API size_t vfr_retrieval_diagnostics(VfrIndex *index, char *json, size_t length);

/* In-place blend that allocates no device memory, for callers that must not
 * call cudaMalloc during a call: a realtime audio callback (cudaMalloc and
 * cudaFree can synchronise the device and take driver locks, an unbounded
 * stall inside a hard deadline) or a host whose device memory budget is fixed
 * up front.  No counterpart in the reference: it is an addition of this
 * library.  Same arguments, checks and results as vocal_faiss_gpu_blend, for
 * an index with the tensor-core layout (flat, engine auto or tensor), at most
 * 256 frames per call and feature width up to 1024.  Its working memory is a
 * 5.3 MiB static device array that every GPU loading the library holds until
 * exit; the first call on a device looks up that array's address, and the
 * first launch of each kernel may load its code (which the driver can back
 * with device memory), so make one warm-up call before any stream capture or
 * deadline-bound use.  All calls share the array: calls whose kernels
 * overlap on the GPU race and must be serialised by the caller. */
VFR_API int vfr_retrieval_blend_noalloc(VfrIndex *index, float *features, size_t frames, int32_t width,
                                        const float *index_rate, VfrStream *stream, char **error);

/* Per-kernel timing with CUDA events recorded on the call's stream around
 * every kernel the index launches (eager calls only; not during capture).
 * enable = 1 clears and starts recording, enable = 0 stops.  Writes JSON
 * {"kernel": {"launches": L, "ms": T}, ...} of what was recorded so far
 * (synchronises the recorded events); returns the length needed. */
VFR_API size_t vfr_retrieval_profile(VfrIndex *index, int32_t enable, char *json, size_t length);

/* Row-sharded multi-GPU building blocks (one process per GPU; the exchange is
 * a collective of the caller's choice, NCCL all-gather in the Python host).
 *
 * vfr_merge_topk: k-way merge of `shards` per-shard top-8 lists
 *   dist/labels [shards][frames][8] -> out [frames][8], ordered by
 *   (distance, label); flat shards carry global row ids as labels, so this is
 *   the single-index scan order.
 * vfr_gather_owned: for every (frame, slot) label in [label_base,
 *   label_base + n) of this shard write its fp32 vector to out[frame][slot][:],
 *   else -0.0 (so a sum over shards reproduces each vector bit-exactly).
 * vfr_blend_gathered: the reference weights + blend from per-frame distances
 *   [frames][8] and gathered neighbour vectors [frames][8][width]. */
VFR_API int vfr_merge_topk(const float *dist, const int64_t *labels, int32_t shards, size_t frames, float *out_dist,
                   int64_t *out_labels, VfrStream *stream, char **error);
VFR_API int vfr_gather_owned(VfrIndex *index, const int64_t *labels, size_t frames, float *out, VfrStream *stream,
                     char **error);
VFR_API int vfr_blend_gathered(const float *queries, float *out, const float *dist, const float *neighbours,
                       size_t frames, int32_t width, const float *index_rate, VfrStream *stream, char **error);
/* vfr_blend_gathered over a compact buffer of gathered rows (rows
 * [row_count][width], e.g. what an all-to-all of the owned winners
 * delivered): slot (frame, k) reads row slot_rows[frame * 8 + k] (device
 * i32 [frames][8]); slots past the frame's count are not read.  Same
 * weights, blend and results as vfr_blend_gathered (the reference's
 * crates/vocal-cpu/src/retrieval.rs:65-81). */
VFR_API int vfr_blend_gathered_rows(const float *queries, float *out, const float *dist, const float *rows,
                                    size_t row_count, const int32_t *slot_rows, size_t frames, int32_t width,
                                    const float *index_rate, VfrStream *stream, char **error);

/* Row-sharded blend over peer memory (one process per GPU of a node).
 * After the merge every rank knows the global labels of its frames'
 * winners; instead of exchanging the winners' rows with a collective, each
 * rank maps the other shards' fp32 row arrays (CUDA IPC) once, and
 * vfr_blend_peer reads every winner straight from the GPU that owns it
 * (plain loads over NVLink; no bulk or tensor copies of peer memory).  No
 * counterpart in the reference, which is single-GPU; the arithmetic is the
 * reference's blend (crates/vocal-cpu/src/retrieval.rs:65-81).
 *
 * vfr_index_ipc_export: the descriptor of this shard (its rows' IPC handle,
 *   label_base, row count, width) for the other ranks; flat indexes only.
 * vfr_peer_rows_open: maps the shards described by descs[0 .. shards) (in
 *   label order, contiguous; descs[self] describes `local`).  Close every
 *   mapping (vfr_peer_rows_close) on every rank before any rank destroys its
 *   index, with the devices idle (e.g. synchronise, barrier, close,
 *   barrier).
 * vfr_blend_peer: queries/out [frames][width] (this rank's frames), dist
 *   [frames][8] and labels [frames][8] their merged top-8 (vfr_merge_topk);
 *   the same results as vfr_blend_gathered on the gathered vectors. */
typedef struct VfrPeerRows VfrPeerRows;
typedef struct VfrIpcRows {
    uint8_t rows_handle[64]; /* cudaIpcMemHandle_t of the fp32 rows */
    uint8_t ids_handle[64];  /* of the label -> row map, when has_ids */
    int64_t label_base;
    int64_t rows;
    int32_t width;
    int32_t has_ids;
    int32_t device;
    int32_t reserved;
} VfrIpcRows;
VFR_API int vfr_index_ipc_export(VfrIndex *index, VfrIpcRows *out, char **error);
VFR_API int vfr_peer_rows_open(VfrIndex *local, int32_t shards, const VfrIpcRows *descs, int32_t self,
                               VfrPeerRows **out, char **error);
VFR_API void vfr_peer_rows_close(VfrPeerRows *peers);
VFR_API int vfr_blend_peer(VfrPeerRows *peers, const float *queries, float *out, const float *dist,
                           const int64_t *labels, size_t frames, int32_t width, const float *index_rate,
                           VfrStream *stream, char **error);

/* Single-process multi-GPU index: one handle over several devices of a node
 * (the reference is single-GPU; this is the C entry its Rust runtime would
 * call to drive several GPUs from one process).  devices[0] is the home
 * device: queries, outputs, index_rate and `stream` belong to it, and every
 * call is ordered on that stream.
 *
 * VFR_SHARD_ROWS (flat indexes): device s holds rows [s n / G, (s + 1) n / G);
 *   every shard searches all frames, the lists are merged by (distance,
 *   global row) -- the single-index scan order -- and the blend reads each
 *   winner's row from the device that owns it over NVLink.  Results equal a
 *   single index's bit for bit.
 * VFR_SHARD_QUERIES: every device holds a replica and serves a contiguous
 *   share of the frames (any index kind).
 * Peer access between the home device and every other device is enabled at
 * create (an error when the hardware has none).  Scratch grows on demand
 * outside stream capture (VfrOptions.max_frames pre-sizes it and the
 * shards' workspaces); calls on one handle are serialised on the host. */
typedef struct VfrShardedIndex VfrShardedIndex;
enum { VFR_SHARD_ROWS = 0, VFR_SHARD_QUERIES = 1 };
VFR_API int vfr_retrieval_create_sharded(int32_t device_count, const int32_t *devices, int32_t mode,
                                         int32_t dimensions, int32_t nlist, int32_t nprobe, size_t vector_count,
                                         const float *centroids, size_t centroid_count, const int32_t *offsets,
                                         size_t offset_count, const float *vectors, size_t vector_value_count,
                                         const int32_t *ids, size_t id_count, const VfrOptions *options,
                                         VfrShardedIndex **out, char **error);
VFR_API void vfr_retrieval_destroy_sharded(VfrShardedIndex *index);
/* k in 1..8; distances [frames][k], labels [frames][k] (FAISS ids, -1 past a frame's count). */
VFR_API int vfr_retrieval_search_sharded(VfrShardedIndex *index, const float *queries, size_t frames,
                                         int32_t width, int32_t k, float *distances, int64_t *labels,
                                         VfrStream *stream, char **error);
/* Out-of-place blend (out may alias queries), as vfr_retrieval_blend_from. */
VFR_API int vfr_retrieval_blend_sharded(VfrShardedIndex *index, const float *queries, float *out, size_t frames,
                                        int32_t width, const float *index_rate, VfrStream *stream, char **error);

/* Self-test of the bounded wait every mbarrier wait in the library's kernels
 * uses (no counterpart in the reference): one thread waits on a barrier that
 * only `arrive` != 0 completes, giving up after limit_ns (at most 2 s).
 * *timed_out = 1 when the wait gave up, 0 when the phase completed;
 * *elapsed_ns = the device time the wait took.  Synchronous; allocates. */
VFR_API int vfr_selftest_bounded_wait(uint64_t limit_ns, int32_t arrive, int32_t *timed_out, uint64_t *elapsed_ns,
                                      char **error);

#ifdef __cplusplus
}
#endif

#endif /* VFR_RETRIEVAL_H */
