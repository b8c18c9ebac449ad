//! Raw bindings of libvfr_retrieval.so (include/vfr_retrieval.h).
//!
//! The first block is the reference's retrieval ABI under the same names and
//! signatures (crates/vocal-tensorrt/src/ffi.rs:174-199, native/bridge.h:
//! 241-251), so the reference's own `GpuRetrievalIndex` can link against
//! this library unchanged; the rest are this library's extensions.  Return
//! codes follow bridge.h:24-32: 0 ok, 1 failure with a malloc'd message in
//! `*error` (free it with `vfr_free_error`), 2 unknown failure.

use std::ffi::{CStr, c_char, c_void};

/// Opaque device-resident index (vocal::RetrievalGpuIndex).
#[repr(C)]
pub struct RetrievalGpuIndex {
    _private: [u8; 0],
}

/// Opaque host-side parsed index.
#[repr(C)]
pub struct VfrHostIndex {
    _private: [u8; 0],
}

/// Opaque set of peer row mappings (row-sharded blend over NVLink).
#[repr(C)]
pub struct VfrPeerRows {
    _private: [u8; 0],
}

/// Opaque single-process multi-GPU index (vfr_retrieval_*_sharded).
#[repr(C)]
pub struct VfrShardedIndex {
    _private: [u8; 0],
}

/// Stream handle with the layout of vocal::Stream (bridge.h:54).
#[repr(C)]
pub struct Stream {
    pub stream: *mut c_void,
}

pub const VFR_ENGINE_AUTO: i32 = 0;
pub const VFR_ENGINE_EXACT: i32 = 1;
pub const VFR_ENGINE_TENSOR: i32 = 2;
pub const VFR_SHARE_STORAGE: i32 = 1;
pub const VFR_SHARD_ROWS: i32 = 0;
pub const VFR_SHARD_QUERIES: i32 = 1;

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct VfrOptions {
    pub struct_size: i32,
    pub engine: i32,
    pub candidates: i32,
    pub flags: i32,
    pub label_base: i64,
    pub max_frames: i64,
}

impl Default for VfrOptions {
    fn default() -> Self {
        Self {
            struct_size: size_of::<Self>() as i32,
            engine: VFR_ENGINE_AUTO,
            candidates: 0,
            flags: 0,
            label_base: 0,
            max_frames: 0,
        }
    }
}

/// One row shard's storage as other processes map it (VfrIpcRows).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct VfrIpcRows {
    pub rows_handle: [u8; 64],
    pub ids_handle: [u8; 64],
    pub label_base: i64,
    pub rows: i64,
    pub width: i32,
    pub has_ids: i32,
    pub device: i32,
    pub reserved: i32,
}

unsafe extern "C" {
    // ---- the reference's retrieval ABI (same names and signatures)
    pub fn vocal_faiss_gpu_create(
        dimensions: i32,
        nlist: i32,
        nprobe: i32,
        vector_count: usize,
        centroids: *const f32,
        centroid_count: usize,
        offsets: *const i32,
        offset_count: usize,
        vectors: *const f32,
        vector_value_count: usize,
        ids: *const i32,
        id_count: usize,
        out: *mut *mut RetrievalGpuIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vocal_faiss_gpu_destroy(index: *mut RetrievalGpuIndex);
    pub fn vocal_faiss_gpu_blend(
        index: *mut RetrievalGpuIndex,
        features: *mut f32,
        frames: usize,
        width: i32,
        index_rate: *const f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vocal_retrieval_protect(
        features: *mut f32,
        raw: *const f32,
        pitchf: *const f32,
        ratio: *const f32,
        protect: *const f32,
        frames: i32,
        hubert_frames: i32,
        width: i32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_free_error(message: *mut c_char);

    // ---- index loading (RetrievalIndex::from_faiss / from_package)
    pub fn vfr_index_parse_faiss(
        bytes: *const u8,
        length: usize,
        out: *mut *mut VfrHostIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_index_from_vfrm(
        image: *const u8,
        length: usize,
        feature_dims: i32,
        out: *mut *mut VfrHostIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_index_free(index: *mut VfrHostIndex);
    pub fn vfr_index_info(
        index: *const VfrHostIndex,
        dimensions: *mut i32,
        nlist: *mut i32,
        nprobe: *mut i32,
        vector_count: *mut i64,
    );
    pub fn vfr_index_centroids(index: *const VfrHostIndex) -> *const f32;
    pub fn vfr_index_offsets(index: *const VfrHostIndex) -> *const i32;
    pub fn vfr_index_vectors(index: *const VfrHostIndex) -> *const f32;
    pub fn vfr_index_ids(index: *const VfrHostIndex) -> *const i32;
    pub fn vfr_index_upload(
        index: *const VfrHostIndex,
        out: *mut *mut RetrievalGpuIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_index_load(
        bytes: *const u8,
        length: usize,
        options: *const VfrOptions,
        out: *mut *mut RetrievalGpuIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_index_load_vfrm(
        image: *const u8,
        length: usize,
        feature_dims: i32,
        options: *const VfrOptions,
        out: *mut *mut RetrievalGpuIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_index_load_file(
        path: *const c_char,
        feature_dims: i32,
        options: *const VfrOptions,
        out: *mut *mut RetrievalGpuIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_index_content_hash(
        bytes: *const u8,
        length: usize,
        hash: *mut u64,
        error: *mut *mut c_char,
    ) -> i32;

    // ---- IVF training (the offline FAISS train/add step)
    pub fn vfr_kmeans(
        x: *const f32,
        n: i64,
        d: i32,
        k: i32,
        niter: i32,
        max_points_per_centroid: i32,
        seed: u64,
        centroids: *mut f32,
        objective: *mut f64,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_ivf_assign(
        centroids: *const f32,
        k: i32,
        x: *const f32,
        n: i64,
        d: i32,
        lists: *mut i32,
        distances: *mut f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_ivf_build(
        centroids: *const f32,
        k: i32,
        x: *const f32,
        n: i64,
        d: i32,
        nprobe: i32,
        options: *const VfrOptions,
        out: *mut *mut RetrievalGpuIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_ivf_write(
        centroids: *const f32,
        k: i32,
        x: *const f32,
        n: i64,
        d: i32,
        lists: *const i32,
        nprobe: i32,
        out: *mut u8,
        capacity: usize,
        size: *mut usize,
        error: *mut *mut c_char,
    ) -> i32;

    // ---- extended retrieval entry points
    pub fn vfr_retrieval_create(
        dimensions: i32,
        nlist: i32,
        nprobe: i32,
        vector_count: usize,
        centroids: *const f32,
        centroid_count: usize,
        offsets: *const i32,
        offset_count: usize,
        vectors: *const f32,
        vector_value_count: usize,
        ids: *const i32,
        id_count: usize,
        options: *const VfrOptions,
        out: *mut *mut RetrievalGpuIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_retrieval_reserve(index: *mut RetrievalGpuIndex, max_frames: usize, error: *mut *mut c_char) -> i32;
    pub fn vfr_retrieval_search(
        index: *mut RetrievalGpuIndex,
        queries: *const f32,
        frames: usize,
        width: i32,
        k: i32,
        distances: *mut f32,
        labels: *mut i64,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_retrieval_blend_from(
        index: *mut RetrievalGpuIndex,
        queries: *const f32,
        out: *mut f32,
        frames: usize,
        width: i32,
        index_rate: *const f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_rvc_frontend(
        hubert: *const f32,
        raw: *const f32,
        f0: *const f32,
        ratio: *const f32,
        protect: *const f32,
        hubert_frames: i32,
        f0_frames: i32,
        width: i32,
        feats: *mut f32,
        pitchf: *mut f32,
        pitch: *mut i32,
        out_frames: *mut i32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_engine_frontend(
        blended: *const f32,
        raw: *const f32,
        hz: *const f32,
        protect: f32,
        frames: i32,
        hz_frames: i32,
        width: i32,
        out: *mut f32,
        coarse: *mut i32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_retrieval_blend_save_raw(
        index: *mut RetrievalGpuIndex,
        features: *mut f32,
        raw: *mut f32,
        frames: usize,
        width: i32,
        index_rate: *const f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_retrieval_diagnostics(index: *mut RetrievalGpuIndex, json: *mut c_char, length: usize) -> usize;
    pub fn vfr_retrieval_blend_noalloc(
        index: *mut RetrievalGpuIndex,
        features: *mut f32,
        frames: usize,
        width: i32,
        index_rate: *const f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_retrieval_profile(index: *mut RetrievalGpuIndex, enable: i32, json: *mut c_char, length: usize)
    -> usize;

    // ---- row-sharded multi-GPU building blocks
    pub fn vfr_merge_topk(
        dist: *const f32,
        labels: *const i64,
        shards: i32,
        frames: usize,
        out_dist: *mut f32,
        out_labels: *mut i64,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_gather_owned(
        index: *mut RetrievalGpuIndex,
        labels: *const i64,
        frames: usize,
        out: *mut f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_blend_gathered(
        queries: *const f32,
        out: *mut f32,
        dist: *const f32,
        neighbours: *const f32,
        frames: usize,
        width: i32,
        index_rate: *const f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_blend_gathered_rows(
        queries: *const f32,
        out: *mut f32,
        dist: *const f32,
        rows: *const f32,
        row_count: usize,
        slot_rows: *const i32,
        frames: usize,
        width: i32,
        index_rate: *const f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_index_ipc_export(index: *mut RetrievalGpuIndex, out: *mut VfrIpcRows, error: *mut *mut c_char) -> i32;
    pub fn vfr_peer_rows_open(
        local: *mut RetrievalGpuIndex,
        shards: i32,
        descs: *const VfrIpcRows,
        own: i32,
        out: *mut *mut VfrPeerRows,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_peer_rows_close(peers: *mut VfrPeerRows);
    pub fn vfr_selftest_bounded_wait(
        limit_ns: u64,
        arrive: i32,
        timed_out: *mut i32,
        elapsed_ns: *mut u64,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_blend_peer(
        peers: *mut VfrPeerRows,
        queries: *const f32,
        out: *mut f32,
        dist: *const f32,
        labels: *const i64,
        frames: usize,
        width: i32,
        index_rate: *const f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_retrieval_create_sharded(
        device_count: i32,
        devices: *const i32,
        mode: i32,
        dimensions: i32,
        nlist: i32,
        nprobe: i32,
        vector_count: usize,
        centroids: *const f32,
        centroid_count: usize,
        offsets: *const i32,
        offset_count: usize,
        vectors: *const f32,
        vector_value_count: usize,
        ids: *const i32,
        id_count: usize,
        options: *const VfrOptions,
        out: *mut *mut VfrShardedIndex,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_retrieval_destroy_sharded(index: *mut VfrShardedIndex);
    pub fn vfr_retrieval_search_sharded(
        index: *mut VfrShardedIndex,
        queries: *const f32,
        frames: usize,
        width: i32,
        k: i32,
        distances: *mut f32,
        labels: *mut i64,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
    pub fn vfr_retrieval_blend_sharded(
        index: *mut VfrShardedIndex,
        queries: *const f32,
        out: *mut f32,
        frames: usize,
        width: i32,
        index_rate: *const f32,
        stream: *mut Stream,
        error: *mut *mut c_char,
    ) -> i32;
}

/// The message of a failed call (freed here), or `fallback` when the library
/// stored none -- the role of crates/vocal-tensorrt/src/ffi.rs:390-400.
pub fn native_message(error: *mut c_char, fallback: &str) -> String {
    if error.is_null() {
        fallback.into()
    } else {
        let message = unsafe { CStr::from_ptr(error) }.to_string_lossy().into_owned();
        unsafe { vfr_free_error(error) };
        message
    }
}

// ---- the CUDA runtime calls the host-buffer paths need (libcudart)
pub type CudaError = i32;
pub const CUDA_MEMCPY_HOST_TO_DEVICE: i32 = 1;
pub const CUDA_MEMCPY_DEVICE_TO_HOST: i32 = 2;

unsafe extern "C" {
    pub fn cudaMalloc(ptr: *mut *mut c_void, bytes: usize) -> CudaError;
    pub fn cudaFree(ptr: *mut c_void) -> CudaError;
    pub fn cudaMemcpyAsync(dst: *mut c_void, src: *const c_void, bytes: usize, kind: i32, stream: *mut c_void)
    -> CudaError;
    pub fn cudaStreamCreate(stream: *mut *mut c_void) -> CudaError;
    pub fn cudaStreamDestroy(stream: *mut c_void) -> CudaError;
    pub fn cudaStreamSynchronize(stream: *mut c_void) -> CudaError;
    pub fn cudaGetDeviceCount(count: *mut i32) -> CudaError;
    pub fn cudaDeviceGetAttribute(value: *mut i32, attribute: i32, device: i32) -> CudaError;
    pub fn cudaGetErrorString(error: CudaError) -> *const c_char;
}

/// cudaDevAttrComputeCapabilityMajor / Minor.
pub const CUDA_ATTR_CC_MAJOR: i32 = 75;
pub const CUDA_ATTR_CC_MINOR: i32 = 76;
