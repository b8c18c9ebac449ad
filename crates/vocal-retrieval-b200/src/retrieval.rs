//! Device-resident retrieval index over libvfr_retrieval.so: the role of
//! crates/vocal-tensorrt/src/retrieval.rs:19-171 (same constructor checks,
//! buffer validation and error kinds), plus the library's extensions
//! (device ingest, search, out-of-place and allocation-free blends,
//! diagnostics).

use std::ffi::{CString, c_void};
use std::path::Path;
use std::ptr;

use vocal_model::RetrievalIndex;

use crate::ffi;

/// NativeBuildError::Argument / ::Api of crates/vocal-tensorrt/src/lib.rs.
#[derive(Debug, thiserror::Error)]
pub enum RetrievalError {
    #[error("{0}")]
    Argument(String),
    #[error("{0}")]
    Api(String),
}

/// A device allocation the caller owns (features, index_rate, outputs).
pub trait DeviceBuffer {
    fn device_ptr(&self) -> u64;
    fn bytes(&self) -> usize;
}

/// A CUDA stream: `vfr_stream` points at a `{ cudaStream_t }` that lives as
/// long as `self` (vocal::Stream has that layout, bridge.h:54).
pub trait DeviceStream {
    fn vfr_stream(&self) -> *mut ffi::Stream;
}

/// Engine selection and workspace sizing (VfrOptions).
#[derive(Clone, Copy, Debug, Default)]
pub struct Options {
    pub engine: Engine,
    /// Re-rank width per frame (16..128, multiple of 16); 0 = 64.
    pub candidates: i32,
    /// Added to every returned label (row-sharded shards).
    pub label_base: i64,
    /// Workspace pre-size; 0 = grow on demand (outside stream capture).
    pub max_frames: i64,
    /// Loaders: share device rows between handles of identical bytes.
    pub share_storage: bool,
}

#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub enum Engine {
    /// Tensor-core candidates + exact fp32 re-rank; exact SIMT where faster.
    #[default]
    Auto,
    /// SIMT exact scan only.
    Exact,
    /// Tensor-core candidates + exact re-rank.
    Tensor,
}

impl Options {
    fn raw(&self) -> ffi::VfrOptions {
        ffi::VfrOptions {
            engine: match self.engine {
                Engine::Auto => ffi::VFR_ENGINE_AUTO,
                Engine::Exact => ffi::VFR_ENGINE_EXACT,
                Engine::Tensor => ffi::VFR_ENGINE_TENSOR,
            },
            candidates: self.candidates,
            flags: if self.share_storage { ffi::VFR_SHARE_STORAGE } else { 0 },
            label_base: self.label_base,
            max_frames: self.max_frames,
            ..ffi::VfrOptions::default()
        }
    }
}

pub struct GpuRetrievalIndex {
    raw: *mut ffi::RetrievalGpuIndex,
    dimensions: usize,
    nlist: usize,
    nprobe: usize,
    vector_count: usize,
}

// One owner moves the index to the realtime worker; calls are stream-ordered
// on the caller's stream (Send, not Sync, as the reference's index).
unsafe impl Send for GpuRetrievalIndex {}

fn to_i32(value: usize, what: &str) -> Result<i32, RetrievalError> {
    i32::try_from(value).map_err(|_| RetrievalError::Argument(format!("retrieval {what} exceeds i32")))
}

fn check(code: i32, error: *mut std::ffi::c_char, fallback: &str) -> Result<(), RetrievalError> {
    if code == 0 { Ok(()) } else { Err(RetrievalError::Api(ffi::native_message(error, fallback))) }
}

impl GpuRetrievalIndex {
    /// GpuRetrievalIndex::new of the reference: uploads a parsed index
    /// through the drop-in `vocal_faiss_gpu_create`.
    pub fn new(index: &RetrievalIndex) -> Result<Self, RetrievalError> {
        Self::with_options(index, None)
    }

    /// `new` with engine / workspace options (`vfr_retrieval_create`).
    pub fn with_options(index: &RetrievalIndex, options: Option<&Options>) -> Result<Self, RetrievalError> {
        if index.is_empty() {
            return Err(RetrievalError::Argument("retrieval index has no vectors".into()));
        }
        let (dimensions, nlist, nprobe) = (index.dimensions(), index.nlist(), index.nprobe());
        if dimensions == 0 || nlist == 0 || nprobe == 0 || nprobe > nlist {
            return Err(RetrievalError::Argument(
                "retrieval index has invalid dimensions or IVF configuration".into(),
            ));
        }
        let (mut raw, mut error) = (ptr::null_mut(), ptr::null_mut());
        let (d, l, p) = (to_i32(dimensions, "width")?, to_i32(nlist, "nlist")?, to_i32(nprobe, "nprobe")?);
        let code = unsafe {
            match options {
                None => ffi::vocal_faiss_gpu_create(
                    d, l, p, index.len(),
                    index.centroids().as_ptr(), index.centroids().len(),
                    index.offsets().as_ptr(), index.offsets().len(),
                    index.vectors().as_ptr(), index.vectors().len(),
                    index.ids().as_ptr(), index.ids().len(),
                    &mut raw, &mut error,
                ),
                Some(o) => {
                    let opt = o.raw();
                    ffi::vfr_retrieval_create(
                        d, l, p, index.len(),
                        index.centroids().as_ptr(), index.centroids().len(),
                        index.offsets().as_ptr(), index.offsets().len(),
                        index.vectors().as_ptr(), index.vectors().len(),
                        index.ids().as_ptr(), index.ids().len(),
                        &opt, &mut raw, &mut error,
                    )
                }
            }
        };
        check(code, error, "create CUDA retrieval index failed")?;
        Self::from_raw(raw)
    }

    /// Device ingest of FAISS bytes (`vfr_index_load`): parse checks on the
    /// host, rows straight to device memory, finite check on the device.
    pub fn load(bytes: &[u8], options: Option<&Options>) -> Result<Self, RetrievalError> {
        let opt = options.map(Options::raw);
        let (mut raw, mut error) = (ptr::null_mut(), ptr::null_mut());
        let code = unsafe {
            ffi::vfr_index_load(
                bytes.as_ptr(), bytes.len(),
                opt.as_ref().map_or(ptr::null(), |o| o as *const _),
                &mut raw, &mut error,
            )
        };
        check(code, error, "load CUDA retrieval index failed")?;
        Self::from_raw(raw)
    }

    /// Device ingest from a FAISS `.index` or a VFRM package on disk
    /// (`vfr_index_load_file`); `None` when a package holds no index.
    pub fn load_file(path: &Path, feature_dims: usize, options: Option<&Options>)
    -> Result<Option<Self>, RetrievalError> {
        let c_path = CString::new(path.as_os_str().as_encoded_bytes())
            .map_err(|_| RetrievalError::Argument("index path contains a NUL byte".into()))?;
        let opt = options.map(Options::raw);
        let (mut raw, mut error) = (ptr::null_mut(), ptr::null_mut());
        let code = unsafe {
            ffi::vfr_index_load_file(
                c_path.as_ptr(), to_i32(feature_dims, "feature width")?,
                opt.as_ref().map_or(ptr::null(), |o| o as *const _),
                &mut raw, &mut error,
            )
        };
        check(code, error, "load CUDA retrieval index failed")?;
        if raw.is_null() { Ok(None) } else { Self::from_raw(raw).map(Some) }
    }

    fn from_raw(raw: *mut ffi::RetrievalGpuIndex) -> Result<Self, RetrievalError> {
        if raw.is_null() {
            return Err(RetrievalError::Api("create CUDA retrieval index returned null handle".into()));
        }
        let mut me = Self { raw, dimensions: 0, nlist: 0, nprobe: 0, vector_count: 0 };
        let diag = me.diagnostics();
        let field = |k: &str| diag.get(k).and_then(serde_json::Value::as_u64).unwrap_or(0) as usize;
        me.dimensions = field("dimensions");
        me.nlist = field("nlist");
        me.nprobe = field("nprobe");
        me.vector_count = field("vectors");
        Ok(me)
    }

    pub fn dimensions(&self) -> usize {
        self.dimensions
    }
    pub fn nlist(&self) -> usize {
        self.nlist
    }
    pub fn nprobe(&self) -> usize {
        self.nprobe
    }
    pub fn len(&self) -> usize {
        self.vector_count
    }
    pub fn is_empty(&self) -> bool {
        self.vector_count == 0
    }
    /// The handle for code that calls ffi directly.
    pub fn as_raw(&self) -> *mut ffi::RetrievalGpuIndex {
        self.raw
    }

    /// Sizes the workspace for `max_frames` frames per call, so that later
    /// calls allocate nothing (needed before CUDA graph capture).
    pub fn reserve(&mut self, max_frames: usize) -> Result<(), RetrievalError> {
        let mut error = ptr::null_mut();
        let code = unsafe { ffi::vfr_retrieval_reserve(self.raw, max_frames, &mut error) };
        check(code, error, "reserve CUDA retrieval workspace failed")
    }

    /// Blend HuBERT features in place (`vocal_faiss_gpu_blend`).
    /// `index_rate` is a one-element device buffer, so changing the ratio
    /// does not invalidate a captured CUDA graph.
    pub fn blend(&self, features: &impl DeviceBuffer, frames: usize, index_rate: &impl DeviceBuffer,
                 stream: &impl DeviceStream) -> Result<(), RetrievalError> {
        if frames == 0 {
            return Ok(());
        }
        validate_blend_buffers(frames, self.dimensions, features.bytes(), index_rate.bytes())?;
        let mut error = ptr::null_mut();
        let code = unsafe {
            ffi::vocal_faiss_gpu_blend(
                self.raw, features.device_ptr() as *mut f32, frames, to_i32(self.dimensions, "width")?,
                index_rate.device_ptr() as *const f32, stream.vfr_stream(), &mut error,
            )
        };
        check(code, error, "CUDA retrieval blend failed")
    }

    /// `blend` without device allocation during the call (static scratch;
    /// at most 256 frames; calls on one device must not overlap).
    pub fn blend_noalloc(&self, features: &impl DeviceBuffer, frames: usize, index_rate: &impl DeviceBuffer,
                         stream: &impl DeviceStream) -> Result<(), RetrievalError> {
        if frames == 0 {
            return Ok(());
        }
        validate_blend_buffers(frames, self.dimensions, features.bytes(), index_rate.bytes())?;
        let mut error = ptr::null_mut();
        let code = unsafe {
            ffi::vfr_retrieval_blend_noalloc(
                self.raw, features.device_ptr() as *mut f32, frames, to_i32(self.dimensions, "width")?,
                index_rate.device_ptr() as *const f32, stream.vfr_stream(), &mut error,
            )
        };
        check(code, error, "CUDA retrieval blend failed")
    }

    /// `blend` with RetrievalProtection::save_raw fused in: `raw` receives
    /// the frames as they are before the blend.
    pub fn blend_save_raw(&self, features: &impl DeviceBuffer, raw: &impl DeviceBuffer, frames: usize,
                          index_rate: &impl DeviceBuffer, stream: &impl DeviceStream) -> Result<(), RetrievalError> {
        if frames == 0 {
            return Ok(());
        }
        validate_blend_buffers(frames, self.dimensions, features.bytes(), index_rate.bytes())?;
        validate_blend_buffers(frames, self.dimensions, raw.bytes(), index_rate.bytes())?;
        let mut error = ptr::null_mut();
        let code = unsafe {
            ffi::vfr_retrieval_blend_save_raw(
                self.raw, features.device_ptr() as *mut f32, raw.device_ptr() as *mut f32, frames,
                to_i32(self.dimensions, "width")?, index_rate.device_ptr() as *const f32, stream.vfr_stream(),
                &mut error,
            )
        };
        check(code, error, "CUDA retrieval blend failed")
    }

    /// Out-of-place blend: reads `queries`, writes `out` (may alias).
    pub fn blend_from(&self, queries: &impl DeviceBuffer, out: &impl DeviceBuffer, frames: usize,
                      index_rate: &impl DeviceBuffer, stream: &impl DeviceStream) -> Result<(), RetrievalError> {
        if frames == 0 {
            return Ok(());
        }
        validate_blend_buffers(frames, self.dimensions, queries.bytes(), index_rate.bytes())?;
        validate_blend_buffers(frames, self.dimensions, out.bytes(), index_rate.bytes())?;
        let mut error = ptr::null_mut();
        let code = unsafe {
            ffi::vfr_retrieval_blend_from(
                self.raw, queries.device_ptr() as *const f32, out.device_ptr() as *mut f32, frames,
                to_i32(self.dimensions, "width")?, index_rate.device_ptr() as *const f32, stream.vfr_stream(),
                &mut error,
            )
        };
        check(code, error, "CUDA retrieval blend failed")
    }

    /// The k (1..8) nearest rows of each frame: exact squared distances
    /// [frames][k] f32 and FAISS labels [frames][k] i64 (+inf / -1 missing).
    pub fn search(&self, queries: &impl DeviceBuffer, frames: usize, k: usize, distances: &impl DeviceBuffer,
                  labels: &impl DeviceBuffer, stream: &impl DeviceStream) -> Result<(), RetrievalError> {
        if !(1..=8).contains(&k) {
            return Err(RetrievalError::Argument("search k must be in 1..8".into()));
        }
        if frames == 0 {
            return Ok(());
        }
        let need = |width: usize| frames.checked_mul(k).and_then(|n| n.checked_mul(width));
        if need(4).is_none_or(|b| b > distances.bytes()) || need(8).is_none_or(|b| b > labels.bytes()) {
            return Err(RetrievalError::Argument("search outputs are smaller than frames x k".into()));
        }
        validate_blend_buffers(frames, self.dimensions, queries.bytes(), size_of::<f32>())?;
        let mut error = ptr::null_mut();
        let code = unsafe {
            ffi::vfr_retrieval_search(
                self.raw, queries.device_ptr() as *const f32, frames, to_i32(self.dimensions, "width")?,
                k as i32, distances.device_ptr() as *mut f32, labels.device_ptr() as *mut i64, stream.vfr_stream(),
                &mut error,
            )
        };
        check(code, error, "CUDA retrieval search failed")
    }

    /// `vfr_retrieval_diagnostics` as JSON: engine, tensor-core layout, last
    /// plan, empty / re-run / certified frame counts, bounded-wait timeouts.
    /// Synchronises the index's device.
    pub fn diagnostics(&self) -> serde_json::Value {
        let need = unsafe { ffi::vfr_retrieval_diagnostics(self.raw, ptr::null_mut(), 0) };
        let mut buf = vec![0u8; need + 1];
        unsafe { ffi::vfr_retrieval_diagnostics(self.raw, buf.as_mut_ptr().cast(), buf.len()) };
        buf.truncate(need);
        serde_json::from_slice(&buf).unwrap_or(serde_json::Value::Null)
    }
}

/// crates/vocal-tensorrt/src/retrieval.rs:147-165: the frame count must fit
/// a CUDA grid and the buffers must hold frames x width floats and the rate.
pub fn validate_blend_buffers(frames: usize, dimensions: usize, feature_bytes: usize, rate_bytes: usize)
-> Result<(), RetrievalError> {
    let required = frames.checked_mul(dimensions).and_then(|n| n.checked_mul(size_of::<f32>()));
    if frames > i32::MAX as usize || required.is_none_or(|bytes| bytes > feature_bytes) || rate_bytes < size_of::<f32>()
    {
        return Err(RetrievalError::Argument("retrieval shape exceeds CUDA grid or buffer capacity".into()));
    }
    Ok(())
}

impl Drop for GpuRetrievalIndex {
    fn drop(&mut self) {
        unsafe { ffi::vocal_faiss_gpu_destroy(self.raw) }
    }
}

/// A device allocation owned by this crate (cudaMalloc / cudaFree).
pub struct DeviceAlloc {
    ptr: *mut c_void,
    bytes: usize,
}

unsafe impl Send for DeviceAlloc {}

impl DeviceAlloc {
    pub fn new(bytes: usize) -> Result<Self, RetrievalError> {
        let mut ptr = ptr::null_mut();
        let rc = unsafe { ffi::cudaMalloc(&mut ptr, bytes.max(1)) };
        if rc != 0 {
            return Err(RetrievalError::Api(cuda_message(rc, "cudaMalloc")));
        }
        Ok(Self { ptr, bytes })
    }
}

impl DeviceBuffer for DeviceAlloc {
    fn device_ptr(&self) -> u64 {
        self.ptr as u64
    }
    fn bytes(&self) -> usize {
        self.bytes
    }
}

impl Drop for DeviceAlloc {
    fn drop(&mut self) {
        unsafe { ffi::cudaFree(self.ptr) };
    }
}

/// A stream owned by this crate, in the `{ cudaStream_t }` layout.
pub struct OwnedStream {
    handle: Box<ffi::Stream>,
}

unsafe impl Send for OwnedStream {}

impl OwnedStream {
    pub fn new() -> Result<Self, RetrievalError> {
        let mut s = ptr::null_mut();
        let rc = unsafe { ffi::cudaStreamCreate(&mut s) };
        if rc != 0 {
            return Err(RetrievalError::Api(cuda_message(rc, "cudaStreamCreate")));
        }
        Ok(Self { handle: Box::new(ffi::Stream { stream: s }) })
    }
    pub fn synchronize(&self) -> Result<(), RetrievalError> {
        let rc = unsafe { ffi::cudaStreamSynchronize(self.handle.stream) };
        if rc != 0 { Err(RetrievalError::Api(cuda_message(rc, "cudaStreamSynchronize"))) } else { Ok(()) }
    }
    pub fn cuda_stream(&self) -> *mut c_void {
        self.handle.stream
    }
}

impl DeviceStream for OwnedStream {
    fn vfr_stream(&self) -> *mut ffi::Stream {
        (&*self.handle as *const ffi::Stream).cast_mut()
    }
}

impl Drop for OwnedStream {
    fn drop(&mut self) {
        unsafe { ffi::cudaStreamDestroy(self.handle.stream) };
    }
}

pub(crate) fn cuda_message(rc: ffi::CudaError, what: &str) -> String {
    let text = unsafe { std::ffi::CStr::from_ptr(ffi::cudaGetErrorString(rc)) }.to_string_lossy().into_owned();
    format!("{what}: {text}")
}
