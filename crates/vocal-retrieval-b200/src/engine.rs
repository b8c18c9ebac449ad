//! The engine-side seam: which implementation serves a voice's retrieval
//! index, and a `FeatureIndex` (crates/vocal-engine/src/pipeline.rs:133-135)
//! for the generic engine backed by the B200 library.
//!
//! Call sites this replaces or extends in the reference:
//! * the TensorRT backend loads the index right after the package
//!   (crates/vocal-engine/src/tensorrt_backend.rs:179-186) and its pipeline
//!   enqueues `vocal_faiss_gpu_blend`; libvfr_retrieval.so exports that ABI
//!   under the same names, so `RetrievalBackend::B200` there means linking
//!   this library in place of native/retrieval.cu;
//! * the generic engine takes any `FeatureIndex`; `B200FeatureIndex` is one
//!   that blends on the GPU from host feature matrices.
//!
//! The model crate's `RetrievalIndex` API (crates/vocal-model/src/
//! retrieval.rs:45-57) is unchanged: every backend starts from it.

use crate::retrieval::{DeviceAlloc, GpuRetrievalIndex, OwnedStream, RetrievalError};
use crate::{ffi, runtime};
use vocal_model::RetrievalIndex;

/// The retrieval implementation a pipeline uses.
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum RetrievalBackend {
    /// The reference's CPU blend (crates/vocal-cpu/src/retrieval.rs:27-83).
    Cpu,
    /// This library on an sm_100 GPU.
    B200,
}

impl RetrievalBackend {
    /// `VOCAL_RETRIEVAL_BACKEND` = `cpu` | `b200` | `auto` (or unset).
    pub const ENV: &'static str = "VOCAL_RETRIEVAL_BACKEND";

    /// The environment's explicit choice, if any.
    pub fn from_env() -> Result<Option<Self>, RetrievalError> {
        match std::env::var(Self::ENV).ok().as_deref().map(str::trim) {
            None | Some("") | Some("auto") => Ok(None),
            Some("cpu") => Ok(Some(Self::Cpu)),
            Some("b200") => Ok(Some(Self::B200)),
            Some(other) => Err(RetrievalError::Argument(format!("{} must be cpu, b200 or auto, not {other}", Self::ENV))),
        }
    }

    /// The explicit choice, else B200 when the library finds an sm_100
    /// device, else the CPU path.  An explicit `b200` on a machine without
    /// one is an error, not a silent fallback.
    pub fn select() -> Result<Self, RetrievalError> {
        let probe = runtime::availability();
        match Self::from_env()? {
            Some(Self::B200) if !probe.available => Err(RetrievalError::Argument(format!(
                "{}=b200 but {}",
                Self::ENV,
                probe.reason.unwrap_or_default()
            ))),
            Some(choice) => Ok(choice),
            None => Ok(if probe.available { Self::B200 } else { Self::Cpu }),
        }
    }
}

/// A `FeatureIndex` that blends host feature matrices on the GPU: frames go
/// to a device buffer, `vocal_faiss_gpu_blend` runs on the index's stream,
/// and the blended frames come back.  Buffers grow to the largest block.
pub struct B200FeatureIndex {
    index: GpuRetrievalIndex,
    stream: OwnedStream,
    features: DeviceAlloc,
    rate: DeviceAlloc,
    capacity: usize,
}

impl B200FeatureIndex {
    pub fn new(index: &RetrievalIndex, max_frames: usize) -> Result<Self, RetrievalError> {
        let mut gpu = GpuRetrievalIndex::new(index)?;
        gpu.reserve(max_frames.max(1))?;
        let features = DeviceAlloc::new(max_frames.max(1) * index.dimensions() * size_of::<f32>())?;
        Ok(Self {
            index: gpu,
            stream: OwnedStream::new()?,
            features,
            rate: DeviceAlloc::new(size_of::<f32>())?,
            capacity: max_frames.max(1),
        })
    }

    pub fn index(&self) -> &GpuRetrievalIndex {
        &self.index
    }

    /// Blends `data` ([frames][width], row-major) in place on the GPU.
    pub fn blend_host(&mut self, data: &mut [f32], frames: usize, index_ratio: f32) -> Result<(), RetrievalError> {
        let width = self.index.dimensions();
        if data.len() != frames.saturating_mul(width) {
            return Err(RetrievalError::Argument("feature matrix width does not match the index".into()));
        }
        if frames == 0 || index_ratio == 0.0 {
            return Ok(()); // the reference's call site skips the blend at ratio 0
        }
        if frames > self.capacity {
            self.stream.synchronize()?;
            self.features = DeviceAlloc::new(frames * width * size_of::<f32>())?;
            self.index.reserve(frames)?;
            self.capacity = frames;
        }
        let bytes = frames * width * size_of::<f32>();
        let s = self.stream.cuda_stream();
        let copy = |dst: u64, src: *const f32, n: usize, kind: i32| unsafe {
            ffi::cudaMemcpyAsync(dst as *mut std::ffi::c_void, src.cast(), n, kind, s)
        };
        let ratio = [index_ratio];
        let rc = copy(self.rate_ptr(), ratio.as_ptr(), size_of::<f32>(), ffi::CUDA_MEMCPY_HOST_TO_DEVICE);
        let rc = if rc == 0 { copy(self.features_ptr(), data.as_ptr(), bytes, ffi::CUDA_MEMCPY_HOST_TO_DEVICE) } else { rc };
        if rc != 0 {
            return Err(RetrievalError::Api(crate::retrieval::cuda_message(rc, "cudaMemcpyAsync")));
        }
        self.index.blend(&self.features, frames, &self.rate, &self.stream)?;
        let rc = unsafe {
            ffi::cudaMemcpyAsync(data.as_mut_ptr().cast(), self.features_ptr() as *const std::ffi::c_void, bytes,
                                 ffi::CUDA_MEMCPY_DEVICE_TO_HOST, s)
        };
        if rc != 0 {
            return Err(RetrievalError::Api(crate::retrieval::cuda_message(rc, "cudaMemcpyAsync")));
        }
        self.stream.synchronize()
    }

    fn features_ptr(&self) -> u64 {
        use crate::retrieval::DeviceBuffer;
        self.features.device_ptr()
    }
    fn rate_ptr(&self) -> u64 {
        use crate::retrieval::DeviceBuffer;
        self.rate.device_ptr()
    }
}

#[cfg(feature = "engine")]
impl vocal_engine::FeatureIndex for B200FeatureIndex {
    fn blend(&mut self, features: &mut vocal_engine::FeatureMatrix, index_ratio: f32)
    -> Result<(), vocal_engine::EngineError> {
        if features.dims != self.index.dimensions() {
            return Err(vocal_engine::EngineError::InvalidInput(
                "feature width does not match the retrieval index".into(),
            ));
        }
        let frames = features.frames;
        self.blend_host(&mut features.data, frames, index_ratio).map_err(|e| match e {
            RetrievalError::Argument(m) => vocal_engine::EngineError::InvalidInput(m),
            RetrievalError::Api(m) => vocal_engine::EngineError::BackendUnavailable(m),
        })
    }
}
