//! vocal-retrieval-b200: the B200 implementation of vocal-fast-rs's feature
//! retrieval (k=8 squared-L2 search of HuBERT/ContentVec frames against a
//! voice's FAISS index, then the inverse-square weighted blend at
//! index_rate), as a thin Rust layer over libvfr_retrieval.so.
//!
//! * `ffi`: the C ABI, including the reference's `vocal_faiss_gpu_*` names;
//! * `retrieval`: `GpuRetrievalIndex` in the shape of the reference's
//!   (crates/vocal-tensorrt/src/retrieval.rs), plus device ingest, search
//!   and the allocation-free blend;
//! * `engine`: `RetrievalBackend` selection and a `FeatureIndex` for the
//!   generic engine;
//! * `runtime`: the backend-catalog availability row and diagnostics.

pub mod engine;
pub mod ffi;
pub mod retrieval;
pub mod runtime;

pub use engine::{B200FeatureIndex, RetrievalBackend};
pub use retrieval::{DeviceBuffer, DeviceStream, Engine, GpuRetrievalIndex, Options, RetrievalError};
