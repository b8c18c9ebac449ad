//! The runtime-side seam: an availability entry for the backend catalog
//! (crates/vocal-runtime/src/capabilities.rs:184-250 lists backends with
//! `available`, `reason`, `device`, `description`) and the index's
//! diagnostics for the runtime's state reports (crates/vocal-runtime/src/
//! state.rs:1439-1524 builds the engine per backend).

use crate::ffi;
use crate::retrieval::GpuRetrievalIndex;

/// One row of the backend catalog.
#[derive(Clone, Debug)]
pub struct Availability {
    pub available: bool,
    pub reason: Option<String>,
    pub device: Option<String>,
    pub description: String,
}

/// Probes the CUDA devices for compute capability 10.0 (B200, sm_100a, the
/// only target libvfr_retrieval.so is built for).
pub fn availability() -> Availability {
    let description = "GPU feature retrieval (k=8 L2 search + inverse-square blend) on B200 tensor cores; \
                       results bit-identical to the CPU path"
        .to_string();
    let mut count = 0;
    let rc = unsafe { ffi::cudaGetDeviceCount(&mut count) };
    if rc != 0 || count == 0 {
        return Availability {
            available: false,
            reason: Some("no CUDA device is available".into()),
            device: None,
            description,
        };
    }
    for dev in 0..count {
        let (mut major, mut minor) = (0, 0);
        let ok = unsafe {
            ffi::cudaDeviceGetAttribute(&mut major, ffi::CUDA_ATTR_CC_MAJOR, dev) == 0
                && ffi::cudaDeviceGetAttribute(&mut minor, ffi::CUDA_ATTR_CC_MINOR, dev) == 0
        };
        if ok && major == 10 && minor == 0 {
            return Availability {
                available: true,
                reason: None,
                device: Some(format!("CUDA device {dev} (sm_100)")),
                description,
            };
        }
    }
    Availability {
        available: false,
        reason: Some("no compute capability 10.0 (B200) device; this library is built for sm_100a only".into()),
        device: None,
        description,
    }
}

/// The index's diagnostics (engine, tensor-core layout, last plan, empty /
/// re-run / certified frames, bounded-wait timeouts) for runtime reports.
pub fn diagnostics(index: &GpuRetrievalIndex) -> serde_json::Value {
    index.diagnostics()
}
