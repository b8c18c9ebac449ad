"""Host-side mirror of the reference retrieval interface over libvfr_retrieval.so.

The compute lives in the CUDA library (csrc/); this package only binds its C
ABI (include/vfr_retrieval.h) with ctypes and mirrors the reference's Rust
types:

* `RetrievalIndex` - crates/vocal-model/src/retrieval.rs:6-57 (parse FAISS /
  VFRM bytes into normalised arrays; the parsing itself runs in the library).
* `GpuRetrievalIndex` - crates/vocal-tensorrt/src/retrieval.rs:19-171
  (device-resident index, `blend` in place with a device ratio scalar).
* `ShardedRetrievalIndex` - one handle over several GPUs of this process
  (row or query sharding; no counterpart in the single-GPU reference).
"""
from .lib import NativeError, load_library  # noqa: F401
from .index import GpuRetrievalIndex, RetrievalIndex, ShardedRetrievalIndex, validate_blend_buffers  # noqa: F401
