"""ctypes binding of libvfr_retrieval.so (include/vfr_retrieval.h).

The library is built in-tree (vocal-fast-rs_b200/build.py) and loaded from
there; there is no fallback implementation, so a missing or stale library is
an error.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "libvfr_retrieval.so")
HEADER = os.path.join(PKG, "..", "include", "vfr_retrieval.h")

ENGINE_AUTO, ENGINE_EXACT, ENGINE_TENSOR = 0, 1, 2
SHARD_ROWS, SHARD_QUERIES = 0, 1
SHARE_STORAGE = 1  # VfrOptions.flags: VFR_SHARE_STORAGE

_lib = None


class NativeError(RuntimeError):
    """A non-zero return code from the library, with its message
    (the role of NativeBuildError::Api, crates/vocal-tensorrt/src/retrieval.rs:69-86)."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class Options(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_int32),
        ("engine", ctypes.c_int32),
        ("candidates", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("label_base", ctypes.c_int64),
        ("max_frames", ctypes.c_int64),
    ]


class Stream(ctypes.Structure):
    _fields_ = [("stream", ctypes.c_void_p)]


class IpcRows(ctypes.Structure):
    """VfrIpcRows: one shard's row storage as other processes map it."""
    _fields_ = [
        ("rows_handle", ctypes.c_uint8 * 64),
        ("ids_handle", ctypes.c_uint8 * 64),
        ("label_base", ctypes.c_int64),
        ("rows", ctypes.c_int64),
        ("width", ctypes.c_int32),
        ("has_ids", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


def declared_symbols() -> list[str]:
    """Function names declared in include/vfr_retrieval.h."""
    text = open(HEADER).read()
    return re.findall(r"^VFR_API [^;(]*?\b([a-z_][a-z0-9_]*)\(", text, re.M)


def load_library(path: str | None = None):
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise OSError(f"libvfr_retrieval.so not built at {path}; run vocal-fast-rs_b200/build.py")
    L = ctypes.CDLL(path)
    P = ctypes.POINTER
    vp, sz, i32, i64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_int64
    err = P(ctypes.c_char_p)
    sig = {
        "vocal_faiss_gpu_create": ([i32, i32, i32, sz, vp, sz, vp, sz, vp, sz, vp, sz, P(vp), err], ctypes.c_int),
        "vocal_faiss_gpu_destroy": ([vp], None),
        "vocal_faiss_gpu_blend": ([vp, vp, sz, i32, vp, P(Stream), err], ctypes.c_int),
        "vocal_retrieval_protect": ([vp, vp, vp, vp, vp, i32, i32, i32, P(Stream), err], ctypes.c_int),
        "vfr_rvc_frontend": ([vp, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp, P(i32), P(Stream), err], ctypes.c_int),
        "vfr_engine_frontend": ([vp, vp, vp, ctypes.c_float, i32, i32, i32, vp, vp, P(Stream), err], ctypes.c_int),
        "vfr_retrieval_blend_save_raw": ([vp, vp, vp, sz, i32, vp, P(Stream), err], ctypes.c_int),
        "vfr_free_error": ([vp], None),
        "vfr_index_parse_faiss": ([ctypes.c_char_p, sz, P(vp), err], ctypes.c_int),
        "vfr_index_from_vfrm": ([ctypes.c_char_p, sz, i32, P(vp), err], ctypes.c_int),
        "vfr_index_free": ([vp], None),
        "vfr_index_info": ([vp, P(i32), P(i32), P(i32), P(i64)], None),
        "vfr_index_centroids": ([vp], vp),
        "vfr_index_offsets": ([vp], vp),
        "vfr_index_vectors": ([vp], vp),
        "vfr_index_ids": ([vp], vp),
        "vfr_index_upload": ([vp, P(vp), err], ctypes.c_int),
        "vfr_index_load": ([vp, sz, P(Options), P(vp), err], ctypes.c_int),
        "vfr_index_load_vfrm": ([vp, sz, i32, P(Options), P(vp), err], ctypes.c_int),
        "vfr_index_load_file": ([ctypes.c_char_p, i32, P(Options), P(vp), err], ctypes.c_int),
        "vfr_index_content_hash": ([vp, sz, vp, err], ctypes.c_int),
        "vfr_kmeans": ([vp, i64, i32, i32, i32, i32, ctypes.c_uint64, vp, vp, P(Stream), err], ctypes.c_int),
        "vfr_ivf_assign": ([vp, i32, vp, i64, i32, vp, vp, P(Stream), err], ctypes.c_int),
        "vfr_ivf_build": ([vp, i32, vp, i64, i32, i32, P(Options), P(vp), err], ctypes.c_int),
        "vfr_ivf_write": ([vp, i32, vp, i64, i32, vp, i32, vp, sz, P(sz), err], ctypes.c_int),
        "vfr_retrieval_create": ([i32, i32, i32, sz, vp, sz, vp, sz, vp, sz, vp, sz, P(Options), P(vp), err],
                                 ctypes.c_int),
        "vfr_retrieval_reserve": ([vp, sz, err], ctypes.c_int),
        "vfr_retrieval_search": ([vp, vp, sz, i32, i32, vp, vp, P(Stream), err], ctypes.c_int),
        "vfr_retrieval_blend_from": ([vp, vp, vp, sz, i32, vp, P(Stream), err], ctypes.c_int),
        "vfr_retrieval_diagnostics": ([vp, ctypes.c_char_p, sz], sz),
        "vfr_retrieval_blend_noalloc": ([vp, vp, sz, i32, vp, P(Stream), err], ctypes.c_int),
        "vfr_retrieval_profile": ([vp, i32, ctypes.c_char_p, sz], sz),
        "vfr_merge_topk": ([vp, vp, i32, sz, vp, vp, P(Stream), err], ctypes.c_int),
        "vfr_gather_owned": ([vp, vp, sz, vp, P(Stream), err], ctypes.c_int),
        "vfr_blend_gathered": ([vp, vp, vp, vp, sz, i32, vp, P(Stream), err], ctypes.c_int),
        "vfr_blend_gathered_rows": ([vp, vp, vp, vp, sz, vp, sz, i32, vp, P(Stream), err], ctypes.c_int),
        "vfr_index_ipc_export": ([vp, P(IpcRows), err], ctypes.c_int),
        "vfr_peer_rows_open": ([vp, i32, P(IpcRows), i32, P(vp), err], ctypes.c_int),
        "vfr_peer_rows_close": ([vp], None),
        "vfr_blend_peer": ([vp, vp, vp, vp, vp, sz, i32, vp, P(Stream), err], ctypes.c_int),
        "vfr_selftest_bounded_wait": ([ctypes.c_uint64, i32, P(i32), P(ctypes.c_uint64), err], ctypes.c_int),
        "vfr_retrieval_create_sharded": ([i32, P(i32), i32, i32, i32, i32, sz, vp, sz, vp, sz, vp, sz, vp, sz,
                                          P(Options), P(vp), err], ctypes.c_int),
        "vfr_retrieval_destroy_sharded": ([vp], None),
        "vfr_retrieval_search_sharded": ([vp, vp, sz, i32, i32, vp, vp, P(Stream), err], ctypes.c_int),
        "vfr_retrieval_blend_sharded": ([vp, vp, vp, sz, i32, vp, P(Stream), err], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def call(fn, *args):
    """Invokes a fallible entry point, translating rc/error into NativeError."""
    L = load_library()
    e = ctypes.c_char_p()
    rc = fn(*args, ctypes.byref(e))
    if rc != 0:
        msg = e.value.decode() if e.value else "native retrieval call failed"
        if e.value:
            L.vfr_free_error(ctypes.cast(e, ctypes.c_void_p))
        raise NativeError(rc, msg)
    return rc


def stream_struct(stream=None) -> Stream:
    """VfrStream for a torch CUDA stream (default: the current stream)."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return Stream(ctypes.c_void_p(s.cuda_stream))
