"""Python mirror of the reference's retrieval types over the C ABI.

`RetrievalIndex` mirrors crates/vocal-model/src/retrieval.rs:6-57: bytes in,
normalised arrays out (the bounded reader runs in the library).
`GpuRetrievalIndex` mirrors crates/vocal-tensorrt/src/retrieval.rs:19-171:
device-resident index with `blend(features, frames, index_rate, stream)` in
place, plus `search` and `blend_from`.  Device buffers are torch CUDA tensors
(plumbing only); every computation is a library call.
"""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np

from . import lib as _l
from .lib import NativeError, call, load_library, stream_struct


def validate_blend_buffers(frames: int, dimensions: int, feature_bytes: int, rate_bytes: int) -> None:
    """crates/vocal-tensorrt/src/retrieval.rs:147-165: buffer-capacity checks
    before the C-ABI call (NativeBuildError::Argument -> ValueError)."""
    int32_max = 2**31 - 1
    required = frames * dimensions * 4
    if frames > int32_max or required > 2**64 - 1 or required > feature_bytes or rate_bytes < 4:
        raise ValueError("retrieval shape exceeds CUDA grid or buffer capacity")


class RetrievalIndex:
    """Parsed FAISS Flat/IVF-Flat index (host arrays, owned by the library)."""

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)
        L = load_library()
        d, nl, npb, n = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
        L.vfr_index_info(self._h, ctypes.byref(d), ctypes.byref(nl), ctypes.byref(npb), ctypes.byref(n))
        self._d, self._nlist, self._nprobe, self._n = d.value, nl.value, npb.value, n.value

    @classmethod
    def from_faiss(cls, data) -> "RetrievalIndex":
        """bytes, or any contiguous buffer (numpy uint8, memoryview)."""
        L = load_library()
        out = ctypes.c_void_p()
        if not isinstance(data, bytes):
            view = np.ascontiguousarray(np.frombuffer(data, np.uint8) if not isinstance(data, np.ndarray)
                                        else data.reshape(-1).view(np.uint8))
            data = ctypes.cast(view.ctypes.data, ctypes.c_char_p) if view.size else b""
            call(L.vfr_index_parse_faiss, data, view.size, ctypes.byref(out))
        else:
            call(L.vfr_index_parse_faiss, data, len(data), ctypes.byref(out))
        return cls(out.value)

    @classmethod
    def from_package(cls, image: bytes, feature_dims: int = 0) -> "RetrievalIndex | None":
        """Index stored in a VFRM image as aux.retrieval.faiss, or None."""
        L = load_library()
        out = ctypes.c_void_p()
        call(L.vfr_index_from_vfrm, image, len(image), int(feature_dims), ctypes.byref(out))
        return cls(out.value) if out.value else None

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value and _l._lib is not None:
            _l._lib.vfr_index_free(self._h)
            self._h = ctypes.c_void_p()

    def dimensions(self) -> int:
        return self._d

    def nlist(self) -> int:
        return self._nlist

    def nprobe(self) -> int:
        return self._nprobe

    def __len__(self) -> int:
        return self._n

    def is_empty(self) -> bool:
        return self._n == 0

    def _array(self, fn, count, dtype, shape=None):
        ptr = fn(self._h)
        ctype = ctypes.c_float if dtype == np.float32 else ctypes.c_int32
        a = np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctype)), (count,)).copy()
        return a.reshape(shape) if shape else a

    def centroids(self) -> np.ndarray:
        return self._array(load_library().vfr_index_centroids, self._nlist * self._d, np.float32,
                           (self._nlist, self._d))

    def offsets(self) -> np.ndarray:
        return self._array(load_library().vfr_index_offsets, self._nlist + 1, np.int32)

    def vectors(self) -> np.ndarray:
        return self._array(load_library().vfr_index_vectors, self._n * self._d, np.float32, (self._n, self._d))

    def ids(self) -> np.ndarray:
        return self._array(load_library().vfr_index_ids, self._n, np.int32)


def _ptr(t) -> int:
    return t.data_ptr()


class GpuRetrievalIndex:
    """Device-resident retrieval index (one per GPU / shard).

    Construct from a `RetrievalIndex` (`upload`) or from arrays (`from_arrays`,
    numpy on the host or torch tensors on the device: the library copies them).
    """

    def __init__(self, handle: int, d: int, nlist: int, nprobe: int, n: int):
        self._h = ctypes.c_void_p(handle)
        self.d, self.nlist, self.nprobe, self.n = d, nlist, nprobe, n

    @classmethod
    def upload(cls, index: RetrievalIndex) -> "GpuRetrievalIndex":
        if index.is_empty():
            raise ValueError("retrieval index has no vectors")
        L = load_library()
        out = ctypes.c_void_p()
        call(L.vfr_index_upload, index._h, ctypes.byref(out))
        return cls(out.value, index.dimensions(), index.nlist(), index.nprobe(), len(index))

    @classmethod
    def load(cls, source, feature_dims: int = 0, engine: int = _l.ENGINE_AUTO, candidates: int = 0,
             label_base: int = 0, max_frames: int = 0, share: bool = False) -> "GpuRetrievalIndex | None":
        """Device ingest of a FAISS index or a VFRM package (`vfr_index_load`,
        `vfr_index_load_vfrm`, `vfr_index_load_file`): `source` is a path or
        a bytes-like image (bytes, bytearray, memoryview, numpy uint8).  The
        rows go from the image to the device without a host copy; errors are
        the parser's (`RetrievalIndex.from_faiss`).  None when a VFRM package
        has no retrieval index.  `share=True` shares the device arrays with
        other handles loaded from the same bytes on this device."""
        L = load_library()
        out = ctypes.c_void_p()
        opt = _l.Options(ctypes.sizeof(_l.Options), engine, candidates, _l.SHARE_STORAGE if share else 0,
                         label_base, max_frames)
        if isinstance(source, (str, os.PathLike)):
            call(L.vfr_index_load_file, os.fsencode(source), int(feature_dims), ctypes.byref(opt), ctypes.byref(out))
        else:
            view = np.frombuffer(source, dtype=np.uint8) if not isinstance(source, np.ndarray) else source
            view = np.ascontiguousarray(view.reshape(-1).view(np.uint8))
            ptr = view.ctypes.data if view.size else None
            if view.size >= 4 and bytes(view[:4]) == b"VFRM":
                call(L.vfr_index_load_vfrm, ptr, view.size, int(feature_dims), ctypes.byref(opt), ctypes.byref(out))
            else:
                call(L.vfr_index_load, ptr, view.size, ctypes.byref(opt), ctypes.byref(out))
        if not out.value:
            return None
        g = cls(out.value, 0, 0, 0, 0)
        diag = g.diagnostics()
        g.d, g.nlist, g.nprobe, g.n = diag["dimensions"], diag["nlist"], diag["nprobe"], diag["vectors"]
        return g

    @classmethod
    def from_arrays(cls, centroids, offsets, vectors, ids, nprobe: int, engine: int = _l.ENGINE_AUTO,
                    candidates: int = 0, label_base: int = 0, max_frames: int = 0, drop_in: bool = False):
        """`drop_in=True` calls the reference-named vocal_faiss_gpu_create."""
        L = load_library()
        keep = []

        def host(a, dtype):
            if hasattr(a, "data_ptr"):  # torch tensor: copy to host (create takes host arrays)
                a = a.detach().cpu().numpy()
            a = np.ascontiguousarray(a, dtype)
            keep.append(a)
            return a

        c = host(centroids, np.float32)
        o = host(offsets, np.int32)
        v = host(vectors, np.float32)
        i = host(ids, np.int32)
        d = c.shape[-1] if c.ndim == 2 else int(v.shape[-1])
        nlist = o.size - 1
        n = i.size
        out = ctypes.c_void_p()
        args = (int(d), int(nlist), int(nprobe), n, c.ctypes.data, c.size, o.ctypes.data, o.size, v.ctypes.data,
                v.size, i.ctypes.data, i.size)
        if drop_in:
            call(L.vocal_faiss_gpu_create, *args, ctypes.byref(out))
        else:
            opt = _l.Options(ctypes.sizeof(_l.Options), engine, candidates, 0, label_base, max_frames)
            call(L.vfr_retrieval_create, *args, ctypes.byref(opt), ctypes.byref(out))
        return cls(out.value, int(d), int(nlist), int(nprobe), int(n))

    def __del__(self):
        self.close()

    def close(self):
        if getattr(self, "_h", None) and self._h.value and _l._lib is not None:
            _l._lib.vocal_faiss_gpu_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __len__(self):
        return self.n

    # -- the path -------------------------------------------------------------
    def blend(self, features, frames: int, index_rate, stream=None) -> None:
        """In place, as GpuRetrievalIndex::blend (retrieval.rs:111-145).
        `features` is a CUDA f32 tensor holding at least frames*d values;
        `index_rate` a CUDA f32 tensor with at least one element."""
        if frames == 0:
            return
        validate_blend_buffers(frames, self.d, features.numel() * features.element_size(),
                               index_rate.numel() * index_rate.element_size())
        L = load_library()
        s = stream_struct(stream)
        call(L.vocal_faiss_gpu_blend, self._h, _ptr(features), frames, self.d, _ptr(index_rate), ctypes.byref(s))

    def blend_save_raw(self, features, raw, frames: int, index_rate, stream=None) -> None:
        """`blend` with RetrievalProtection::save_raw fused in
        (crates/vocal-tensorrt/src/pipeline.rs:1842-1853): `raw` (a CUDA f32
        tensor of at least frames*d values) receives the frames as they are
        before the blend."""
        if frames == 0:
            return
        validate_blend_buffers(frames, self.d, features.numel() * features.element_size(),
                               index_rate.numel() * index_rate.element_size())
        if raw.numel() < frames * self.d:
            raise ValueError("raw feature buffer is smaller than frames x width")
        L = load_library()
        s = stream_struct(stream)
        call(L.vfr_retrieval_blend_save_raw, self._h, _ptr(features), _ptr(raw), frames, self.d, _ptr(index_rate),
             ctypes.byref(s))

    def blend_from(self, queries, out, index_rate, stream=None) -> None:
        frames = queries.shape[0]
        if frames == 0:
            return
        validate_blend_buffers(frames, self.d, out.numel() * out.element_size(),
                               index_rate.numel() * index_rate.element_size())
        L = load_library()
        s = stream_struct(stream)
        call(L.vfr_retrieval_blend_from, self._h, _ptr(queries), _ptr(out), frames, self.d, _ptr(index_rate),
             ctypes.byref(s))

    def search(self, queries, k: int = 8, stream=None):
        """(distances [Q,k] f32, labels [Q,k] i64) as CUDA tensors."""
        import torch

        frames = queries.shape[0]
        dist = torch.empty((frames, k), dtype=torch.float32, device=queries.device)
        labels = torch.empty((frames, k), dtype=torch.int64, device=queries.device)
        if frames:
            L = load_library()
            s = stream_struct(stream)
            call(L.vfr_retrieval_search, self._h, _ptr(queries), frames, self.d, int(k), _ptr(dist), _ptr(labels),
                 ctypes.byref(s))
        return dist, labels

    def reserve(self, max_frames: int) -> None:
        call(load_library().vfr_retrieval_reserve, self._h, int(max_frames))

    def diagnostics(self) -> dict:
        L = load_library()
        need = L.vfr_retrieval_diagnostics(self._h, None, 0)
        buf = ctypes.create_string_buffer(need + 1)
        L.vfr_retrieval_diagnostics(self._h, buf, need + 1)
        return json.loads(buf.value.decode())

    def profile(self, enable: bool) -> dict:
        """Per-kernel CUDA-event times recorded since the last call; `enable`
        starts (True) or stops (False) recording from now on."""
        L = load_library()
        buf = ctypes.create_string_buffer(4096)  # one call: reading also resets
        need = L.vfr_retrieval_profile(self._h, int(enable), buf, 4096)
        if need >= 4096:
            raise RuntimeError("profile report truncated")
        return json.loads(buf.value.decode())

    # -- row-sharded helpers ----------------------------------------------------
    def gather_owned(self, labels, out, stream=None) -> None:
        L = load_library()
        s = stream_struct(stream)
        call(L.vfr_gather_owned, self._h, _ptr(labels), labels.shape[0], _ptr(out), ctypes.byref(s))


def merge_topk(dist, labels, out_dist, out_labels, stream=None) -> None:
    """dist/labels [shards, Q, 8] -> out [Q, 8] by (distance, label)."""
    L = load_library()
    s = stream_struct(stream)
    call(L.vfr_merge_topk, _ptr(dist), _ptr(labels), dist.shape[0], dist.shape[1], _ptr(out_dist), _ptr(out_labels),
         ctypes.byref(s))


def blend_gathered(queries, out, dist, neighbours, index_rate, stream=None) -> None:
    L = load_library()
    s = stream_struct(stream)
    call(L.vfr_blend_gathered, _ptr(queries), _ptr(out), _ptr(dist), _ptr(neighbours), queries.shape[0],
         queries.shape[1], _ptr(index_rate), ctypes.byref(s))


def blend_gathered_rows(queries, out, dist, rows, slot_rows, index_rate, stream=None) -> None:
    """vfr_blend_gathered over a compact row buffer: slot (f, k) reads
    rows[slot_rows[f, k]] (int32 CUDA tensor [frames, 8])."""
    L = load_library()
    s = stream_struct(stream)
    call(L.vfr_blend_gathered_rows, _ptr(queries), _ptr(out), _ptr(dist), _ptr(rows) if rows.numel() else 0,
         rows.shape[0], _ptr(slot_rows), queries.shape[0], queries.shape[1], _ptr(index_rate), ctypes.byref(s))


class ShardedRetrievalIndex:
    """One handle over several GPUs of this process (vfr_retrieval_*_sharded):
    `mode` SHARD_ROWS splits a flat index's rows across `devices` (results
    equal a single index's bit for bit), SHARD_QUERIES gives every device a
    replica and a share of the frames.  Frames, outputs, the ratio and the
    stream belong to devices[0]."""

    def __init__(self, handle: int, d: int, devices, mode: int):
        self._h = ctypes.c_void_p(handle)
        self.d = d
        self.devices = list(devices)
        self.mode = mode

    @classmethod
    def from_arrays(cls, devices, mode, centroids, offsets, vectors, ids, nprobe: int, engine: int = _l.ENGINE_AUTO,
                    max_frames: int = 0):
        L = load_library()
        keep = []

        def host(a, dtype):
            if hasattr(a, "data_ptr"):
                a = a.detach().cpu().numpy()
            a = np.ascontiguousarray(a, dtype)
            keep.append(a)
            return a

        c = host(centroids, np.float32)
        o = host(offsets, np.int32)
        v = host(vectors, np.float32)
        i = host(ids, np.int32)
        dev = (ctypes.c_int32 * len(devices))(*devices)
        d = c.shape[-1] if c.ndim == 2 else int(v.shape[-1])
        out = ctypes.c_void_p()
        opt = _l.Options(ctypes.sizeof(_l.Options), engine, 0, 0, 0, max_frames)
        call(L.vfr_retrieval_create_sharded, len(devices), dev, int(mode), int(d), int(o.size - 1), int(nprobe),
             i.size, c.ctypes.data, c.size, o.ctypes.data, o.size, v.ctypes.data, v.size, i.ctypes.data, i.size,
             ctypes.byref(opt), ctypes.byref(out))
        return cls(out.value, int(d), devices, mode)

    def __del__(self):
        self.close()

    def close(self):
        if getattr(self, "_h", None) and self._h.value and _l._lib is not None:
            _l._lib.vfr_retrieval_destroy_sharded(self._h)
            self._h = ctypes.c_void_p()

    def search(self, queries, k: int = 8, stream=None):
        """(distances [Q,k] f32, labels [Q,k] i64) on devices[0]."""
        import torch

        frames = queries.shape[0]
        dist = torch.empty((frames, k), dtype=torch.float32, device=queries.device)
        labels = torch.empty((frames, k), dtype=torch.int64, device=queries.device)
        if frames:
            s = stream_struct(stream)
            call(load_library().vfr_retrieval_search_sharded, self._h, _ptr(queries), frames, self.d, int(k),
                 _ptr(dist), _ptr(labels), ctypes.byref(s))
        return dist, labels

    def blend_from(self, queries, out, index_rate, stream=None) -> None:
        frames = queries.shape[0]
        if frames:
            s = stream_struct(stream)
            call(load_library().vfr_retrieval_blend_sharded, self._h, _ptr(queries), _ptr(out), frames, self.d,
                 _ptr(index_rate), ctypes.byref(s))
