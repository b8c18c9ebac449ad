"""IVF training on the device over libvfr_retrieval.so.

The reference builds its IVF-Flat indexes offline with FAISS
(`IndexIVFFlat.train` + `add`; crates/vocal-directml/tests/fixtures/README.md,
scripts/benchmark-retrieval.py:56-65).  `train_ivf` does the same on the GPU
and returns the FAISS bytes any reader of the format (the reference's
`RetrievalIndex::from_faiss` included) loads; `build_ivf_index` skips the
bytes and builds the device index directly.  Results are deterministic for a
given seed.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import lib as _l
from .lib import call, load_library, stream_struct


def _ptr(t) -> int:
    return t.data_ptr()


def _check_rows(x):
    import torch

    if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.float32 and x.dim() == 2
            and x.is_contiguous()):
        raise ValueError("expected a contiguous CUDA float32 tensor [rows, width]")


def _stream(stream):
    """The call's stream: a side stream ordered after the current one when
    none is given (the library's calls here return after their work)."""
    import torch

    if stream is not None:
        return stream
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    return side


def kmeans(x, k: int, niter: int = 10, max_points_per_centroid: int = 256, seed: int = 1234, stream=None):
    """(centroids [k, d] CUDA tensor, objective per iteration as numpy f64)."""
    import torch

    _check_rows(x)
    n, d = x.shape
    centroids = torch.empty((k, d), dtype=torch.float32, device=x.device)
    objective = np.zeros(max(niter, 1), np.float64)
    s = stream_struct(_stream(stream))
    call(load_library().vfr_kmeans, _ptr(x), n, d, int(k), int(niter), int(max_points_per_centroid),
         ctypes.c_uint64(seed), _ptr(centroids), objective.ctypes.data, ctypes.byref(s))
    return centroids, objective[:niter]


def assign(centroids, x, stream=None):
    """(lists [n] int32, squared distances [n] float32), CUDA tensors."""
    import torch

    _check_rows(x)
    _check_rows(centroids)
    n, d = x.shape
    lists = torch.empty(n, dtype=torch.int32, device=x.device)
    dist = torch.empty(n, dtype=torch.float32, device=x.device)
    s = stream_struct(_stream(stream))
    call(load_library().vfr_ivf_assign, _ptr(centroids), centroids.shape[0], _ptr(x), n, d, _ptr(lists), _ptr(dist),
         ctypes.byref(s))
    return lists, dist


def write_ivf(centroids: np.ndarray, x: np.ndarray, lists: np.ndarray, nprobe: int = 1) -> bytes:
    """FAISS IndexIVFFlat bytes from host arrays (`vfr_ivf_write`)."""
    c = np.ascontiguousarray(centroids, dtype=np.float32)
    v = np.ascontiguousarray(x, dtype=np.float32)
    lst = np.ascontiguousarray(lists, dtype=np.int32)
    L = load_library()
    size = ctypes.c_size_t(0)
    args = (c.ctypes.data, c.shape[0], v.ctypes.data, v.shape[0], v.shape[1], lst.ctypes.data, int(nprobe))
    call(L.vfr_ivf_write, *args, None, 0, ctypes.byref(size))
    out = np.empty(size.value, np.uint8)
    call(L.vfr_ivf_write, *args, out.ctypes.data, out.size, ctypes.byref(size))
    return out.tobytes()


def train_ivf(x, nlist: int, nprobe: int = 1, niter: int = 10, max_points_per_centroid: int = 256, seed: int = 1234,
              stream=None) -> bytes:
    """IndexIVFFlat(train + add) of the rows of `x` (CUDA float32 [n, d]):
    FAISS IwFl bytes, labels the row numbers."""
    centroids, _ = kmeans(x, nlist, niter, max_points_per_centroid, seed, stream)
    lists, _ = assign(centroids, x, stream)
    return write_ivf(centroids.cpu().numpy(), x.cpu().numpy(), lists.cpu().numpy(), nprobe)


def build_ivf_index(x, centroids, nprobe: int = 1, engine: int = _l.ENGINE_AUTO, candidates: int = 0,
                    label_base: int = 0, max_frames: int = 0):
    """A GpuRetrievalIndex with every row of `x` in the list of its nearest
    centroid (`vfr_ivf_build`), without a host round trip."""
    import torch

    from .index import GpuRetrievalIndex

    _check_rows(x)
    _check_rows(centroids)
    n, d = x.shape
    torch.cuda.current_stream().synchronize()  # the build runs on its own stream
    out = ctypes.c_void_p()
    opt = _l.Options(ctypes.sizeof(_l.Options), engine, candidates, 0, label_base, max_frames)
    call(load_library().vfr_ivf_build, _ptr(centroids), centroids.shape[0], _ptr(x), n, d, int(nprobe),
         ctypes.byref(opt), ctypes.byref(out))
    return GpuRetrievalIndex(out.value, d, centroids.shape[0], int(nprobe), n)
