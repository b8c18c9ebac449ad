"""ctypes loader for the CPU oracle (oracle/vfr_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py, never by the product package.  The C code restates
crates/vocal-model/src/retrieval.rs:62-268 (FAISS reader) and
crates/vocal-cpu/src/retrieval.rs:5-83 (search + blend) of the reference.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

OK, ERR_CONFIG, ERR_NO_CANDIDATE = 0, 1, 2


class _Index(ctypes.Structure):
    _fields_ = [
        ("d", ctypes.c_int64),
        ("nprobe", ctypes.c_int64),
        ("nlist", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("centroids", ctypes.POINTER(ctypes.c_float)),
        ("offsets", ctypes.POINTER(ctypes.c_int32)),
        ("vectors", ctypes.POINTER(ctypes.c_float)),
        ("ids", ctypes.POINTER(ctypes.c_int32)),
    ]


def build() -> str:
    """Compiles liboracle.so with the committed Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.POINTER
        L.orc_parse_faiss.argtypes = [ctypes.c_char_p, ctypes.c_size_t, P(_Index), ctypes.c_char_p, ctypes.c_size_t]
        L.orc_parse_faiss.restype = ctypes.c_int
        L.orc_free.argtypes = [P(_Index)]
        L.orc_vfrm_find_faiss.argtypes = [ctypes.c_char_p, ctypes.c_size_t, P(ctypes.c_uint64), P(ctypes.c_uint64)]
        L.orc_vfrm_find_faiss.restype = ctypes.c_int
        for name in ("orc_l2_scalar", "orc_l2_avx2", "orc_l2_lanes"):
            fn = getattr(L, name)
            fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
            fn.restype = ctypes.c_float
        L.orc_blend_row.argtypes = [P(_Index), ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int]
        L.orc_blend_row.restype = ctypes.c_int
        L.orc_blend_batch.argtypes = [P(_Index), ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.orc_blend_batch.restype = ctypes.c_int
        L.orc_search_batch.argtypes = [P(_Index), ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int64,
                                       ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p]
        L.orc_search_batch.restype = ctypes.c_int
        L.orc_protect.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_float,
                                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
        L.orc_protect.restype = None
        L.orc_rvc_frontend.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float,
                                       ctypes.c_float, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.orc_rvc_frontend.restype = ctypes.c_int64
        L.orc_engine_frontend.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float,
                                          ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                          ctypes.c_void_p]
        L.orc_engine_frontend.restype = ctypes.c_int64
        L.orc_kmeans.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                 ctypes.c_int32, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.orc_kmeans.restype = ctypes.c_int
        L.orc_ivf_assign.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                                     ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.orc_ivf_assign.restype = None
        L.orc_view.argtypes = [P(_Index), ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class OracleIndex:
    """Normalised RetrievalIndex arrays as the reference parser produces them.

    Either parsed from FAISS bytes (`from_faiss`) or wrapped from arrays
    (`from_arrays`, no copy beyond contiguity).
    """

    def __init__(self):
        self._c = _Index()
        self._owned = False
        self._keep = ()

    @classmethod
    def from_faiss(cls, data: bytes) -> "OracleIndex":
        L = lib()
        self = cls()
        err = ctypes.create_string_buffer(256)
        rc = L.orc_parse_faiss(data, len(data), ctypes.byref(self._c), err, 256)
        if rc != 0:
            raise ValueError(err.value.decode())
        self._owned = True
        return self

    @classmethod
    def from_arrays(cls, centroids, offsets, vectors, ids, nprobe: int) -> "OracleIndex":
        self = cls()
        c = np.ascontiguousarray(centroids, np.float32)
        o = np.ascontiguousarray(offsets, np.int32)
        v = np.ascontiguousarray(vectors, np.float32)
        i = np.ascontiguousarray(ids, np.int32)
        d = c.shape[1]
        lib().orc_view(ctypes.byref(self._c), d, c.shape[0], int(nprobe), v.shape[0], _ptr(c), _ptr(o), _ptr(v),
                       _ptr(i))
        self._keep = (c, o, v, i)
        return self

    def __del__(self):
        if self._owned and _lib is not None:
            _lib.orc_free(ctypes.byref(self._c))
            self._owned = False

    # accessors mirroring RetrievalIndex (crates/vocal-model/src/retrieval.rs:16-43)
    @property
    def d(self) -> int:
        return int(self._c.d)

    @property
    def nlist(self) -> int:
        return int(self._c.nlist)

    @property
    def nprobe(self) -> int:
        return int(self._c.nprobe)

    def __len__(self) -> int:
        return int(self._c.n)

    def centroids(self) -> np.ndarray:
        return np.ctypeslib.as_array(self._c.centroids, (self.nlist * self.d,)).reshape(self.nlist, self.d).copy()

    def offsets(self) -> np.ndarray:
        return np.ctypeslib.as_array(self._c.offsets, (self.nlist + 1,)).copy()

    def vectors(self) -> np.ndarray:
        n = len(self)
        return np.ctypeslib.as_array(self._c.vectors, (n * self.d,)).reshape(n, self.d).copy()

    def ids(self) -> np.ndarray:
        return np.ctypeslib.as_array(self._c.ids, (len(self),)).copy()

    # the path itself
    def blend(self, feats: np.ndarray, ratio: float, simd: bool = True, threads: int = 1):
        """Reference call site semantics: in place on a copy; returns
        (blended, per-frame status) where status 2 means the reference
        returned `IVF search selected no candidate` for that frame (its row is
        left untouched)."""
        out = np.ascontiguousarray(feats, np.float32).copy()
        frames = out.shape[0]
        status = np.zeros(frames, np.int32)
        lib().orc_blend_batch(ctypes.byref(self._c), _ptr(out), frames, out.shape[1], ctypes.c_float(ratio),
                              int(simd), int(threads), _ptr(status))
        return out, status

    def search(self, queries: np.ndarray, simd: bool = True, nprobe: int = 0, threads: int = 1):
        """Top-8 (squared distance, storage row, FAISS label, count)."""
        q = np.ascontiguousarray(queries, np.float32)
        frames = q.shape[0]
        dist = np.empty((frames, 8), np.float32)
        rows = np.empty((frames, 8), np.int64)
        labels = np.empty((frames, 8), np.int64)
        count = np.empty(frames, np.int32)
        lib().orc_search_batch(ctypes.byref(self._c), _ptr(q), frames, int(simd), int(nprobe), int(threads),
                               _ptr(dist), _ptr(rows), _ptr(labels), _ptr(count))
        return dist, rows, labels, count


def l2(a: np.ndarray, b: np.ndarray, kind: str = "avx2") -> float:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    fn = {"avx2": lib().orc_l2_avx2, "scalar": lib().orc_l2_scalar, "lanes": lib().orc_l2_lanes}[kind]
    return float(fn(_ptr(a), _ptr(b), a.shape[0]))


def vfrm_find_faiss(image: bytes):
    """(offset, length) of aux.retrieval.faiss, None when absent; raises on a
    malformed container."""
    off = ctypes.c_uint64()
    n = ctypes.c_uint64()
    rc = lib().orc_vfrm_find_faiss(image, len(image), ctypes.byref(off), ctypes.byref(n))
    if rc < 0:
        raise ValueError("malformed VFRM container")
    return (off.value, n.value) if rc == 1 else None


def protect(features: np.ndarray, raw: np.ndarray, pitchf: np.ndarray, ratio: float, amount: float,
            hubert_frames: int) -> np.ndarray:
    """Restated protect_features (crates/vocal-tensorrt/native/retrieval_protection.cu:4-16)
    on a copy of `features` [frames][width]; `raw` holds hubert_frames rows."""
    out = np.ascontiguousarray(features, dtype=np.float32).copy()
    raw = np.ascontiguousarray(raw, dtype=np.float32)
    pitchf = np.ascontiguousarray(pitchf, dtype=np.float32)
    frames, width = out.shape
    assert pitchf.shape[0] >= frames and raw.shape[0] >= hubert_frames and raw.shape[1] == width
    lib().orc_protect(_ptr(out), _ptr(raw), _ptr(pitchf), ctypes.c_float(ratio), ctypes.c_float(amount),
                      frames, hubert_frames, width)
    return out


def rvc_frontend(hubert: np.ndarray, raw, f0: np.ndarray, ratio: float, amount: float):
    """Restated frontend.cpp:36-75 plus the protection (raw=None skips it):
    (feats [target][w], pitchf [target], pitch [target] i32, coarse [target]
    unrounded and unclamped)."""
    hubert = np.ascontiguousarray(hubert, dtype=np.float32)
    f0 = np.ascontiguousarray(f0, dtype=np.float32)
    h, w = hubert.shape
    target = min(2 * (h + 1), f0.shape[0])
    feats = np.empty((target, w), np.float32)
    pitchf = np.empty(target, np.float32)
    pitch = np.empty(target, np.int32)
    coarse = np.empty(target, np.float32)
    rawp = None
    if raw is not None:
        raw = np.ascontiguousarray(raw, dtype=np.float32)
        rawp = _ptr(raw)
    got = lib().orc_rvc_frontend(_ptr(hubert), rawp, _ptr(f0), ctypes.c_float(ratio), ctypes.c_float(amount), h,
                                 f0.shape[0], w, _ptr(feats), _ptr(pitchf), _ptr(pitch), _ptr(coarse))
    assert got == target
    return feats, pitchf, pitch, coarse


def engine_frontend(blended: np.ndarray, raw, hz, protect: float):
    """Restated generic-engine frontend (crates/vocal-engine/src/pipeline.rs:
    75-96, 312-333, 625-633): (features [2 frames][w], coarse [min(2 frames,
    len(hz))] i32 or None)."""
    blended = np.ascontiguousarray(blended, dtype=np.float32)
    frames, w = blended.shape
    out = np.empty((2 * frames, w), np.float32)
    rawp = hzp = None
    hz_frames = 0
    coarse = None
    if raw is not None:
        raw = np.ascontiguousarray(raw, dtype=np.float32)
        rawp = _ptr(raw)
    if hz is not None:
        hz = np.ascontiguousarray(hz, dtype=np.float32)
        hzp, hz_frames = _ptr(hz), hz.shape[0]
        coarse = np.empty(min(2 * frames, hz_frames), np.int32)
    got = lib().orc_engine_frontend(_ptr(blended), rawp, hzp, ctypes.c_float(protect), frames, hz_frames, w, _ptr(out),
                                    None if coarse is None else _ptr(coarse))
    assert got == (0 if coarse is None else coarse.shape[0])
    return out, coarse


def kmeans(x: np.ndarray, k: int, niter: int = 10, max_points_per_centroid: int = 256, seed: int = 1234,
           threads: int = 1):
    """Restated vfr_kmeans: (centroids [k][d] f32, objective [niter] f64)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, d = x.shape
    c = np.empty((k, d), np.float32)
    obj = np.empty(max(niter, 1), np.float64)
    rc = lib().orc_kmeans(_ptr(x), n, d, k, niter, max_points_per_centroid, ctypes.c_uint64(seed), _ptr(c), _ptr(obj),
                          threads)
    if rc != 0:
        raise ValueError("invalid k-means arguments")
    return c, obj[:niter]


def ivf_assign(centroids: np.ndarray, x: np.ndarray, threads: int = 1):
    """Restated vfr_ivf_assign: (lists [n] i32, squared distances [n] f32)."""
    c = np.ascontiguousarray(centroids, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, d = x.shape
    lists = np.empty(n, np.int32)
    dist = np.empty(n, np.float32)
    lib().orc_ivf_assign(_ptr(c), c.shape[0], _ptr(x), n, d, _ptr(lists), _ptr(dist), threads)
    return lists, dist
