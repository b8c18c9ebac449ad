"""C-ABI boundary checks that need no GPU: the library loads, exports every
entry point declared in include/vfr_retrieval.h, and the argument validation
of the drop-in entry points (crates/vocal-tensorrt/native/retrieval.cu:42-59,
100-105) fails with the reference's messages and error convention
(bridge.h:24-32: rc 1 + malloc'd message)."""
import ctypes

import numpy as np
import pytest


def test_exports_every_declared_symbol(native):
    from vfr import lib

    declared = lib.declared_symbols()
    assert len(declared) >= 21
    for name in declared:
        assert hasattr(native, name), name
    for name in ("vocal_faiss_gpu_create", "vocal_faiss_gpu_destroy", "vocal_faiss_gpu_blend"):
        assert name in declared


def _create(native, d=4, nlist=1, nprobe=1, n=3, centroid_count=None, offsets=None, vec_count=None, id_count=None):
    c = np.zeros(nlist * d, np.float32)
    o = np.array(offsets if offsets is not None else [0] + [n] * nlist, np.int32)
    v = np.zeros(max(n * d, 1), np.float32)
    i = np.arange(max(n, 1), dtype=np.int32)
    out = ctypes.c_void_p()
    err = ctypes.c_char_p()
    rc = native.vocal_faiss_gpu_create(d, nlist, nprobe, n, c.ctypes.data,
                                       c.size if centroid_count is None else centroid_count, o.ctypes.data, o.size,
                                       v.ctypes.data, n * d if vec_count is None else vec_count, i.ctypes.data,
                                       n if id_count is None else id_count, ctypes.byref(out), ctypes.byref(err))
    msg = err.value.decode() if err.value else None
    if err.value:
        native.vfr_free_error(ctypes.cast(err, ctypes.c_void_p))
    return rc, msg, out.value


@pytest.mark.parametrize("kwargs,message", [
    (dict(d=0), "invalid FAISS GPU index dimension"),
    (dict(d=4097), "invalid FAISS GPU index dimension"),
    (dict(nlist=2, nprobe=3), "invalid FAISS GPU IVF configuration"),
    (dict(nlist=40, nprobe=33), "invalid FAISS GPU IVF configuration"),
    (dict(n=0), "invalid FAISS GPU vector count"),
    (dict(centroid_count=3), "invalid FAISS centroid payload"),
    (dict(vec_count=5), "invalid FAISS vector payload"),
    (dict(id_count=2), "invalid FAISS id payload"),
    (dict(offsets=[0, 2]), "FAISS list offsets do not cover vectors"),
    (dict(nlist=2, offsets=[0, 3, 2, 9]), "invalid FAISS list offsets"),
])
def test_create_validation(native, kwargs, message):
    rc, msg, handle = _create(native, **kwargs)
    assert rc == 1 and msg == message and not handle


def test_non_monotone_offsets(native):
    rc, msg, _ = _create(native, nlist=2, offsets=[0, 3, 3])
    # offsets cover n=3 and are monotone: that one is valid up to the device
    # step; a decreasing pair is rejected before any CUDA call
    rc, msg, _ = _create(native, nlist=3, n=3, offsets=[0, 2, 1, 3])
    assert rc == 1 and msg == "FAISS list offsets are not monotonic"


def test_blend_argument_validation(native):
    from vfr import lib

    err = ctypes.c_char_p()
    s = lib.Stream(ctypes.c_void_p(0))
    rc = native.vocal_faiss_gpu_blend(None, None, 0, 768, None, ctypes.byref(s), ctypes.byref(err))
    assert rc == 1 and err.value.decode() == "invalid FAISS GPU blend arguments"
    native.vfr_free_error(ctypes.cast(err, ctypes.c_void_p))
    # diagnostics of a null handle is a no-op
    assert native.vfr_retrieval_diagnostics(None, None, 0) == 0


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_reports(cuda):
    """The bounded mbarrier wait every kernel of the library uses: waiting on
    a barrier nothing completes returns a timeout status after the limit
    (the context stays usable), and a completed phase returns at once."""
    import ctypes

    from vfr import lib

    L = lib.load_library()
    flag, ns = ctypes.c_int32(-1), ctypes.c_uint64(0)
    lib.call(L.vfr_selftest_bounded_wait, 50_000_000, 0, ctypes.byref(flag), ctypes.byref(ns))
    assert flag.value == 1
    assert 50_000_000 <= ns.value < 1_000_000_000
    lib.call(L.vfr_selftest_bounded_wait, 50_000_000, 1, ctypes.byref(flag), ctypes.byref(ns))
    assert flag.value == 0 and ns.value < 50_000_000
    # the device still runs work afterwards
    t = cuda.arange(8, device="cuda", dtype=cuda.float32)
    assert float(t.sum().item()) == 28.0
