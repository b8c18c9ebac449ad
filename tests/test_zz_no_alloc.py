"""The no-allocation blend (vfr_retrieval_blend_noalloc) against the
allocating drop-in entry point (vocal_faiss_gpu_blend), through the C ABI.

The no-allocation entry point serves callers that cannot call cudaMalloc
during a call (a realtime audio callback, a fixed device-memory budget): its
scratch is a static device array shared by all calls.  Two calls in a row,
with different frames and frame counts, must each equal the allocating entry
point bit for bit (the tolerance of every parity test here), so nothing left
in the shared scratch by one call leaks into the next.  This file is collected
last so a failure here comes after every other test has run.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call_blend(fn, index, feats, rate, stream):
    from vfr import lib

    err = ctypes.c_char_p()
    s = lib.Stream(ctypes.c_void_p(stream.cuda_stream))
    rc = fn(index._h, feats.data_ptr(), feats.shape[0], feats.shape[1], rate.data_ptr(), ctypes.byref(s),
            ctypes.byref(err))
    msg = err.value.decode() if err.value else ""
    if err.value:
        lib.load_library().vfr_free_error(ctypes.cast(err, ctypes.c_void_p))
    return rc, msg


def test_noalloc_blend_matches_allocating_blend_twice(cuda):
    torch = cuda
    from vfr import GpuRetrievalIndex, lib, synth

    L = lib.load_library()
    ix, q = synth.make_np("c1", n=20_000, q=140 + 34)
    g = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1)
    assert g.diagnostics()["tensor_cores"]
    rate = torch.tensor([0.75], device="cuda")
    stream = torch.cuda.Stream()
    for frames in (q[:140], q[140:]):  # an RVC 140-frame block, then a 34-frame one
        src = torch.from_numpy(np.ascontiguousarray(frames)).cuda()
        expected = src.clone()
        got = src.clone()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            assert _call_blend(L.vocal_faiss_gpu_blend, g, expected, rate, stream) == (0, "")
            assert _call_blend(L.vfr_retrieval_blend_noalloc, g, got, rate, stream) == (0, "")
        stream.synchronize()
        e, o = expected.cpu().numpy(), got.cpu().numpy()
        assert not np.array_equal(e, frames)  # the blend did change the frames
        assert np.array_equal(o.view(np.uint32), e.view(np.uint32))


def _two_calls_match(torch, L, g, q, rate, stream, splits):
    """For each frame range in `splits` (two calls in a row): the allocating
    blend and the no-allocation blend of the same frames agree bit for bit."""
    for lo, hi in splits:
        src = torch.from_numpy(np.ascontiguousarray(q[lo:hi])).cuda()
        expected = src.clone()
        got = src.clone()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            assert _call_blend(L.vocal_faiss_gpu_blend, g, expected, rate, stream) == (0, "")
            assert _call_blend(L.vfr_retrieval_blend_noalloc, g, got, rate, stream) == (0, "")
        stream.synchronize()
        e, o = expected.cpu().numpy(), got.cpu().numpy()
        assert not np.array_equal(e, q[lo:hi])
        assert np.array_equal(o.view(np.uint32), e.view(np.uint32))
    return g.diagnostics()["last_plan"]


@pytest.mark.parametrize("rows,frames,keep,layout", [
    (260_000, 256, 16, "full"),   # 16 candidates per list, 73 segments x 2 frame tiles
    (492_000, 128, 16, "full"),   # exactly the 148-work-item cap: the key region is full
    (492_000, 16, 16, "spread"),  # a small block (spread A layout) with long work items
    (100_000, 32, 8, "spread"),   # a realtime block against c4's database size
])
def test_noalloc_blend_plans_at_the_scratch_limits(cuda, rows, frames, keep, layout):
    torch = cuda
    from vfr import GpuRetrievalIndex, lib, synth

    L = lib.load_library()
    arrays, q = synth.make_torch("c4", "cuda", n=rows, q=2 * frames)
    g = GpuRetrievalIndex.from_arrays(arrays["centroids"], arrays["offsets"], arrays["vectors"], arrays["ids"], 1)
    del arrays
    q = q.cpu().numpy()
    rate = torch.tensor([0.75], device="cuda")
    stream = torch.cuda.Stream()
    plan = _two_calls_match(torch, L, g, q, rate, stream, [(0, frames), (frames, 2 * frames)])
    assert plan["keep"] == keep and plan["layout"] == layout, plan
    if rows == 492_000 and frames == 128:
        assert plan["segments"] == 148, plan
    g.close()


def test_noalloc_blend_allocates_no_device_memory(cuda):
    """A fresh index that only ever sees the no-allocation entry point keeps
    no workspace, and device free memory does not move across its calls
    (after one warm-up call, which may load kernel code on first use)."""
    torch = cuda
    from vfr import GpuRetrievalIndex, lib, synth

    L = lib.load_library()
    ix, q = synth.make_np("c1", n=30_000, q=3 * 64)
    g = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1)
    rate = torch.tensor([0.75], device="cuda")
    stream = torch.cuda.Stream()
    bufs = [torch.from_numpy(np.ascontiguousarray(q[i * 64:(i + 1) * 64])).cuda() for i in range(3)]
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        assert _call_blend(L.vfr_retrieval_blend_noalloc, g, bufs[0], rate, stream) == (0, "")
    stream.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    with torch.cuda.stream(stream):
        for b in bufs[1:]:
            assert _call_blend(L.vfr_retrieval_blend_noalloc, g, b, rate, stream) == (0, "")
    stream.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    diag = g.diagnostics()
    assert diag["workspace_bytes"] == 0 and diag["workspace_frames"] == 0, diag
    g.close()


def test_noalloc_blend_rejects_what_it_cannot_hold(cuda):
    torch = cuda
    from vfr import GpuRetrievalIndex, lib, synth

    L = lib.load_library()
    ix, q = synth.make_np("c1", n=4096, q=257)
    g = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1)
    rate = torch.tensor([0.75], device="cuda")
    stream = torch.cuda.Stream()
    feats = torch.from_numpy(q).cuda()
    torch.cuda.synchronize()
    rc, msg = _call_blend(L.vfr_retrieval_blend_noalloc, g, feats, rate, stream)
    assert rc == 1 and "at most 256 frames" in msg
    exact = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1, engine=lib.ENGINE_EXACT)
    rc, msg = _call_blend(L.vfr_retrieval_blend_noalloc, exact, feats[:8].contiguous(), rate, stream)
    assert rc == 1 and "tensor-core layout" in msg
