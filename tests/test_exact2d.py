"""The 2-D exact engine (small IVF batches under the default engine) against
the oracle, bit for bit: search distances and labels, and the blend.

Cases: the stand-in for the reference's published shape (IVF511,Flat, 19,949
x 768, nprobe 1, blocks of 34 and 140 frames, ratio 0.5 --
docs/faiss-gpu-retrieval.md:59-79 of the reference), the same index probed
at nprobe 8, an index with more than 1,024 lists (so a lane of the merging
warp owns several coarse slices), and ratio 0 / empty probed lists.  The
engine that served each call is read back from vfr_retrieval_diagnostics.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module")
def ivf511(cuda):
    from vfr import synth

    arrays, q = synth.make_torch("ivf511", "cuda", q=140)
    ix = synth.IndexArrays(arrays["centroids"].cpu().numpy(), arrays["offsets"].cpu().numpy(),
                           arrays["vectors"].cpu().numpy(), arrays["ids"].cpu().numpy(), 1)
    return ix, q.cpu().numpy()


def _run(torch, ix, q, ratio, nprobe, engine=None):
    from vfr import GpuRetrievalIndex, lib

    g = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, nprobe,
                                      engine=lib.ENGINE_AUTO if engine is None else engine)
    s = torch.cuda.Stream()
    qd = torch.from_numpy(np.ascontiguousarray(q)).cuda()
    feats = qd.clone()
    rate = torch.tensor([ratio], device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        gd, gl = g.search(qd, stream=s)
        g.blend(feats, q.shape[0], rate, stream=s)
    s.synchronize()
    return g, gd.cpu().numpy(), gl.cpu().numpy(), feats.cpu().numpy()


def _check(oracle, ix, q, ratio, nprobe, gd, gl, out):
    o = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, nprobe)
    dist, _, labels, _ = o.search(q, threads=THREADS)
    expected, status = o.blend(q, ratio, threads=THREADS)
    assert np.array_equal(gl, labels)
    assert np.array_equal(gd.view(np.uint32), dist.view(np.uint32))
    ok = status == 0
    assert np.array_equal(out[ok].view(np.uint32), expected[ok].view(np.uint32))
    # no candidate (every probed list empty): the reference CPU errors, the
    # library keeps the frame
    assert np.array_equal(out[~ok].view(np.uint32), q[~ok].view(np.uint32))
    return status


@pytest.mark.parametrize("frames", [34, 140])
@pytest.mark.parametrize("nprobe", [1, 8])
def test_published_shape_blocks(cuda, oracle, ivf511, frames, nprobe):
    ix, q = ivf511
    q = q[:frames]
    g, gd, gl, out = _run(cuda, ix, q, 0.5, nprobe)
    # the published shape (nprobe 1) always fits the 2-D engine; at nprobe 8
    # the 140-frame block reads enough rows to go to the tensor-core path
    engine = g.diagnostics()["last_engine"]
    assert engine == "exact2d" if nprobe == 1 or frames == 34 else engine in ("exact2d", "tensor")
    _check(oracle, ix, q, 0.5, nprobe, gd, gl, out)
    g.close()


def test_empty_lists_keep_the_frame(cuda, oracle, ivf511):
    """Frames placed on the centroids of empty lists (the stand-in index has
    some): at nprobe 1 their probed list is empty and the frame is kept."""
    ix, q = ivf511
    sizes = np.diff(ix.offsets)
    empty = np.flatnonzero(sizes == 0)
    assert len(empty) > 0
    qq = np.concatenate([ix.centroids[empty[:8]], q[:24]]).astype(np.float32)
    g, gd, gl, out = _run(cuda, ix, qq, 0.5, 1)
    status = _check(oracle, ix, qq, 0.5, 1, gd, gl, out)
    assert (status[: min(8, len(empty))] == 2).all()
    assert g.diagnostics()["empty_frames"] >= min(8, len(empty))
    g.close()


def test_many_lists(cuda, oracle):
    """1,100 lists (35 coarse slices): the coarse merge where a lane holds
    several slices' lists, at nprobe 4."""
    from vfr import synth

    rng = np.random.default_rng(77)
    x = rng.standard_normal((6000, 96), dtype=np.float32)
    centroids = x[rng.choice(len(x), 1100, replace=False)].copy()
    ix = synth.ivf_arrays(x, centroids, 4)
    q = rng.standard_normal((50, 96), dtype=np.float32)
    q[0] = x[10]  # an exact match
    g, gd, gl, out = _run(cuda, ix, q, 0.75, 4)
    assert g.diagnostics()["last_engine"] == "exact2d"
    _check(oracle, ix, q, 0.75, 4, gd, gl, out)
    g.close()


def test_ratio_zero_leaves_frames(cuda, ivf511):
    ix, q = ivf511
    q = q[:34]
    g, _, _, out = _run(cuda, ix, q, 0.0, 1)
    assert np.array_equal(out.view(np.uint32), q.view(np.uint32))
    g.close()


def test_graph_replay_and_reserve(cuda, oracle, ivf511):
    """Reserved up front, captured in a CUDA graph, replayed with a changed
    ratio (device scalar): equal to the oracle at the new ratio."""
    torch = cuda
    from vfr import GpuRetrievalIndex

    ix, q = ivf511
    q = q[:140]
    g = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1, max_frames=140)
    rate = torch.tensor([0.5], device="cuda")
    src = torch.from_numpy(q).cuda()
    feats = src.clone()
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            g.blend(feats, 140, rate, stream=s)
        rate.fill_(0.8)
        feats.copy_(src)
        graph.replay()
    s.synchronize()
    del graph
    o = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1)
    expected, status = o.blend(q, 0.8, threads=THREADS)
    out = feats.cpu().numpy()
    ok = status == 0
    assert np.array_equal(out[ok].view(np.uint32), expected[ok].view(np.uint32))
    g.close()
