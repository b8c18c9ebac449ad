"""GPU parity: libvfr_retrieval.so through its C ABI against the CPU oracle
(restatement of crates/vocal-cpu/src/retrieval.rs:27-83) on the same seeded
inputs.

The bar is bit-exact: distances (reference AVX2 summation order), the top-8
rows with scan-order ties, FAISS labels, and blended features (f64 weights,
f32 blend) must equal the oracle's bits.  The single documented divergence is
the reference CPU error `IVF search selected no candidate`: there the library
follows the reference CUDA kernels and leaves the frame unchanged.
"""
import os

import numpy as np
import pytest

from parity_cases import make_scaled, reference_fixtures, scaled_configs, tie_fixture

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1
ENGINES = ["exact", "auto", "tensor"]


def _engine(name):
    from vfr import lib

    return {"exact": lib.ENGINE_EXACT, "auto": lib.ENGINE_AUTO, "tensor": lib.ENGINE_TENSOR}[name]


def gpu_index(ix, engine="exact", **kw):
    from vfr import GpuRetrievalIndex

    return GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, ix.nprobe,
                                         engine=_engine(engine), **kw)


def oracle_index(oracle, ix):
    return oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, ix.nprobe)


def gpu_blend(cuda, g, q, ratio):
    s = cuda.cuda.Stream()
    feats = cuda.from_numpy(q.copy()).cuda()
    rate = cuda.tensor([ratio], dtype=cuda.float32, device="cuda")
    cuda.cuda.synchronize()  # inputs were staged on the default stream
    with cuda.cuda.stream(s):
        g.blend(feats, q.shape[0], rate, stream=s)
    s.synchronize()
    return feats.cpu().numpy()


def assert_blend_parity(oracle_out, status, gpu_out, queries):
    ok = status == 0
    assert np.array_equal(gpu_out[ok].view(np.uint32), oracle_out[ok].view(np.uint32)), (
        f"max diff {np.abs(gpu_out[ok] - oracle_out[ok]).max()}")
    # no candidate: the CPU reference errors, the library keeps the query
    assert np.array_equal(gpu_out[~ok].view(np.uint32), queries[~ok].view(np.uint32))
    assert set(np.unique(status)) <= {0, 2}


@pytest.mark.parametrize("engine", ENGINES)
@pytest.mark.parametrize("case", [c[0] for c in reference_fixtures()])
@pytest.mark.parametrize("ratio", [0.5, 1.0])
def test_reference_fixture_blend(cuda, oracle, engine, case, ratio):
    name, ix, q = next(c for c in reference_fixtures() if c[0] == case)
    expected, status = oracle_index(oracle, ix).blend(q, ratio, threads=THREADS)
    got = gpu_blend(cuda, gpu_index(ix, engine), q, ratio)
    assert_blend_parity(expected, status, got, q)
    if case == "empty-list":
        assert (status == 2).all()


@pytest.mark.parametrize("engine", ENGINES)
@pytest.mark.parametrize("key", list(scaled_configs()))
def test_scaled_config_blend(cuda, oracle, engine, key):
    ix, q, ratio = make_scaled(key)
    expected, status = oracle_index(oracle, ix).blend(q, ratio, threads=THREADS)
    got = gpu_blend(cuda, gpu_index(ix, engine), q, ratio)
    assert_blend_parity(expected, status, got, q)


@pytest.mark.parametrize("engine", ENGINES)
@pytest.mark.parametrize("key", ["c1", "c3-np8", "c2"])
def test_search_distances_and_labels(cuda, oracle, engine, key):
    ix, q, _ = make_scaled(key)
    dist, rows, labels, count = oracle_index(oracle, ix).search(q, threads=THREADS)
    g = gpu_index(ix, engine)
    s = cuda.cuda.Stream()
    qd = cuda.from_numpy(q).cuda()
    cuda.cuda.synchronize()  # inputs were staged on the default stream
    with cuda.cuda.stream(s):
        gd, gl = g.search(qd, k=8, stream=s)
    s.synchronize()
    gd, gl = gd.cpu().numpy(), gl.cpu().numpy()
    assert np.array_equal(gl, labels)
    assert np.array_equal(gd.view(np.uint32), dist.view(np.uint32))
    cuda.cuda.synchronize()  # inputs were staged on the default stream
    with cuda.cuda.stream(s):
        gd3, gl3 = g.search(qd, k=3, stream=s)
    s.synchronize()
    assert np.array_equal(gl3.cpu().numpy(), labels[:, :3])


def test_ties_resolve_in_scan_order(cuda, oracle):
    ix, q = tie_fixture()
    dist, rows, labels, _ = oracle_index(oracle, ix).search(q, threads=1)
    for engine in ENGINES:
        g = gpu_index(ix, engine)
        s = cuda.cuda.Stream()
        cuda.cuda.synchronize()  # inputs were staged on the default stream
        with cuda.cuda.stream(s):
            gd, gl = g.search(cuda.from_numpy(q).cuda(), stream=s)
        s.synchronize()
        assert np.array_equal(gl.cpu().numpy(), labels), engine
        expected, status = oracle_index(oracle, ix).blend(q, 0.75)
        assert_blend_parity(expected, status, gpu_blend(cuda, g, q, 0.75), q)


def test_dml_fixtures_keep_query_on_empty_list(cuda, oracle):
    """crates/vocal-directml/src/runtime.rs:596-625 queries at ratio 1."""
    from conftest import golden
    from vfr import GpuRetrievalIndex, RetrievalIndex

    queries = np.array([[0, 1], [10, 1.2], [21, 0], [30, 1.5]], np.float32)
    for name in ("ivf-small-probe1.index", "ivf-small-probe2.index"):
        g = GpuRetrievalIndex.upload(RetrievalIndex.from_faiss(golden(name)))
        out = gpu_blend(cuda, g, queries, 1.0)
        expected, status = oracle.OracleIndex.from_faiss(golden(name)).blend(queries, 1.0)
        assert_blend_parity(expected, status, out, queries)
        assert np.abs(out[0] - [0, 1]).max() < 1e-20
        if g.nprobe == 1:
            assert out[2].tolist() == [21.0, 0.0]
            assert g.diagnostics()["empty_frames"] >= 1
        else:
            assert abs(out[2, 0] - 30.0) < 2e-5


@pytest.mark.parametrize("engine", ENGINES)
def test_ratio_zero_and_clamp(cuda, oracle, engine):
    ix, q, _ = make_scaled("c4")
    g = gpu_index(ix, engine)
    for r in (0.0, -1.0, float("nan")):
        out = gpu_blend(cuda, g, q, r)
        assert np.array_equal(out.view(np.uint32), q.view(np.uint32))
    # r > 1 clamps to 1 (reference CUDA kernels, retrieval_block.cuh:30)
    one, status = oracle_index(oracle, ix).blend(q, 1.0, threads=THREADS)
    assert_blend_parity(one, status, gpu_blend(cuda, g, q, 1.7), q)


@pytest.mark.parametrize("engine", ENGINES)
def test_graph_replay_sees_ratio_changes(cuda, oracle, engine):
    """crates/vocal-tensorrt/src/retrieval/tests.rs:36-83: a captured graph
    observes index_rate updates; ratio 0 replays preserve the query bits."""
    import torch

    ix, q, ratio = make_scaled("c4")
    g = gpu_index(ix, engine)
    g.reserve(q.shape[0])
    src = torch.from_numpy(q).cuda()
    feats = src.clone()
    rate = torch.tensor([ratio], dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()  # inputs were staged on the default stream
    with torch.cuda.stream(s):
        g.blend(feats, q.shape[0], rate, stream=s)  # warm-up outside capture
        graph = torch.cuda.CUDAGraph()
        feats.copy_(src)
        with torch.cuda.graph(graph, stream=s):
            g.blend(feats, q.shape[0], rate, stream=s)
        for value in (ratio, 0.0, 0.3):
            rate.fill_(value)
            feats.copy_(src)
            graph.replay()
            s.synchronize()
            out = feats.cpu().numpy()
            if value == 0.0:
                assert np.array_equal(out.view(np.uint32), q.view(np.uint32))
            else:
                expected, status = oracle_index(oracle, ix).blend(q, value, threads=THREADS)
                assert_blend_parity(expected, status, out, q)
    del graph


def test_blend_from_matches_in_place(cuda, oracle):
    import torch

    ix, q, ratio = make_scaled("c1")
    g = gpu_index(ix, "auto")
    src = torch.from_numpy(q).cuda()
    out = torch.empty_like(src)
    rate = torch.tensor([ratio], dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()  # inputs were staged on the default stream
    with torch.cuda.stream(s):
        g.blend_from(src, out, rate, stream=s)
    s.synchronize()
    assert np.array_equal(src.cpu().numpy(), q)  # input untouched
    assert np.array_equal(out.cpu().numpy().view(np.uint32), gpu_blend(cuda, g, q, ratio).view(np.uint32))


def test_argument_errors(cuda):
    import torch
    from vfr import NativeError, lib

    ix, q, _ = make_scaled("c4")
    g = gpu_index(ix, "exact")
    feats = torch.from_numpy(q).cuda()
    rate = torch.tensor([0.5], device="cuda")
    with pytest.raises(NativeError, match="invalid FAISS CUDA stream"):
        g.blend(feats, q.shape[0], rate, stream=torch.cuda.default_stream())
    import ctypes
    s = torch.cuda.Stream()
    st = lib.Stream(ctypes.c_void_p(s.cuda_stream))
    with pytest.raises(NativeError, match="feature width mismatch"):
        lib.call(lib.load_library().vocal_faiss_gpu_blend, g._h, feats.data_ptr(), q.shape[0], 767,
                 rate.data_ptr(), ctypes.byref(st))
    with pytest.raises(ValueError):
        g.blend(feats, q.shape[0] + 1, rate, stream=s)


@pytest.mark.parametrize("engine", ENGINES)
def test_row_sharded_blocks_reproduce_single_index(cuda, oracle, engine):
    """Two row shards on one GPU (the multi-GPU exchange emulated by stacking):
    per-shard search with global labels -> k-way merge -> owned-vector gather
    -> sum over shards -> blend equals the single-index results bitwise."""
    import torch
    from vfr import synth
    from vfr.index import blend_gathered, merge_topk

    ix, q, ratio = make_scaled("c1")
    n = ix.n
    cut = [0, n // 3, n]
    s = torch.cuda.Stream()
    qd = torch.from_numpy(q).cuda()
    rate = torch.tensor([ratio], device="cuda")
    dists, labels, shards = [], [], []
    torch.cuda.synchronize()  # inputs were staged on the default stream
    with torch.cuda.stream(s):
        for a, b in zip(cut[:-1], cut[1:]):
            part = synth.flat_arrays(ix.vectors[a:b])
            g = gpu_index(part, engine, label_base=a)
            shards.append(g)
            d8, l8 = g.search(qd, stream=s)
            dists.append(d8)
            labels.append(l8)
        D = torch.stack(dists).contiguous()
        L = torch.stack(labels).contiguous()
        md = torch.empty_like(D[0])
        ml = torch.empty_like(L[0])
        merge_topk(D, L, md, ml, stream=s)
        # -0.0 is the identity of the sum for every value, -0.0 included
        gathered = torch.full((q.shape[0], 8, q.shape[1]), -0.0, device="cuda")
        for g in shards:
            part = torch.empty_like(gathered)
            g.gather_owned(ml, part, stream=s)
            gathered += part
        out = torch.empty_like(qd)
        blend_gathered(qd, out, md, gathered, rate, stream=s)
    s.synchronize()
    dist, rows, olabels, _ = oracle_index(oracle, ix).search(q, threads=THREADS)
    assert np.array_equal(ml.cpu().numpy(), olabels)
    assert np.array_equal(md.cpu().numpy().view(np.uint32), dist.view(np.uint32))
    expected, status = oracle_index(oracle, ix).blend(q, ratio, threads=THREADS)
    assert_blend_parity(expected, status, out.cpu().numpy(), q)


def test_row_sharded_winner_exchange_on_one_gpu(cuda, oracle):
    """The multi-GPU winner exchange emulated on one GPU with three row
    shards: every shard packs the winners it owns by destination
    (LibraryOps.gather_rows over the compact label list), the receive buffer
    of each destination is assembled source by source as the all-to-all
    delivers it, and vfr_blend_gathered_rows blends each destination's
    frames through its slot -> row map; the concatenated output equals the
    single-index blend bit for bit."""
    import torch
    from vfr.sharded import LibraryOps, _send_labels, _slot_rows, exchange_plan, shard_rows

    ix, q, ratio = make_scaled("c1")
    world = 3
    q = q[:249]  # a multiple of the world size
    m = q.shape[0] // world
    bounds = [shard_rows(ix.n, world, r)[0] for r in range(world)] + [ix.n]
    s = torch.cuda.Stream()
    qd = torch.from_numpy(q).cuda()
    rate = torch.tensor([ratio], device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        ops = [LibraryOps(ix.vectors[bounds[r]:bounds[r + 1]], bounds[r]) for r in range(world)]
        results = [o.search(qd, s) for o in ops]
        md, ml = ops[0].merge(torch.stack([r[0] for r in results]).contiguous(),
                              torch.stack([r[1] for r in results]).contiguous(), s)
        counts, owner = exchange_plan(ml, bounds, world, 0)
        counts = counts.cpu().tolist()
        sends = [o.gather_rows(_send_labels(ml, owner, r, sum(counts[r])), s) for r, o in enumerate(ops)]
        outs = []
        for t in range(world):
            recv = torch.cat([sends[o][sum(counts[o][:t]):sum(counts[o][:t + 1])] for o in range(world)])
            slots = _slot_rows(owner, t, m, world)
            outs.append(ops[t].blend_rows(qd[t * m:(t + 1) * m], md[t * m:(t + 1) * m].contiguous(), recv, slots,
                                          rate, s))
        out = torch.cat(outs)
    s.synchronize()
    expected, status = oracle_index(oracle, ix).blend(q, ratio, threads=THREADS)
    assert_blend_parity(expected, status, out.cpu().numpy(), q)


@pytest.mark.parametrize("key", ["c1", "c3-np1", "c3-np8"])
def test_tensor_core_stage_serves_the_frames(cuda, oracle, key):
    """The certified tensor-core stage (not the exact re-run) settles the
    frames of the seeded configs, flat and IVF, and stays bit-exact."""
    ix, q, ratio = make_scaled(key)
    g = gpu_index(ix, "tensor")
    expected, status = oracle_index(oracle, ix).blend(q, ratio, threads=THREADS)
    assert_blend_parity(expected, status, gpu_blend(cuda, g, q, ratio), q)
    diag = g.diagnostics()
    assert diag["tensor_cores"]
    assert diag["candidate_frames"] >= 0.95 * len(q)
    assert diag["candidate_frames"] + diag["fallback_frames"] == len(q)
