"""Re-runs of uncertified frames (the exact kernel behind the tensor-core
engine).  Frames whose candidate set cannot be certified -- here more than
kRerankMax rows at exactly the same distance -- are re-run exactly; when at
most 64 frames fall back, each frame's probed rows are split across many
CTAs and the slices' top-8 lists merged (exact_split), otherwise one CTA
scans each frame.  400 frames put the merge on its one-warp-per-frame form.  Both must give the reference's results bit for bit:
search (distances, scan-order ties, labels) and blend against the oracle
(crates/vocal-cpu/src/retrieval.rs:27-83), flat and IVF.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def tie_heavy(n, d, nlist, seed, copies=150, clusters=3):
    """Random rows plus `clusters` rows repeated `copies` times each, so a
    query next to one of them has >kRerankMax exactly tied neighbours."""
    from vfr import synth

    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((n, d), dtype=np.float32)
    tied = rng.standard_normal((clusters, d), dtype=np.float32) * 3
    pos = rng.choice(n, clusters * copies, replace=False)
    rows[pos] = np.repeat(tied, copies, axis=0)
    if nlist == 1:
        ix = synth.flat_arrays(rows)
    else:
        centroids = rows[rng.choice(n, nlist, replace=False)].copy()
        ix = synth.ivf_arrays(rows, centroids, 1)
    return ix, tied, rng


@pytest.mark.parametrize("nlist,nprobe", [(1, 1), (16, 4), (16, 8), (16, 16)])
@pytest.mark.parametrize("frames,tied_frames", [(40, 10), (70, 70), (12, 1), (400, 100)])
def test_rerun_matches_oracle(cuda, oracle, nlist, nprobe, frames, tied_frames):
    from vfr import GpuRetrievalIndex, lib

    ix, tied, rng = tie_heavy(60_000, 64, nlist, 100 + nlist + frames)
    q = rng.standard_normal((frames, 64), dtype=np.float32)
    sel = rng.choice(frames, tied_frames, replace=False)
    q[sel] = tied[rng.integers(0, len(tied), tied_frames)] + np.float32(1e-3)
    g = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, nprobe, engine=lib.ENGINE_TENSOR)
    o = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, nprobe)
    torch = cuda
    s = torch.cuda.Stream()
    dq = torch.from_numpy(q).cuda()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        gd, gl = g.search(dq, stream=s)
    s.synchronize()
    dist, _, labels, count = o.search(q, threads=8)
    assert np.array_equal(gl.cpu().numpy(), labels)
    assert np.array_equal(gd.cpu().numpy().view(np.uint32), dist.view(np.uint32))
    # nprobe > 8 runs on the exact engine from the start: nothing falls back
    tensor_path = nprobe <= 8
    before = g.diagnostics()["fallback_frames"]
    assert before >= tied_frames if tensor_path else before == 0
    feats = torch.from_numpy(q.copy()).cuda()
    rate = torch.tensor([0.75], device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        g.blend(feats, frames, rate, stream=s)
    s.synchronize()
    expected, status = o.blend(q, 0.75, threads=8)
    ok = status == 0
    assert np.array_equal(feats.cpu().numpy()[ok].view(np.uint32), expected[ok].view(np.uint32))
    if tensor_path:
        assert g.diagnostics()["fallback_frames"] - before >= tied_frames
    g.close()


def crowded_ivf(n, d, nlist, seed, crowd=40, near=3, filler=2000):
    """An IVF index where list 0 holds a crowd of `crowd` rows all within a
    hair of a point b (far closer together than the candidate stage's error
    bound), list 1 holds `near` rows closer still to b, and both lists also
    hold `filler` far rows.  A query at b finds its exact top 8 as the
    `near` rows plus crowd rows; list 0 keeps only 16 of the crowd, so its
    threshold cannot certify the frame, while list 1's can."""
    from vfr import synth

    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((n, d), dtype=np.float32)
    b = rng.standard_normal(d).astype(np.float32) * 3
    u = rng.standard_normal(d).astype(np.float32)
    centroids = rows[rng.choice(n, nlist, replace=False)].copy()
    centroids[0] = b + np.float32(0.1) * u
    centroids[1] = b - np.float32(0.1) * u
    rows[:crowd] = b + np.float32(0.01) * rng.standard_normal((crowd, d), dtype=np.float32)
    rows[crowd:crowd + near] = b + np.float32(0.005) * rng.standard_normal((near, d), dtype=np.float32)
    lists = synth.assign_np(centroids, rows)
    lists[:crowd] = 0
    lists[crowd:crowd + near] = 1
    far = crowd + near + rng.choice(n - crowd - near, 2 * filler, replace=False)
    lists[far[:filler]] = 0
    lists[far[filler:]] = 1
    return synth.ivf_arrays(rows, centroids, 1, lists=lists), b, rng


@pytest.mark.parametrize("nprobe", [4, 8])
@pytest.mark.parametrize("frames,crowded", [(48, 12), (120, 100)])
def test_partial_rerun_matches_oracle(cuda, oracle, nprobe, frames, crowded):
    """Frames that fail only on one list's threshold are re-run on that
    probe's rows alone (at most 64 such frames: the split re-run), with the
    other probes' re-ranked top 8 handed over by the merge; with more, every
    frame is rescanned in full.  Bit-exact against the oracle either way, and
    the re-run's row count shows which happened."""
    from vfr import GpuRetrievalIndex, lib

    torch = cuda
    d = 64
    ix, b, rng = crowded_ivf(60_000, d, 16, 7 + frames + nprobe)
    q = rng.standard_normal((frames, d), dtype=np.float32)
    sel = rng.choice(frames, crowded, replace=False)
    q[sel] = b + np.float32(1e-4) * rng.standard_normal((crowded, d), dtype=np.float32)
    g = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, nprobe, engine=lib.ENGINE_TENSOR)
    o = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, nprobe)
    s = torch.cuda.Stream()
    dq = torch.from_numpy(q).cuda()
    before = g.diagnostics()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        gd, gl = g.search(dq, stream=s)
    s.synchronize()
    after = g.diagnostics()
    dist, _, labels, _ = o.search(q, threads=8)
    assert np.array_equal(gl.cpu().numpy(), labels)
    assert np.array_equal(gd.cpu().numpy().view(np.uint32), dist.view(np.uint32))
    # the crowded frames' top 8: the near rows first, then crowd rows
    assert np.isin(labels[sel][:, :3], [40, 41, 42]).all()
    fell_back = after["fallback_frames"] - before["fallback_frames"]
    assert fell_back == crowded
    sizes = np.diff(ix.offsets)
    cd = ((ix.centroids - b) ** 2).sum(1)
    full = int(sizes[np.argsort(cd, kind="stable")[:nprobe]].sum())  # the crowded frames' probed rows
    scanned = after["rerun_rows"] - before["rerun_rows"]
    if crowded <= 64:
        assert scanned < crowded * full
        assert scanned <= crowded * (sizes[0] + sizes[1])
    else:
        assert scanned == crowded * full
    feats = torch.from_numpy(q.copy()).cuda()
    rate = torch.tensor([0.75], device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        g.blend(feats, frames, rate, stream=s)
    s.synchronize()
    expected, status = o.blend(q, 0.75, threads=8)
    assert (status == 0).all()
    assert np.array_equal(feats.cpu().numpy().view(np.uint32), expected.view(np.uint32))
    assert g.diagnostics()["fallback_frames"] - after["fallback_frames"] == crowded
    g.close()
