"""IVF training on the device (`vfr_kmeans`, `vfr_ivf_assign`,
`vfr_ivf_build`, `vfr_ivf_write`): the offline FAISS step of the reference
(IndexIVFFlat::train + add; crates/vocal-directml/tests/fixtures/README.md,
scripts/benchmark-retrieval.py:56-65).  FAISS is not vendored by the
reference, so the trainer is deterministic by design and parity is pinned to
the CPU restatement in oracle/vfr_oracle.c, itself checked here against an
independent numpy statement and against the reference's IVF fixture.

CPU: the oracle's k-means against numpy (sampling, initial centroids, exact
assignment, fixed-point means, empty-cluster splits); the FAISS writer
byte-identical to the test writer (tests' faiss_io, FAISS's layout) and read
back by the parser; argument errors.
GPU: centroids and objectives bit-exact against the oracle (with and without
sampling, d = 768, forced splits), assignments bit-exact, the directly built
index equal to loading the written bytes, the reference fixture's lists
reproduced.
"""
import ctypes

import numpy as np
import pytest

from conftest import golden


def _splitmix(state):
    mask = (1 << 64) - 1
    state = (state + 0x9E3779B97F4A7C15) & mask
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
    return state, z ^ (z >> 31)


def _prefix(n, m, seed):
    p = list(range(n))
    st = seed
    for i in range(m):
        st, r = _splitmix(st)
        j = i + r % (n - i)
        p[i], p[j] = p[j], p[i]
    return p[:m]


def numpy_kmeans(x, k, niter, max_ppc, seed, oracle):
    """An independent statement of the trainer (distances from the oracle's
    avx2_l2 restatement)."""
    n, d = x.shape
    m = k * max_ppc if max_ppc > 0 and n > k * max_ppc else n
    train = x[_prefix(n, m, seed)] if m < n else x
    c = train[_prefix(m, k, seed + 1)].copy()
    maxabs = float(np.abs(train).max())
    e = int(np.frexp(np.float32(maxabs))[1])
    bits = 0
    while (1 << bits) < m:
        bits += 1
    s = 62 - bits - e
    scale, inv = 2.0 ** s, 2.0 ** -s
    q = np.rint(train.astype(np.float64) * scale).astype(np.int64)
    split = seed + 2
    objs = []
    for _ in range(niter):
        dist = np.array([[oracle.l2(row, cj) for cj in c] for row in train], np.float32)
        lists = dist.argmin(axis=1)
        objs.append(float(sum(float(v) for v in dist[np.arange(m), lists])))
        counts = np.bincount(lists, minlength=k)
        sums = np.zeros((k, d), np.int64)
        np.add.at(sums, lists, q)
        with np.errstate(invalid="ignore", divide="ignore"):
            means = ((sums.astype(np.float64) / counts[:, None]) * inv).astype(np.float32)
        c = np.where(counts[:, None] > 0, means, np.float32(0.0)).astype(np.float32)
        w = counts.astype(np.float64)
        for ci in range(k):
            if w[ci] != 0:
                continue
            cj, found = 0, False
            for _t in range(64 * k + 1024):
                p = (w[cj] - 1.0) / float(m - k) if m != k else (np.inf if w[cj] > 1 else np.nan)
                split, r = _splitmix(split)
                if float(np.float32((r >> 40) * 2.0 ** -24)) < p:
                    found = True
                    break
                cj = (cj + 1) % k
            if not found:
                cj = int(np.argmax(w))
            c[ci] = c[cj]
            up, down = np.float32(1 + 1 / 1024), np.float32(1 - 1 / 1024)
            even = np.arange(d) % 2 == 0
            c[ci] = np.where(even, c[ci] * up, c[ci] * down)
            c[cj] = np.where(even, c[cj] * down, c[cj] * up)
            w[ci] = w[cj] / 2.0
            w[cj] -= w[ci]
    return c, np.array(objs)


@pytest.mark.parametrize("n,d,k,niter,max_ppc", [(120, 7, 5, 4, 0), (300, 9, 4, 3, 40), (40, 3, 8, 5, 0)])
def test_oracle_kmeans_matches_numpy_statement(oracle, n, d, k, niter, max_ppc):
    rng = np.random.default_rng(n + d + k)
    x = rng.standard_normal((n, d), dtype=np.float32)
    if n == 40:
        x = np.repeat(x[:5], 8, axis=0)  # five distinct rows, eight clusters: splits
    want_c, want_obj = numpy_kmeans(x, k, niter, max_ppc, 77, oracle)
    c, obj = oracle.kmeans(x, k, niter, max_ppc, 77)
    assert np.array_equal(c.view(np.uint32), want_c.view(np.uint32))
    assert np.array_equal(obj, want_obj)


@pytest.mark.parametrize("sizes_kind", ["full", "sprs"])
def test_writer_matches_faiss_layout(oracle, sizes_kind):
    from vfr import RetrievalIndex, faiss_io
    from vfr.training import write_ivf

    rng = np.random.default_rng(4)
    k, n, d = 12, 200, 5
    c = rng.standard_normal((k, d), dtype=np.float32)
    v = rng.standard_normal((n, d), dtype=np.float32)
    lists = rng.integers(0, k if sizes_kind == "full" else 4, n).astype(np.int32)
    got = write_ivf(c, v, lists, nprobe=3)
    assert got == faiss_io.ivf_bytes(c, v, 3, lists=lists)
    ix = RetrievalIndex.from_faiss(got)
    assert ix.nprobe() == 3 and np.array_equal(ix.centroids(), c)
    order = np.argsort(lists, kind="stable")
    assert np.array_equal(ix.ids(), order) and np.array_equal(ix.vectors(), v[order])


def test_writer_reproduces_reference_fixture():
    """The reference's ivf-small fixtures (fixtures/README.md): centroids
    (0,0),(10,0),(20,0),(30,0), rows added to their nearest list."""
    from vfr.training import write_ivf

    c = np.array([[0, 0], [10, 0], [20, 0], [30, 0]], np.float32)
    v = np.array([[0, 1], [0, 2], [10, 1], [10, 2], [30, 1], [30, 2]], np.float32)
    lists = np.array([0, 0, 1, 1, 3, 3], np.int32)
    for probes in (1, 2):
        assert write_ivf(c, v, lists, nprobe=probes) == golden(f"ivf-small-probe{probes}.index")


def test_oracle_assignment_reproduces_fixture_lists(oracle):
    c = np.array([[0, 0], [10, 0], [20, 0], [30, 0]], np.float32)
    v = np.array([[0, 1], [0, 2], [10, 1], [10, 2], [30, 1], [30, 2]], np.float32)
    lists, dist = oracle.ivf_assign(c, v)
    assert lists.tolist() == [0, 0, 1, 1, 3, 3] and dist.tolist() == [1, 4, 1, 4, 1, 4]
    # ties go to the lower centroid
    lists, _ = oracle.ivf_assign(c, np.array([[5, 0], [25, 0]], np.float32))
    assert lists.tolist() == [0, 2]


def test_trainer_argument_errors():
    from vfr import lib

    L = lib.load_library()
    s = lib.Stream(None)
    p = ctypes.c_void_p(16)
    with pytest.raises(lib.NativeError, match="invalid FAISS CUDA stream"):
        lib.call(L.vfr_kmeans, p, 10, 4, 2, 1, 0, ctypes.c_uint64(1), p, None, ctypes.byref(s))
    size = ctypes.c_size_t(0)
    c = np.zeros((2, 2), np.float32)
    bad = np.array([0, 2], np.int32)
    with pytest.raises(lib.NativeError, match="out of range"):
        lib.call(L.vfr_ivf_write, c.ctypes.data, 2, c.ctypes.data, 2, 2, bad.ctypes.data, 1, None, 0,
                 ctypes.byref(size))
    with pytest.raises(lib.NativeError, match="invalid IVF write arguments"):
        lib.call(L.vfr_ivf_write, c.ctypes.data, 2, c.ctypes.data, 2, 2, bad.ctypes.data, 3, None, 0,
                 ctypes.byref(size))


# ------------------------------------------------------------------- GPU


@pytest.mark.gpu
@pytest.mark.parametrize("n,d,k,niter,max_ppc", [(20000, 64, 64, 8, 256), (50000, 32, 32, 6, 256),
                                                 (4000, 768, 16, 5, 0), (3000, 7, 40, 6, 0)])
def test_kmeans_bit_exact_against_oracle(cuda, oracle, n, d, k, niter, max_ppc):
    from vfr.training import assign, kmeans

    torch = cuda
    rng = np.random.default_rng(n + k)
    means = rng.standard_normal((max(4, k // 2), d), dtype=np.float32) * 3
    x = (means[rng.integers(0, means.shape[0], n)] + 0.3 * rng.standard_normal((n, d), dtype=np.float32))
    if d == 7:
        x = np.repeat(x[:25], n // 25, axis=0)  # 25 distinct rows for 40 clusters: splits every iteration
    x = np.ascontiguousarray(x, dtype=np.float32)
    want_c, want_obj = oracle.kmeans(x, k, niter, max_ppc, 1234, threads=8)
    dx = torch.from_numpy(x).cuda()
    c, obj = kmeans(dx, k, niter, max_ppc, 1234)
    assert np.array_equal(c.cpu().numpy().view(np.uint32), want_c.view(np.uint32))
    assert np.array_equal(obj, want_obj)
    lists, dist = assign(c, dx)
    want_lists, want_dist = oracle.ivf_assign(want_c, x, threads=8)
    assert np.array_equal(lists.cpu().numpy(), want_lists)
    assert np.array_equal(dist.cpu().numpy().view(np.uint32), want_dist.view(np.uint32))


@pytest.mark.gpu
def test_build_equals_loading_written_bytes(cuda):
    from vfr import GpuRetrievalIndex
    from vfr.training import assign, build_ivf_index, kmeans, write_ivf

    torch = cuda
    rng = np.random.default_rng(12)
    x = rng.standard_normal((30000, 128), dtype=np.float32)
    dx = torch.from_numpy(x).cuda()
    c, _ = kmeans(dx, 50, 5)
    lists, _ = assign(c, dx)
    data = write_ivf(c.cpu().numpy(), x, lists.cpu().numpy(), nprobe=4)
    loaded = GpuRetrievalIndex.load(data)
    built = build_ivf_index(dx, c, nprobe=4)
    q = x[:300] + 0.05 * rng.standard_normal((300, 128), dtype=np.float32)
    for g in (loaded, built):
        assert g.diagnostics()["nlist"] == 50
    outs = []
    s = torch.cuda.Stream()
    for g in (loaded, built):
        dq = torch.from_numpy(q).cuda()
        rate = torch.tensor([0.75], device="cuda")
        torch.cuda.synchronize()
        with torch.cuda.stream(s):
            g.blend(dq, q.shape[0], rate, stream=s)
            dist, labels = g.search(torch.from_numpy(q).cuda(), stream=s)
        s.synchronize()
        outs.append((dq.cpu().numpy(), dist.cpu().numpy(), labels.cpu().numpy()))
    for a, b in zip(*outs):
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8))
    loaded.close()
    built.close()


@pytest.mark.gpu
def test_train_ivf_fixture_and_errors(cuda):
    from vfr import lib
    from vfr.training import assign, build_ivf_index, kmeans, write_ivf

    torch = cuda
    c = torch.tensor([[0, 0], [10, 0], [20, 0], [30, 0]], dtype=torch.float32, device="cuda")
    v = np.array([[0, 1], [0, 2], [10, 1], [10, 2], [30, 1], [30, 2]], np.float32)
    lists, _ = assign(c, torch.from_numpy(v).cuda())
    assert write_ivf(c.cpu().numpy(), v, lists.cpu().numpy(), 2) == golden("ivf-small-probe2.index")
    g = build_ivf_index(torch.from_numpy(v).cuda(), c, nprobe=2)
    assert g.diagnostics()["vectors"] == 6
    g.close()
    with pytest.raises(lib.NativeError, match="at least as large as number of clusters"):
        kmeans(torch.zeros((3, 4), device="cuda"), 4)
    bad = torch.zeros((10, 4), device="cuda")
    bad[3, 1] = float("nan")
    with pytest.raises(lib.NativeError, match="non-finite training vector"):
        kmeans(bad, 2)
    with pytest.raises(lib.NativeError, match="invalid FAISS GPU IVF configuration"):
        build_ivf_index(torch.from_numpy(v).cuda(), c, nprobe=5)
