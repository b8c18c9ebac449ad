"""Seeded synthetic retrieval workloads with the shapes of the benchmark configs.

No public dataset is involved: every database is an isotropic Gaussian
mixture (component means ~ N(0,1)^d, within-component sigma 0.3), queries are
drawn from the same mixture plus N(0, 0.1) noise, and streaming blocks are a
random walk (step N(0, 0.05)) from the previous block.  IVF coarse centroids
come from seeded Lloyd k-means.  The numpy path (CPU, tests) and the torch path
(device, benchmark) use the same formulas and seeds but different generators,
so they produce different - individually deterministic - data.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class Workload:
    key: str
    name: str
    n: int
    d: int
    q: int
    components: int
    ratio: float
    nlist: int = 1
    nprobe: tuple = (1,)
    kmeans_iters: int = 0
    blocks: int = 1
    walk: float = 0.0
    extra: dict = field(default_factory=dict)


CONFIGS = {
    "c1": Workload("c1", "rvc-v2-flat-20k", 20_000, 768, 250, 256, 0.75),
    "c2": Workload("c2", "rvc-v1-flat-50k", 50_000, 256, 1_000, 512, 0.5),
    "c3": Workload("c3", "rvc-v2-ivf-200k", 200_000, 768, 30_000, 1_024, 0.75, nlist=256, nprobe=(1, 8),
                   kmeans_iters=20),
    "c4": Workload("c4", "rvc-v2-stream-100k", 100_000, 768, 32, 512, 0.75, blocks=1_000, walk=0.05),
    "c5": Workload("c5", "rvc-v2-flat-4m", 4_000_000, 768, 30_000, 4_096, 0.75),
    # Stand-in for the one shape the reference publishes timings on
    # (docs/faiss-gpu-retrieval.md:59-79: a real IVF511,Flat nprobe=1 index of
    # 19,949 768-d vectors, blocks of 34 and 140 frames, ratio 0.5): seeded
    # mixture rows, 511 lists from 20 seeded k-means iterations.
    "ivf511": Workload("ivf511", "rvc-v2-ivf511-20k", 19_949, 768, 140, 256, 0.5, nlist=511, nprobe=(1,),
                       kmeans_iters=20, extra={"blocks": (34, 140)}),
}

_SEEDS = {"ivf511": (1511, 2511, 3511)}

SIGMA = 0.3
QUERY_NOISE = 0.1


def seeds(key: str):
    if key in _SEEDS:
        return _SEEDS[key]
    c = int(key[1:])
    return 1000 + c, 2000 + c, 3000 + c


# --------------------------------------------------------------------------- numpy
def mixture_np(n: int, d: int, components: int, seed: int, chunk: int = 65536):
    rng = np.random.default_rng(seed)
    means = rng.standard_normal((components, d), dtype=np.float32)
    x = np.empty((n, d), np.float32)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        comp = rng.integers(0, components, m)
        x[s:s + m] = means[comp] + np.float32(SIGMA) * rng.standard_normal((m, d), dtype=np.float32)
    return x, means


def queries_np(means: np.ndarray, q: int, seed: int):
    rng = np.random.default_rng(seed)
    comp = rng.integers(0, means.shape[0], q)
    d = means.shape[1]
    out = means[comp] + np.float32(SIGMA) * rng.standard_normal((q, d), dtype=np.float32)
    out += np.float32(QUERY_NOISE) * rng.standard_normal((q, d), dtype=np.float32)
    return out


def walk_np(block: np.ndarray, step: float, seed: int):
    rng = np.random.default_rng(seed)
    return block + np.float32(step) * rng.standard_normal(block.shape, dtype=np.float32)


def kmeans_np(x: np.ndarray, k: int, iters: int, seed: int):
    rng = np.random.default_rng(seed)
    c = x[rng.choice(len(x), k, replace=False)].astype(np.float32)
    for _ in range(iters):
        lab = assign_np(c, x)
        sums = np.zeros_like(c, dtype=np.float64)
        np.add.at(sums, lab, x)
        cnt = np.bincount(lab, minlength=k)
        nz = cnt > 0
        c[nz] = (sums[nz] / cnt[nz, None]).astype(np.float32)
    return c


def assign_np(c: np.ndarray, x: np.ndarray, chunk: int = 16384):
    cn = (c.astype(np.float64) ** 2).sum(1)
    out = np.empty(len(x), np.int64)
    for s in range(0, len(x), chunk):
        xs = x[s:s + chunk].astype(np.float64)
        out[s:s + chunk] = (cn[None, :] - 2.0 * xs @ c.T.astype(np.float64)).argmin(1)
    return out


@dataclass
class IndexArrays:
    """Normalised RetrievalIndex arrays (crates/vocal-model/src/retrieval.rs:6-14):
    centroids [nlist, d], offsets [nlist+1] i32, vectors [n, d] in inverted-list
    order, ids [n] i32 (FAISS labels, a permutation), and the persisted nprobe."""
    centroids: np.ndarray
    offsets: np.ndarray
    vectors: np.ndarray
    ids: np.ndarray
    nprobe: int

    @property
    def d(self):
        return self.centroids.shape[1]

    @property
    def nlist(self):
        return self.centroids.shape[0]

    @property
    def n(self):
        return self.vectors.shape[0]


def flat_arrays(x: np.ndarray) -> IndexArrays:
    """What the reference parser makes of an IxF2 index (retrieval.rs:67-82)."""
    n, d = x.shape
    return IndexArrays(np.zeros((1, d), np.float32), np.array([0, n], np.int32), np.ascontiguousarray(x),
                       np.arange(n, dtype=np.int32), 1)


def ivf_arrays(x: np.ndarray, centroids: np.ndarray, nprobe: int, lists: np.ndarray | None = None) -> IndexArrays:
    """Inverted-list layout of an IwFl index built by adding `x` in order."""
    if lists is None:
        lists = assign_np(centroids, x)
    order = np.argsort(lists, kind="stable")
    sizes = np.bincount(lists, minlength=centroids.shape[0])
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    return IndexArrays(np.ascontiguousarray(centroids, np.float32), offsets, np.ascontiguousarray(x[order]),
                       order.astype(np.int32), nprobe)


def make_np(key: str, n: int | None = None, q: int | None = None, nprobe: int | None = None):
    """(IndexArrays, queries) for config `key`, optionally resized (tests)."""
    w = CONFIGS[key]
    n = n or w.n
    q = q or w.q
    s_db, s_q, s_km = seeds(key)
    x, means = mixture_np(n, w.d, w.components, s_db)
    queries = queries_np(means, q, s_q)
    if w.nlist > 1:
        k = min(w.nlist, n)
        c = kmeans_np(x, k, w.kmeans_iters, s_km)
        ix = ivf_arrays(x, c, nprobe or w.nprobe[0])
    else:
        ix = flat_arrays(x)
    return ix, queries


# --------------------------------------------------------------------------- torch (device)
def make_torch(key: str, device, n: int | None = None, q: int | None = None, nprobe: int | None = None):
    """Device-generated (IndexArrays-like dict of torch tensors, queries)."""
    import torch

    w = CONFIGS[key]
    n = n or w.n
    q = q or w.q
    s_db, s_q, s_km = seeds(key)
    g = torch.Generator(device=device)
    g.manual_seed(s_db)
    means = torch.randn((w.components, w.d), generator=g, device=device, dtype=torch.float32)
    x = torch.empty((n, w.d), device=device, dtype=torch.float32)
    chunk = 1 << 18
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        comp = torch.randint(0, w.components, (m,), generator=g, device=device)
        x[s:s + m] = means[comp] + SIGMA * torch.randn((m, w.d), generator=g, device=device)
    g.manual_seed(s_q)
    comp = torch.randint(0, w.components, (q,), generator=g, device=device)
    queries = means[comp] + SIGMA * torch.randn((q, w.d), generator=g, device=device)
    queries += QUERY_NOISE * torch.randn((q, w.d), generator=g, device=device)
    if w.nlist > 1:
        g.manual_seed(s_km)
        perm = torch.randperm(n, generator=g, device=device)[: w.nlist]
        c = x[perm].clone()
        for _ in range(w.kmeans_iters):
            lab = _assign_torch(c, x)
            sums = torch.zeros_like(c, dtype=torch.float64).index_add_(0, lab, x.double())
            cnt = torch.bincount(lab, minlength=w.nlist)
            nz = cnt > 0
            c[nz] = (sums[nz] / cnt[nz, None]).float()
        lab = _assign_torch(c, x)
        order = torch.sort(lab, stable=True).indices
        sizes = torch.bincount(lab, minlength=w.nlist)
        offsets = torch.cat([torch.zeros(1, device=device, dtype=torch.int64), sizes.cumsum(0)]).int()
        arrays = dict(centroids=c, offsets=offsets, vectors=x[order].contiguous(), ids=order.int(),
                      nprobe=nprobe or w.nprobe[0])
        del x
    else:
        arrays = dict(centroids=torch.zeros((1, w.d), device=device), offsets=torch.tensor([0, n], device=device,
                      dtype=torch.int32), vectors=x, ids=torch.arange(n, device=device, dtype=torch.int32), nprobe=1)
    return arrays, queries


def _assign_torch(c, x, chunk: int = 1 << 16):
    import torch

    cn = (c.double() ** 2).sum(1)
    out = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    for s in range(0, x.shape[0], chunk):
        xs = x[s:s + chunk].double()
        out[s:s + chunk] = (cn[None, :] - 2.0 * xs @ c.double().T).argmin(1)
    return out
