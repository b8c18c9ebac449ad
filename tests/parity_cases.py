"""Seeded parity cases shared by the GPU tests, smoke() and the benchmark.

The fixture recipes follow the reference's retrieval benchmark driver
(scripts/benchmark-retrieval.py:43-72): Flat widths 33/256/768/4096 with
3/65/257/17 rows whose last row duplicates the first and whose first query is
an exact match (seed 812); a width-33 IVF index with 8 lists trained on 1024
vectors holding 19 of them, probed at nprobe 1/4/8; and an IVF index whose
nearest list is empty.  FAISS is not available, so training uses this
repository's seeded k-means and list assignment instead of faiss.train/add.
"""
from __future__ import annotations

import numpy as np

from vfr import synth


def reference_fixtures():
    """[(name, IndexArrays, queries)]"""
    rng = np.random.default_rng(812)
    out = []
    for width, count in [(33, 3), (256, 65), (768, 257), (4096, 17)]:
        vectors = rng.standard_normal((count, width), dtype=np.float32)
        vectors[-1] = vectors[0]
        q = rng.standard_normal((7, width), dtype=np.float32)
        q[0] = vectors[0]
        out.append((f"flat-{width}", synth.flat_arrays(vectors), q))
    width = 33
    vectors = rng.standard_normal((1024, width), dtype=np.float32)
    centroids = synth.kmeans_np(vectors, 8, 10, 812)
    q = rng.standard_normal((9, width), dtype=np.float32)
    q[0] = vectors[0]
    for probes in (1, 4, 8):
        out.append((f"ivf-{probes}", synth.ivf_arrays(vectors[:19], centroids, probes), q))
    coarse = np.stack([np.zeros(width), np.ones(width) * 10]).astype(np.float32)
    empty = synth.ivf_arrays(np.ones((1, width), np.float32) * 10, coarse, 1)
    out.append(("empty-list", empty, np.zeros((3, width), np.float32)))
    return out


def tie_fixture():
    """Exact distance ties across rows and lists: duplicated rows in two
    lists, queries equidistant from several rows."""
    d = 16
    base = np.eye(d, dtype=np.float32)[:6] * 2.0
    vectors = np.concatenate([base, base, base[:3]], 0)  # duplicates in storage order
    centroids = np.stack([base[:3].mean(0), base[3:].mean(0), base.mean(0)]).astype(np.float32)
    lists = np.array([0, 0, 0, 1, 1, 1, 2, 2, 2, 2, 2, 2, 1, 0, 2])
    q = np.zeros((4, d), np.float32)
    q[1] = base[0]
    q[2] = (base[0] + base[1]) / 2
    q[3] = base.mean(0)
    return synth.ivf_arrays(vectors, centroids, 3, lists=lists), q


def scaled_configs():
    """BASELINE configs at sizes the oracle finishes in seconds."""
    return {
        "c1": dict(n=20_000, q=250),
        "c2": dict(n=20_000, q=200),
        "c3-np1": dict(n=20_000, q=200, nprobe=1),
        "c3-np8": dict(n=20_000, q=200, nprobe=8),
        "c4": dict(n=20_000, q=32),
    }


def make_scaled(key: str):
    spec = dict(scaled_configs()[key])
    base = key.split("-")[0]
    w = synth.CONFIGS[base]
    if base == "c3":
        # smaller k-means: nlist 64 over 20k rows, same seeds
        ix, q = _ivf_small(spec["n"], spec["q"], spec["nprobe"])
        return ix, q, w.ratio
    ix, q = synth.make_np(base, n=spec["n"], q=spec["q"])
    return ix, q, w.ratio


def _ivf_small(n, q, nprobe, nlist=64):
    s_db, s_q, s_km = synth.seeds("c3")
    x, means = synth.mixture_np(n, 768, 1024, s_db)
    queries = synth.queries_np(means, q, s_q)
    c = synth.kmeans_np(x, nlist, 5, s_km)
    return synth.ivf_arrays(x, c, nprobe), queries
