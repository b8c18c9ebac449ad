"""Row-sharded multi-GPU retrieval: one process per GPU over torch.distributed.

Every rank holds a contiguous slice of the database rows (rank r: rows
[r*N/G, (r+1)*N/G)) as its own device index whose labels are global rows.
For a batch of Q frames (replicated on every rank) one step is:

  1. local exact top-8 of all Q frames against the rank's rows
     (tensor-core candidates + exact re-rank, C ABI `vfr_retrieval_search`);
  2. all-gather of the G per-shard top-8 lists (NCCL, 12 B per entry);
  3. k-way merge by (distance, global row) -> the single-index top-8, which is
     the reference's scan order for a flat index (`vfr_merge_topk`);
  4. each rank writes the winning vectors it owns, -0.0 elsewhere
     (`vfr_gather_owned`), and a reduce-scatter (sum) hands rank r the exact
     fp32 neighbour vectors of its Q/G frames (x + -0.0 == x bit for bit);
  5. the reference's f64 weights + f32 blend for those frames
     (`vfr_blend_gathered`).

Frames are therefore blended exactly as by a single index; the output of
rank r is frames [r*Q/G, (r+1)*Q/G).  The reference is single-GPU; this is the
multi-GPU extension of its path.  Collectives are taken in the same order on
every rank.  `ops` selects the per-rank compute: `LibraryOps` (CUDA library,
the product) or a test double with the same interface.

Query sharding (`query_sharded_blend`) is the other mode, for large offline
batches against an index that fits one GPU (c3): every rank holds a full
replica and blends its contiguous share of the frames; no collective is
needed unless every rank wants the whole output (`gather=True`).
"""
from __future__ import annotations

import numpy as np

from . import lib as _l
from .index import GpuRetrievalIndex, blend_gathered, merge_topk


def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous row range of `rank` (sizes differ by at most one)."""
    return n * rank // world, n * (rank + 1) // world


def padded_frames(q: int, world: int) -> int:
    return (q + world - 1) // world * world


class LibraryOps:
    """Per-rank compute through libvfr_retrieval.so on CUDA tensors."""

    def __init__(self, vectors_slice, label_base: int, engine: int = _l.ENGINE_AUTO, max_frames: int = 0):
        n_local, d = vectors_slice.shape
        self.index = GpuRetrievalIndex.from_arrays(
            np.zeros((1, d), np.float32), np.array([0, n_local], np.int32), vectors_slice,
            np.arange(n_local, dtype=np.int32), 1, engine=engine, label_base=label_base, max_frames=max_frames)
        self.d = d

    def search(self, q, stream):
        return self.index.search(q, k=8, stream=stream)

    def merge(self, dists, labels, stream):
        import torch

        md = torch.empty_like(dists[0])
        ml = torch.empty_like(labels[0])
        merge_topk(dists, labels, md, ml, stream=stream)
        return md, ml

    def gather_owned(self, labels, stream):
        import torch

        out = torch.empty((labels.shape[0], 8, self.d), dtype=torch.float32, device=labels.device)
        self.index.gather_owned(labels, out, stream=stream)
        return out

    def blend(self, q, dist, neighbours, rate, stream):
        import torch

        out = torch.empty_like(q)
        blend_gathered(q, out, dist, neighbours, rate, stream=stream)
        return out


def _all_gather(t, group, world):
    import torch
    import torch.distributed as dist

    if dist.get_backend(group) == "nccl":
        out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
        return out
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.stack(parts)


def _reduce_scatter_sum(t, group, world, rank):
    """Sum over ranks of t [world*m, ...], returning this rank's m rows."""
    import torch
    import torch.distributed as dist

    m = t.shape[0] // world
    if dist.get_backend(group) == "nccl":
        out = torch.empty((m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.reduce_scatter_tensor(out, t.contiguous(), op=dist.ReduceOp.SUM, group=group)
        return out
    full = t.clone()
    dist.all_reduce(full, op=dist.ReduceOp.SUM, group=group)
    return full[rank * m:(rank + 1) * m].clone()


def sharded_blend(ops, queries, rate, group, world: int, rank: int, stream=None):
    """One row-sharded step for `queries` [Q, d] (Q a multiple of world, the
    same tensor on every rank).  Returns (this rank's blended frames
    [Q/world, d], merged distances [Q, 8], merged labels [Q, 8])."""
    q = queries.shape[0]
    if q % world:
        raise ValueError("frame count must be a multiple of the world size; pad with padded_frames()")
    d8, l8 = ops.search(queries, stream)
    dists = _all_gather(d8, group, world)
    labels = _all_gather(l8, group, world)
    md, ml = ops.merge(dists, labels, stream)
    owned = ops.gather_owned(ml, stream)
    mine = _reduce_scatter_sum(owned, group, world, rank)
    m = q // world
    lo = rank * m
    out = ops.blend(queries[lo:lo + m], md[lo:lo + m].contiguous(), mine, rate, stream)
    return out, md, ml


def shard_frames(q: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous frame range of `rank` in query sharding (sizes differ by at
    most one)."""
    return q * rank // world, q * (rank + 1) // world


def query_sharded_blend(index, queries, rate, group, world: int, rank: int, stream=None, gather: bool = False):
    """Query-sharded blend: `index` is this rank's full replica (a
    GpuRetrievalIndex, or a test double with its `blend`), `queries` [Q, d]
    the whole batch on every rank.  Returns this rank's blended frames
    [hi - lo, d] (frames [lo, hi) of shard_frames), or with gather=True the
    whole blended batch [Q, d] on every rank (one all-gather of equal-size,
    padded slices)."""
    q = queries.shape[0]
    lo, hi = shard_frames(q, world, rank)
    out = queries[lo:hi].clone()
    if hi > lo:
        index.blend(out, hi - lo, rate, stream=stream)
    if not gather:
        return out
    import torch

    m = (q + world - 1) // world
    padded = torch.zeros((m,) + tuple(queries.shape[1:]), dtype=queries.dtype, device=queries.device)
    padded[: hi - lo] = out
    parts = _all_gather(padded, group, world)
    return torch.cat([parts[r][: shard_frames(q, world, r)[1] - shard_frames(q, world, r)[0]] for r in range(world)])
