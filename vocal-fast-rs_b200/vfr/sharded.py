"""Row-sharded multi-GPU retrieval: one process per GPU over torch.distributed.

Every rank holds a contiguous slice of the database rows (rank r: rows
[r*N/G, (r+1)*N/G)) as its own device index whose labels are global rows.
For a batch of Q frames (replicated on every rank) one step is:

  1. local exact top-8 of all Q frames against the rank's rows
     (tensor-core candidates + exact re-rank, C ABI `vfr_retrieval_search`);
  2. all-gather of the G per-shard top-8 lists (NCCL, 12 B per entry);
  3. k-way merge by (distance, global row) -> the single-index top-8, which is
     the reference's scan order for a flat index (`vfr_merge_topk`);
  4. the reference's f64 weights + f32 blend of the rank's Q/G frames, with
     the winners' fp32 rows read where they live.  Default (NCCL groups, the
     GPUs of one node): every rank has mapped the other shards' row arrays
     once (CUDA IPC) and `vfr_blend_peer` loads each winner from its owner's
     HBM over NVLink inside the blend kernel -- no staging, no collective, no
     host wait.  Otherwise (`exchange="all_to_all"`, and gloo): every rank
     knows who owns each winner and who needs it, packs the winners it owns
     by destination (`vfr_gather_owned` on the compact label list), one
     all-to-all with those uneven splits delivers them, and
     `vfr_blend_gathered_rows` reads them through a slot -> row map.

Frames are therefore blended exactly as by a single index; the output of
rank r is frames [r*Q/G, (r+1)*Q/G).  The reference is single-GPU; this is the
multi-GPU extension of its path.  Collectives are taken in the same order on
every rank.  With a `timeout_s` every host wait of a step is a bounded poll
(the peer path waits once, for the step's end; the all-to-all path for its G x
G split sizes and for the all-to-all): if a peer never joins before the
deadline, the process group is aborted and `ShardTimeout` is raised instead
of waiting forever.
`ops` selects the per-rank compute: `LibraryOps` (CUDA library, the product)
or a test double with the same interface.

Query sharding (`query_sharded_blend`) is the other mode, for large offline
batches against an index that fits one GPU (c3): every rank holds a full
replica and blends its contiguous share of the frames; no collective is
needed unless every rank wants the whole output (`gather=True`).
"""
from __future__ import annotations

import contextlib
import time

import numpy as np

from . import lib as _l
from .index import GpuRetrievalIndex, blend_gathered_rows, merge_topk


class ShardTimeout(RuntimeError):
    """A peer rank did not take part in a collective before the deadline;
    the process group has been aborted."""


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
        self.label_base = label_base
        self.rows = n_local

    def search(self, q, stream):
        return self.index.search(q, k=8, stream=stream)

    def merge(self, dists, labels, stream):
        import torch

        md = torch.empty_like(dists[0])
        ml = torch.empty_like(labels[0])
        merge_topk(dists, labels, md, ml, stream=stream)
        return md, ml

    def gather_rows(self, labels, stream):
        """[L, d] fp32 vectors of the (owned, global) labels [L], in order."""
        import torch

        count = labels.shape[0]
        padded = (count + 7) // 8 * 8
        lab = torch.full((padded,), -1, dtype=torch.int64, device=labels.device)
        lab[:count] = labels
        out = torch.empty((padded, self.d), dtype=torch.float32, device=labels.device)
        if padded:
            self.index.gather_owned(lab.view(-1, 8), out.view(-1, 8, self.d), stream=stream)
        return out[:count]

    def blend_rows(self, q, dist, rows, slot_rows, rate, stream):
        import torch

        out = torch.empty_like(q)
        blend_gathered_rows(q, out, dist, rows, slot_rows, rate, stream=stream)
        return out

    # -- peer-memory exchange (NCCL process groups: the GPUs of one node)
    peers = None

    def open_peers(self, group, world: int, rank: int, deadline=None):
        """Maps every shard's rows into this process (collective: every rank
        calls it once, in the same step)."""
        self.peers = PeerRows(self.index, group, world, rank, deadline)

    def blend_peer(self, q, dist, labels, rate, stream):
        import torch

        out = torch.empty_like(q)
        self.peers.blend(q, out, dist, labels, rate, stream)
        return out

    def close(self, group=None):
        """Releases the peer mappings on every rank before any rank frees its
        rows (collective when peers are open): synchronise, barrier, close,
        barrier."""
        if self.peers is None:
            return
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group=group)
        self.peers.close()
        self.peers = None
        torch.cuda.synchronize()
        dist.barrier(group=group)


class PeerRows:
    """This rank's mappings of every row shard's fp32 rows
    (vfr_index_ipc_export on each rank, an all-gather of the descriptors,
    vfr_peer_rows_open), used by vfr_blend_peer."""

    def __init__(self, index, group, world: int, rank: int, deadline=None):
        import ctypes

        import torch
        import torch.distributed as dist

        L = _l.load_library()
        desc = _l.IpcRows()
        _l.call(L.vfr_index_ipc_export, index._h, ctypes.byref(desc))
        raw = torch.frombuffer(bytearray(bytes(desc)), dtype=torch.uint8)
        if dist.get_backend(group) == "nccl":
            raw = raw.cuda()
        every = _all_gather(raw, group, world, deadline, "peer row descriptors").cpu().numpy()
        descs = (_l.IpcRows * world)()
        for r in range(world):
            ctypes.memmove(ctypes.addressof(descs[r]), every[r].tobytes(), ctypes.sizeof(_l.IpcRows))
        self._h = ctypes.c_void_p()
        _l.call(L.vfr_peer_rows_open, index._h, world, descs, rank, ctypes.byref(self._h))

    def blend(self, q, out, dist, labels, rate, stream=None):
        import ctypes

        from .index import _ptr

        L = _l.load_library()
        s = _l.stream_struct(stream)
        _l.call(L.vfr_blend_peer, self._h, _ptr(q), _ptr(out), _ptr(dist), _ptr(labels), q.shape[0], q.shape[1],
                _ptr(rate), ctypes.byref(s))

    def close(self):
        if getattr(self, "_h", None) and self._h.value:
            _l.load_library().vfr_peer_rows_close(self._h)
            self._h = None

    def __del__(self):
        self.close()


def _stream_ctx(stream):
    """Runs the torch ops of a step on `stream` (a CUDA stream) so they are
    ordered with the library calls made on it; no-op for CPU tensors."""
    if stream is None:
        return contextlib.nullcontext()
    import torch

    return torch.cuda.stream(stream)


def _abort(group):
    import torch.distributed as dist

    try:
        dist.distributed_c10d._abort_process_group(group)
    except Exception:  # noqa: BLE001 - best effort: the caller raises ShardTimeout either way
        pass


def _poll(done, deadline, group, what):
    """Spins on `done()` (a CUDA event query or a collective's completion)
    until it holds or the deadline passes; then aborts the group and raises.
    Busy for the first millisecond, so a wait that ends soon costs
    microseconds, then in 50 us sleeps."""
    spin_until = time.monotonic() + 1e-3
    while not done():
        now = time.monotonic()
        if now > deadline:
            _abort(group)
            raise ShardTimeout(f"{what}: a peer rank did not join before the deadline; process group aborted")
        if now > spin_until:
            time.sleep(5e-5)


def _all_gather(t, group, world, deadline=None, what="all-gather"):
    import torch
    import torch.distributed as dist

    if dist.get_backend(group) == "nccl":
        out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        work = dist.all_gather_into_tensor(out, t.contiguous(), group=group, async_op=deadline is not None)
    else:
        parts = [torch.empty_like(t) for _ in range(world)]
        work = dist.all_gather(parts, t.contiguous(), group=group, async_op=deadline is not None)
    if deadline is not None:
        _poll(work.is_completed, deadline, group, what)
        work.wait()
    return out if dist.get_backend(group) == "nccl" else torch.stack(parts)


def _bounds(ops, group, world, deadline=None):
    """Global row bounds [G+1] of the shards (gathered once, cached on ops)."""
    import torch
    import torch.distributed as dist

    b = getattr(ops, "_shard_bounds", None)
    if b is None:
        mine = torch.tensor([ops.label_base, ops.label_base + ops.rows], dtype=torch.int64)
        if dist.get_backend(group) == "nccl":
            mine = mine.cuda()
        spans = _all_gather(mine, group, world, deadline, "row-shard bounds").cpu()
        b = [int(spans[0, 0])] + [int(spans[r, 1]) for r in range(world)]
        if any(int(spans[r, 0]) != b[r] for r in range(world)):
            raise ValueError("row shards must be contiguous and in rank order")
        ops._shard_bounds = b
    return b


def exchange_plan(ml, bounds, world: int, rank: int):
    """Who sends which winner where, from the merged labels ml [Q, 8]
    (identical on every rank).  Entry e = f*8 + k belongs to destination
    rank f // (Q/G) and is owned by the shard whose rows hold ml[f, k].
    Returns (counts [G, G] int64 on ml's device: counts[o, t] entries owned
    by o for destination t; owner [Q*8] with G for empty slots)."""
    import torch

    q = ml.shape[0]
    m = q // world
    flat = ml.reshape(-1)
    inner = torch.tensor(bounds[1:-1], dtype=torch.int64, device=ml.device)
    owner = torch.searchsorted(inner, flat, right=True)
    owner = torch.where(flat >= 0, owner, torch.full_like(owner, world))
    dest = torch.arange(flat.numel(), device=ml.device) // (8 * m)
    key = torch.where(owner < world, owner * world + dest, torch.full_like(owner, world * world))
    counts = torch.bincount(key, minlength=world * world + 1)[: world * world].view(world, world)
    return counts, owner


def _send_labels(ml, owner, rank, total):
    """The labels this rank owns, in entry order (destination-major),
    without a host-side mask (the count is already known)."""
    import torch

    flat = ml.reshape(-1)
    own = owner == rank
    pos = torch.cumsum(own.to(torch.int64), 0) - 1
    tgt = torch.where(own, pos, torch.full_like(pos, total))
    idx = torch.zeros(total + 1, dtype=torch.int64, device=ml.device)
    idx.scatter_(0, tgt, torch.arange(flat.numel(), device=ml.device))
    return flat[idx[:total]]


def _slot_rows(owner, rank, m, world):
    """Receive-buffer row of every slot of this rank's frames: the buffer
    holds, source by source, that source's entries in entry order, which is
    the stable order of the owners; empty slots get -1."""
    import torch

    share = owner[rank * m * 8:(rank + 1) * m * 8]
    perm = torch.sort(share, stable=True).indices
    pos = torch.empty_like(perm)
    pos[perm] = torch.arange(perm.numel(), device=owner.device)
    pos = torch.where(share < world, pos, torch.full_like(pos, -1))
    return pos.to(torch.int32).view(m, 8)


def sharded_blend(ops, queries, rate, group, world: int, rank: int, stream=None, timeout_s: float | None = None,
                  exchange: str = "auto"):
    """One row-sharded step for `queries` [Q, d] (Q a multiple of world, the
    same tensor on every rank).  Returns (this rank's blended frames
    [Q/world, d], merged distances [Q, 8], merged labels [Q, 8]).

    exchange: "peer" reads the winners from their owners' memory in the blend
    kernel (NCCL groups with LibraryOps; the peer mappings are opened on the
    first call, so every rank must make it), "all_to_all" sends them with a
    collective, "auto" takes "peer" where it can.  With `timeout_s` the
    step's host waits are bounded: ShardTimeout (and an aborted group) if a
    peer never joins."""
    import torch
    import torch.distributed as dist

    q = queries.shape[0]
    if q % world:
        raise ValueError("frame count must be a multiple of the world size; pad with padded_frames()")
    deadline = time.monotonic() + timeout_s if timeout_s is not None else None
    nccl = dist.get_backend(group) == "nccl"
    if exchange == "auto":
        exchange = "peer" if nccl and hasattr(ops, "open_peers") else "all_to_all"
    m = q // world
    lo = rank * m
    with _stream_ctx(stream):
        bounds = _bounds(ops, group, world, deadline)
        if exchange == "peer" and ops.peers is None:
            ops.open_peers(group, world, rank, deadline)
        d8, l8 = ops.search(queries, stream)
        # on NCCL the two gathers are only enqueued here: the bounded wait for
        # the count matrix below (or the end of the step) covers them
        gloo_deadline = deadline if not nccl else None
        dists = _all_gather(d8, group, world, gloo_deadline, "top-8 distance all-gather")
        labels = _all_gather(l8, group, world, gloo_deadline, "top-8 label all-gather")
        md, ml = ops.merge(dists, labels, stream)
        if exchange == "peer":
            out = ops.blend_peer(queries[lo:lo + m], md[lo:lo + m].contiguous(), ml[lo:lo + m].contiguous(), rate,
                                 stream)
            if deadline is not None:
                ev = torch.cuda.Event()
                ev.record()
                _poll(ev.query, deadline, group, "row-sharded step")
            return out, md, ml
        counts_dev, owner = exchange_plan(ml, bounds, world, rank)
        if deadline is not None and counts_dev.is_cuda:
            host = torch.empty(counts_dev.shape, dtype=counts_dev.dtype, pin_memory=True)
            host.copy_(counts_dev, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            _poll(ev.query, deadline, group, "row-sharded top-8 exchange")
            counts = host.tolist()
        else:
            counts = counts_dev.cpu().tolist()
        send_n = counts[rank]
        recv_n = [counts[o][rank] for o in range(world)]
        send = ops.gather_rows(_send_labels(ml, owner, rank, sum(send_n)), stream)
        recv = torch.empty((sum(recv_n), queries.shape[1]), dtype=torch.float32, device=queries.device)
        work = dist.all_to_all_single(recv, send.contiguous(), recv_n, send_n, group=group,
                                      async_op=deadline is not None)
        if deadline is not None:
            _poll(work.is_completed, deadline, group, "row-sharded winner exchange")
            work.wait()
        slots = _slot_rows(owner, rank, m, world)
        out = ops.blend_rows(queries[lo:lo + m], md[lo:lo + m].contiguous(), recv, slots, rate, stream)
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
