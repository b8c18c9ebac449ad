"""World-size-2 `gloo` test of the row-sharded choreography (vfr/sharded.py)
on CPU: shard ranges, the all-gather of per-shard top-8 lists, the merge by
(distance, global row), the all-to-all of the owned winners (each vector sent once, to the
rank that blends its frame), and the per-rank output slices.  The per-rank compute is
a test double over the CPU oracle; the CUDA kernels of the same steps are
covered by tests/test_parity.py::test_row_sharded_blocks_reproduce_single_index.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleOps:
    """Test double of vfr.sharded.LibraryOps on CPU tensors."""

    def __init__(self, vectors_slice, label_base):
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [os.path.join(root, "vocal-fast-rs_b200"), root]
        from oracle import oracle
        from vfr import synth

        flat = synth.flat_arrays(vectors_slice)
        self.ix = oracle.OracleIndex.from_arrays(flat.centroids, flat.offsets, flat.vectors, flat.ids, 1)
        self.base = label_base
        self.label_base = label_base
        self.rows = len(vectors_slice)
        self.vectors = vectors_slice

    def search(self, q, stream):
        dist, rows, labels, _ = self.ix.search(q.numpy())
        labels = np.where(labels >= 0, labels + self.base, -1)
        return torch.from_numpy(dist), torch.from_numpy(labels)

    def merge(self, dists, labels, stream):
        D, L = dists.numpy(), labels.numpy()
        shards, q, _ = D.shape
        md = np.full((q, 8), np.inf, np.float32)
        ml = np.full((q, 8), -1, np.int64)
        for f in range(q):
            cand = [(D[s, f, k], L[s, f, k]) for s in range(shards) for k in range(8) if L[s, f, k] >= 0]
            cand.sort(key=lambda t: (float(t[0]), int(t[1])))
            for k, (dd, ll) in enumerate(cand[:8]):
                md[f, k], ml[f, k] = dd, ll
        return torch.from_numpy(md), torch.from_numpy(ml)

    def gather_rows(self, labels, stream):
        local = labels.numpy() - self.base
        assert ((local >= 0) & (local < len(self.vectors))).all(), "a rank was asked for rows it does not own"
        return torch.from_numpy(np.ascontiguousarray(self.vectors[local]))

    def blend_rows(self, q, dist, rows, slot_rows, rate, stream):
        """The reference's f64 weights + f32 blend in numpy (IEEE, same order)."""
        sr = slot_rows.numpy()
        rn = rows.numpy()
        nb = np.zeros(sr.shape + (rn.shape[1] if rn.ndim == 2 else q.shape[1],), np.float32)
        nb[sr >= 0] = rn[sr[sr >= 0]]
        qn, dn = q.numpy(), dist.numpy()
        r = np.float32(min(max(float(rate[0]), 0.0), 1.0))
        out = qn.copy()
        for f in range(qn.shape[0]):
            count = int(np.argmax(~np.isfinite(np.append(dn[f], np.inf))))
            if count == 0 or not r > 0:
                continue
            w = [1.0 / (float(max(dn[f, k], np.float32(1e-12))) ** 2) for k in range(count)] + [0.0] * (8 - count)
            s = -0.0
            for x in w:
                s = s + x
            acc = np.full(qn.shape[1], -0.0)
            for k in range(count):
                acc = acc + (nb[f, k].astype(np.float64) * w[k]) / s
            out[f] = qn[f] * (np.float32(1) - r) + acc.astype(np.float32) * r
        return torch.from_numpy(out)


def _worker(rank, world, port, vectors, queries, ratio, results):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "vocal-fast-rs_b200"), root, os.path.join(root, "tests")]
    import datetime

    import torch.distributed as dist
    from test_sharded_cpu import OracleOps
    from vfr.sharded import shard_rows, sharded_blend

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    lo, hi = shard_rows(len(vectors), world, rank)
    ops = OracleOps(vectors[lo:hi], lo)
    out, md, ml = sharded_blend(ops, torch.from_numpy(queries), torch.tensor([ratio]), dist.group.WORLD, world, rank)
    results[rank] = (out.numpy(), md.numpy(), ml.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_sharded_choreography_matches_single_index(oracle, world):
    from vfr import synth

    ix, q = synth.make_np("c1", n=3001, q=42)
    q[3] = ix.vectors[17]  # exact match
    ix.vectors[2999] = ix.vectors[5]  # duplicate rows in different shards: tie -> lower row
    q[4] = ix.vectors[5]
    ratio = 0.75
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, ix.vectors, q, ratio, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    orc = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1)
    expected, status = orc.blend(q, ratio)
    dist, rows, labels, _ = orc.search(q)
    got = np.concatenate([results[r][0] for r in range(world)])
    assert (status == 0).all()
    assert np.array_equal(got.view(np.uint32), expected.view(np.uint32))
    for r in range(world):
        assert np.array_equal(results[r][2], labels)
        assert np.array_equal(results[r][1].view(np.uint32), dist.view(np.uint32))
    assert labels[4, 0] == 5 and labels[4, 1] == 2999


def _absent_peer_worker(rank, world, port, vectors, queries, timeout_s, results):
    """Rank 0 runs a bounded step; rank 1 never takes part in it (it stays
    alive, idle, past rank 0's deadline, then leaves)."""
    import sys
    import time

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "vocal-fast-rs_b200"), root, os.path.join(root, "tests")]
    import datetime

    import torch.distributed as dist
    from test_sharded_cpu import OracleOps
    from vfr.sharded import ShardTimeout, shard_rows, sharded_blend

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    lo, hi = shard_rows(len(vectors), world, rank)
    ops = OracleOps(vectors[lo:hi], lo)
    ops._shard_bounds = [shard_rows(len(vectors), world, r)[0] for r in range(world)] + [len(vectors)]
    if rank != 0:
        time.sleep(timeout_s + 4.0)
        results[rank] = ("idle", 0.0)
        os._exit(0)
    t0 = time.monotonic()
    try:
        sharded_blend(ops, torch.from_numpy(queries), torch.tensor([0.75]), dist.group.WORLD, world, rank,
                      timeout_s=timeout_s)
        results[rank] = ("returned", time.monotonic() - t0)
    except ShardTimeout as e:
        results[rank] = (str(e), time.monotonic() - t0)
    os._exit(0)


def test_absent_peer_gives_bounded_error(oracle):
    """A rank that never joins the step's collectives: the other rank's
    sharded_blend raises ShardTimeout at its deadline (the process group is
    aborted) instead of waiting for the group's 120 s timeout."""
    from vfr import synth

    ix, q = synth.make_np("c1", n=1000, q=8)
    timeout_s = 3.0
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, 2, port, ix.vectors, q, timeout_s, results))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    msg, elapsed = results[0]
    assert "did not join before the deadline" in msg, msg
    assert timeout_s <= elapsed < timeout_s + 5.0, elapsed
    assert results[1][0] == "idle"


def test_exchange_plan_counts_and_slots():
    """The owner / destination bookkeeping of the winner exchange on a
    hand-made label matrix: 3 ranks, 2 frames each, shards of 10 rows."""
    from vfr.sharded import _send_labels, _slot_rows, exchange_plan

    world, m = 3, 2
    bounds = [0, 10, 20, 30]
    rng = np.random.default_rng(5)
    ml = torch.from_numpy(rng.integers(0, 30, (world * m, 8)).astype(np.int64))
    ml[1, 6:] = -1  # a frame with six neighbours
    counts, owner = exchange_plan(ml, bounds, world, 0)
    L = ml.numpy()
    for o in range(world):
        for t in range(world):
            block = L[t * m:(t + 1) * m]
            assert counts[o, t] == ((block >= bounds[o]) & (block < bounds[o + 1])).sum()
    assert counts.sum() == (L >= 0).sum()
    # what rank r sends, in destination-major entry order
    for r in range(world):
        sent = _send_labels(ml, owner, r, int(counts[r].sum())).numpy()
        flat = L.reshape(-1)
        assert np.array_equal(sent, flat[(flat >= bounds[r]) & (flat < bounds[r + 1])])
    # what rank t receives: source by source; its slots map back to the labels
    for t in range(world):
        recv = np.concatenate([_send_labels(ml, owner, o, int(counts[o].sum())).numpy()[
            int(counts[o, :t].sum()):int(counts[o, :t + 1].sum())] for o in range(world)])
        slots = _slot_rows(owner, t, m, world).numpy()
        block = L[t * m:(t + 1) * m]
        assert np.array_equal(np.where(slots >= 0, recv[np.maximum(slots, 0)], -1), block)


def test_shard_rows_cover_everything():
    from vfr.sharded import padded_frames, shard_rows

    for n in (1, 7, 4_000_000):
        for world in (1, 2, 3, 8):
            spans = [shard_rows(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert padded_frames(30000, 8) == 30000 and padded_frames(30001, 8) == 30008


class OracleReplica:
    """A full replica for query sharding: the oracle's blend on CPU tensors."""

    def __init__(self, oracle_index, ratio):
        self.o = oracle_index
        self.ratio = ratio

    def blend(self, feats, frames, rate, stream=None):
        out, _ = self.o.blend(feats.numpy()[:frames], float(rate[0]))
        feats[:frames] = torch.from_numpy(out)


def _query_worker(rank, world, port, arrays, queries, ratio, gather, results):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "vocal-fast-rs_b200"), root, os.path.join(root, "tests")]
    import datetime

    import torch.distributed as dist
    from oracle import oracle as orc
    from test_sharded_cpu import OracleReplica
    from vfr.sharded import query_sharded_blend

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    centroids, offsets, vectors, ids, nprobe = arrays
    replica = OracleReplica(orc.OracleIndex.from_arrays(centroids, offsets, vectors, ids, nprobe), ratio)
    out = query_sharded_blend(replica, torch.from_numpy(queries), torch.tensor([ratio]), dist.group.WORLD, world,
                              rank, gather=gather)
    results[rank] = out.numpy()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,frames,gather", [(2, 41, False), (2, 41, True), (3, 10, True)])
def test_query_sharded_choreography_matches_single_index(oracle, world, frames, gather):
    """Each rank blends its contiguous share of the frames against a full
    replica (here the oracle); the shares in rank order, or the gathered
    batch on every rank, equal the single-index blend (an IVF index, so the
    mode's use case, offline IVF batches, is the one exercised)."""
    from vfr import synth

    ix, q = synth.make_np("c3", n=4000, q=frames, nprobe=2)
    ratio = 0.75
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    arrays = (ix.centroids, ix.offsets, ix.vectors, ix.ids, ix.nprobe)
    procs = [ctx.Process(target=_query_worker, args=(r, world, port, arrays, q, ratio, gather, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    expected, status = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, ix.nprobe).blend(
        q, ratio)
    if gather:
        for r in range(world):
            assert np.array_equal(results[r].view(np.uint32), expected.view(np.uint32))
    else:
        got = np.concatenate([results[r] for r in range(world)])
        assert np.array_equal(got.view(np.uint32), expected.view(np.uint32))


def test_shard_frames_cover_everything():
    from vfr.sharded import shard_frames

    for q in (0, 1, 7, 30_000):
        for world in (1, 2, 3, 8):
            spans = [shard_frames(q, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == q
            assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
