"""Row-sharded retrieval on 2 GPUs over NCCL (one process per GPU) against
the single-index oracle: every rank's blended frames and the merged
distances/labels must equal the oracle bit for bit.  Skipped on a machine
with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, vectors, queries, ratio, results, exchange="auto"):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "vocal-fast-rs_b200"), root]
    import torch
    import torch.distributed as dist
    from vfr.sharded import LibraryOps, shard_rows, sharded_blend

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    lo, hi = shard_rows(len(vectors), world, rank)
    ops = LibraryOps(vectors[lo:hi], lo)
    q = torch.from_numpy(queries).to(dev)
    rate = torch.tensor([ratio], device=dev)
    s = torch.cuda.Stream(dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        out, md, ml = sharded_blend(ops, q, rate, dist.group.WORLD, world, rank, stream=s, timeout_s=60.0,
                                    exchange=exchange)
        # a second step with other frames through the same (already open) exchange
        out2, _, _ = sharded_blend(ops, q.flip(0).contiguous(), rate, dist.group.WORLD, world, rank, stream=s,
                                   timeout_s=60.0, exchange=exchange)
    s.synchronize()
    results[rank] = (out.cpu().numpy(), md.cpu().numpy(), ml.cpu().numpy(), out2.cpu().numpy())
    ops.close(dist.group.WORLD)  # peer mappings released on every rank before any index is freed
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["peer", "all_to_all"])
def test_two_gpu_row_sharded_blend_matches_oracle(oracle, exchange):
    """Both winner exchanges: rows read from the owner GPU inside the blend
    kernel (peer), and packed rows sent with an NCCL all-to-all."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from vfr import synth

    ix, q = synth.make_np("c1", n=20_000, q=256)
    ix.vectors[19_999] = ix.vectors[11]  # duplicate across the shard boundary: tie -> lower row
    q[5] = ix.vectors[11]
    ratio = 0.75
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ix.vectors, q, ratio, results, exchange))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    orc = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1)
    expected, status = orc.blend(q, ratio, threads=os.cpu_count() or 1)
    dist, rows, labels, _ = orc.search(q, threads=os.cpu_count() or 1)
    got = np.concatenate([results[r][0] for r in range(2)])
    assert (status == 0).all()
    assert np.array_equal(got.view(np.uint32), expected.view(np.uint32))
    for r in range(2):
        assert np.array_equal(results[r][2], labels)
        assert np.array_equal(results[r][1].view(np.uint32), dist.view(np.uint32))
    assert labels[5, 0] == 11 and labels[5, 1] == 19_999
    expected2, _ = orc.blend(q[::-1].copy(), ratio, threads=os.cpu_count() or 1)
    got2 = np.concatenate([results[r][3] for r in range(2)])
    assert np.array_equal(got2.view(np.uint32), expected2.view(np.uint32))


def _query_worker(rank, world, port, arrays, queries, ratio, results):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "vocal-fast-rs_b200"), root]
    import torch
    import torch.distributed as dist
    from vfr import GpuRetrievalIndex
    from vfr.sharded import query_sharded_blend

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    centroids, offsets, vectors, ids, nprobe = arrays
    replica = GpuRetrievalIndex.from_arrays(centroids, offsets, vectors, ids, nprobe)
    q = torch.from_numpy(queries).to(dev)
    rate = torch.tensor([ratio], device=dev)
    s = torch.cuda.Stream(dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        out = query_sharded_blend(replica, q, rate, dist.group.WORLD, world, rank, stream=s, gather=True)
    s.synchronize()
    results[rank] = out.cpu().numpy()
    replica.close()
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_query_sharded_ivf_blend_matches_oracle(oracle):
    """Query sharding of an offline IVF batch: a replica per GPU, each blends
    its share, an all-gather gives every rank the whole batch."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from vfr import synth

    ix, q = synth.make_np("c3", n=20_000, q=301, nprobe=8)
    ratio = 0.75
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    arrays = (ix.centroids, ix.offsets, ix.vectors, ix.ids, ix.nprobe)
    procs = [ctx.Process(target=_query_worker, args=(r, 2, port, arrays, q, ratio, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    orc = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, ix.nprobe)
    expected, status = orc.blend(q, ratio, threads=os.cpu_count() or 1)
    ok = status == 0
    for r in range(2):
        assert np.array_equal(results[r][ok].view(np.uint32), expected[ok].view(np.uint32))
        assert np.array_equal(results[r][~ok].view(np.uint32), q[~ok].view(np.uint32))
