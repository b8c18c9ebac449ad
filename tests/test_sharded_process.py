"""The single-process multi-GPU index (vfr_retrieval_*_sharded) against one
index on one GPU, bit for bit.

Row sharding splits a flat index's rows over the handle's devices and
merges the shards' top-8 lists by (distance, global row), the single-index
scan order (crates/vocal-cpu/src/retrieval.rs:33-61); the blend reads each
winner from the device that owns it.  Query sharding gives every device a
replica and a share of the frames.  On a one-GPU box the shards share
device 0 (the same code path, with peer access trivially present); the
two-GPU case runs when the box has two.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _single(torch, ix, q, ratio):
    from vfr import GpuRetrievalIndex

    g = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, ix.nprobe)
    s = torch.cuda.Stream()
    qd = torch.from_numpy(q).cuda()
    out = torch.empty_like(qd)
    rate = torch.tensor([ratio], device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        d, l = g.search(qd, stream=s)
        g.blend_from(qd, out, rate, stream=s)
    s.synchronize()
    g.close()
    return d.cpu().numpy(), l.cpu().numpy(), out.cpu().numpy()


def _sharded(torch, ix, q, ratio, devices, mode, k=8):
    from vfr import ShardedRetrievalIndex

    h = ShardedRetrievalIndex.from_arrays(devices, mode, ix.centroids, ix.offsets, ix.vectors, ix.ids, ix.nprobe)
    s = torch.cuda.Stream()
    qd = torch.from_numpy(q).cuda()
    out = torch.empty_like(qd)
    rate = torch.tensor([ratio], device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        d, l = h.search(qd, k=k, stream=s)
        h.blend_from(qd, out, rate, stream=s)
        # in place, a second time: the same frames again
        again = qd.clone()
        h.blend_from(again, again, rate, stream=s)
    s.synchronize()
    h.close()
    return d.cpu().numpy(), l.cpu().numpy(), out.cpu().numpy(), again.cpu().numpy()


def _check(single, sharded, k=8):
    d1, l1, o1 = single
    d2, l2, o2, a2 = sharded
    assert np.array_equal(l2, l1[:, :k])
    assert np.array_equal(d2.view(np.uint32), d1[:, :k].view(np.uint32))
    assert np.array_equal(o2.view(np.uint32), o1.view(np.uint32))
    assert np.array_equal(a2.view(np.uint32), o1.view(np.uint32))


@pytest.fixture(scope="module")
def flat():
    from vfr import synth

    ix, q = synth.make_np("c1", n=20_000, q=300)
    # FAISS ids that are not the storage rows: labels come back as ids
    rng = np.random.default_rng(5)
    ix = synth.IndexArrays(ix.centroids, ix.offsets, ix.vectors, rng.permutation(ix.vectors.shape[0]).astype(np.int32),
                           1)
    return ix, q


@pytest.mark.parametrize("shards,frames", [(2, 300), (3, 300), (2, 32), (5, 7)])
def test_row_shards_match_one_index(cuda, flat, shards, frames):
    from vfr import lib

    ix, q = flat
    q = np.ascontiguousarray(q[:frames])
    single = _single(cuda, ix, q, 0.75)
    _check(single, _sharded(cuda, ix, q, 0.75, [0] * shards, lib.SHARD_ROWS))


def test_row_shards_k_below_8(cuda, flat):
    from vfr import lib

    ix, q = flat
    q = np.ascontiguousarray(q[:64])
    single = _single(cuda, ix, q, 0.5)
    _check(single, _sharded(cuda, ix, q, 0.5, [0, 0], lib.SHARD_ROWS, k=3), k=3)


def test_row_shards_against_the_oracle(cuda, oracle, flat):
    from vfr import lib

    ix, q = flat
    q = np.ascontiguousarray(q[:48])
    d, l, out, _ = _sharded(cuda, ix, q, 0.75, [0, 0, 0], lib.SHARD_ROWS)
    o = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1)
    od, _, ol, _ = o.search(q, threads=8)
    expected, status = o.blend(q, 0.75, threads=8)
    assert np.array_equal(l, ol)
    assert np.array_equal(d.view(np.uint32), od.view(np.uint32))
    assert (status == 0).all()
    assert np.array_equal(out.view(np.uint32), expected.view(np.uint32))


def test_query_shards_ivf(cuda):
    from vfr import lib, synth

    ix, q = synth.make_np("c3", n=20_000, q=203, nprobe=4)
    single = _single(cuda, ix, q, 0.75)
    _check(single, _sharded(cuda, ix, q, 0.75, [0, 0, 0], lib.SHARD_QUERIES))


def test_row_sharding_needs_a_flat_index(cuda):
    from vfr import NativeError, ShardedRetrievalIndex, lib, synth

    ix, _ = synth.make_np("c3", n=4_000, q=8, nprobe=2)
    with pytest.raises(NativeError, match="flat index"):
        ShardedRetrievalIndex.from_arrays([0, 0], lib.SHARD_ROWS, ix.centroids, ix.offsets, ix.vectors, ix.ids,
                                          ix.nprobe)


def test_two_devices(cuda, flat):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from vfr import lib

    ix, q = flat
    q = np.ascontiguousarray(q[:300])
    single = _single(cuda, ix, q, 0.75)
    _check(single, _sharded(cuda, ix, q, 0.75, [0, 1], lib.SHARD_ROWS))
    _check(single, _sharded(cuda, ix, q, 0.75, [0, 1], lib.SHARD_QUERIES))
