"""The CTA-pair candidate kernel (clusters of two CTAs, one M = 256
cta_group::2 MMA; large flat launches) against the one-CTA kernel and the
oracle, bit for bit.

4,224 frames are 33 query tiles, so the last pair holds a padding tile; the
same index is built twice, once with the pair layout switched on
(VFR_PAIR=1 at creation; it is opt-in) and once without, and both must
return the same distances, labels and blended frames; frames at both ends
are also checked against the oracle's exact scan
(crates/vocal-cpu/src/retrieval.rs:27-83).
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _index(torch, ix, pair):
    from vfr import GpuRetrievalIndex

    old = os.environ.get("VFR_PAIR")
    try:
        if pair:
            os.environ["VFR_PAIR"] = "1"
        else:
            os.environ.pop("VFR_PAIR", None)
        return GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1)
    finally:
        if old is None:
            os.environ.pop("VFR_PAIR", None)
        else:
            os.environ["VFR_PAIR"] = old


def _run(torch, g, q, ratio):
    s = torch.cuda.Stream()
    qd = torch.from_numpy(q).cuda()
    out = torch.empty_like(qd)
    rate = torch.tensor([ratio], device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        d, l = g.search(qd, stream=s)
        plan = None
        g.blend_from(qd, out, rate, stream=s)
    s.synchronize()
    plan = g.diagnostics()["last_plan"]
    return d.cpu().numpy(), l.cpu().numpy(), out.cpu().numpy(), plan


@pytest.fixture(scope="module")
def case():
    from vfr import synth

    return synth.make_np("c1", n=100_000, q=4224)


def test_pair_matches_one_cta_and_oracle(cuda, oracle, case):
    ix, q = case
    gp = _index(cuda, ix, pair=True)
    d1, l1, o1, plan1 = _run(cuda, gp, q, 0.75)
    diag = gp.diagnostics()
    gp.close()
    g1 = _index(cuda, ix, pair=False)
    d0, l0, o0, plan0 = _run(cuda, g1, q, 0.75)
    g1.close()
    assert plan0["layout"] == "full"
    assert plan1["layout"] == "pair"
    assert plan1["keep"] == 16
    assert np.array_equal(l1, l0)
    assert np.array_equal(d1.view(np.uint32), d0.view(np.uint32))
    assert np.array_equal(o1.view(np.uint32), o0.view(np.uint32))
    assert diag["timeouts"] == 0
    o = oracle.OracleIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, 1)
    pick = np.r_[0:24, 4096:4128, 4200:4224]
    qq = np.ascontiguousarray(q[pick])
    od, _, ol, _ = o.search(qq, threads=os.cpu_count() or 1)
    expected, status = o.blend(qq, 0.75, threads=os.cpu_count() or 1)
    assert np.array_equal(l1[pick], ol)
    assert np.array_equal(d1[pick].view(np.uint32), od.view(np.uint32))
    assert (status == 0).all()
    assert np.array_equal(o1[pick].view(np.uint32), expected.view(np.uint32))
