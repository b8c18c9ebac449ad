"""Unvoiced-frame protection, the step after the retrieval blend
(crates/vocal-tensorrt/native/retrieval_protection.cu:4-33,
crates/vocal-tensorrt/src/retrieval/protection.rs:7-121).

CPU: the oracle restatement reproduces the reference's known-answer test
(protection.rs:108-184: a voiced/unvoiced boundary, the appended frame that
maps past the last HuBERT row, ratio 0 and protect >= 0.5 as no-ops).
GPU: `vocal_retrieval_protect` against the oracle, bit-exact, on both kernel
variants (float4 rows and scalar rows), the known-answer sequence replayed
from a captured graph with device scalars, and the blend with the raw copy
fused in (`vfr_retrieval_blend_save_raw`) against the plain blend.
"""
import numpy as np
import pytest

from parity_cases import make_scaled

RAW = np.array([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]], dtype=np.float32)  # protection.rs:135
F0 = np.array([0.0, 100.0, 0.0, 100.0, 0.0], dtype=np.float32)       # protection.rs:139


def kat_expected(amount: float) -> np.ndarray:
    """protection.rs:152-164: odd frames are voiced; frame 4 maps past the
    last HuBERT row and takes row 1."""
    out = np.full((5, 3), 10.0, dtype=np.float32)
    for frame in range(0, 5, 2):
        for channel in range(3):
            out[frame, channel] = np.float32(10.0 * amount + (min(frame // 2, 1) * 3 + channel + 1) * (1 - amount))
    return out


def test_oracle_reproduces_reference_kat(oracle):
    feats = np.full((5, 3), 10.0, dtype=np.float32)
    got = oracle.protect(feats, RAW, F0, 0.5, 0.33, hubert_frames=2)
    assert np.abs(got - kat_expected(0.33)).max() < 1e-6
    # ratio 0 and protect >= 0.5 leave the features alone (protection.rs:167-181)
    assert np.array_equal(oracle.protect(feats, RAW, F0, 0.0, 0.33, hubert_frames=2), feats)
    assert np.array_equal(oracle.protect(feats, RAW, F0, 0.5, 0.5, hubert_frames=2), feats)
    # protect 0 copies the raw row (protection.rs:185-190)
    assert np.array_equal(oracle.protect(feats, RAW, F0, 0.5, 0.0, hubert_frames=2)[0], RAW[0])


def test_set_amount_validation():
    from vfr.protection import RetrievalProtection

    p = RetrievalProtection(2, 3, device="cpu")
    for bad in (float("nan"), -0.1, 1.5, float("inf")):
        with pytest.raises(ValueError, match="finite and in"):
            p.set_amount(bad)
    p.set_amount(0.5)
    assert p.last_amount == 0.5 and float(p.amount[0]) == 0.5


@pytest.mark.gpu
def test_protect_kat_through_captured_graph(cuda, oracle):
    """protection.rs:126-190 step by step, the graph captured once."""
    from vfr.protection import RetrievalProtection

    torch = cuda
    dev = "cuda"
    raw = torch.from_numpy(RAW.reshape(-1).copy()).to(dev)
    feats = torch.full((15,), 10.0, device=dev)
    f0 = torch.from_numpy(F0).to(dev)
    ratio = torch.tensor([0.5], device=dev)
    prot = RetrievalProtection(2, 3)
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        prot.save_raw(raw, 2, stream=s)
        prot.apply(feats, f0, ratio, 5, 2, stream=s)
    s.synchronize()
    got = feats.cpu().numpy().reshape(5, 3)
    assert np.abs(got - kat_expected(0.33)).max() < 1e-6
    assert np.array_equal(got, oracle.protect(np.full((5, 3), 10.0, np.float32), RAW, F0, 0.5, 0.33, 2))

    ratio.fill_(0.0)
    feats.fill_(10.0)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        prot.save_raw(raw, 2, stream=s)
        prot.apply(feats, f0, ratio, 5, 2, stream=s)
    graph.replay()
    torch.cuda.synchronize()
    assert np.array_equal(feats.cpu().numpy(), np.full(15, 10.0, np.float32))
    ratio.fill_(0.5)
    graph.replay()
    torch.cuda.synchronize()
    got = feats.cpu().numpy()
    assert abs(got[0] - 3.97) < 1e-6 and np.array_equal(got[3:6], np.full(3, 10.0, np.float32))
    for amount in (0.5, 0.0, 0.33, 1.0, 0.33):
        feats.fill_(10.0)
        prot.set_amount(amount)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        got = feats.cpu().numpy().reshape(5, 3)
        want = oracle.protect(np.full((5, 3), 10.0, np.float32), RAW, F0, 0.5, amount, 2)
        assert np.array_equal(got, want), amount
    del graph


@pytest.mark.gpu
@pytest.mark.parametrize("width,offset", [(768, 0), (256, 0), (7, 0), (768, 1)])
@pytest.mark.parametrize("ratio,amount", [(0.75, 0.33), (0.75, 0.0), (float("nan"), 0.2), (0.75, 0.5), (0.0, 0.3)])
def test_protect_matches_oracle(cuda, oracle, width, offset, ratio, amount):
    """Random features, raw rows and pitch (voiced, unvoiced, negative, NaN)
    over an appended frame: the float4 kernel (width % 4 == 0, aligned) and
    the scalar one (odd width, or rows shifted off 16-byte alignment)."""
    torch = cuda
    rng = np.random.default_rng(7000 + width)
    hubert = 34
    frames = 2 * hubert + 1
    feats = rng.standard_normal((frames, width)).astype(np.float32)
    raw = rng.standard_normal((hubert, width)).astype(np.float32)
    pitch = rng.choice(np.array([0.0, 120.0, -1.0, np.nan, 230.5], dtype=np.float32), size=frames)
    want = oracle.protect(feats, raw, pitch, ratio, amount, hubert)

    from vfr import lib

    L = lib.load_library()
    buf = torch.zeros(offset + frames * width, device="cuda")
    buf[offset:] = torch.from_numpy(feats.reshape(-1))
    rbuf = torch.zeros(offset + hubert * width, device="cuda")
    rbuf[offset:] = torch.from_numpy(raw.reshape(-1))
    f0 = torch.from_numpy(pitch).cuda()
    r = torch.tensor([ratio], dtype=torch.float32, device="cuda")
    p = torch.tensor([amount], dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    s = lib.stream_struct(torch.cuda.current_stream())
    import ctypes

    lib.call(L.vocal_retrieval_protect, buf[offset:].data_ptr(), rbuf[offset:].data_ptr(), f0.data_ptr(),
             r.data_ptr(), p.data_ptr(), frames, hubert, width, ctypes.byref(s))
    torch.cuda.synchronize()
    got = buf[offset:].cpu().numpy().reshape(frames, width)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_protect_argument_errors(cuda):
    import ctypes

    from vfr import lib

    L = lib.load_library()
    t = cuda.zeros(16, device="cuda")
    s = lib.stream_struct(cuda.cuda.current_stream())
    with pytest.raises(lib.NativeError, match="null retrieval protection binding"):
        lib.call(L.vocal_retrieval_protect, t.data_ptr(), None, t.data_ptr(), t.data_ptr(), t.data_ptr(), 2, 1, 4,
                 ctypes.byref(s))
    for frames, hub, width in ((0, 1, 4), (2, 0, 4), (2, 1, 0), (2**30, 1, 4)):
        with pytest.raises(lib.NativeError, match="invalid retrieval protection dimensions"):
            lib.call(L.vocal_retrieval_protect, t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(),
                     t.data_ptr(), frames, hub, width, ctypes.byref(s))


@pytest.mark.gpu
@pytest.mark.parametrize("engine", ["tensor", "exact"])
@pytest.mark.parametrize("key", ["c4", "c1", "c3-np1"])
def test_blend_save_raw_equals_copy_then_blend(cuda, key, engine):
    """The fused raw copy: raw holds the frames before the blend and the
    blended frames equal the plain in-place blend, on the flat tensor-core
    path (raw written by the merge kernel), IVF and the exact engine (device
    copy before the blend)."""
    from vfr import GpuRetrievalIndex, lib

    ix, q, ratio = make_scaled(key)
    eng = {"tensor": lib.ENGINE_TENSOR, "exact": lib.ENGINE_EXACT}[engine]
    g = GpuRetrievalIndex.from_arrays(ix.centroids, ix.offsets, ix.vectors, ix.ids, ix.nprobe, engine=eng)
    torch = cuda
    rate = torch.tensor([ratio], device="cuda")
    plain = torch.from_numpy(q.copy()).cuda()
    fused = torch.from_numpy(q.copy()).cuda()
    raw = torch.full_like(fused, float("nan"))
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        g.blend(plain, q.shape[0], rate, stream=s)
        g.blend_save_raw(fused, raw, q.shape[0], rate, stream=s)
    s.synchronize()
    assert np.array_equal(raw.cpu().numpy().view(np.uint32), q.view(np.uint32))
    assert np.array_equal(fused.cpu().numpy().view(np.uint32), plain.cpu().numpy().view(np.uint32))
    rate.fill_(0.0)  # ratio 0: the raw copy is still taken, features unchanged
    raw.fill_(float("nan"))
    fused.copy_(torch.from_numpy(q))
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        g.blend_save_raw(fused, raw, q.shape[0], rate, stream=s)
    s.synchronize()
    assert np.array_equal(raw.cpu().numpy().view(np.uint32), q.view(np.uint32))
    assert np.array_equal(fused.cpu().numpy().view(np.uint32), q.view(np.uint32))
    with pytest.raises(lib.NativeError, match="overlaps"):
        g.blend_save_raw(fused, fused, q.shape[0], rate, stream=s)
    g.close()
