"""The RVC frontend after the retrieval blend, with the unvoiced-frame
protection fused (crates/vocal-tensorrt/native/frontend.cpp:36-75; resize
mode from crates/vocal-tensorrt/native/graph/layers.cpp:385; protection from
crates/vocal-tensorrt/native/retrieval_protection.cu:4-16).

CPU: the oracle restatement against an independent numpy statement of the
graph (append the last HuBERT frame, nearest asymmetric 2x, crop to
min(2 (h + 1), f0 frames), coarse mel pitch) and the mapping's end points
(50 Hz -> 1, 1100 Hz -> 255, unvoiced -> 1).
GPU: `vfr_rvc_frontend` against the oracle: feats and pitchf bit-exact, with
and without the protection, over crops that drop or keep the appended frame;
the coarse pitch exact wherever the unrounded mel bin is not within 1e-3 of a
rounding boundary (the graph's log is the device's `logf`, within 1 ulp of
the host's), and never off by more than one there.
"""
import ctypes

import numpy as np
import pytest


def numpy_frontend(hubert, f0):
    h = np.concatenate([hubert, hubert[-1:]], axis=0)
    resized = np.repeat(h, 2, axis=0)
    target = min(resized.shape[0], f0.shape[0])
    return resized[:target], f0[:target]


def test_oracle_matches_numpy_statement(oracle):
    rng = np.random.default_rng(11)
    for h, f in ((5, 12), (5, 9), (5, 40), (1, 1), (1, 4), (33, 66)):
        hubert = rng.standard_normal((h, 7)).astype(np.float32)
        f0 = rng.uniform(0.0, 1200.0, f).astype(np.float32)
        feats, pitchf, pitch, coarse = oracle.rvc_frontend(hubert, None, f0, 0.5, 0.33)
        want_feats, want_f0 = numpy_frontend(hubert, f0)
        assert np.array_equal(feats, want_feats) and np.array_equal(pitchf, want_f0)
        mel = 1127.0 * np.log1p(f0[: len(pitch)].astype(np.float64) / 700.0)
        lo, hi = 1127.0 * np.log1p(50.0 / 700.0), 1127.0 * np.log1p(1100.0 / 700.0)
        exact = (mel - lo) * 254.0 / (hi - lo) + 1.0
        assert np.abs(coarse - exact).max() < 1e-3
        clear = np.abs(exact - np.floor(exact) - 0.5) > 1e-3
        assert np.array_equal(pitch[clear], np.clip(np.rint(exact[clear]), 1, 255).astype(np.int32))


def test_oracle_pitch_end_points_and_protection(oracle):
    hubert = np.arange(6, dtype=np.float32).reshape(2, 3)
    raw = -np.ones((2, 3), dtype=np.float32)
    f0 = np.array([0.0, 50.0, 1100.0, 2000.0, np.nan, -5.0], dtype=np.float32)
    feats, pitchf, pitch, _ = oracle.rvc_frontend(hubert, raw, f0, 0.5, 0.25)
    assert pitch.tolist() == [1, 1, 255, 255, 1, 1]
    # frames 0, 4 and 5 are unvoiced (0, NaN, negative): 0.25 f + 0.75 raw
    assert np.array_equal(feats[1], hubert[0]) and np.array_equal(feats[2], hubert[1])
    assert np.array_equal(feats[0], np.float32(0.25) * hubert[0] - np.float32(0.75))
    assert np.array_equal(feats[4], np.float32(0.25) * hubert[1] - np.float32(0.75))  # appended frame
    plain, *_ = oracle.rvc_frontend(hubert, raw, f0, 0.0, 0.25)
    assert np.array_equal(plain, numpy_frontend(hubert, f0)[0])


def _run(torch, hubert, raw, f0, ratio, amount, stream):
    from vfr.protection import RetrievalProtection, rvc_frontend

    h, w = hubert.shape
    dev_hubert = torch.from_numpy(hubert).cuda()
    dev_f0 = torch.from_numpy(f0).cuda()
    prot = rate = None
    if raw is not None:
        prot = RetrievalProtection(h, w)
        prot.raw.copy_(torch.from_numpy(raw))
        prot.set_amount(amount)
        rate = torch.tensor([ratio], dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        out = rvc_frontend(dev_hubert, dev_f0, h, prot, rate, stream=stream)
    stream.synchronize()
    return [t.cpu().numpy() for t in out]


@pytest.mark.gpu
@pytest.mark.parametrize("h,f0_frames,width", [(32, 66, 768), (32, 64, 768), (32, 70, 768), (47, 95, 256),
                                               (1, 2, 768), (9, 17, 7)])
@pytest.mark.parametrize("protect", [None, (0.75, 0.33), (0.75, 0.5), (0.0, 0.2)])
def test_frontend_matches_oracle(cuda, oracle, h, f0_frames, width, protect):
    torch = cuda
    rng = np.random.default_rng(h * 1000 + f0_frames + width)
    hubert = rng.standard_normal((h, width)).astype(np.float32)
    raw = rng.standard_normal((h, width)).astype(np.float32)
    f0 = rng.uniform(40.0, 1200.0, f0_frames).astype(np.float32)
    f0[rng.random(f0_frames) < 0.3] = 0.0
    f0[rng.random(f0_frames) < 0.05] = np.nan
    ratio, amount = protect if protect else (0.0, 0.0)
    use_raw = raw if protect else None
    feats, pitchf, pitch = _run(torch, hubert, use_raw, f0, ratio, amount, torch.cuda.Stream())
    want_feats, want_f0, want_pitch, coarse = oracle.rvc_frontend(hubert, use_raw, f0, ratio, amount)
    assert feats.shape == want_feats.shape
    assert np.array_equal(feats.view(np.uint32), want_feats.view(np.uint32))
    assert np.array_equal(pitchf.view(np.uint32), want_f0.view(np.uint32))
    near = np.abs(coarse - np.floor(coarse) - 0.5) < 1e-3
    assert np.array_equal(pitch[~near], want_pitch[~near])
    assert np.abs(pitch.astype(np.int64) - want_pitch).max() <= 1


@pytest.mark.gpu
def test_frontend_pitch_sweep(cuda, oracle):
    """Every f0 on a 1/64 Hz grid from 0 to 1200 Hz through one call."""
    torch = cuda
    f0 = (np.arange(0, 1200 * 64, dtype=np.float32) / np.float32(64.0)).astype(np.float32)
    h = f0.shape[0] // 2
    hubert = np.zeros((h, 4), dtype=np.float32)
    _, pitchf, pitch = _run(torch, hubert, None, f0, 0.0, 0.0, torch.cuda.Stream())
    _, _, want, coarse = oracle.rvc_frontend(hubert, None, f0, 0.0, 0.0)
    near = np.abs(coarse - np.floor(coarse) - 0.5) < 1e-3
    assert near.mean() < 0.01
    assert np.array_equal(pitch[~near], want[~near])
    assert np.abs(pitch.astype(np.int64) - want).max() <= 1
    assert np.array_equal(pitchf, f0)


@pytest.mark.gpu
def test_frontend_argument_errors(cuda):
    from vfr import lib

    L = lib.load_library()
    t = cuda.zeros(64, device="cuda")
    i = cuda.zeros(64, dtype=cuda.int32, device="cuda")
    s = lib.stream_struct(cuda.cuda.Stream())
    out = ctypes.c_int32(0)
    p = t.data_ptr()
    with pytest.raises(lib.NativeError, match="null RVC frontend binding"):
        lib.call(L.vfr_rvc_frontend, None, None, p, None, None, 2, 4, 4, p, p, i.data_ptr(), ctypes.byref(out),
                 ctypes.byref(s))
    with pytest.raises(lib.NativeError, match="null retrieval protection binding"):
        lib.call(L.vfr_rvc_frontend, p, p, p, None, None, 2, 4, 4, p, p, i.data_ptr(), ctypes.byref(out),
                 ctypes.byref(s))
    for h, f, w in ((0, 4, 4), (2, 0, 4), (2, 4, 0), (2**30, 2**30, 4)):
        with pytest.raises(lib.NativeError, match="invalid RVC frontend dimensions"):
            lib.call(L.vfr_rvc_frontend, p, None, p, None, None, h, f, w, p, p, i.data_ptr(), ctypes.byref(out),
                     ctypes.byref(s))
