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
The generic engine's frontend (crates/vocal-engine/src/pipeline.rs:75-96,
312-333, 625-633; `vfr_engine_frontend`) the same way: linear 2x, protection
on every frame, f0_to_coarse with Rust's rounding and NaN cast.
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


# ----------------------------------------------------------- engine frontend
# crates/vocal-engine/src/pipeline.rs: interpolate_2x (75-96), the protection
# of RvcPipeline::run (312-333) and f0_to_coarse (625-633).


def numpy_engine_frontend(blended, raw, hz, protect):
    """An independent numpy statement of the Rust code, in f32 with each
    operation rounded."""
    f32 = np.float32
    frames, width = blended.shape

    def interp(x):
        out = np.empty((2 * frames, width), np.float32)
        for t in range(2 * frames):
            source = f32(t) / f32(2.0)
            left = int(np.floor(source))
            right = min(left + 1, frames - 1)
            w = f32(source - f32(left))
            out[t] = x[left] * (f32(1.0) - w) + x[right] * w
        return out

    feats = interp(blended)
    coarse = None
    if hz is not None:
        limit = min(2 * frames, hz.shape[0])
        if raw is not None and protect < 0.5:
            before = interp(raw)
            p = f32(min(max(protect, 0.0), 1.0))
            for t in range(limit):
                v = f32(1.0) if hz[t] > 0 else p
                feats[t] = feats[t] * v + before[t] * (f32(1.0) - v)
        coarse = np.empty(limit, np.int32)
        with np.errstate(invalid="ignore"):
            for t in range(limit):
                coarse[t] = numpy_f0_to_coarse(hz[t])
    return feats, coarse


def numpy_f0_to_coarse(f0):
    f32 = np.float32
    f0 = f32(f0)
    if f0 <= 0:
        return 1
    lo = f32(1127.0) * np.log(f32(1.0) + f32(50.0) / f32(700.0))
    hi = f32(1127.0) * np.log(f32(1.0) + f32(1100.0) / f32(700.0))
    mel = f32(1127.0) * np.log(f32(1.0) + f0 / f32(700.0))
    x = (mel - lo) * f32(254.0) / (hi - lo) + f32(1.0)
    if np.isnan(x):
        return 0
    r = np.floor(np.abs(x) + f32(0.5)) * np.sign(x)  # half away from zero
    return int(min(max(r, 1.0), 255.0))


def test_engine_oracle_matches_numpy_statement(oracle):
    rng = np.random.default_rng(21)
    for frames, hz_frames, width, protect in ((5, 10, 3, 0.33), (5, 7, 3, 0.2), (5, 14, 4, 0.0), (1, 2, 6, 0.4),
                                             (6, 12, 5, 0.5), (3, 0, 2, 0.1)):
        blended = rng.standard_normal((frames, width)).astype(np.float32)
        raw = rng.standard_normal((frames, width)).astype(np.float32)
        hz = rng.uniform(-50.0, 1300.0, hz_frames).astype(np.float32)
        hz[::3] = 0.0
        want, want_c = numpy_engine_frontend(blended, raw, hz, protect)
        got, got_c = oracle.engine_frontend(blended, raw, hz, protect)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert np.array_equal(got_c, want_c)
    got, coarse = oracle.engine_frontend(blended, None, None, 0.33)
    assert coarse is None and np.array_equal(got, numpy_engine_frontend(blended, None, None, 0.33)[0])


def test_engine_coarse_end_points(oracle):
    """f0_to_coarse at its edges: unvoiced and negative -> 1, NaN -> 0 (the
    saturating cast), 50 Hz -> 1, 1100 Hz and above -> 255, and agreement
    with the reference's own numpy mapping (scripts/compare-native-python.py
    quantize_f0) away from rounding ties."""
    hz = np.array([0.0, -3.0, np.nan, 50.0, 1100.0, 5000.0, 140.0], dtype=np.float32)
    _, coarse = oracle.engine_frontend(np.zeros((4, 1), np.float32), None, hz, 0.33)
    assert coarse.tolist()[:6] == [1, 1, 0, 1, 255, 255]
    f0 = np.linspace(1.0, 1200.0, 5000, dtype=np.float32)
    _, coarse = oracle.engine_frontend(np.zeros((2500, 1), np.float32), None, f0, 0.33)
    mel = 1127.0 * np.log1p(f0.astype(np.float64) / 700.0)
    lo, hi = 1127.0 * np.log1p(50.0 / 700.0), 1127.0 * np.log1p(1100.0 / 700.0)
    exact = (mel - lo) * 254.0 / (hi - lo) + 1.0
    clear = np.abs(exact - np.floor(exact) - 0.5) > 1e-3
    assert np.array_equal(coarse[clear], np.clip(np.rint(exact[clear]), 1, 255).astype(np.int32))


@pytest.mark.gpu
@pytest.mark.parametrize("frames,hz_frames,width", [(32, 64, 768), (32, 50, 768), (32, 90, 256), (1, 2, 768),
                                                    (9, 18, 7), (47, 94, 256)])
@pytest.mark.parametrize("mode", ["plain", "protect", "pitch-only", "protect-0.5"])
def test_engine_frontend_matches_oracle(cuda, oracle, frames, hz_frames, width, mode):
    from vfr.protection import engine_frontend

    torch = cuda
    rng = np.random.default_rng(frames * 100 + hz_frames + width)
    blended = rng.standard_normal((frames, width)).astype(np.float32)
    blended[0, 0] = -0.0  # signed zeros survive a (1 - 0) + b 0 only when computed literally
    raw = rng.standard_normal((frames, width)).astype(np.float32)
    hz = rng.uniform(40.0, 1200.0, hz_frames).astype(np.float32)
    hz[rng.random(hz_frames) < 0.3] = 0.0
    hz[rng.random(hz_frames) < 0.05] = np.nan
    use_raw = raw if mode in ("protect", "protect-0.5") else None
    use_hz = None if mode == "plain" else hz
    protect = 0.5 if mode == "protect-0.5" else 0.33
    want, want_c = oracle.engine_frontend(blended, use_raw, use_hz, protect)
    s = torch.cuda.Stream()
    b = torch.from_numpy(blended).cuda()
    r = None if use_raw is None else torch.from_numpy(use_raw).cuda()
    h = None if use_hz is None else torch.from_numpy(use_hz).cuda()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        got, coarse = engine_frontend(b, frames, r, h, protect, stream=s)
    s.synchronize()
    got = got.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    if use_hz is None:
        assert coarse is None
        return
    coarse = coarse.cpu().numpy()
    mel = 1127.0 * np.log1p(use_hz[: len(want_c)].astype(np.float64) / 700.0)
    lo, hi = 1127.0 * np.log1p(50.0 / 700.0), 1127.0 * np.log1p(1100.0 / 700.0)
    with np.errstate(invalid="ignore"):
        exact = (mel - lo) * 254.0 / (hi - lo) + 1.0
        near = np.abs(exact - np.floor(exact) - 0.5) < 1e-3
    assert np.array_equal(coarse[~near], want_c[~near])
    assert np.abs(coarse.astype(np.int64) - want_c).max() <= 1


@pytest.mark.gpu
def test_engine_frontend_argument_errors(cuda):
    from vfr import lib

    L = lib.load_library()
    t = cuda.zeros(64, device="cuda")
    s = lib.stream_struct(cuda.cuda.Stream())
    p = t.data_ptr()
    with pytest.raises(lib.NativeError, match="null engine frontend binding"):
        lib.call(L.vfr_engine_frontend, p, None, p, ctypes.c_float(0.3), 2, 4, 4, p, None, ctypes.byref(s))
    for bad in (float("nan"), -0.1, 1.5):
        with pytest.raises(lib.NativeError, match="finite and in"):
            lib.call(L.vfr_engine_frontend, p, None, None, ctypes.c_float(bad), 2, 0, 4, p, None, ctypes.byref(s))
    for frames, width in ((0, 4), (2, 0), (1 << 23 + 1, 1), (1 << 20, 2048)):
        with pytest.raises(lib.NativeError, match="invalid engine frontend dimensions"):
            lib.call(L.vfr_engine_frontend, p, None, None, ctypes.c_float(0.3), frames, 0, width, p, None,
                     ctypes.byref(s))
