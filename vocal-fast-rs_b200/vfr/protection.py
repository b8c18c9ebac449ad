"""Unvoiced-frame protection over libvfr_retrieval.so.

Mirrors `RetrievalProtection` (crates/vocal-tensorrt/src/retrieval/
protection.rs:7-121): the raw HuBERT features are saved before the retrieval
blend and, after the frontend's 2x interpolation, unvoiced frames are mixed
back toward them by `vocal_retrieval_protect`.  The protection amount is a
device scalar, so a captured CUDA graph follows `set_amount`.  The save can
also be fused into the blend (`GpuRetrievalIndex.blend_save_raw`), which
replaces `save_raw`'s device copy.
"""
from __future__ import annotations

import ctypes
import math

from .lib import call, load_library, stream_struct


def _ptr(t) -> int:
    return t.data_ptr()


class RetrievalProtection:
    def __init__(self, max_hubert_frames: int, width: int, device="cuda"):
        import torch

        if max_hubert_frames <= 0 or width <= 0:
            raise ValueError("protection allocation overflow")
        self.width = width
        self.raw = torch.zeros((max_hubert_frames, width), dtype=torch.float32, device=device)
        self.amount = torch.full((1,), 0.33, dtype=torch.float32, device=device)
        self.last_amount = 0.33

    def set_amount(self, value: float) -> None:
        """protection.rs:27-40: finite and in [0, 1]; uploads only on change."""
        if not math.isfinite(value) or not 0.0 <= value <= 1.0:
            raise ValueError("protect must be finite and in [0,1]")
        if value != self.last_amount:
            self.amount.fill_(value)
            self.last_amount = value

    def save_raw(self, features, frames: int, stream=None) -> None:
        """protection.rs:42-50: device copy of the first `frames` rows."""
        import torch

        s = stream if stream is not None else torch.cuda.current_stream()
        with torch.cuda.stream(s):
            self.raw.view(-1)[: frames * self.width].copy_(features.reshape(-1)[: frames * self.width])

    def apply(self, features, pitchf, ratio, frames: int, hubert_frames: int, stream=None) -> None:
        """protection.rs:52-97, with the same geometry checks."""
        elements = frames * self.width
        feature_bytes = features.numel() * features.element_size()
        if (frames == 0 or hubert_frames == 0 or elements > 2**31 - 1 or elements * 4 > feature_bytes
                or hubert_frames * self.width * 4 > self.raw.numel() * 4
                or frames * 4 > pitchf.numel() * pitchf.element_size() or ratio.numel() * ratio.element_size() < 4):
            raise ValueError("invalid protection buffer geometry")
        load_library()
        s = stream_struct(stream)
        call(load_library().vocal_retrieval_protect, _ptr(features), _ptr(self.raw), _ptr(pitchf), _ptr(ratio),
             _ptr(self.amount), ctypes.c_int32(frames), ctypes.c_int32(hubert_frames), ctypes.c_int32(self.width),
             ctypes.byref(s))


def rvc_frontend(hubert, f0, hubert_frames: int, protection: "RetrievalProtection | None" = None, ratio=None,
                 stream=None):
    """The RVC frontend after the blend (crates/vocal-tensorrt/native/
    frontend.cpp:36-75) with the protection fused when `protection` is given
    (its raw rows and amount, with the device `ratio`): returns CUDA tensors
    (feats [target, width], pitchf [target], pitch [target] int32)."""
    import torch

    width = hubert.shape[-1]
    f0_frames = f0.numel()
    target = min(2 * (hubert_frames + 1), f0_frames)
    feats = torch.empty((target, width), dtype=torch.float32, device=hubert.device)
    pitchf = torch.empty(target, dtype=torch.float32, device=hubert.device)
    pitch = torch.empty(target, dtype=torch.int32, device=hubert.device)
    out = ctypes.c_int32(0)
    L = load_library()
    s = stream_struct(stream)
    raw = amount = rate = None
    if protection is not None:
        raw, amount, rate = _ptr(protection.raw), _ptr(protection.amount), _ptr(ratio)
    call(L.vfr_rvc_frontend, _ptr(hubert), raw, _ptr(f0), rate, amount, ctypes.c_int32(hubert_frames),
         ctypes.c_int32(f0_frames), ctypes.c_int32(width), _ptr(feats), _ptr(pitchf), _ptr(pitch), ctypes.byref(out),
         ctypes.byref(s))
    assert out.value == target
    return feats, pitchf, pitch


def engine_frontend(blended, frames: int, raw=None, hz=None, protect: float = 0.33, stream=None):
    """The generic engine's frontend (crates/vocal-engine/src/pipeline.rs:
    75-96, 312-333, 625-633) on the device: returns (features [2 frames,
    width], coarse [min(2 frames, hz frames)] int32 or None)."""
    import torch

    width = blended.shape[-1]
    out = torch.empty((2 * frames, width), dtype=torch.float32, device=blended.device)
    coarse = None
    hz_frames = 0
    if hz is not None:
        hz_frames = hz.numel()
        coarse = torch.empty(min(2 * frames, hz_frames), dtype=torch.int32, device=blended.device)
    s = stream_struct(stream)
    call(load_library().vfr_engine_frontend, _ptr(blended), None if raw is None else _ptr(raw),
         None if hz is None else _ptr(hz), ctypes.c_float(protect), ctypes.c_int32(frames), ctypes.c_int32(hz_frames),
         ctypes.c_int32(width), _ptr(out), None if coarse is None or coarse.numel() == 0 else _ptr(coarse),
         ctypes.byref(s))
    return out, coarse
