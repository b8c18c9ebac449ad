#!/usr/bin/env python
"""Benchmark of the feature-retrieval hot path (k=8 L2 search + inverse-square
gather-blend) on B200, one process per GPU.

Headline workload (`--workload c5`, default): flat index of N=4,000,000 x 768
fp32 rows from a seeded 4,096-component Gaussian mixture, Q=30,000 query
frames per step, k=8, blend at index_rate 0.75.  With --gpus N>1 the rows are
sharded across ranks (NCCL all-gather of per-shard top-8 + merge + exact
blend), so the total work per step is fixed (strong scaling).  A step is one
blend of the Q frames (out of place, so every step sees the same inputs).

Printed JSON line (rank 0): value = frames/s of the whole job over K timed
steps (device time, max over ranks); e2e = the same metric through the
drop-in C ABI (vocal_faiss_gpu_blend) with pinned host buffers and the
host<->device copies inside the timed region; roofline = the candidate GEMM
kernel (cand_kernel) timed with CUDA events on its stream during the timed
steps; cpu_baseline = the CPU oracle (restatement of the reference's CPU
retrieval) on a bounded sample of frames against the same database, all host
cores; streaming = the c4 realtime config (Q=32 frames per block, N=100,000)
replayed as a CUDA graph, p50/p95 per-block latency over 1,000 blocks; ivf =
the c3 IVF-Flat config (200k rows, nlist 256, 30k frames) at nprobe 1 and 8,
each with a roofline from the lists the frames actually probe; c1 / c2 = those
configs' blends (graph replay, L2 flushed or warm) with the candidate
kernel's roofline; published_shape = a seeded stand-in for the reference's
published IVF511 timings (34 and 140 frames); parity (every N) = rank 0's
first 64 output frames of a full-size step against the CPU oracle's exact
scan of all rows.

`--impl reference` times the reference's CPU retrieval (the oracle port; the
Rust original cannot be built here) on the same workload instead.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import struct
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "vocal-fast-rs_b200"), ROOT]

METRIC = "kNN queries/s (768-d, k=8) at 1/2/4/8 B200; p50 per-block latency"
UNIT = "queries/s"


def args_parse():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["vfr", "reference"], default="vfr")
    ap.add_argument("--workload", default="c5", choices=["c1", "c2", "c4", "c5"])
    ap.add_argument("--queries", type=int, default=0, help="override frames per step")
    ap.add_argument("--rows", type=int, default=0, help="override database rows (testing only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-streaming", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-ingest", action="store_true", help="skip the c5 index-ingest timing")
    ap.add_argument("--no-training", action="store_true", help="skip the IVF training timing")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of rank 0's first frames")
    ap.add_argument("--no-configs", action="store_true", help="skip the c1/c2/published-shape timings")
    ap.add_argument("--no-cublas", action="store_true", help="skip the same-box cuBLAS reference")
    return ap.parse_args()


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self, devices):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in devices:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None, "samples": len(sm), "reasons": sorted(reasons)}


def cublas_same_box(device):
    """torch.matmul bf16 8192^3 (cuBLAS) back to back for about 2 s on this
    GPU with the SM clock sampled: the same-box reference for the candidate
    kernel's tensor rate (the measured peaks come from another box, and the
    clock under the power cap differs between boxes)."""
    import torch

    a = torch.randn(8192, 8192, dtype=torch.bfloat16, device=device)
    b = torch.randn_like(a)
    c = torch.empty_like(a)
    for _ in range(20):
        torch.matmul(a, b, out=c)
    torch.cuda.synchronize()
    sampler = ClockSampler()
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 2500
    e0.record()
    for _ in range(reps):
        torch.matmul(a, b, out=c)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop({torch.cuda.current_device()})
    ms = e0.elapsed_time(e1) / reps
    del a, b, c
    torch.cuda.empty_cache()
    return {"tflops": 2 * 8192 ** 3 / ms / 1e9, "ms_per_gemm": ms, "clocks": clocks,
            "what": "torch.matmul bf16 8192^3, 2,500 back to back on this GPU after the timed steps"}


def dist_setup(gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    return world, rank, local


# ---------------------------------------------------------------------------- reference arm
def run_reference(a, world, rank):
    if rank != 0:
        return  # rank 0 alone runs the CPU reference
    import numpy as np
    import torch

    from oracle import oracle
    from vfr import synth

    w = synth.CONFIGS[a.workload]
    n = a.rows or w.n
    dev = "cuda" if torch.cuda.is_available() else None
    if dev:
        arrays, queries = synth.make_torch(a.workload, dev, n=n, q=a.queries or w.q)
        vectors = arrays["vectors"].cpu().numpy()
        queries = queries.cpu().numpy()
        del arrays
        torch.cuda.empty_cache()
    else:
        ix, queries = synth.make_np(a.workload, n=n, q=a.queries or w.q)
        vectors = ix.vectors
    flat = synth.flat_arrays(vectors)
    orc = oracle.OracleIndex.from_arrays(flat.centroids, flat.offsets, flat.vectors, flat.ids, 1)
    cores = os.cpu_count() or 1
    sample = max(cores, 8)
    times = []
    for step in range(a.warmup + a.steps):
        s0 = (step * sample) % max(1, queries.shape[0] - sample)
        t0 = time.perf_counter()
        orc.blend(queries[s0:s0 + sample], w.ratio, threads=cores)
        dt = time.perf_counter() - t0
        if step >= a.warmup:
            times.append(dt)
    value = sample * len(times) / sum(times)
    desc = f"{sample} frames per step against all {n} rows, {cores} threads, AVX2 order"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": 1000 * sum(times) / len(times), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(a, w, n, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(a, w, n, world):
    return {"workload": f"{w.key} {w.name}: flat N={n} x {w.d} fp32, Q={a.queries or w.q} frames/step, k=8, "
                        f"index_rate={w.ratio}",
            "rows": n, "dims": w.d, "frames_per_step": a.queries or w.q, "k": 8, "index_rate": w.ratio,
            "sharding": f"rows/{world}" if world > 1 else "none",
            "l2": "inputs larger than L2 (fp16 row shadow alone exceeds 126 MB)"}


# ---------------------------------------------------------------------------- our arm
def cpu_baseline(vectors, queries, ratio, n):
    from oracle import oracle
    from vfr import synth

    cores = os.cpu_count() or 1
    flat = synth.flat_arrays(vectors)
    orc = oracle.OracleIndex.from_arrays(flat.centroids, flat.offsets, flat.vectors, flat.ids, 1)
    sample = max(cores, 8)
    t0 = time.perf_counter()
    orc.blend(queries[:sample], ratio, threads=cores)
    dt = time.perf_counter() - t0
    # the reference's own loop is serial (crates/vocal-cpu/src/pipeline.rs:295-299): one thread, two frames
    t1 = time.perf_counter()
    orc.blend(queries[:2], ratio, threads=1)
    dt1 = time.perf_counter() - t1
    return {"value": sample / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"first {sample} frames against all {n} rows ({dt:.1f} s), AVX2-order C restatement, "
                      f"{cores} threads",
            "single_core": {"value": 2 / dt1, "unit": UNIT, "cores": 1,
                            "sample": f"first 2 frames against all {n} rows ({dt1:.2f} s), one thread, the "
                                      "reference's serial loop"}}


PARITY_FRAMES = 64
STEP_TIMEOUT_S = 120.0  # host deadline of one row-sharded step's collectives


def parity_check(vectors, q, out, dist, labels, ratio, n):
    """Bit-level comparison of the benchmarked path's output for frames
    `q` (blended `out`, top-8 `dist`/`labels` of the same full-size step)
    with the oracle (C restatement of crates/vocal-cpu/src/retrieval.rs:27-83)
    scanning all n rows on every host thread."""
    import numpy as np

    from oracle import oracle
    from vfr import synth

    cores = os.cpu_count() or 1
    flat = synth.flat_arrays(vectors)
    orc = oracle.OracleIndex.from_arrays(flat.centroids, flat.offsets, flat.vectors, flat.ids, 1)
    t0 = time.perf_counter()
    expected, status = orc.blend(q, ratio, threads=cores)
    od, _, ol, _ = orc.search(q, threads=cores)
    dt = time.perf_counter() - t0
    return {"frames": int(q.shape[0]), "rows": n, "label_mismatches": int((ol != labels).any(1).sum()),
            "distance_bit_mismatches": int((od.view(np.uint32) != dist.view(np.uint32)).any(1).sum()),
            "blend_bit_mismatches": int((expected.view(np.uint32) != out.view(np.uint32)).any(1).sum()),
            "oracle_status_nonzero": int((status != 0).sum()), "oracle_s": dt, "oracle_threads": cores,
            "what": "rank 0's first output frames of one full-size step vs the CPU oracle's exact scan of all rows"}


def streaming(device):
    """c4: Q=32-frame blocks against 100k rows, CUDA-graph replay, per-block latency."""
    import numpy as np
    import torch

    from vfr import GpuRetrievalIndex, synth

    w = synth.CONFIGS["c4"]
    arrays, block0 = synth.make_torch("c4", device, q=w.q)
    g = torch.Generator(device=device)
    g.manual_seed(4004)
    blocks = torch.empty((w.blocks, w.q, w.d), device=device)
    blocks[0] = block0
    for b in range(1, w.blocks):
        blocks[b] = blocks[b - 1] + w.walk * torch.randn((w.q, w.d), generator=g, device=device)
    idx = GpuRetrievalIndex.from_arrays(arrays["centroids"], arrays["offsets"], arrays["vectors"], arrays["ids"], 1,
                                        max_frames=w.q)
    del arrays
    feats = torch.empty((w.q, w.d), device=device)
    rate = torch.tensor([w.ratio], device=device)
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        feats.copy_(blocks[0])
        idx.blend(feats, w.q, rate, stream=s)
        graph = torch.cuda.CUDAGraph()
        feats.copy_(blocks[0])
        with torch.cuda.graph(graph, stream=s):
            idx.blend(feats, w.q, rate, stream=s)
        start = [torch.cuda.Event(enable_timing=True) for _ in range(w.blocks)]
        end = [torch.cuda.Event(enable_timing=True) for _ in range(w.blocks)]
        for b in range(20):
            feats.copy_(blocks[b])
            graph.replay()
        for b in range(w.blocks):
            feats.copy_(blocks[b])  # reset outside the events, as the reference benchmark does
            start[b].record(s)
            graph.replay()
            end[b].record(s)
    s.synchronize()
    lat = sorted(start[b].elapsed_time(end[b]) for b in range(w.blocks))
    diag = idx.diagnostics()
    del graph
    idx.close()
    p50 = lat[len(lat) // 2]
    hbm_bytes = 100_000 * 768 * 2 + 100_000 * 4 + w.q * 64 * 768 * 4
    peak = measured_peaks()[0].get("hbm_gbs", 6650.0)
    return {"workload": "c4 rvc-v2-stream-100k: flat N=100000 x 768, 1000 blocks of Q=32 (random walk), graph replay",
            "p50_block_ms": p50, "p95_block_ms": lat[int(len(lat) * 0.95)], "mean_block_ms": sum(lat) / len(lat),
            "blocks": w.blocks, "frames_per_s_at_p50": w.q / (p50 / 1000),
            "hbm_bytes_per_block": hbm_bytes, "hbm_gbs_at_p50": hbm_bytes / (p50 / 1000) / 1e9,
            "hbm_frac_at_p50": hbm_bytes / (p50 / 1000) / 1e9 / peak,
            "fallback_frames": diag["fallback_frames"]}


def protection(device):
    """The step after the blend on the realtime path: the raw copy fused into
    the blend (vfr_retrieval_blend_save_raw) against the reference's separate
    device copy + blend, and vocal_retrieval_protect on the interpolated block
    (2 x 32 + 1 frames x 768, half of them unvoiced), and the frontend with
    the protection fused (vfr_rvc_frontend) against frontend + protect, each
    replayed from a CUDA graph (p50 over 200 replays)."""
    import torch

    from vfr import GpuRetrievalIndex, synth
    from vfr.protection import RetrievalProtection, engine_frontend, rvc_frontend

    w = synth.CONFIGS["c4"]
    arrays, block = synth.make_torch("c4", device, q=w.q)
    idx = GpuRetrievalIndex.from_arrays(arrays["centroids"], arrays["offsets"], arrays["vectors"], arrays["ids"], 1,
                                        max_frames=w.q)
    del arrays
    rate = torch.tensor([w.ratio], device=device)
    feats = block.clone()
    prot = RetrievalProtection(w.q, w.d, device=device)
    frames = 2 * w.q + 1
    interp = torch.randn((frames, w.d), device=device)
    g = torch.Generator(device=device)
    g.manual_seed(5005)
    pitch = torch.where(torch.rand(frames, generator=g, device=device) < 0.5, 0.0, 150.0)
    s = torch.cuda.Stream()

    def p50(fn):
        torch.cuda.synchronize()
        with torch.cuda.stream(s):
            fn()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                fn()
            for _ in range(20):
                graph.replay()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(200)]
            for a, b in ev:
                a.record(s)
                graph.replay()
                b.record(s)
        s.synchronize()
        lat = sorted(a.elapsed_time(b) for a, b in ev)
        del graph
        return lat[len(lat) // 2] * 1000.0

    def copy_then_blend():
        prot.save_raw(feats, w.q, stream=s)
        idx.blend(feats, w.q, rate, stream=s)

    t_copy = p50(copy_then_blend)
    t_fused = p50(lambda: idx.blend_save_raw(feats, prot.raw, w.q, rate, stream=s))
    t_protect = p50(lambda: prot.apply(interp, pitch, rate, frames, w.q, stream=s))
    # the frontend (append, 2x, crop, coarse pitch) on the same block, f0 of
    # 2 (q + 1) frames: separate frontend + protect as in the reference's
    # pipeline, then the fused kernel
    f0 = torch.where(torch.rand(2 * (w.q + 1), generator=g, device=device) < 0.5, 0.0, 150.0)

    def frontend_then_protect():
        out, pf, _ = rvc_frontend(feats, f0, w.q, stream=s)
        prot.apply(out, pf, rate, out.shape[0], w.q, stream=s)

    t_front_sep = p50(frontend_then_protect)
    t_front = p50(lambda: rvc_frontend(feats, f0, w.q, prot, rate, stream=s))
    # the generic engine's linear frontend with its protection and coarse pitch
    hz = torch.where(torch.rand(2 * w.q, generator=g, device=device) < 0.5, 0.0, 150.0)
    t_engine = p50(lambda: engine_frontend(feats, w.q, prot.raw, hz, 0.33, stream=s))
    idx.close()
    unvoiced = int((pitch <= 0).sum().item())
    bytes_protect = unvoiced * w.d * 4 * 3 + frames * 4
    return {"workload": f"c4 block: {w.q} HuBERT frames, {frames} interpolated frames x {w.d}, {unvoiced} unvoiced",
            "copy_then_blend_us_p50": t_copy, "blend_save_raw_us_p50": t_fused,
            "protect_us_p50": t_protect, "protect_bytes": bytes_protect,
            "protect_gbs_at_p50": bytes_protect / (t_protect * 1e-6) / 1e9,
            "frontend_then_protect_us_p50": t_front_sep, "frontend_fused_us_p50": t_front,
            "engine_frontend_us_p50": t_engine}


def ingest(device):
    """Index ingest for c5 (flat 4,000,000 x 768, a 12.3 GB FAISS image in
    host memory): the reference's route (host parse RetrievalIndex::from_faiss,
    then create from the host arrays with pageable copies) against
    vfr_index_load (rows straight from the image through pinned staging
    buffers on several host threads, row check on the device), and a
    shared-storage hit (content hash, no upload).  Wall-clock seconds of one
    load each, device synchronised on both sides."""
    import time

    import numpy as np
    import torch

    from vfr import GpuRetrievalIndex, RetrievalIndex, faiss_io, synth

    arrays, _ = synth.make_torch("c5", device, q=1)
    v = arrays["vectors"]
    n, d = v.shape
    head = faiss_io._index_header(b"IxF2", d, n) + struct.pack("<Q", n * d)
    raw = np.empty(len(head) + n * d * 4 + 64, np.uint8)
    # rows 64-byte aligned in the buffer, as a page-aligned file mapping would leave them
    start = (-(raw.ctypes.data + len(head))) % 64
    image = raw[start:start + len(head) + n * d * 4]
    image[:len(head)] = np.frombuffer(head, np.uint8)
    torch.from_numpy(image[len(head):].view(np.float32).reshape(n, d)).copy_(v)
    del arrays, v
    torch.cuda.empty_cache()

    def timed(fn):
        torch.cuda.synchronize()
        t = time.perf_counter()
        r = fn()
        torch.cuda.synchronize()
        return r, time.perf_counter() - t

    host, t_parse = timed(lambda: RetrievalIndex.from_faiss(image))
    g, t_create = timed(lambda: GpuRetrievalIndex.upload(host))
    g.close()
    del host
    g, t_load = timed(lambda: GpuRetrievalIndex.load(image))
    g.close()
    first, t_first = timed(lambda: GpuRetrievalIndex.load(image, share=True))
    hit, t_hit = timed(lambda: GpuRetrievalIndex.load(image, share=True))
    shared = hit.diagnostics()["shared_handles"]
    hit.close()
    first.close()
    nbytes = int(image.size)
    return {"workload": f"c5 image: flat {n} x {d} FAISS IxF2, {nbytes} bytes in host memory",
            "reference_parse_s": t_parse, "create_from_host_arrays_s": t_create,
            "reference_route_s": t_parse + t_create, "load_s": t_load, "load_gbs": nbytes / t_load / 1e9,
            "load_shared_first_s": t_first, "load_shared_hit_s": t_hit, "shared_handles": shared}


def training(device, cpu_threads: int):
    """IVF training, the reference's offline FAISS step (IndexIVFFlat train +
    add), on c5's rows: the first 200,000 into 256 lists and all 4,000,000
    into 4,096 lists; vfr_kmeans (10 iterations on at most 256 sampled rows
    per list) then vfr_ivf_build (every row assigned and gathered into its
    list).  Wall-clock seconds with the device synchronised.  The CPU
    restatement (oracle) runs one k-means iteration of the 256-list case on
    the host threads for scale."""
    import time

    import torch

    from vfr import synth
    from vfr.training import build_ivf_index, kmeans

    arrays, _ = synth.make_torch("c5", device, q=1)
    x = arrays["vectors"]
    del arrays
    out = {"workload": "c5 rows (Gaussian mixture, 768-d): 200k rows -> 256 lists, 4M rows -> 4096 lists; "
                       "10 k-means iterations, <= 256 sampled rows per list, then every row assigned"}
    for name, rows, lists in (("lists256_rows200k", 200_000, 256), ("lists4096_rows4m", x.shape[0], 4096)):
        xs = x[:rows].contiguous()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        c, obj = kmeans(xs, lists, niter=10, max_points_per_centroid=256, seed=1234)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        g = build_ivf_index(xs, c, nprobe=8)
        torch.cuda.synchronize()
        t2 = time.perf_counter()
        g.close()
        out[name] = {"kmeans_s": t1 - t0, "build_s": t2 - t1, "total_s": t2 - t0,
                     "objective_first": float(obj[0]), "objective_last": float(obj[-1])}
        del xs, c
    if cpu_threads > 0:
        from oracle import oracle as orc

        xs = x[:200_000].cpu().numpy()
        t0 = time.perf_counter()
        orc.kmeans(xs, 256, niter=1, max_points_per_centroid=256, seed=1234, threads=cpu_threads)
        out["cpu_baseline_one_iteration_lists256_s"] = time.perf_counter() - t0
        out["cpu_threads"] = cpu_threads
    del x
    torch.cuda.empty_cache()
    return out


def _replay_latency(fn, s, reps, pre=None):
    """Captures fn() into a CUDA graph on stream s, replays it 20 times, then
    times `reps` replays with CUDA events on s; `pre` (an L2 flush, an input
    reset) runs before each timed replay, outside the events.  Returns
    (p50, p95, mean) in ms."""
    import torch

    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        fn()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            fn()
        for _ in range(20):
            graph.replay()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for a, b in ev:
            if pre is not None:
                pre()
            a.record(s)
            graph.replay()
            b.record(s)
    s.synchronize()
    lat = sorted(a.elapsed_time(b) for a, b in ev)
    del graph
    return lat[len(lat) // 2], lat[int(len(lat) * 0.95)], sum(lat) / len(lat)


L2_FLUSH_BYTES = 256 << 20  # written between timed replays: twice the 126 MB L2


def _flat_roofline(q, n, d, kernel_s, peaks, peak_kind, flops_key="bf16_tflops"):
    """Roofline of one flat candidate launch: 2*Q*N*d FLOP on the tensor pipe
    against N*(2*d_pad + 4) bytes of streamed fp16 rows and fp32 norms; the
    bound is whichever takes longer at the measured peaks."""
    d_pad = (d + 63) // 64 * 64
    flops = 2.0 * q * n * d
    nbytes = float(n) * (2 * d_pad + 4)
    tf = peaks.get(flops_key, 1590.0)
    hbm = peaks.get("hbm_gbs", 6650.0)
    t_f, t_b = flops / (tf * 1e12), nbytes / (hbm * 1e9)
    if t_f >= t_b:
        ach = flops / kernel_s / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": tf, "unit": "TFLOP/s", "frac": ach / tf,
                "peak_source": f"{peak_kind} {flops_key}", "algorithmic_flop": flops, "algorithmic_bytes": nbytes,
                "bound_us": t_f * 1e6, "kernel_us": kernel_s * 1e6}
    ach = nbytes / kernel_s / 1e9
    return {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
            "peak_source": f"{peak_kind} hbm_gbs", "algorithmic_flop": flops, "algorithmic_bytes": nbytes,
            "bound_us": t_b * 1e6, "kernel_us": kernel_s * 1e6}


def flat_config(device, key):
    """c1 (20,000 x 768, 250 frames, ratio 0.75) or c2 (50,000 x 256, 1,000
    frames, ratio 0.5): one out-of-place blend of the config's frames,
    replayed from a CUDA graph.  `cold` overwrites a 256 MB buffer between
    replays (outside the events), so the index (30.7 / 25.6 MB of fp16 rows)
    is not left in L2 by the previous call; `warm` leaves it there, as back
    to back realtime blocks would.  The roofline is the candidate kernel's
    CUDA-event time over 20 eager calls (L2 flushed before each) against the
    larger of the tensor and HBM bounds at the burst peaks (a kernel timed
    on its own)."""
    import torch

    from vfr import GpuRetrievalIndex, synth

    w = synth.CONFIGS[key]
    arrays, queries = synth.make_torch(key, device)
    idx = GpuRetrievalIndex.from_arrays(arrays["centroids"], arrays["offsets"], arrays["vectors"], arrays["ids"], 1,
                                        max_frames=w.q)
    del arrays
    out = torch.empty_like(queries)
    rate = torch.tensor([w.ratio], device=device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    s = torch.cuda.Stream()

    def call():
        idx.blend_from(queries, out, rate, stream=s)

    cold = _replay_latency(call, s, 200, pre=lambda: flush.fill_(1.0))
    warm = _replay_latency(call, s, 200)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        idx.profile(True)
        for _ in range(20):
            flush.fill_(1.0)
            call()
    s.synchronize()
    prof = idx.profile(False)
    diag = idx.diagnostics()
    idx.close()
    cand = prof["cand_kernel"]
    cand_s = cand["ms"] / max(1, cand["launches"]) / 1000.0
    peaks, peak_kind = measured_peaks()
    roof = _flat_roofline(w.q, w.n, w.d, cand_s, peaks, peak_kind)
    roof["kernel"] = "cand_kernel"
    roof["call_frac_at_cold_p50"] = roof["bound_us"] / (cold[0] * 1000.0)
    return {"workload": f"{w.key} {w.name}: flat N={w.n} x {w.d}, Q={w.q} frames per call, k=8, "
                        f"index_rate={w.ratio}, graph replay (200 timed)",
            "queries_per_s_cold_p50": w.q / (cold[0] / 1000.0), "cold_p50_ms": cold[0], "cold_p95_ms": cold[1],
            "queries_per_s_warm_p50": w.q / (warm[0] / 1000.0), "warm_p50_ms": warm[0], "warm_p95_ms": warm[1],
            "l2": f"cold: {L2_FLUSH_BYTES >> 20} MB written between replays; warm: index left L2-resident",
            "kernels_ms": {k: v["ms"] / max(1, v["launches"]) for k, v in prof.items()},
            "plan": diag["last_plan"], "fallback_frames": diag["fallback_frames"], "roofline": roof}


def published_shape(device):
    """Stand-in for the reference's only published timings of this path
    (docs/faiss-gpu-retrieval.md:59-79: RTX 3060, a real IVF511,Flat
    nprobe=1 index of 19,949 768-d vectors, ratio 0.5, CUDA-graph replay
    medians 0.127 ms for 34 frames and 0.242 ms for 140): a seeded mixture
    index of the same shape (511 lists from 20 k-means iterations), the same
    block sizes and ratio, graph replay of vocal_faiss_gpu_blend with the
    frames reset before each replay (outside the events), p50/p95 over 500
    replays, for the default engine and the exact SIMT engine."""
    import torch

    from vfr import GpuRetrievalIndex, lib, synth

    w = synth.CONFIGS["ivf511"]
    arrays, queries = synth.make_torch("ivf511", device, q=max(w.extra["blocks"]))
    rate = torch.tensor([w.ratio], device=device)
    s = torch.cuda.Stream()
    out = {"workload": f"IVF-Flat N={w.n} x {w.d}, nlist={w.nlist}, nprobe=1, ratio {w.ratio}; seeded stand-in "
                       f"for the reference's published IVF511 index",
           "reference_published_ms_p50": {"34": 0.127, "140": 0.242},
           "reference_hardware": "RTX 3060 (docs/faiss-gpu-retrieval.md:69-72)"}
    for name, engine in (("auto", lib.ENGINE_AUTO), ("exact", lib.ENGINE_EXACT)):
        idx = GpuRetrievalIndex.from_arrays(arrays["centroids"], arrays["offsets"], arrays["vectors"], arrays["ids"],
                                            1, engine=engine, max_frames=max(w.extra["blocks"]))
        res = {}
        for frames in w.extra["blocks"]:
            src = queries[:frames].contiguous()
            feats = src.clone()
            p50, p95, mean = _replay_latency(lambda: idx.blend(feats, frames, rate, stream=s), s, 500,
                                             pre=lambda: feats.copy_(src))
            res[str(frames)] = {"p50_ms": p50, "p95_ms": p95, "mean_ms": mean}
        diag = idx.diagnostics()
        res["fallback_frames"] = diag["fallback_frames"]
        res["engine_used"] = diag["last_engine"]
        out[name] = res
        idx.close()
    return out


def _ivf_roofline(arrays, queries, nprobe, ms, peaks, peak_kind):
    """c3 bounds from the lists the frames actually probe (coarse order
    computed here in float64 with torch; a work count, not a parity claim):
    FLOP = 2 d (Q nlist + sum over frames of the probed lists' rows); bytes =
    the fp16 rows and fp32 norms of every list probed at least once, the
    fp16 centroids, the fp32 frames read and written, and the fp32 rows of
    each frame's 8 neighbours read by the blend.  The bound is the larger of
    the two times at the measured sustained tensor and HBM peaks."""
    import torch

    c = arrays["centroids"].double()
    q = queries.double()
    sizes = (arrays["offsets"][1:] - arrays["offsets"][:-1]).long()
    nq, d = queries.shape
    nlist = c.shape[0]
    probed = torch.empty((nq, nprobe), dtype=torch.long, device=queries.device)
    cn = (c * c).sum(1)
    for s0 in range(0, nq, 4096):
        dq = cn[None, :] - 2.0 * q[s0:s0 + 4096] @ c.T
        probed[s0:s0 + 4096] = dq.topk(nprobe, largest=False).indices
    scanned = int(sizes[probed].sum().item())
    touched = torch.zeros(nlist, dtype=torch.bool, device=queries.device)
    touched[probed.flatten()] = True
    d_pad = (d + 63) // 64 * 64
    flops = 2.0 * d * (nq * nlist + scanned)
    nbytes = (float(sizes[touched].sum().item()) * (2 * d_pad + 4) + nlist * d_pad * 2 + 2.0 * nq * d * 4
              + nq * 8.0 * d * 4)
    tf = peaks.get("bf16_tflops_sustained", 1400.0)
    hbm = peaks.get("hbm_gbs", 6650.0)
    t_f, t_b = flops / (tf * 1e12), nbytes / (hbm * 1e9)
    bound_s = max(t_f, t_b)
    return {"bound": "tensor" if t_f >= t_b else "hbm", "rows_scanned": scanned,
            "rows_scanned_per_frame": scanned / nq, "lists_touched": int(touched.sum().item()),
            "algorithmic_flop": flops, "algorithmic_bytes": nbytes, "t_flop_us": t_f * 1e6, "t_bytes_us": t_b * 1e6,
            "bound_us": bound_s * 1e6, "measured_us": ms * 1000.0, "frac": bound_s / (ms / 1000.0),
            "peak_source": f"{peak_kind} bf16_tflops_sustained and hbm_gbs"}


def ivf(device):
    """c3: IVF-Flat 200k x 768, nlist 256 (20 seeded k-means iterations), 30k
    frames, nprobe 1 and 8; frames/s of the blend (CUDA events)."""
    import torch

    from vfr import GpuRetrievalIndex, synth

    w = synth.CONFIGS["c3"]
    arrays, queries = synth.make_torch("c3", device)
    out = {"workload": "c3 rvc-v2-ivf-200k: IVF-Flat N=200000 x 768, nlist=256, Q=30000 frames, k=8, "
                       "index_rate=0.75, 5 timed blends after 1 warm-up"}
    rate = torch.tensor([w.ratio], device=device)
    dst = torch.empty_like(queries)
    s = torch.cuda.Stream()
    for nprobe in w.nprobe:
        idx = GpuRetrievalIndex.from_arrays(arrays["centroids"], arrays["offsets"], arrays["vectors"], arrays["ids"],
                                            nprobe, max_frames=queries.shape[0])
        torch.cuda.synchronize()
        with torch.cuda.stream(s):
            idx.blend_from(queries, dst, rate, stream=s)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(5):
                idx.blend_from(queries, dst, rate, stream=s)
            e1.record(s)
        s.synchronize()
        ms = e0.elapsed_time(e1) / 5
        diag = idx.diagnostics()
        out[f"nprobe{nprobe}"] = {"ms_per_30k_frames": ms, "frames_per_s": queries.shape[0] / (ms / 1000.0),
                                  "exact_rerun_frames": diag["fallback_frames"] // 6,
                                  "exact_rerun_rows": diag["rerun_rows"] // 6,
                                  "certified_frames": diag["candidate_frames"] // 6}
        idx.close()
        peaks, peak_kind = measured_peaks()
        out[f"nprobe{nprobe}"]["roofline"] = _ivf_roofline(arrays, queries, nprobe, ms, peaks, peak_kind)
    return out


def main():
    a = args_parse()
    world, rank, local = dist_setup(a.gpus)
    if a.impl == "reference":
        run_reference(a, world, rank)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    from vfr import GpuRetrievalIndex, synth
    from vfr.sharded import LibraryOps, padded_frames, shard_rows, sharded_blend

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        group = dist.group.WORLD
    w = synth.CONFIGS[a.workload]
    n = a.rows or w.n
    q = padded_frames(a.queries or w.q, world)
    peaks, peak_kind = measured_peaks()

    # ---- data (seeded, identical on every rank) and index
    arrays, queries = synth.make_torch(a.workload, device, n=n, q=q)
    lo, hi = shard_rows(n, world, rank)
    host_vectors = arrays["vectors"][lo:hi].cpu().numpy()
    # rank 0 keeps every row on the host for the oracle (parity check and,
    # at N=1, the CPU baseline)
    full_host = None
    if rank == 0 and (not a.no_parity or (world == 1 and not a.no_cpu_baseline)):
        full_host = host_vectors if world == 1 else arrays["vectors"].cpu().numpy()
    del arrays
    torch.cuda.empty_cache()
    ops = LibraryOps(host_vectors, label_base=lo, max_frames=q)
    del host_vectors
    rate = torch.tensor([w.ratio], device=device)
    out = torch.empty_like(queries)
    s = torch.cuda.Stream(device)
    torch.cuda.synchronize()

    def step():
        if world == 1:
            ops.index.blend_from(queries, out, rate, stream=s)
            return 4  # prep_queries, cand_kernel, merge_kernel, exact_kernel
        sharded_blend(ops, queries, rate, group, world, rank, stream=s, timeout_s=STEP_TIMEOUT_S)
        return 6  # + merge_topk, blend_peer

    with torch.cuda.stream(s):
        for _ in range(a.warmup):
            step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    launches = 0
    ops.index.profile(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(a.steps):
            launches += step()
        e1.record(s)
    torch.cuda.synchronize()
    ms_local = e0.elapsed_time(e1)
    prof = ops.index.profile(False)
    clocks = sampler.stop(set(range(8))) if rank == 0 else None
    if world > 1:
        dist.barrier()
    t = torch.tensor([ms_local], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = q * a.steps / (ms / 1000.0)

    # ---- roofline of the dominant kernel: the distance GEMM is tensor-bound
    # for large frame blocks; for small ones (c4's 32 frames) it streams the
    # fp16 row shadow and norms once per launch and is HBM-bound
    cand = prof["cand_kernel"]
    n_local = hi - lo
    d_pad = (w.d + 63) // 64 * 64
    cand_s = cand["ms"] / max(1, cand["launches"]) / 1000.0
    traffic = None  # DRAM bytes of one full-size launch, when profiles/traffic.json has a capture of it
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            tj = json.load(f).get(f"cand_kernel/{a.workload}", {})
        if tj.get("captured_rows") == n_local and tj.get("captured_frames") == q:
            traffic = tj["dram_bytes_read"] + tj["dram_bytes_write"]
    common = {"kernel": "cand_kernel", "traffic": traffic, "kernel_ms": cand_s * 1000,
              "step_share": cand["ms"] / ms_local if ms_local else None,
              "kernels_ms": {k: v["ms"] / max(1, v["launches"]) for k, v in prof.items()}}
    if q <= 32:
        bytes_per_launch = float(n_local) * (d_pad * 2 + 4)
        achieved = bytes_per_launch / cand_s / 1e9 if cand["launches"] else None
        peak = peaks.get("hbm_gbs", 6650.0)
        roofline = dict(common, bound="hbm", achieved=achieved, peak=peak, unit="GB/s",
                        frac=achieved / peak if achieved else None,
                        peak_source=f"{peak_kind} hbm_gbs (copy bandwidth)",
                        algorithmic=f"N*(2*d_pad + 4) = {bytes_per_launch:.4g} bytes per launch (fp16 row shadow "
                                    f"and fp32 norms, N={n_local}, d_pad={d_pad})")
    else:
        flops_per_launch = 2.0 * q * n_local * w.d
        achieved = flops_per_launch / cand_s / 1e12 if cand["launches"] else None
        peak = peaks.get("bf16_tflops_sustained", 1400.0)
        roofline = dict(common, bound="tensor", achieved=achieved, peak=peak, unit="TFLOP/s",
                        frac=achieved / peak if achieved else None,
                        peak_source=f"{peak_kind} bf16_tflops_sustained (dense fp16 and bf16 share the rate)",
                        algorithmic=f"2*Q*N*d = {flops_per_launch:.4g} FLOP per launch (Q={q}, N={n_local}, d={w.d})")

    # ---- e2e through the drop-in C ABI with pinned host buffers
    e2e = None
    if not a.no_e2e:
        # each rank uploads its own share of the frames from pinned host
        # memory and the shares are all-gathered over NVLink; each rank
        # reads back the frames it blended
        m = q // world
        host_in = queries[rank * m:(rank + 1) * m].cpu().pin_memory()
        host_out = torch.empty((m, w.d), dtype=torch.float32).pin_memory()
        feats = torch.empty_like(queries)
        feats_local = torch.empty((m, w.d), dtype=torch.float32, device=device)

        def e2e_step():
            if world == 1:
                feats.copy_(host_in, non_blocking=True)
                ops.index.blend(feats, q, rate, stream=s)  # vocal_faiss_gpu_blend, in place
                host_out.copy_(feats, non_blocking=True)
            else:
                feats_local.copy_(host_in, non_blocking=True)
                dist.all_gather_into_tensor(feats, feats_local, group=group)
                o, _, _ = sharded_blend(ops, feats, rate, group, world, rank, stream=s, timeout_s=STEP_TIMEOUT_S)
                host_out.copy_(o, non_blocking=True)

        with torch.cuda.stream(s):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world == 1:
            # a serving loop's pipeline: the frames of step i+1 go up and the
            # blended frames of step i come back on a copy stream while the
            # GPU blends (two device frame buffers); the timed region runs
            # from before the first upload to after the last read-back
            cs = torch.cuda.Stream()
            bufs = [feats, torch.empty_like(feats)]
            up = [torch.cuda.Event() for _ in range(2)]
            done = [torch.cuda.Event() for _ in range(2)]
            f0.record(cs)
            with torch.cuda.stream(cs):
                bufs[0].copy_(host_in, non_blocking=True)
                up[0].record(cs)
            for i in range(a.steps):
                cur, nxt = i % 2, (i + 1) % 2
                s.wait_event(up[cur])
                with torch.cuda.stream(s):
                    ops.index.blend(bufs[cur], q, rate, stream=s)  # vocal_faiss_gpu_blend, in place
                    done[cur].record(s)
                with torch.cuda.stream(cs):
                    if i + 1 < a.steps:  # the other buffer's read-back is already queued before this
                        bufs[nxt].copy_(host_in, non_blocking=True)
                        up[nxt].record(cs)
                    cs.wait_event(done[cur])
                    host_out.copy_(bufs[cur], non_blocking=True)
            f1.record(cs)
        else:
            with torch.cuda.stream(s):
                f0.record(s)
                for _ in range(a.steps):
                    e2e_step()
                f1.record(s)
        torch.cuda.synchronize()
        te = torch.tensor([f0.elapsed_time(f1)], device=device)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": q * a.steps / (float(te.item()) / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": int(host_in.numel() * 4) * world,
               "d2h_bytes_per_step": int(host_out.numel() * 4) * world,
               "bytes": "summed over ranks (each rank copies its own share of the frames each way)",
               "pipeline": "uploads and read-backs on a copy stream overlapping the neighbouring steps' blends "
                           "(two device frame buffers)" if world == 1 else "serial per step",
               "api": "vocal_faiss_gpu_blend" if world == 1 else
               "NCCL all-gather of the frames + vfr_retrieval_search + NCCL top-8 all-gather + vfr_merge_topk + "
               "vfr_blend_peer (winners read from their owner GPU over NVLink)"}

    # ---- correctness beside the timed numbers: rank 0's first PARITY_FRAMES
    # output frames of a full-size step (labels from the same step's search)
    # against the oracle's exact scan of every row
    parity_out = None
    if not a.no_parity:
        with torch.cuda.stream(s):
            if world == 1:
                ops.index.blend_from(queries, out, rate, stream=s)
                pd, pl = ops.index.search(queries, k=8, stream=s)
                mine = out
            else:
                mine, pd, pl = sharded_blend(ops, queries, rate, group, world, rank, stream=s,
                                             timeout_s=STEP_TIMEOUT_S)
        torch.cuda.synchronize()
        if rank == 0:
            f = min(PARITY_FRAMES, mine.shape[0])
            parity_out = (mine[:f].cpu().numpy(), pd[:f].cpu().numpy(), pl[:f].cpu().numpy())

    diag = ops.index.diagnostics()
    extra = {}
    if rank == 0 and world == 1 and not a.no_streaming:
        extra["streaming"] = streaming(device)
        extra["protection"] = protection(device)
        extra["ivf"] = ivf(device)
        if not a.no_ingest:
            extra["ingest"] = ingest(device)
        if not a.no_training:
            extra["training"] = training(device, 0 if a.no_cpu_baseline else (os.cpu_count() or 1))
    if rank == 0 and world == 1 and not a.no_configs and not a.no_streaming:
        extra["c1"] = flat_config(device, "c1")
        extra["c2"] = flat_config(device, "c2")
        extra["published_shape"] = published_shape(device)
    if rank == 0 and world == 1 and not a.no_cublas and roofline and roofline.get("unit") == "TFLOP/s":
        ref = cublas_same_box(device)
        extra["cublas_same_box"] = ref
        mhz, ref_mhz = (clocks or {}).get("sm_mhz"), ref["clocks"].get("sm_mhz")
        if roofline.get("achieved") and mhz and ref_mhz:
            # per clock: the kernel's TFLOP/s per MHz over cuBLAS's on this box
            roofline["per_clock_vs_cublas_same_box"] = (roofline["achieved"] / mhz) / (ref["tflops"] / ref_mhz)
    cpu = None
    if rank == 0 and world == 1 and full_host is not None and not a.no_cpu_baseline:
        cpu = cpu_baseline(full_host, queries.cpu().numpy(), w.ratio, n)
    if parity_out is not None:
        extra["parity"] = parity_check(full_host, queries[:parity_out[0].shape[0]].cpu().numpy(), *parity_out,
                                       w.ratio, n)
    if world > 1:
        ops.close(group)  # peer mappings released on every rank before any rank frees its rows
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f16 candidates, f32 exact distances, f64 weights", "data": "synthetic",
        "config": workload_config(a, w, n, world), "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu,
        "clocks": clocks, "gpu_launches": launches,
        "exactness": {"fallback_frames": diag["fallback_frames"], "certified_frames": diag["candidate_frames"],
                      "timeouts": diag["timeouts"]},
    }
    line.update(extra)
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
