#!/usr/bin/env python
"""Benchmark of the Token2Wav DiT/CFM flow-matching solve on B200 (BASELINE.json metric: chunk mel frames/s per full
CFG ODE solve at 1/2/4/8 GPUs, with p50 / p95 per-chunk latency).

Default workload: benchmark config 5 — 1024 independent streams, each a 300-frame prompt + 50-frame chunk (seed 3),
sharded by stream across the N ranks by the product's own scheduler (``b200t2w.scheduler.shard_streams``, contiguous),
one process per GPU, no collective on the data path (only a gloo barrier and a max over ranks of the device-timed
region).  Total work is fixed as N grows: strong scaling.  Each rank solves its shard in batches of ``--batch`` streams
(64: the north star's target shape, 64 x (300 + 50), bf16), one CUDA-graph-replayed full 10-step CFG solve per batch,
back to back.  One "step" = the whole job: every stream's chunk solved once.

    value          = 1024 x 50 chunk mel frames / (max over ranks of the step's device time)
    latency_ms     = per-chunk latency: a chunk's solve ends with its batch, so each chunk's latency is the time from
                     the step's start to its batch's end; p50 / p95 over all chunks of all timed steps and ranks
    e2e            = the same job through the public API (``B200Solver.solve_streams`` on per-stream host tensors:
                     host -> device copies of every input and a device -> host read of every chunk mel inside the
                     timed region)
    roofline       = the bf16 GEMMs of one batch solve (FLOPs from the path's formula / their event-timed time in an
                     eager profiling solve) against MEASURED_PEAKS.json bf16_tflops_sustained
    subrecords     = (N = 1, rank 0) config 2, config 3, config 4 (FP8), the steady-state form at 32 and 64 windows,
                     each with its own ms, frames/s and GEMM fraction
    reference_gpu  = (N = 1) the reference's own GPU PyTorch path on this GPU (``BatchedToken2Wav._solve``, fp16,
                     run by ``bench.py --impl reference --reference-gpu`` in a child process), with the speed-up of this
                     build at the target shape and at config 2

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c5|c2|target|c3|c4|steady] [--impl b200|reference]

``--impl reference`` times the reference's algorithm on the host cores (the fp32 CPU oracle port of the reference
solver on all threads), one stream of the workload per step, on rank 0 only.  ``--impl reference --reference-gpu``
prints the reference GPU path's timings instead (used by the default arm).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "minicpm-o-4.5-single-gpu-engine_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402

from b200t2w.config import REFERENCE, DiTConfig  # noqa: E402
from b200t2w.workload import C2, C3, C4, C5, TARGET, Workload, make_streams  # noqa: E402

METRIC = "DiT mel frames/s per full CFG ODE solve"
UNIT = "mel frames/s"
L2_FLUSH_BYTES = 256 << 20


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="c5", choices=["c5", "c2", "target", "c3", "c4", "steady", "encoder", "hift"])
    ap.add_argument("--batch", type=int, default=64, help="streams per solve on a rank (c5) / windows per call (steady)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-profile", action="store_true")
    ap.add_argument("--no-subrecords", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true")
    ap.add_argument("--reference-gpu", action="store_true",
                    help="with --impl reference: time the reference's GPU PyTorch path and print its record")
    ap.add_argument("--reference-fastdit", action="store_true",
                    help="with --reference-gpu: also time the reference's FastDiT (FlashInfer + Triton + cuBLAS)")
    ap.add_argument("--timeline", action="store_true",
                    help="also record one graph-replayed solve with torch.profiler (CUPTI) and report each kernel "
                         "position's share of the solve's span (the time by which it extends the critical path)")
    return ap.parse_args()


def rank_streams(name: str, rank: int, world: int) -> tuple[Workload, list]:
    """This rank's workload and stream indices.  c5: the 1024 streams split by the product's scheduler (contiguous
    blocks, strong scaling); the fixed-size configs: every rank runs the whole config (replicas, weak scaling)."""
    from b200t2w.scheduler import shard_streams

    if name == "c5":
        return C5, shard_streams(list(C5.lengths), world, contiguous=True)[rank]
    wl = {"c2": C2, "target": TARGET, "c3": C3, "c4": C4, "steady": C2}[name]
    return wl, list(range(wl.streams))


def timeline_from_events(evs: list) -> dict:
    """Per-position time of one solve from its kernels' (name, GPU start us, GPU end us).  Kernels are named by their
    place in a DiT block: a GEMM by its epilogue (k_gemm<BN, EPI, ...>: EPI 0 in_proj, 2 fc1 with GELU, 4 QKV,
    BN 80 the final linear) or, for the plain bf16 ones, by the kernel before it (attention -> proj, add_ln_mod ->
    conv1, ln_mish -> conv2, fc1 -> fc2); a LayerNorm kernel by the GEMM it follows.  "exposed" is the time by which a
    kernel extends the end of the solve so far, so the exposed times add up to the solve's span (kernels overlap
    through programmatic dependent launch and early starts on completion counters)."""
    import re

    evs = sorted(evs, key=lambda e: e[1])
    if not evs:
        return {}
    names = []
    for n, _, _ in evs:
        m = re.search(r"k_gemm<(\d+), (\d+)", n)
        mp = re.search(r"k_gemm(?:_pair|8)<(\d+)>", n)  # the CTA-pair and FP8 GEMMs: k_gemm_pair<EPI>, k_gemm8<EPI>
        if m or mp:
            bn, epi = (int(m.group(1)), int(m.group(2))) if m else (256, int(mp.group(1)))
            # the kernel before it, skipping the slot-pool solve's cache-scatter kernels
            prev = next((x.split(" after ")[0] for x in reversed(names) if x not in ("conv_cache", "kv_scatter")), "")
            nm = ("final" if bn == 80 else "in_proj" if epi == 0 else "fc1" if epi == 2 else "qkv" if epi == 4
                  else {"attn": "proj", "ln_mish": "conv2", "fc1": "fc2"}.get(prev, "conv1"))
        elif "k_add_ln_mod" in n or "k_ln_mish" in n:
            nm = ("add_ln_mod" if "add_ln_mod" in n else "ln_mish") + (f" after {names[-1]}" if names else "")
        else:
            m = re.search(r"k_(\w+)", n)
            nm = m.group(1) if m else "other"
            nm = "attn" if nm.startswith("attn") else nm
        names.append(nm)
    exposed, busy, last = {}, {}, evs[0][1]
    for (_, s0, e0), nm in zip(evs, names):
        busy[nm] = busy.get(nm, 0.0) + (e0 - s0)
        if e0 > last:
            exposed[nm] = exposed.get(nm, 0.0) + (e0 - last)
            last = e0
    return {"solve_ms": round((evs[-1][2] - evs[0][1]) / 1000, 3), "kernels": len(evs),
            "exposed_ms": {k: round(v / 1000, 3) for k, v in sorted(exposed.items(), key=lambda x: -x[1])},
            "kernel_ms": {k: round(v / 1000, 3) for k, v in sorted(busy.items(), key=lambda x: -x[1])}}


def timeline(solve) -> dict:
    """One solve under torch.profiler with CUDA activities only (CUPTI records the kernels inside the CUDA graph with
    their GPU start and end): ``timeline_from_events`` of it."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as pr:
        solve()
        torch.cuda.synchronize()
    return timeline_from_events([(e.name, e.time_range.start, e.time_range.end) for e in pr.events()
                                 if e.device_type.name == "CUDA"])


def flops_per_solve(cfg: DiTConfig, lengths) -> tuple[float, float]:
    """(GEMM FLOPs, attention FLOPs) of one full CFG solve, from the per-token / per-key formulas of the path:
    per token per block 2H(10H + 2F) GEMM FLOPs (QKV 3H, proj H, two 3-tap convs 3H each, fc1 / fc2 F), plus in_proj
    (2 * 4mel * H) and the final linear (2 H mel) per token; attention 4 H per (query, key) pair; tokens count both CFG
    halves; a packed row (P, T) has P^2 + T (P + T) (query, key) pairs per half."""
    H, F, Dp, S = cfg.hidden, cfg.ffn, cfg.depth, cfg.steps
    gemm = attn = 0.0
    for P, T in lengths:
        tok = 2 * (P + T)
        gemm += S * tok * (Dp * 2 * H * (10 * H + 2 * F) + 2 * cfg.in_dim * H + 2 * H * cfg.mel)
        attn += S * Dp * 4 * H * 2 * (P * P + T * (P + T))
    return gemm, attn


class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.p = None
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                                       "-i", str(index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def physical_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local_rank])
        except (ValueError, IndexError):
            return local_rank
    return local_rank


def cpu_oracle_time(cfg: DiTConfig, streams: list, reps: int, warm: int) -> tuple[list, int]:
    """Seconds per one-stream solve of the CPU oracle (fp32, all host threads)."""
    from oracle import dit_oracle

    threads = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    model = dit_oracle.build_model(cfg, seed=0)
    ts = []
    for i in range(warm + reps):
        s = streams[i % len(streams)]
        t0 = time.perf_counter()
        dit_oracle.solve_packed(model, s["x0"], s["mu"], s["cond"], s["spk"], s["P"], s["T"])
        if i >= warm:
            ts.append(time.perf_counter() - t0)
    torch.set_num_threads(prev)  # the launch-bound records after this one keep the host's default pool
    return ts, threads


def reference_arm(a, rank: int, world: int) -> None:
    """The reference's solver algorithm on the host cores (the fp32 CPU oracle port), one stream of the workload per
    step, rank 0 only; the other ranks exit without work."""
    if rank != 0:
        return
    wl, _ = rank_streams(a.workload, 0, 1)
    streams = make_streams(wl, count=min(4, wl.streams))
    ts, threads = cpu_oracle_time(REFERENCE, streams, a.steps, a.warmup)
    T = [streams[i % len(streams)]["T"] for i in range(a.steps)]
    value = sum(T) / sum(ts)
    sample = f"1 stream of {wl.name} (P={streams[0]['P']}, T={streams[0]['T']}) per step, fp32 CPU oracle port"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": 1000 * statistics.mean(ts), "higher_is_better": True,
        "scaling": "strong" if a.workload == "c5" else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": wl.name, "streams_per_step": 1, "model": "reference-config DiT (unverified), random init"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)


def _reference_modules():
    """The reference checkout installed in baseline/_ref (its engine package) plus the one symbol its solver imports
    from the absent stepaudio2 package (``decoder_dit.modulate``), and the restated estimator modules it drives."""
    import types

    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "engine")):
        raise RuntimeError("baseline/_ref is not installed")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    from oracle import dit_oracle

    names = ["stepaudio2", "stepaudio2.cosyvoice2", "stepaudio2.cosyvoice2.flow", "stepaudio2.cosyvoice2.flow.decoder_dit"]
    for n in names:
        sys.modules.setdefault(n, types.ModuleType(n))
    sys.modules["stepaudio2.cosyvoice2.flow.decoder_dit"].modulate = dit_oracle.modulate
    return dit_oracle


def reference_gpu_eager(wl: Workload, steps: int, warm: int, dev) -> dict:
    """The reference's own GPU PyTorch path, ``BatchedToken2Wav._solve`` (engine/runtime/token2wav_batch.py:632-702),
    unmodified, on this GPU in fp16 (the reference's FP16 flow): the prompt setup of every stream (prompt mel as the
    condition, empty caches) then its chunk against the caches it left, over the whole batch at once — the two-stage
    form of one full 10-step CFG solve of a chunk with its prompt.  Event-timed per two-stage solve."""
    from types import SimpleNamespace

    dit_oracle = _reference_modules()
    from engine.models.token2wav import StreamState
    from engine.runtime.token2wav_batch import BatchedToken2Wav

    cfg = REFERENCE
    P, T = wl.lengths[0]
    assert all(x == (P, T) for x in wl.lengths)
    n = wl.streams
    model = dit_oracle.build_model(cfg, seed=0, noise_frames=P + T + 8).to(dev).half()
    bt = BatchedToken2Wav.__new__(BatchedToken2Wav)
    bt.flow = SimpleNamespace(decoder=model)
    bt.t2w = SimpleNamespace(n_timesteps=cfg.steps)
    bt.graphs = bt.euler = None
    ss = make_streams(wl, cfg.mel)
    h = lambda k, a, b: torch.stack([s[k][:, a:b] for s in ss]).to(dev, torch.float16).contiguous()  # noqa: E731
    mu_p, mu_c, cond_p = h("mu", 0, P), h("mu", P, P + T), h("cond", 0, P)
    spk = torch.stack([s["spk"] for s in ss]).to(dev, torch.float16)

    def solve():
        sts = [StreamState(prompt=None, hift_cache={}, flow_cache={
            "estimator_cnn_cache": torch.zeros(cfg.steps, cfg.depth, 2, 2 * cfg.hidden, 2, device=dev, dtype=torch.float16),
            "estimator_att_cache": torch.zeros(cfg.steps, cfg.depth, 2, cfg.heads, 0, 2 * cfg.head_dim, device=dev,
                                               dtype=torch.float16)}) for _ in range(n)]
        bt._solve(sts, mu_p, spk, cond=cond_p, keep_cache=True)
        return bt._solve(sts, mu_c, spk, cond=None, keep_cache=True)

    st = torch.cuda.current_stream(dev)
    with torch.inference_mode():
        for _ in range(warm):
            solve()
        torch.cuda.synchronize(dev)
        ms = []
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            solve()
            e1.record(st)
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
    m = statistics.median(ms)
    return {"path": "BatchedToken2Wav._solve (engine/runtime/token2wav_batch.py:632-702), eager, fp16, two-stage "
                    "(prompt setup then chunk)", "workload": wl.name, "streams": n, "ms_per_solve": m,
            "chunk_frames_per_s": n * T / (m / 1000), "timed_solves": steps}


def reference_gpu_fastdit(wl: Workload, steps: int, warm: int, dev) -> dict:
    """The reference's production form, ``FastDiT.solve`` (engine/runtime/dit_fast.py:432-495: FlashInfer paged
    prefill, Triton norm kernels, cuBLAS linears, CUDA graphs per row bucket), fp16: every stream's prompt setup then
    its chunk window, timed as one two-stage solve, and the chunk window alone (the steady-state call)."""
    dit_oracle = _reference_modules()
    from engine.runtime.dit_fast import FastDiT

    cfg = REFERENCE
    P, T = wl.lengths[0]
    n = wl.streams
    model = dit_oracle.build_model(cfg, seed=0, noise_frames=P + T + 8).to(dev).half()
    fd = FastDiT(model, cfg.steps, n_slots=2 * n * (P + T + 8), max_streams=max(96, n), device=dev, use_graphs=True,
                 fused_residual=True, fused_conv=True)
    ss = make_streams(wl, cfg.mel)
    mu_p = [s["mu"][:, :P].to(dev, torch.float16) for s in ss]
    mu_c = [s["mu"][:, P:].to(dev, torch.float16) for s in ss]
    cond_p = [s["cond"][:, :P].to(dev, torch.float16) for s in ss]
    spk = torch.stack([s["spk"] for s in ss]).to(dev, torch.float16)
    st = torch.cuda.current_stream(dev)
    two, win = [], []
    with torch.inference_mode():
        for i in range(warm + steps):
            caches = [fd.new_cache() for _ in range(n)]
            for c in caches:
                c.keep = P
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(st)
            fd.solve(caches, mu_p, spk, cond_p, [True] * n)
            e1.record(st)
            fd.solve(caches, mu_c, spk, None, [True] * n)
            e2.record(st)
            e2.synchronize()
            if i >= warm:
                two.append(e0.elapsed_time(e2))
                win.append(e1.elapsed_time(e2))
            for c in caches:
                fd.release(c)
    m, mw = statistics.median(two), statistics.median(win)
    return {"path": "FastDiT.solve (engine/runtime/dit_fast.py:432-495), FlashInfer + Triton + cuBLAS, fp16, graphs",
            "workload": wl.name, "streams": n, "ms_per_solve": m, "chunk_frames_per_s": n * T / (m / 1000),
            "window_ms": mw, "window_frames_per_s": n * T / (mw / 1000), "timed_solves": steps,
            "graph_calls": dict(fd.counts)}


def reference_gpu_encoder(n: int, prompt_tokens: int, steps: int, warm: int, dev, batched_io: bool) -> dict:
    """The reference's own flow-encoder path on this GPU in fp16, unmodified: ``BatchedToken2Wav._setup_encoder_batched``
    for ``n`` prompts (one padded batch), then steady windows of 25 + 3 tokens through ``_flow_encode``'s steps
    (``input_embedding``, ``_encoder`` with left-padded caches, ``encoder_proj``) and ``_flow_finish``'s trim
    (engine/runtime/token2wav_batch.py:365-478,566-616), over the restated flow module.  ``batched_io``: the engine's
    ``t2w_encoder_batched_io`` option (Triton cache gather / scatter, engine/runtime/encoder_io.py)."""
    _reference_modules()
    from engine.runtime import token2wav_batch as tb

    from b200t2w.config import ENCODER
    from oracle import encoder_oracle as eo

    flow = eo.build_flow(ENCODER, seed=0).to(dev).half()
    bt = tb.BatchedToken2Wav.__new__(tb.BatchedToken2Wav)
    bt.flow, bt.fast, bt.enc_graphs, bt.encoder_batched_io = flow, None, None, batched_io
    bt.profile = bt.trace = None
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, ENCODER.vocab, (1, prompt_tokens), generator=g).to(dev) for _ in range(n)]
    feats = [(p, None, None, None, None) for p in prompts]
    wins = [torch.randint(0, ENCODER.vocab, (n, 28), generator=g).to(dev) for _ in range(4)]
    keep = 2 * prompt_tokens

    class St:  # the parts of StreamState the encoder driver reads
        def __init__(self, cnn, att):
            self.flow_cache = {"conformer_cnn_cache": cnn, "conformer_att_cache": att}
            self.prompt = type("Prompt", (), {"mels": torch.zeros(1, keep, 1)})()

    st = torch.cuda.current_stream(dev)
    with torch.inference_mode():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        encs = bt._setup_encoder_batched(feats)
        e1.record(st)
        e1.synchronize()
        setup_ms = e0.elapsed_time(e1)
        sts = [St(cnn, att) for _, cnn, att in encs]

        def call(k):
            h = flow.encoder_proj(bt._encoder(sts, flow.input_embedding(wins[k % 4]), False))
            for s in sts:
                c = s.flow_cache
                c["conformer_att_cache"] = tb._trim(c["conformer_att_cache"], keep, 3)
            return h

        for k in range(max(warm, 4)):
            call(k)
        torch.cuda.synchronize(dev)
        ms = []
        for k in range(steps):
            e0.record(st)
            call(k)
            e1.record(st)
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
    m = statistics.median(ms)
    return {"path": "BatchedToken2Wav._encoder + encoder_proj + _flow_finish trim (token2wav_batch.py:365-478), fp16, "
                    + ("encoder_batched_io" if batched_io else "per-stream cache I/O"),
            "streams": n, "ms_per_call": m, "mu_frames_per_s": n * 50 / (m / 1000), "setup_ms": setup_ms,
            "setup_mu_frames_per_s": n * 2 * prompt_tokens / (setup_ms / 1000), "timed_calls": steps}


def reference_gpu_hift(n: int, steps: int, warm: int, dev, tf32: bool, graphs: bool = False) -> dict:
    """The reference's own vocoder path on this GPU, unmodified: ``BatchedToken2Wav._vocode``
    (engine/runtime/token2wav_batch.py:813-848) with ``hift_forward`` (engine/models/token2wav.py:230-245), strict fp32
    (cuDNN TF32 off, as the reference runs Token2Wav) or with its ``decode_tf32`` option, over the restated vocoder:
    ``n`` streams, 50-frame windows, every call one window per stream.  ``graphs``: its ``t2w_graphs`` option, the
    vocoder replayed from ``HiFTGraphs`` (engine/runtime/hift_graph.py:22-88; default row buckets, 64 rows in slices of
    16), the warm-up calls capturing the graphs."""
    _reference_modules()
    from types import SimpleNamespace

    import numpy as np
    from engine.models.token2wav import StreamState, strict_fp32
    from engine.runtime import token2wav_batch as tb

    from b200t2w.config import HIFT
    from oracle import hift_oracle as ho

    hift = ho.build_hift(HIFT, seed=0).to(dev)
    bt = tb.BatchedToken2Wav.__new__(tb.BatchedToken2Wav)
    bt.hift, bt.hift_graphs, bt.hift_decode_tf32 = hift, None, tf32
    if graphs:
        from engine.runtime.hift_graph import HiFTGraphs

        bt.hift_graphs = HiFTGraphs(hift, decode_tf32=tf32)
    bt.t2w = SimpleNamespace(window=torch.from_numpy(np.hamming(2 * ho.SOURCE_CACHE)).to(dev))
    sts = [StreamState(prompt=None, flow_cache={}, noise_seed=1000 + i,
                       hift_cache=dict(mel=torch.zeros(1, HIFT.mel, 0, device=dev), source=torch.zeros(1, 1, 0, device=dev),
                                       speech=torch.zeros(1, 0, device=dev))) for i in range(n)]
    g = torch.Generator().manual_seed(13)
    mels = [[(torch.randn(1, HIFT.mel, 50, generator=g) - 2.0).to(dev) for _ in range(n)] for _ in range(3)]
    st = torch.cuda.current_stream(dev)
    ms = []
    with torch.inference_mode(), strict_fp32():
        for k in range(warm + steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            bt._vocode([(s, None, False) for s in sts], mels[k % 3])
            e1.record(st)
            e1.synchronize()
            if k >= warm:
                ms.append(e0.elapsed_time(e1))
    m = statistics.median(ms)
    return {"path": "BatchedToken2Wav._vocode + " + ("HiFTGraphs replay (hift_graph.py:22-88)" if graphs else
                                                      "hift_forward (token2wav.py:230-245)")
                    + " (token2wav_batch.py:813-848), " + ("decode_tf32" if tf32 else "strict fp32"),
            "streams": n, "ms_per_call": m, "mel_frames_per_s": n * 50 / (m / 1000), "timed_calls": steps,
            **({"graph_counts": dict(bt.hift_graphs.counts)} if graphs else {})}


def reference_gpu_arm(a) -> None:
    """``--impl reference --reference-gpu``: one JSON record of the reference's GPU PyTorch path at the target shape
    and at config 2 (a child process of the default arm; nothing of this build's library is loaded here)."""
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    rec = {"impl": "reference_gpu", "gpu": torch.cuda.get_device_name(dev)}
    # the reference's decode calls carry at most 32 streams (BatchedToken2Wav.max_flow_streams, token2wav_batch.py:196):
    # its graph-replayed window solve is timed at that size too, beside this build's 32-window steady call
    w32 = Workload("ref_w32_32x(300+50)", 1, C2.lengths[:1] * 32)
    for name, wl in (("target", TARGET), ("c2", C2), ("w32", w32)):
        if name != "w32":
            try:
                rec[name] = reference_gpu_eager(wl, steps=3, warm=1, dev=dev)
            except Exception as e:  # reported, not raised: the default arm's own numbers stand without it
                rec[name] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
        if a.reference_fastdit:
            try:
                rec[name + "_fastdit"] = reference_gpu_fastdit(wl, steps=3, warm=2, dev=dev)
            except Exception as e:
                rec[name + "_fastdit"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    for graphs in (False, True):
        for tf32 in (False, True):
            key = "hift_64" + ("_graphs" if graphs else "") + ("_tf32" if tf32 else "")
            try:
                rec[key] = reference_gpu_hift(64, steps=3, warm=2, dev=dev, tf32=tf32, graphs=graphs)
            except Exception as e:
                rec[key] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
            torch.cuda.empty_cache()
    for io in (False, True):
        key = "encoder_64" + ("_batched_io" if io else "")
        try:
            rec[key] = reference_gpu_encoder(64, 150, steps=5, warm=4, dev=dev, batched_io=io)
        except Exception as e:
            rec[key] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.empty_cache()
    print(json.dumps(rec), flush=True)


def steady_record(cfg: DiTConfig, dev, n: int, steps: int, warmup: int, seed: int, timeline_on: bool = False) -> dict:
    """Steady-state windows through ``B200FastDiT`` (the reference's ``FastDiT.solve`` form): ``n`` streams with
    300-frame prompts set up, then one 50-frame window per stream per call against the slot-pool caches (trimmed to the
    prompt plus the last 100 keys).  Window inputs sit in pinned host memory and each call's mel is read back to pinned
    host memory, inside the timed region.  Throughput: calls back to back (a call's host work overlaps the previous
    call's GPU work); latency: one call at a time."""
    from b200t2w.fastdit import B200FastDiT
    from b200t2w.solver import B200Solver
    from b200t2w.weights import random_state_dict

    P, T = 300, 50
    g = torch.Generator().manual_seed(seed)
    noise = torch.randn(cfg.mel, 8192, generator=g)
    solver = B200Solver(cfg, random_state_dict(cfg, seed=0, device=dev), device=dev)
    fd = B200FastDiT(solver, noise, n_slots=2 * n * (P + 100 + T + 8), max_streams=n)
    spk = torch.randn(n, cfg.mel, generator=g)
    caches = [fd.new_cache() for _ in range(n)]
    for c in caches:
        c.keep = P
    for i0 in range(0, n, 16):  # prompt setups, 16 per call
        cs = caches[i0:i0 + 16]
        fd.solve(cs, [torch.randn(cfg.mel, P, generator=g) for _ in cs], spk[i0:i0 + 16],
                 [torch.randn(cfg.mel, P, generator=g) for _ in cs], [True] * len(cs))
    mus = [[torch.randn(cfg.mel, T, generator=g).pin_memory() for _ in range(n)] for _ in range(4)]
    spk_d = spk.to(dev)
    host_out = torch.empty(n, cfg.mel, T).pin_memory()

    def step(k):
        outs = fd.solve(caches, mus[k % 4], spk_d, None, [True] * n)
        host_out.copy_(torch.stack(outs), non_blocking=True)

    # caches reach the trimmed steady length (P + 100) after three windows; the steady structure's CUDA graph is
    # captured on its second call, so two more warm-up windows keep the capture out of the timed region
    for k in range(max(warmup, 3) + 2):
        step(k)
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for k in range(steps):
        step(k)
    e1.record(st)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    lat = []
    for k in range(min(steps, 5)):
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0.record(st)
        step(k)
        l1.record(st)
        l1.synchronize()
        lat.append(l0.elapsed_time(l1))
    solver.check()
    tl = timeline(lambda: step(0)) if timeline_on else None
    keys = caches[0].length
    # per stream per window: S [2T (Dp 36 H^2 + 800 H) + Dp 4H 2T (keys)], keys = cache (P + 100) + T
    flop = n * cfg.steps * (2 * T * (cfg.depth * 2 * cfg.hidden * (10 * cfg.hidden + 2 * cfg.ffn) + 800 * cfg.hidden)
                            + cfg.depth * 4 * cfg.hidden * 2 * T * keys)
    rec = {"workload": f"steady_{n}x{T} (P={P} cached, keys per row {keys})", "streams": n, "ms_per_call": ms,
           "chunk_frames_per_s": n * T / (ms / 1000), "latency_ms_p50": statistics.median(lat),
           "tflops": flop / (ms / 1000) / 1e12, "solve_calls": dict(fd.counts),
           "h2d_bytes_per_call": n * T * cfg.mel * 4, "d2h_bytes_per_call": n * T * cfg.mel * 4}
    if tl:
        rec["timeline"] = tl
    fd.close()
    solver.close()
    return rec


def encoder_flops(ecfg, T: int, K1: int, K2: int) -> float:
    """Algorithmic FLOPs of one flow-encoder window of T token frames (first stack: T queries over K1 keys; second
    stack: 2T over K2): per frame and layer 2H(5H + 2F) for [q + u | q + v | k | v], linear_out, w_1, w_2; per
    (query, key) 6H for (q + u) k, (q + v) P(r) and P V; the embed linear and the 4- and 3-tap pre-lookahead convs
    over the T + 3 / T frames; the 5-tap up conv, up embed and encoder_proj over the 2T upsampled frames."""
    H, F = ecfg.hidden, ecfg.ffn
    layer = 2 * H * (5 * H + 2 * F)
    s1 = ecfg.blocks1 * (T * layer + 6 * H * T * K1)
    s2 = ecfg.blocks2 * (2 * T * layer + 6 * H * 2 * T * K2)
    convs = (T + 3) * 2 * H * H + T * 2 * H * H * (4 + 3) + 2 * T * (2 * H * H * 5 + 2 * H * H + 2 * H * ecfg.mel)
    return float(s1 + s2 + convs)


def encoder_record(dev, n: int, prompt_tokens: int, steps: int, warmup: int, seed: int, peak_tf: float,
                   cpu: bool = True) -> dict:
    """The flow encoder (row f3: speech tokens -> mu) at the reference config, random init: ``n`` streams set up with
    ``prompt_tokens``-token prompts in one call (the batched prompt setup), then steady windows of 25 tokens + 3
    look-ahead tokens, one per stream per call, once the caches have reached their trimmed length.  Window tokens are
    copied from pinned host memory and every call's mu is read back to pinned host memory inside the timed region
    (device events around the calls, back to back).  The fp32 CPU oracle times one stream's window beside it."""
    from b200t2w.config import ENCODER
    from b200t2w.encoder import B200FlowEncoder
    from oracle import encoder_oracle as eo

    g = torch.Generator().manual_seed(seed)
    flow = eo.build_flow(ENCODER, seed=0)
    enc = B200FlowEncoder.from_flow(flow, device=dev, max_frames=2048, n_slots1=n * 512, n_slots2=n * 1024,
                                    n_streams=n, use_graphs=True)
    prompts = [torch.randint(0, ENCODER.vocab, (prompt_tokens,), generator=g) for _ in range(n)]
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    handles, _ = enc.setup(prompts)
    e1.record(st)
    e1.synchronize()
    setup_ms = e0.elapsed_time(e1)
    W, T = 28, 25
    wins = [[torch.randint(0, ENCODER.vocab, (W,), generator=g).tolist() for _ in range(n)] for _ in range(4)]
    host_out = torch.empty(n * 2 * T, ENCODER.mel).pin_memory()
    out = torch.empty(n * 2 * T, ENCODER.mel, device=dev)

    def call(k):
        enc.encode_packed(handles, wins[k % 4], [False] * n, out=out)
        host_out.copy_(out, non_blocking=True)

    for k in range(max(warmup, 4) + 2):  # caches reach the trimmed length after a few windows; then the capture
        call(k)
    torch.cuda.synchronize(dev)
    k1, k2, keep = enc.stream_info(handles[0])
    e0.record(st)
    for k in range(steps):
        call(k)
    e1.record(st)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    enc.check()
    flop = n * encoder_flops(ENCODER, T, k1 + T, k2 + 2 * T)
    rec = {"workload": f"flow encoder, {n} streams, steady windows of {W} tokens ({T} + 3 look-ahead) after "
                       f"{prompt_tokens}-token prompts (keys per stream: stack 1 {k1} + {T}, stack 2 {k2} + {2 * T})",
           "ms_per_call": ms, "mu_frames_per_s": n * 2 * T / (ms / 1000), "tflops": flop / (ms / 1000) / 1e12,
           "frac_of_bf16_peak": flop / (ms / 1000) / 1e12 / peak_tf,
           "setup_ms": setup_ms, "setup_mu_frames_per_s": n * 2 * prompt_tokens / (setup_ms / 1000),
           "h2d_bytes_per_call": n * W * 4, "d2h_bytes_per_call": n * 2 * T * ENCODER.mel * 4,
           "calls": enc.counts, "note": "setup_ms is the first call (includes its workspace allocation); steady "
                                           "calls replay one CUDA graph per launch structure"}
    if cpu:
        threads = os.cpu_count() or 1
        prev = torch.get_num_threads()
        torch.set_num_threads(threads)
        _, s = eo.encode_prompt(flow, prompts[0])
        ts = []
        for k in range(5):
            t0 = time.perf_counter()
            eo.encode_window(flow, s, torch.tensor(wins[k % 4][0]), False)
            ts.append(time.perf_counter() - t0)
        torch.set_num_threads(prev)
        cpu_s = statistics.median(ts[2:])
        rec["cpu_baseline"] = {"value": 2 * T / cpu_s, "unit": "mu frames/s", "cores": threads, "kind": "port",
                               "sample": "1 stream's steady window, fp32 CPU oracle (median of 3 after 2 warm-up)"}
    for h in handles:
        enc.release(h)
    enc.close()
    return rec


def hift_flops(hcfg, F: int) -> float:
    """Algorithmic FLOPs of one HiFT window of F mel frames (the convolutions; the source, STFT and iSTFT are O(samples)):
    f0 predictor, conv_pre, the three transposed convs, the source branches (strided conv + ResBlock) and the three
    ResBlocks of every stage, conv_post."""
    C, Cf, mel = hcfg.channels, hcfg.f0_channels, hcfg.mel
    fl = 2 * F * 3 * (mel * Cf + (hcfg.f0_layers - 1) * Cf * Cf) + 2 * F * Cf + 2 * F * 7 * mel * C
    L, cin = F, C
    for s, (u, k) in enumerate(zip(hcfg.upsample_rates, hcfg.upsample_kernels)):
        cout = cin // 2
        fl += 2 * L * cin * cout * k  # transposed conv: each input row meets every tap once
        L *= u
        Ls = L + (1 if s == 2 else 0)
        ks = hcfg.source_kernels[s]
        fl += 2 * Ls * cout * cout * 6 * ks + 2 * Ls * cout * (hcfg.n_fft + 2) * (1 if s == 2 else 2 * (15 if s == 0 else 3))
        fl += sum(2 * Ls * cout * cout * 6 * kr for kr in hcfg.resblock_kernels)
        cin = cout
    fl += 2 * (L + 1) * cin * (hcfg.n_fft + 2) * 7
    return float(fl)


def hift_record(dev, n: int, steps: int, warmup: int, seed: int, peak_tf: float, split_fp32: bool = False,
                use_graphs: bool = False) -> dict:
    """The HiFT vocoder (row f4: mel -> 24 kHz waveform) at the reference config, random init, the upsampling stages on
    TF32 tensor cores (the reference's decode_tf32 option; f0 predictor, source, conv_pre / conv_post fp32): ``n``
    streams, every call one 50-frame window per stream (58 frames with the 8 cached ones once the stream has started),
    the windows' mel from pinned host memory and every call's samples read back to pinned host memory inside the timed
    region, calls back to back."""
    from b200t2w.config import HIFT
    from b200t2w.hift import B200HiFT
    from oracle import hift_oracle as ho

    g = torch.Generator().manual_seed(seed)
    voc = B200HiFT.from_module(ho.build_hift(HIFT, seed=0), HIFT, device=dev, max_frames=64, n_streams=n,
                               split_fp32=split_fp32, use_graphs=use_graphs)
    hs = [voc.new_stream(1000 + i) for i in range(n)]
    T = 50
    mels = [(torch.randn(n * T, HIFT.mel, generator=g) - 2.0).pin_memory() for _ in range(3)]
    dmel = torch.empty(n * T, HIFT.mel, device=dev)
    host = torch.empty(n * 480 * (T + 8), dtype=torch.float32).pin_memory()

    def call(k):
        dmel.copy_(mels[k % 3], non_blocking=True)
        flat, _ = voc.vocode_packed(hs, dmel, [T] * n, [False] * n, flat=True)
        host[:flat.numel()].copy_(flat, non_blocking=True)

    for k in range(max(warmup, 3)):
        call(k)
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    t0 = time.perf_counter()
    for k in range(steps):
        call(k)
    host_ms = (time.perf_counter() - t0) * 1000 / steps
    e1.record(st)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    flop = n * hift_flops(HIFT, T + 8)
    for h in hs:
        voc.release(h)
    voc.close()
    return {"workload": f"HiFT vocoder, {n} streams, steady 50-frame windows (58 with the cached 8), "
                        + ("every convolution in split form (3xTF32, fp32-level)" if split_fp32 else
                           "upsampling stages in TF32"),
            "ms_per_call": ms, "host_enqueue_ms_per_call": host_ms, "audio_s_per_s": n * T * 480 / 24000 / (ms / 1000),
            "mel_frames_per_s": n * T / (ms / 1000), "tflops": flop / (ms / 1000) / 1e12,
            "h2d_bytes_per_call": n * T * HIFT.mel * 4, "d2h_bytes_per_call": n * T * 480 * 4}


def packed_record(solver, wl: Workload, steps: int, warm: int, flush: torch.Tensor, peak_tf: float) -> dict:
    """One packed workload as a sub-record: device-resident inputs, ``steps`` graph-replayed solves with L2 flushed
    between them (median event time), and the GEMM fraction from one eager profiling solve."""
    from b200t2w.solver import Layout

    dev = solver.device
    streams = make_streams(wl, solver.cfg.mel)
    layout = Layout(tuple(x["P"] for x in streams), tuple(x["T"] for x in streams))
    b = solver.static_buffers(layout)
    for k in ("x0", "mu", "cond"):
        b[k].copy_(torch.cat([x[k].t() for x in streams]))
    b["spk"].copy_(torch.stack([x["spk"] for x in streams]))
    st = torch.cuda.current_stream(dev)

    def solve():
        solver.solve_packed_dev(layout, b["x0"], b["mu"], b["cond"], b["spk"], b["out"], workspace=b["ws"])

    for _ in range(warm):
        solve()
    ms = []
    for _ in range(steps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        solve()
        e1.record(st)
        e1.synchronize()
        ms.append(e0.elapsed_time(e1))
    solver.check()
    prof = solver.profile(layout, b)
    gemm_flops, attn_flops = flops_per_solve(solver.cfg, list(zip(layout.prompt, layout.chunk)))
    gemm_ms = sum(v for k, (v, _) in prof.items() if k.startswith("gemm"))
    m = statistics.median(ms)
    return {"workload": wl.name, "precision": solver.precision, "streams": wl.streams, "ms_per_solve": m,
            "chunk_frames_per_s": wl.chunk_frames / (m / 1000), "gemm_tflops": gemm_flops / (gemm_ms / 1000) / 1e12,
            "gemm_frac": gemm_flops / (gemm_ms / 1000) / 1e12 / peak_tf, "gemm_ms_per_solve": gemm_ms,
            "attn_ms_per_solve": prof["attn"][0], "solve_tflops": (gemm_flops + attn_flops) / (m / 1000) / 1e12,
            "launches_per_solve": sum(c for _, c in prof.values())}


def reference_gpu_child(a) -> dict:
    """Run ``bench.py --impl reference --reference-gpu`` as a child process (this process never loads the reference
    or its restated modules) and return its record."""
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--reference-gpu", "--reference-fastdit"]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env={**os.environ, "WORLD_SIZE": "1",
                                                                                  "RANK": "0"})
        lines = [x for x in r.stdout.strip().splitlines() if x.startswith("{")]
        if r.returncode or not lines:
            return {"unavailable": f"exit {r.returncode}: {(r.stderr or r.stdout)[-300:]}"}
        return json.loads(lines[-1])
    except subprocess.TimeoutExpired:
        return {"unavailable": "timed out after 900 s"}


def packed_job(a, rank: int, world: int, local: int) -> None:
    """The default arm: this rank's streams in batches of ``--batch`` (one graph-replayed solve each), timed as one
    whole-job step; then the same job end to end through the public API; then (N = 1, rank 0) the sub-records, the
    CPU baseline and the reference GPU path."""
    import torch.distributed as dist

    from b200t2w.solver import B200Solver, Layout
    from b200t2w.weights import random_state_dict

    cfg = REFERENCE
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    wl, idx = rank_streams(a.workload, rank, world)
    fp8 = a.workload == "c4"
    batch = a.batch if a.workload == "c5" else max(len(idx), 1)
    streams = make_streams(wl, cfg.mel, first=idx[0], count=len(idx)) if idx else []
    assert [x["index"] for x in streams] == idx
    groups = [streams[i:i + batch] for i in range(0, len(streams), batch)]
    solver = B200Solver(cfg, random_state_dict(cfg, seed=0, device=dev), precision="fp8" if fp8 else "bf16", device=dev)
    jobs = []
    for g in groups:  # device-resident inputs: one buffer set (and graph) per batch
        layout = Layout(tuple(x["P"] for x in g), tuple(x["T"] for x in g))
        b = {k: torch.cat([x[k].t() for x in g]).to(dev).contiguous() for k in ("x0", "mu", "cond")}
        b["spk"] = torch.stack([x["spk"] for x in g]).to(dev)
        b["out"] = torch.empty_like(b["x0"])
        b["ws"] = solver.workspace(layout, key=(layout.prompt, layout.chunk))
        jobs.append((layout, b))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    def step(evs=None):
        for j, (layout, b) in enumerate(jobs):
            solver.solve_packed_dev(layout, b["x0"], b["mu"], b["cond"], b["spk"], b["out"], workspace=b["ws"])
            if evs is not None:
                evs[j + 1].record(st)

    # ---- device-resident throughput and per-chunk latency (inputs already in HBM)
    for _ in range(a.warmup):
        step()
    barrier()
    clocks = Clocks(physical_index(local))
    recs = []
    for _ in range(a.steps):
        flush.fill_(1)  # L2 flush between timed steps (outside the timed interval)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(jobs) + 1)]
        evs[0].record(st)
        step(evs)
        recs.append(evs)
    barrier()
    clk = clocks.stop()
    solver.check()
    step_ms = [e[0].elapsed_time(e[-1]) if len(e) > 1 else 0.0 for e in recs]
    lat = [e[0].elapsed_time(e[j + 1]) for e in recs for j, g in enumerate(groups) for _ in g]  # one per chunk
    batch_ms = [e[j].elapsed_time(e[j + 1]) for e in recs for j in range(len(jobs))]

    # ---- end to end through the public API: per-stream host tensors -> solve_streams -> chunk mels on the host
    # one contiguous pinned block per batch: an asynchronous device -> host copy into a strided slice would be staged
    # synchronously and hold the host until the batch's solve is done
    host_out = [torch.empty(cfg.mel, sum(x["T"] for x in g), dtype=torch.float32).pin_memory() for g in groups]
    h2d = sum(4 * (3 * x["x0"].numel() + x["spk"].numel()) for x in streams)
    d2h = sum(t.numel() * 4 for t in host_out)
    e2e_ms = []
    for i in range(1 + a.steps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for gi, g in enumerate(groups):
            outs = solver.solve_streams(g)
            chunk = torch.cat([y[:, x["P"]:] for x, y in zip(g, outs)], dim=1)
            host_out[gi].copy_(chunk, non_blocking=True)
        e1.record(st)
        e1.synchronize()
        if i >= 1:
            e2e_ms.append(e0.elapsed_time(e1))
    barrier()

    # ---- max over ranks of the device-timed regions; every chunk's latency to rank 0
    red = torch.tensor([sum(step_ms), sum(e2e_ms)], dtype=torch.float64)
    all_lat = [lat]
    if world > 1:
        dist.all_reduce(red, op=dist.ReduceOp.MAX)
        all_lat = [None] * world
        dist.all_gather_object(all_lat, lat)
    max_ms, max_e2e = float(red[0]), float(red[1])
    frames = sum(t for _, t in wl.lengths) if a.workload == "c5" else world * wl.chunk_frames
    value = frames * a.steps / (max_ms / 1000)
    e2e_value = frames * a.steps / (max_e2e / 1000)

    roofline = prof = None
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    peak_tf = peaks.get("bf16_tflops_sustained", 1400.0)
    peak_src = ("MEASURED_PEAKS.json bf16_tflops_sustained (measured)" if "bf16_tflops_sustained" in peaks
                else "fallback 1400 TFLOP/s")
    if fp8:  # no measured e4m3 peak: twice the measured bf16 figure (the dense e4m3 / bf16 ratio of the part)
        peak_tf, peak_src = 2 * peak_tf, "2 x " + peak_src + " (no measured e4m3 peak)"
    if not a.no_profile and jobs:
        layout, b = jobs[0]
        prof = solver.profile(layout, b)
        gemm_flops, attn_flops = flops_per_solve(cfg, list(zip(layout.prompt, layout.chunk)))
        gemm_ms = sum(v for k, (v, _) in prof.items() if k.startswith("gemm"))
        achieved = gemm_flops / (gemm_ms / 1000) / 1e12
        roofline = {"bound": "tensor", "kernel": "k_gemm (all tcgen05 GEMM launches of one batch solve)",
                    "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                    "peak_source": peak_src, "traffic": None,
                    "traffic_note": "not captured in this run: per-kernel DRAM bytes come from ncu (profiles/)",
                    "units": f"one solve of {len(layout.prompt)} streams "
                             f"({layout.prompt[0]} + {layout.chunk[0]} frames)",
                    "gemm_tflop_per_solve": gemm_flops / 1e12, "gemm_ms_per_solve": gemm_ms,
                    "solve_tflops": (gemm_flops + attn_flops) / (statistics.median(batch_ms) / 1000) / 1e12,
                    "kernel_ms_per_solve": {k: round(v, 4) for k, (v, _) in prof.items()}}
    tl = None
    if a.timeline and rank == 0 and jobs:
        layout, b = jobs[0]
        tl = timeline(lambda: solver.solve_packed_dev(layout, b["x0"], b["mu"], b["cond"], b["spk"], b["out"],
                                                      workspace=b["ws"]))
    sub, cpu, ref_gpu = {}, None, None
    if rank == 0 and world == 1:
        if not a.no_subrecords:
            if a.workload != "c2":
                sub["c2"] = packed_record(solver, C2, 5, 2, flush, peak_tf)
            sub["c3"] = packed_record(solver, C3, 3, 1, flush, peak_tf)
            if a.workload == "c5":
                sub["target"] = {"workload": TARGET.name, "streams": TARGET.streams,
                                 "ms_per_solve": statistics.median(batch_ms),
                                 "chunk_frames_per_s": TARGET.chunk_frames / (statistics.median(batch_ms) / 1000),
                                 "gemm_frac": roofline["frac"] if roofline else None,
                                 "note": "the c5 job's batches are the target shape (64 x (300 + 50))"}
        if not a.no_cpu_baseline:
            sample = make_streams(wl, cfg.mel, count=1)
            ts, threads = cpu_oracle_time(cfg, sample, reps=2, warm=0)
            cpu = {"value": sample[0]["T"] / statistics.mean(ts), "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"1 stream (P={sample[0]['P']}, T={sample[0]['T']}) of {wl.name}, fp32 CPU oracle, "
                             "2 solves"}
    launches = sum(c for _, c in prof.values()) * len(jobs) * a.steps if prof else None
    solver_precision = solver.precision
    solver.close()
    del jobs
    if rank == 0 and world == 1 and not a.no_subrecords:
        torch.cuda.empty_cache()
        fp8s = B200Solver(cfg, random_state_dict(cfg, seed=0, device=dev), precision="fp8", device=dev)
        sub["c4_fp8"] = packed_record(fp8s, C4, 3, 1, flush, 2 * peaks.get("bf16_tflops_sustained", 1400.0))
        fp8s.close()
        torch.cuda.empty_cache()
        for n in (32, 64):
            sub[f"steady_{n}"] = steady_record(cfg, dev, n, steps=10, warmup=3, seed=11)
            torch.cuda.empty_cache()
        sub["encoder_64"] = encoder_record(dev, 64, 150, steps=10, warmup=4, seed=12, peak_tf=peak_tf)
        torch.cuda.empty_cache()
        sub["hift_64"] = hift_record(dev, 64, steps=5, warmup=2, seed=14, peak_tf=peak_tf)
        torch.cuda.empty_cache()
        sub["hift_64_split_fp32"] = hift_record(dev, 64, steps=5, warmup=2, seed=14, peak_tf=peak_tf, split_fp32=True)
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not a.no_reference_gpu:
        torch.cuda.empty_cache()
        ref_gpu = reference_gpu_child(a)
        ours = {"target": sub.get("target", {}).get("ms_per_solve"), "c2": (sub.get("c2") or {}).get("ms_per_solve")}
        w_ours = (sub.get("steady_32") or {}).get("ms_per_call")
        w_ref = (ref_gpu.get("w32_fastdit") or {}).get("window_ms")
        if w_ours and w_ref:  # steady-state windows, 32 per call: FastDiT's graph-replayed window vs this build's call
            ref_gpu["steady_32_speedup_vs_fastdit_window"] = w_ref / w_ours
        h_ours = (sub.get("hift_64") or {}).get("ms_per_call")
        for k in ("hift_64", "hift_64_tf32", "hift_64_graphs", "hift_64_graphs_tf32"):  # the vocoder's steady call
            h_ref = (ref_gpu.get(k) or {}).get("ms_per_call")
            if h_ours and h_ref:
                ref_gpu.setdefault("hift_speedup", {})[k] = h_ref / h_ours
        h32 = (sub.get("hift_64_split_fp32") or {}).get("ms_per_call")
        for k in ("hift_64", "hift_64_graphs"):  # fp32 numerics on both sides: the reference's default precision
            h_ref = (ref_gpu.get(k) or {}).get("ms_per_call")
            if h32 and h_ref:
                ref_gpu.setdefault("hift_speedup_fp32", {})[k] = h_ref / h32
        e_ours = (sub.get("encoder_64") or {}).get("ms_per_call")
        for k in ("encoder_64", "encoder_64_batched_io"):  # the flow encoder's steady window call, 64 streams
            e_ref = (ref_gpu.get(k) or {}).get("ms_per_call")
            if e_ours and e_ref:
                ref_gpu.setdefault("encoder_speedup", {})[k] = e_ref / e_ours
        if a.workload == "c2":
            ours["c2"] = statistics.median(batch_ms)
        for k, v in ours.items():
            r = (ref_gpu.get(k) or {}).get("ms_per_solve")
            if v and r:
                ref_gpu.setdefault("speedup", {})[k] = r / v
            rf = (ref_gpu.get(k + "_fastdit") or {}).get("ms_per_solve")
            if v and rf:
                ref_gpu.setdefault("speedup_vs_fastdit", {})[k] = rf / v
    if rank == 0:
        flat = sorted(x for r in all_lat for x in r)
        pct = lambda q: flat[min(len(flat) - 1, int(round(q * (len(flat) - 1))))] if flat else None  # noqa: E731
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": max_ms / a.steps, "higher_is_better": True,
            "scaling": "strong" if a.workload == "c5" else "weak", "vs_baseline": None,
            "dtype": "e4m3 (block projections) + bf16" if solver_precision == "fp8" else "bf16", "data": "synthetic",
            "config": {"workload": wl.name, "streams_total": len(wl.lengths) if a.workload == "c5" else world * wl.streams,
                       "streams_per_gpu": len(idx), "batch_streams": batch, "prompt_frames": wl.lengths[0][0],
                       "chunk_frames": wl.lengths[0][1], "chunk_frames_per_step": frames, "mel": cfg.mel,
                       "euler_steps": cfg.steps, "cfg": True,
                       "model": "reference-config DiT (H=512, depth 16, 8x64 heads, unverified), random init",
                       "precision": solver_precision,
                       "sharding": "b200t2w.scheduler.shard_streams (contiguous), one process per GPU, no collectives"
                       if a.workload == "c5" else f"replicas x{world}",
                       "l2": "flushed between timed steps (256 MiB write, untimed); each step's inputs and working set "
                             "exceed L2"},
            "latency_ms": {"p50": pct(0.5), "p95": pct(0.95), "per": "chunk (its batch's end - the step's start)",
                           "batch_solve_ms_p50": statistics.median(batch_ms)},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "B200Solver.solve_streams on per-stream host tensors, chunk mels read back to pinned host"},
            "gpu_launches": launches, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk}
        if sub:
            line["subrecords"] = sub
        if ref_gpu is not None:
            line["reference_gpu"] = ref_gpu
        if tl:
            line["timeline"] = tl
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()


def main() -> None:
    a = args_()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if a.impl == "reference" and a.reference_gpu:
        reference_gpu_arm(a)
        return
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    try:
        if a.impl == "reference":
            reference_arm(a, rank, world)
        elif a.workload == "encoder":
            torch.cuda.set_device(local)
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
                os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
            rec = encoder_record(torch.device("cuda", local), a.batch, 150, a.steps, a.warmup, seed=12 + rank,
                                 peak_tf=peaks.get("bf16_tflops_sustained", 1400.0), cpu=not a.no_cpu_baseline)
            if rank == 0:
                print(json.dumps({"metric": "flow encoder mu frames/s (steady windows)", "value": rec["mu_frames_per_s"],
                                  "unit": "mu frames/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
                                  "ms_per_step": rec["ms_per_call"], "higher_is_better": True, "dtype": "bf16",
                                  "data": "synthetic", "config": {"workload": rec["workload"]}, "encoder": rec}),
                      flush=True)
        elif a.workload == "hift":
            torch.cuda.set_device(local)
            pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
            peak_tf = json.load(open(pk)).get("bf16_tflops_sustained", 1400.0) if os.path.exists(pk) else 1400.0
            rec = hift_record(torch.device("cuda", local), a.batch, a.steps, a.warmup, seed=14, peak_tf=peak_tf)
            if rank == 0:
                print(json.dumps({"metric": "HiFT mel frames/s (steady windows)", "value": rec["mel_frames_per_s"],
                                  "unit": "mel frames/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
                                  "ms_per_step": rec["ms_per_call"], "higher_is_better": True, "dtype": "f32",
                                  "data": "synthetic", "config": {"workload": rec["workload"]}, "hift": rec}), flush=True)
        elif a.workload == "steady":
            torch.cuda.set_device(local)
            rec = steady_record(REFERENCE, torch.device("cuda", local), a.batch, a.steps, a.warmup, seed=11 + rank,
                                timeline_on=a.timeline and rank == 0)
            red = torch.tensor([rec["ms_per_call"]], dtype=torch.float64)
            if world > 1:
                torch.distributed.all_reduce(red, op=torch.distributed.ReduceOp.MAX)
            if rank == 0:
                value = world * rec["streams"] * 50 / (float(red[0]) / 1000)
                print(json.dumps({
                    "metric": "DiT mel frames/s, steady-state windows (slot-pool solve)", "value": value, "unit": UNIT,
                    "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": float(red[0]),
                    "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                    "data": "synthetic", "config": {"workload": rec["workload"], "streams_per_gpu": rec["streams"]},
                    "latency_ms": {"p50": rec["latency_ms_p50"]}, "tflops": rec["tflops"],
                    "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": rec["h2d_bytes_per_call"],
                            "d2h_bytes_per_step": rec["d2h_bytes_per_call"]}, "steady": rec}), flush=True)
        else:
            packed_job(a, rank, world, local)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
