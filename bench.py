#!/usr/bin/env python
"""Benchmark of the Token2Wav DiT/CFM flow-matching solve on B200 (BASELINE.json metric: chunk mel frames/s per full
CFG ODE solve, with p50 / p95 per-chunk latency).

One "step" is one full S-step CFG Euler solve (one CUDA-graph replay) over one batch of packed ``[prompt | chunk]``
streams.  Default workload (N = 1): benchmark config 2, 16 streams of a 300-frame prompt + 50-frame chunk, bf16,
random-init reference-config weights, seeded synthetic inputs.  With ``--gpus N`` (launched by torchrun) every rank is
an independent replica with its own 16 streams (weak scaling; streams never cross GPUs, so there is no collective on the
data path, only a gloo barrier and a max over ranks of the device-timed region).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2|target|c5|c3|c4] [--impl b200|reference]

``--workload steady`` times the steady-state form (the reference's ``FastDiT.solve``): 64 streams with 300-frame
prompts already set up, one 50-frame window per stream per call against the slot-pool caches (trimmed to the prompt
plus the last 100 keys, as the reference trims them); a step is one such call, timed through the public API.

``--workload c4`` is benchmark config 4: config 2's shapes at 128 streams on the FP8 path (e4m3 block projections with
power-of-two block scales; bf16 in_proj, attention and final layer).

``--impl reference`` times the reference's own algorithm on the host cores (the CPU oracle port of the reference
solver, all threads), one stream of the workload per step, on rank 0 only.
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
from b200t2w.workload import C2, C3, C4, C5, TARGET, Workload, make_streams, uniform_streams  # noqa: E402

METRIC = "DiT mel frames/s per full CFG ODE solve"
UNIT = "mel frames/s"
L2_FLUSH_BYTES = 256 << 20


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c2", "target", "c5", "c3", "c4", "steady"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-profile", action="store_true")
    ap.add_argument("--timeline", action="store_true",
                    help="also record one graph-replayed solve with torch.profiler (CUPTI) and report each kernel "
                         "position's share of the solve's span (the time by which it extends the critical path)")
    return ap.parse_args()


def shard(name: str, rank: int, world: int) -> Workload:
    """This rank's streams.  c2 / target: a fixed per-GPU batch (weak scaling); c5: 1024 streams split by rank."""
    if name == "c5":
        n = C5.streams // world
        return Workload(f"{C5.name}[rank {rank}/{world}]", C5.seed, C5.lengths[rank * n:(rank + 1) * n])
    base = {"c2": C2, "target": TARGET, "c3": C3, "c4": C4, "steady": C2}[name]
    if world == 1:
        return base
    return Workload(f"{base.name}[rank {rank}]", base.seed + 1000 * rank, base.lengths)


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
    torch.set_num_threads(threads)
    model = dit_oracle.build_model(cfg, seed=0)
    ts = []
    for i in range(warm + reps):
        s = streams[i % len(streams)]
        t0 = time.perf_counter()
        dit_oracle.solve_packed(model, s["x0"], s["mu"], s["cond"], s["spk"], s["P"], s["T"])
        if i >= warm:
            ts.append(time.perf_counter() - t0)
    return ts, threads


def reference_arm(a, rank: int, world: int) -> None:
    if rank != 0:
        return
    wl = shard(a.workload, 0, 1)
    streams = make_streams(wl, count=min(4, wl.streams))
    ts, threads = cpu_oracle_time(REFERENCE, streams, a.steps, a.warmup)
    T = [streams[i % len(streams)]["T"] for i in range(a.steps)]
    value = sum(T) / sum(ts)
    sample = f"1 stream of {wl.name} (P={streams[0]['P']}, T={streams[0]['T']}) per step, fp32 CPU oracle port"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": 1000 * statistics.mean(ts), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.name, "streams_per_step": 1, "model": "reference-config DiT (unverified), random init"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)


def steady_arm(a, rank: int, world: int) -> None:
    """Steady-state windows through ``B200FastDiT`` (one process per GPU, each with its own 64 streams)."""
    from b200t2w.fastdit import B200FastDiT
    from b200t2w.solver import B200Solver
    from b200t2w.weights import random_state_dict

    cfg = REFERENCE
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n, P, T = 64, 300, 50
    g = torch.Generator().manual_seed(11 + rank)
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
    # window inputs in pinned host memory (copied in by each call), each call's mel read back to pinned host memory
    mus = [[torch.randn(cfg.mel, T, generator=g).pin_memory() for _ in range(n)] for _ in range(4)]
    spk_d = spk.to(dev)
    host_out = torch.empty(n, cfg.mel, T).pin_memory()

    def step(k):
        outs = fd.solve(caches, mus[k % 4], spk_d, None, [True] * n)
        host_out.copy_(torch.stack(outs), non_blocking=True)

    # caches reach the trimmed steady length (P + 100) after three windows; the steady structure's CUDA graph is
    # captured on its second call, so two more warm-up windows keep the capture out of the timed region
    for k in range(max(a.warmup, 3) + 2):
        step(k)
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    # throughput: calls back to back, as a serving loop issues them (a call's host planning overlaps the previous
    # call's GPU work); one event pair around the K calls
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for k in range(a.steps):
        step(k)
    e1.record(st)
    e1.synchronize()
    times = [e0.elapsed_time(e1) / a.steps] * a.steps
    # latency: one call at a time, host planning inside
    lat = []
    for k in range(min(a.steps, 5)):
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0.record(st)
        step(k)
        l1.record(st)
        l1.synchronize()
        lat.append(l0.elapsed_time(l1))
    solver.check()
    tl = timeline(lambda: step(0)) if a.timeline and rank == 0 else None
    frames = n * T
    red = torch.tensor([sum(times)], dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(red, op=torch.distributed.ReduceOp.MAX)
    value = world * frames * a.steps / (float(red[0]) / 1000)
    # per stream per window: S [2T (Dp 36 H^2 + 800 H) + Dp 4H 2T (keys)], keys = cache (P + 100) + T
    keys = caches[0].length
    flop = n * cfg.steps * (2 * T * (cfg.depth * 2 * cfg.hidden * (10 * cfg.hidden + 2 * cfg.ffn) + 800 * cfg.hidden)
                            + cfg.depth * 4 * cfg.hidden * 2 * T * keys)
    if rank == 0:
        print(json.dumps({
            "metric": "DiT mel frames/s, steady-state windows (slot-pool solve)", "value": value, "unit": UNIT,
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": statistics.mean(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"steady_{n}x{T} (P={P} cached, keys per row {keys})", "streams_per_gpu": n,
                       "window_frames": T, "prompt_frames": P, "model": "reference-config DiT (unverified), random init",
                       "timing": "CUDA events around K back-to-back public-API calls (host planning, the pinned "
                                 "host -> device input copies and the device -> host mel read-back inside)",
                       "solve_calls": dict(fd.counts)},
            "latency_ms": {"p50": statistics.median(lat)}, "tflops": flop / (statistics.mean(times) / 1000) / 1e12,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": n * T * cfg.mel * 4,
                    "d2h_bytes_per_step": n * T * cfg.mel * 4}, **({"timeline": tl} if tl else {})}), flush=True)
    fd.close()
    solver.close()


def main() -> None:
    a = args_()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    if a.impl == "reference":
        reference_arm(a, rank, world)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    if a.workload == "steady":
        steady_arm(a, rank, world)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return

    from b200t2w.solver import B200Solver, Layout
    from b200t2w.weights import random_state_dict

    cfg = REFERENCE
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    wl = shard(a.workload, rank, world)
    streams = make_streams(wl, cfg.mel)
    layout = Layout(tuple(s["P"] for s in streams), tuple(s["T"] for s in streams))
    fp8 = a.workload == "c4"
    solver = B200Solver(cfg, random_state_dict(cfg, seed=0, device=dev), precision="fp8" if fp8 else "bf16", device=dev)
    bufs = solver.static_buffers(layout)
    host = {k: torch.cat([s[k].t() for s in streams]).contiguous().pin_memory() for k in ("x0", "mu", "cond")}
    host["spk"] = torch.stack([s["spk"] for s in streams]).contiguous().pin_memory()
    host_out = torch.empty(layout.n_tok, cfg.mel, dtype=torch.float32).pin_memory()
    for k in ("x0", "mu", "cond", "spk"):
        bufs[k].copy_(host[k])
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev)

    def solve():
        solver.solve_packed_dev(layout, bufs["x0"], bufs["mu"], bufs["cond"], bufs["spk"], bufs["out"], workspace=bufs["ws"])

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()

    # ---- device-resident throughput (inputs already in HBM)
    for _ in range(a.warmup):
        solve()
    barrier()
    clocks = Clocks(physical_index(local))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    for e0, e1 in evs:
        flush.fill_(1)  # L2 flush between timed solves (outside the timed interval)
        e0.record(st)
        solve()
        e1.record(st)
    barrier()
    clk = clocks.stop()
    solver.check()
    times = [e0.elapsed_time(e1) for e0, e1 in evs]  # ms
    total_ms = sum(times)

    # ---- end to end through the public API: pinned host inputs -> device -> solve -> host result
    h2d = sum(host[k].numel() * 4 for k in ("x0", "mu", "cond", "spk"))
    d2h = host_out.numel() * 4
    e2e_t = []
    for i in range(a.warmup + a.steps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for k in ("x0", "mu", "cond", "spk"):
            bufs[k].copy_(host[k], non_blocking=True)
        solve()
        host_out.copy_(bufs["out"], non_blocking=True)
        e1.record(st)
        e1.synchronize()
        if i >= a.warmup:
            e2e_t.append(e0.elapsed_time(e1))
    barrier()

    # ---- max over ranks of the device-timed regions
    red = torch.tensor([total_ms, sum(e2e_t)], dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(red, op=torch.distributed.ReduceOp.MAX)
    max_ms, max_e2e_ms = float(red[0]), float(red[1])
    chunk_frames = wl.chunk_frames  # per rank per solve
    value = world * chunk_frames * a.steps / (max_ms / 1000)
    e2e_value = world * chunk_frames * a.steps / (max_e2e_ms / 1000)

    prof = solver.profile(layout, bufs) if not a.no_profile else {}
    tl = timeline(solve) if a.timeline and rank == 0 else None
    gemm_flops, attn_flops = flops_per_solve(cfg, layout_pairs := list(zip(layout.prompt, layout.chunk)))
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    peak_tf = peaks.get("bf16_tflops_sustained", 1400.0)
    peak_src = "MEASURED_PEAKS.json bf16_tflops_sustained" if "bf16_tflops_sustained" in peaks else "fallback"
    if fp8:  # no measured e4m3 peak: twice the measured bf16 figure (the dense e4m3 / bf16 ratio of the part)
        peak_tf *= 2
        peak_src = "2 x " + peak_src + " (no measured e4m3 peak)"
    launches = sum(c for _, c in prof.values()) if prof else None
    gemm_ms = sum(ms for k, (ms, _) in prof.items() if k.startswith("gemm")) if prof else None
    roofline = None
    if prof:
        achieved = gemm_flops / (gemm_ms / 1000) / 1e12
        traffic = None
        try:
            traffic = json.load(open(os.path.join(ROOT, "profiles", "traffic.json"))).get("gemm_bytes_per_solve")
        except (OSError, ValueError):
            pass
        roofline = {"bound": "tensor", "kernel": "k_gemm (all tcgen05 GEMM launches of one solve)", "achieved": achieved,
                    "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf, "peak_source": peak_src,
                    "traffic": traffic, "gemm_ms_per_solve": gemm_ms, "gemm_tflop_per_solve": gemm_flops / 1e12,
                    "solve_tflops": (gemm_flops + attn_flops) / (statistics.mean(times) / 1000) / 1e12,
                    "kernel_ms_per_solve": {k: round(ms, 4) for k, (ms, _) in prof.items()}}
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        sample = make_streams(wl, cfg.mel, count=1)
        ts, threads = cpu_oracle_time(cfg, sample, reps=2, warm=0)
        cpu = {"value": sample[0]["T"] / statistics.mean(ts), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"1 stream (P={sample[0]['P']}, T={sample[0]['T']}) of {wl.name}, fp32 CPU oracle, 2 solves"}
    if rank == 0:
        srt = sorted(times)
        lat = {"p50": statistics.median(times), "p95": srt[min(len(srt) - 1, int(round(0.95 * (len(srt) - 1))))]}
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": max_ms / a.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3 (block projections) + bf16" if fp8 else "bf16", "data": "synthetic",
            "config": {"workload": wl.name, "streams_per_gpu": wl.streams, "prompt_frames": layout.prompt[0],
                       "chunk_frames": layout.chunk[0], "chunk_frames_per_solve_per_gpu": chunk_frames,
                       "packed_frames_per_solve_per_gpu": 2 * wl.packed_frames, "mel": cfg.mel, "euler_steps": cfg.steps,
                       "cfg": True, "model": "reference-config DiT (H=512, depth 16, 8x64 heads, unverified), random init",
                       "precision": "fp8" if fp8 else "bf16",
                       "l2": "flushed between timed solves (256 MiB write, untimed)",
                       "parallelism": f"replicas x{world} (streams sharded by request, no collectives)"},
            "latency_ms": lat, "processed_frames_per_s": value * 2 * wl.packed_frames / chunk_frames,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "latency_ms_p50": statistics.median(e2e_t)},
            "gpu_launches": launches * a.steps if launches else None, "roofline": roofline, "cpu_baseline": cpu,
            "clocks": clk, **({"timeline": tl} if tl else {})}), flush=True)
    solver.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
