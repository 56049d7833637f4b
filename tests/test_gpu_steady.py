"""GPU: the steady-state (slot-pool) solve through the C ABI, driven like the reference's FastDiT.

Windows of several streams ride one call (ragged T, prompt setups beside steady windows and final flushes); each
window's mel must match the reference driver's own streaming solve (``tests/golden/steady_tiny.pt``: ``_solve`` with
its caches and ``_trim``) and the oracle's ``solve_window`` within the bf16 tolerance (rel-L2 <= 1e-2), cache lengths
must follow the reference's trim, and the slot pool must account for every key."""

import os

import pytest
import torch

from b200t2w.config import REFERENCE, TINY
from b200t2w.fastdit import B200FastDiT
from b200t2w.solver import B200Solver, state_dict_from_module
from oracle import dit_oracle

pytestmark = pytest.mark.gpu
TOL_BF16 = 1e-2


def rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm())


def run_interleaved(fd, streams):
    """Every stream's k-th window in one call per k; returns {(stream, k): mel}."""
    caches = []
    for s in streams:
        c = fd.new_cache()
        c.keep = s["P"]
        caches.append(c)
    out = {}
    for k in range(max(len(s["windows"]) for s in streams)):
        ids = [i for i, s in enumerate(streams) if k < len(s["windows"])]
        ws = [streams[i]["windows"][k] for i in ids]
        mels = fd.solve([caches[i] for i in ids], [w["mu"] for w in ws], torch.stack([streams[i]["spk"] for i in ids]),
                        [w["cond"] for w in ws] if any(w["cond"] is not None for w in ws) else None,
                        [w["keep"] for w in ws])
        fd.solver.check()
        for i, w, m in zip(ids, ws, mels):
            out[(i, k)] = m
            assert caches[i].length == w["cache_len_after"], (i, k, caches[i].length, w["cache_len_after"])
    return out, caches


def test_steady_tiny_vs_reference_driver(golden_dir):
    rec = torch.load(os.path.join(golden_dir, "steady_tiny.pt"))
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=2048)
    fd = B200FastDiT(B200Solver(TINY, state_dict_from_module(m)), m.rand_noise[0], n_slots=4096, max_streams=8)
    out, caches = run_interleaved(fd, rec["streams"])
    for i, s in enumerate(rec["streams"]):
        for k, w in enumerate(s["windows"]):
            e = rel(out[(i, k)], w["ref_mel"])
            print(f"stream {i} window {k} (T={w['T']}, keep={w['keep']}, offset={w['offset']}): rel-L2 {e:.3e}")
            assert e < TOL_BF16, (i, k, e)
    assert fd.pool.in_use() == 2 * sum(c.length for c in caches)
    for c in caches:
        fd.release(c)
    assert fd.pool.in_use() == 0


def test_steady_clone_is_independent(golden_dir):
    rec = torch.load(os.path.join(golden_dir, "steady_tiny.pt"))
    s = rec["streams"][1]
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=2048)
    fd = B200FastDiT(B200Solver(TINY, state_dict_from_module(m)), m.rand_noise[0], n_slots=2048, max_streams=4)
    c = fd.new_cache()
    c.keep = s["P"]
    for w in s["windows"][:4]:
        fd.solve([c], [w["mu"]], s["spk"][None], [w["cond"]], [True])
    d = fd.clone(c)
    w = s["windows"][4]
    a = fd.solve([c], [w["mu"]], s["spk"][None], None, [True])[0]
    b = fd.solve([d], [w["mu"]], s["spk"][None], None, [True])[0]
    assert torch.equal(a, b)
    assert rel(a, w["ref_mel"]) < TOL_BF16
    fd.release(c)
    fd.release(d)
    assert fd.pool.in_use() == 0


def test_steady_reference_config_vs_oracle():
    """Reference config: two streams with trims, against the oracle's window solve."""
    torch.set_num_threads(os.cpu_count() or 1)
    m = dit_oracle.build_model(REFERENCE, seed=0, noise_frames=2048)
    fd = B200FastDiT(B200Solver(REFERENCE, state_dict_from_module(m)), m.rand_noise[0], n_slots=2048, max_streams=4)
    g = torch.Generator().manual_seed(5)
    mel = REFERENCE.mel
    streams = []
    for P, Ts in ((120, (50, 50, 50, 7)), (60, (33, 50, 41, 50))):
        ws = [{"mu": torch.randn(mel, P, generator=g), "cond": torch.randn(mel, P, generator=g), "keep": True}]
        ws += [{"mu": torch.randn(mel, t, generator=g), "cond": None, "keep": j < len(Ts) - 1} for j, t in enumerate(Ts)]
        streams.append({"P": P, "spk": torch.randn(mel, generator=g), "windows": ws})
    # oracle, stream by stream
    for s in streams:
        cache = dit_oracle.StreamCache(REFERENCE, keep=s["P"])
        for w in s["windows"]:
            x0 = m.rand_noise[0, :, cache.length:cache.length + w["mu"].shape[1]]
            w["ref_mel"] = dit_oracle.solve_window(m, cache, x0, w["mu"], s["spk"], w["cond"], keep_cache=w["keep"])
            w["cache_len_after"] = cache.length
    out, caches = run_interleaved(fd, streams)
    for i, s in enumerate(streams):
        for k, w in enumerate(s["windows"]):
            e = rel(out[(i, k)], w["ref_mel"])
            print(f"reference config stream {i} window {k}: rel-L2 {e:.3e}")
            assert e < TOL_BF16


def test_steady_graph_replay_equals_eager():
    """use_graphs: once the windows reach the trimmed steady length the call structure repeats, its graph is captured
    on the second sight and replayed; every window's mel equals the eager solve's bit for bit."""
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=4096)
    solver = B200Solver(TINY, state_dict_from_module(m))
    fds = {g: B200FastDiT(solver, m.rand_noise[0], n_slots=4096, max_streams=4, use_graphs=g) for g in (False, True)}
    gen = torch.Generator().manual_seed(9)
    mel, n, P, T = TINY.mel, 3, 40, 32  # caches trimmed to P + 100 keys from the fifth window on
    spk = torch.randn(n, mel, generator=gen)
    windows = [([torch.randn(mel, P, generator=gen) for _ in range(n)], [torch.randn(mel, P, generator=gen) for _ in range(n)])]
    windows += [([torch.randn(mel, T, generator=gen) for _ in range(n)], None) for _ in range(10)]
    outs = {}
    for g, fd in fds.items():
        caches = [fd.new_cache() for _ in range(n)]
        for c in caches:
            c.keep = P
        outs[g] = [fd.solve(caches, mu, spk, cond, [True] * n) for mu, cond in windows]
        fd.solver.check()
        for c in caches:
            fd.release(c)
        assert fd.pool.in_use() == 0
    assert fds[False].counts["graph"] == 0
    assert fds[True].counts["graph"] >= 3, fds[True].counts
    for wa, wb in zip(outs[False], outs[True]):
        for a, b in zip(wa, wb):
            assert torch.equal(a, b)


def test_forward_chunk_with_caches_vs_oracle():
    """The reference's module-level forward_chunk(mu, spks, cond, n_timesteps, temperature, cnn_cache, att_cache): a
    prompt window with empty caches, then chunk windows fed the caches the previous call returned, against the
    oracle's window solve: the mel, the new attention cache (keys [new, old], nothing trimmed) and the conv cache
    within the bf16 tolerance; the slots are all returned."""
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=2048)
    fd = B200FastDiT(B200Solver(TINY, state_dict_from_module(m)), m.rand_noise[0], n_slots=1024, max_streams=2)
    gen = torch.Generator().manual_seed(21)
    mel = TINY.mel
    spk = torch.randn(1, mel, generator=gen)
    cache = dit_oracle.StreamCache(TINY, keep=10 ** 6)
    att = cnn = None
    for j, (T, temp) in enumerate(((40, 1.0), (24, 1.0), (24, 0.7))):
        mu = torch.randn(1, mel, T, generator=gen)
        cond = torch.randn(1, mel, T, generator=gen) if j == 0 else None
        out, cnn, att = fd.forward_chunk(mu, spk, cond, TINY.steps, temp, cnn, att)
        x0 = m.rand_noise[0, :, cache.length:cache.length + T] * temp
        ref = dit_oracle.solve_window(m, cache, x0, mu[0], spk[0], cond[0] if cond is not None else None)
        assert out.shape == (1, mel, T) and out.dtype == torch.float32
        assert att.shape == cache.att.shape and cnn.shape == cache.cnn.shape
        e = (rel(out[0], ref), rel(att, cache.att), rel(cnn, cache.cnn))
        print(f"window {j} (T={T}, temperature {temp}): rel-L2 mel {e[0]:.2e}, att cache {e[1]:.2e}, cnn cache {e[2]:.2e}")
        assert max(e) < TOL_BF16, e
    assert fd.pool.in_use() == 0


def test_from_cfm_vs_reference_driver(golden_dir):
    """Built the reference's way, ``FastDiT(cfm, steps, n_slots, max_streams, device, use_graphs, ...)``: the same
    windows as the reference driver within the bf16 tolerance, and the attributes its worker reads
    (``pool.in_use() - scratch``, ``cnn_free``, ``counts``, ``capture_all()``)."""
    rec = torch.load(os.path.join(golden_dir, "steady_tiny.pt"))
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=2048)
    fd = B200FastDiT.from_cfm(m, TINY.steps, n_slots=4096, max_streams=8, device="cuda", use_graphs=True,
                              setup_tokens=64, fused_residual=True, fused_conv=True)
    assert fd.cfg == TINY and fd.capture_all() == 0
    free0 = len(fd.cnn_free)
    out, caches = run_interleaved(fd, rec["streams"])
    for i, s in enumerate(rec["streams"]):
        for k, w in enumerate(s["windows"]):
            e = rel(out[(i, k)], w["ref_mel"])
            assert e < TOL_BF16, (i, k, e)
    assert fd.pool.in_use() - fd.scratch == 2 * sum(c.length for c in caches)
    assert len(fd.cnn_free) == free0 - 2 * len(caches)
    assert fd.counts["graph"] + fd.counts["eager"] == max(len(s["windows"]) for s in rec["streams"])
    for c in caches:
        fd.release(c)
    assert fd.pool.in_use() == 0 and len(fd.cnn_free) == free0
