"""GPU: the whole CFG Euler solve through the C ABI against the CPU oracle and the golden fixtures.

Tolerance (bf16 path, stated per the north star): final-mel relative L2 <= 1e-2 against the fp32 oracle; the
max-abs error is reported beside it.  Streams are independent, so at full benchmark sizes the GPU solves the whole
batch and a sample of its streams is checked against the oracle (a size-independent property: per-stream results do
not depend on the batch they ride in)."""

import os

import pytest
import torch

from b200t2w.config import REFERENCE, TINY
from b200t2w.solver import B200Solver, Layout, state_dict_from_module
from b200t2w.workload import C1, C2, C3, C4, TARGET, Workload, make_streams
from oracle import dit_oracle

pytestmark = pytest.mark.gpu
TOL_BF16 = 1e-2


def rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm())


def maxabs(a, b):
    return float((a.float().cpu() - b.float().cpu()).abs().max())


@pytest.fixture(scope="module")
def tiny():
    m = dit_oracle.build_model(TINY, seed=0)
    return m, B200Solver(TINY, state_dict_from_module(m))


@pytest.fixture(scope="module")
def ref():
    torch.set_num_threads(os.cpu_count() or 1)
    m = dit_oracle.build_model(REFERENCE, seed=0)
    return m, B200Solver(REFERENCE, state_dict_from_module(m))


def test_modulation_tables_match_oracle(tiny):
    """The time-embedding kernel's adaLN tables equal the oracle module's (t_embedder + adaLN_modulation)."""
    m, s = tiny
    mods, fmods, dts = s.mods()
    from b200t2w.config import t_schedule

    ts, dts_ref = t_schedule(TINY.steps)
    est = m.estimator
    with torch.no_grad():
        for i, t in enumerate(ts):
            temb = est.t_embedder(torch.tensor([t]))
            for b, blk in enumerate(est.blocks):
                r = blk.adaLN_modulation(temb).view(9, -1)
                r[[1, 4, 7]] += 1
                assert rel(mods[i, b], r) < 1e-5, (i, b)
            f = est.final_layer.adaLN_modulation(temb).view(2, -1)
            f[1] += 1
            assert rel(fmods[i], f) < 1e-5
    assert torch.allclose(dts.cpu(), torch.tensor(dts_ref))


def test_tiny_ragged_vs_golden(tiny, golden_dir):
    _, s = tiny
    rec = torch.load(os.path.join(golden_dir, "tiny_ragged.pt"))
    outs = s.solve_streams(rec["streams"])
    s.check()
    for o, g in zip(outs, rec["streams"]):
        P = g["P"]
        e_p, e_c = rel(o[:, :P], g["ref_prompt_mel"]), rel(o[:, P:], g["ref_chunk_mel"])
        assert e_p < TOL_BF16 and e_c < TOL_BF16, (P, g["T"], e_p, e_c, maxabs(o[:, P:], g["ref_chunk_mel"]))


def test_graph_replay_equals_eager(tiny):
    _, s = tiny
    streams = make_streams(Workload("g", 5, ((40, 12), (9, 30))), TINY.mel)
    a = s.solve_streams(streams, graph=False)
    b = s.solve_streams(streams, graph=True)
    c = s.solve_streams(streams, graph=True)
    for x, y, z in zip(a, b, c):
        assert torch.equal(x, y) and torch.equal(y, z)
    n = s.counts()
    assert n["graph"] >= 2 and n["captures"] >= 1 and n["eager"] >= 1


def test_c1_full_size_vs_golden(ref, golden_dir):
    _, s = ref
    rec = torch.load(os.path.join(golden_dir, "c1_reference.pt"))
    st = make_streams(C1)[0]
    out = s.solve_streams([st])[0]
    s.check()
    g = rec["streams"][0]
    e = rel(out[:, st["P"]:], g["ref_chunk_mel"])
    print(f"C1 chunk mel rel-L2 {e:.3e} max-abs {maxabs(out[:, st['P']:], g['ref_chunk_mel']):.3e}")
    assert e < TOL_BF16


# Config 3's sample covers its ragged extremes: stream 25 is the shortest packed row (P=100, T=41), stream 58 the
# longest (P=492, T=91), stream 40 the shortest chunk (P=419, T=26), stream 9 the longest chunk (T=99), stream 24 a
# middle row (P=314, T=69), plus streams 0 and 37.  Those rows exercise the block-causal mask's partial 64-key tiles
# at both ends of the prompt / chunk boundary and the conv pads between short and long neighbours.
@pytest.mark.parametrize("wl,sample", [(C2, (0, 15)), (C3, (0, 9, 24, 25, 37, 40, 58)), (TARGET, (0, 63))])
def test_batch_streams_vs_oracle(ref, wl, sample):
    m, s = ref
    streams = make_streams(wl)
    outs = s.solve_streams(streams)
    s.check()
    for i in sample:
        st = streams[i]
        o = dit_oracle.solve_packed(m, st["x0"], st["mu"], st["cond"], st["spk"], st["P"], st["T"])
        e = rel(outs[i][:, st["P"]:], o[:, st["P"]:])
        print(f"{wl.name} stream {i} (P={st['P']}, T={st['T']}): chunk rel-L2 {e:.3e} "
              f"max-abs {maxabs(outs[i][:, st['P']:], o[:, st['P']:]):.3e}")
        assert e < TOL_BF16


def test_workspace_and_bad_shapes_raise(tiny):
    _, s = tiny
    lay = Layout((5,), (3,))
    z = torch.zeros(8, TINY.mel, device="cuda")
    with pytest.raises(ValueError):
        s.solve_packed_dev(lay, z, z, z, torch.zeros(2, TINY.mel, device="cuda"), z)
    from b200t2w.lib import T2WError

    with pytest.raises(T2WError):
        s.solve_packed_dev(lay, z, z, z, torch.zeros(1, TINY.mel, device="cuda"), z,
                           workspace=torch.empty(256, dtype=torch.uint8, device="cuda"))


TOL_FP8 = 3e-2


def test_fp8_small_config_vs_oracle():
    """The FP8 path (e4m3 block projections) end to end on a small config whose projections tile by 256."""
    from b200t2w.config import DiTConfig

    cfg = DiTConfig(hidden=256, depth=2, heads=4)
    m = dit_oracle.build_model(cfg, seed=0)
    s = B200Solver(cfg, state_dict_from_module(m), precision="fp8")
    streams = make_streams(Workload("fp8s", 7, ((60, 20), (33, 17), (130, 40))), cfg.mel)
    outs = s.solve_streams(streams)
    s.check()
    for st, o in zip(streams, outs):
        ref = dit_oracle.solve_packed(m, st["x0"], st["mu"], st["cond"], st["spk"], st["P"], st["T"])
        e = rel(o, ref)
        print(f"fp8 small (P={st['P']}, T={st['T']}): rel-L2 {e:.3e} max-abs {maxabs(o, ref):.3e}")
        assert e < TOL_FP8


def test_fp8_c1_full_size_vs_golden(ref, golden_dir):
    """Reference config on the FP8 path against the reference driver's fp32 chunk mel."""
    m, _ = ref
    s = B200Solver(REFERENCE, state_dict_from_module(m), precision="fp8")
    rec = torch.load(os.path.join(golden_dir, "c1_reference.pt"))
    st = make_streams(C1)[0]
    out = s.solve_streams([st])[0]
    s.check()
    g = rec["streams"][0]
    e = rel(out[:, st["P"]:], g["ref_chunk_mel"])
    print(f"C1 FP8 chunk mel rel-L2 {e:.3e} max-abs {maxabs(out[:, st['P']:], g['ref_chunk_mel']):.3e}")
    assert e < TOL_FP8


def test_fp8_c4_full_shape_vs_oracle(ref):
    """Config 4 at its real shape: 128 streams of (300 + 50) frames solved as one batch on the FP8 path (2 x 45,056
    packed rows, so the large-M tile schedule of the e4m3 GEMMs runs), streams 0, 63 and 127 against the fp32 oracle
    at the FP8 tolerance."""
    m, _ = ref
    s = B200Solver(REFERENCE, state_dict_from_module(m), precision="fp8")
    streams = make_streams(C4)
    assert len(streams) == 128
    outs = s.solve_streams(streams)
    s.check()
    for i in (0, 63, 127):
        st = streams[i]
        o = dit_oracle.solve_packed(m, st["x0"], st["mu"], st["cond"], st["spk"], st["P"], st["T"])
        e = rel(outs[i][:, st["P"]:], o[:, st["P"]:])
        print(f"{C4.name} stream {i}: FP8 chunk rel-L2 {e:.3e} max-abs {maxabs(outs[i][:, st['P']:], o[:, st['P']:]):.3e}")
        assert e < TOL_FP8
    s.close()
