"""GPU: the flow encoder (speech tokens -> mu) through the C ABI.

Kernels against plain fp32 PyTorch statements of the same op on the same bf16 inputs (relative-position attention
rel-L2 <= 1e-2, P is rounded to bf16 before the P V product; the position table and the LayerNorm <= 1e-5 / 5e-3; the
new GEMM epilogues <= 5e-3).  The whole encoder against the golden fixtures made by the reference's own encoder driver
(``tests/golden/make_encoder_golden.py``: ``_setup_encoder_batched``, ``_encoder`` with left-padded caches, masks,
merged finals and ``_flow_finish``'s trim) and against the fp32 oracle on ragged batches at the reference config:
mu rel-L2 <= 1e-2 (bf16 activations, fp32 residual stream and accumulation), with each stream's cache lengths equal to
the reference's after every call."""

import copy
import ctypes
import math
import os

import pytest
import torch
import torch.nn.functional as F

from b200t2w import lib as L
from b200t2w.config import ENCODER, ENCODER_TINY
from b200t2w.encoder import B200FlowEncoder
from oracle import encoder_oracle as eo

pytestmark = pytest.mark.gpu

TOL = 1e-2


def P(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def S():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm().clamp_min(1e-30))


@pytest.fixture(scope="module", autouse=True)
def _dev():
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    assert L.load().t2w_device_ok(torch.cuda.current_device()) == 1
    torch.manual_seed(0)


def pe_table(H, max_frames, max_period=10000.0):
    r = torch.arange(-(max_frames - 1), max_frames, dtype=torch.float32)[:, None]
    w = torch.exp(torch.arange(0, H, 2, dtype=torch.float32) * -(math.log(max_period) / H))
    pe = torch.zeros(2 * max_frames - 1, H)
    pe[:, 0::2] = torch.sin(r * w)
    pe[:, 1::2] = torch.cos(r * w)
    return pe


@pytest.mark.parametrize("H", [128, 512])
def test_pos_table(H):
    mf = 300
    w = (torch.rand(H, H) * 2 - 1) / math.sqrt(H)
    pos = torch.empty(2 * mf - 1, H, dtype=torch.bfloat16, device="cuda")
    L.call("t2w_enc_pos_table", P(w.cuda()), H, mf, ctypes.c_float(10000.0), P(pos), S())
    torch.cuda.synchronize()
    ref = pe_table(H, mf).double() @ w.double().t()
    assert rel(pos, ref) < 5e-3


def test_enc_ln():
    rows, C = 333, 512
    x = torch.randn(rows, C, device="cuda") * 2 + 0.5
    w, b = 1 + 0.1 * torch.randn(C, device="cuda"), 0.1 * torch.randn(C, device="cuda")
    pad = (torch.rand(rows, device="cuda") < 0.2).to(torch.uint8)
    of = torch.empty_like(x)
    ob = torch.empty(rows, C, dtype=torch.bfloat16, device="cuda")
    L.call("t2w_enc_ln", P(x), P(w), P(b), ctypes.c_float(1e-12), rows, C, P(of), P(ob), P(pad), S())
    torch.cuda.synchronize()
    ref = F.layer_norm(x, (C,), w, b, eps=1e-12)
    ref[pad.bool()] = 0
    assert rel(of, ref) < 1e-5 and rel(ob, ref) < 5e-3
    # in place
    L.call("t2w_enc_ln", P(x), P(w), P(b), ctypes.c_float(1e-12), rows, C, P(x), P(None), P(None), S())
    torch.cuda.synchronize()
    assert rel(x[~pad.bool()], ref[~pad.bool()]) < 1e-5


@pytest.mark.parametrize("epi", ["silu", "leaky"])
def test_gemm_new_epilogues(epi):
    M, N, K = 384, 512, 512
    A = (torch.randn(M, K, device="cuda")).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda") / math.sqrt(K)).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda") * 0.1
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    slope = 0.01
    L.call("t2w_gemm", P(A), K, M, P(W), P(bias), M, N, K, 1, 0, L.EPI[epi], P(out), N, None, ctypes.c_float(slope), S())
    torch.cuda.synchronize()
    y = A.float() @ W.float().t() + bias
    ref = F.silu(y) if epi == "silu" else F.leaky_relu(y, slope)
    assert rel(out, ref) < 5e-3


def relattn_ref(qkv4, pool, pos, mf, seqs, kv_idx, heads):
    H = heads * 64
    out = torch.zeros(qkv4.shape[0], H, device="cuda")
    for q_row, T, K, off in seqs:
        kv = pool[torch.tensor(kv_idx[off:off + K], device="cuda").long()].float()
        i = torch.arange(T, device="cuda")[:, None]
        j = torch.arange(K, device="cuda")[None, :]
        r = (K - T + i) - j + mf - 1
        for h in range(heads):
            c = slice(h * 64, (h + 1) * 64)
            qu = qkv4[q_row:q_row + T, c].float()
            qv = qkv4[q_row:q_row + T, H + h * 64:H + (h + 1) * 64].float()
            k, v = kv[:, c], kv[:, H + h * 64:H + (h + 1) * 64]
            pr = pos[r, h * 64:(h + 1) * 64].float()
            s = (qu @ k.t() + (qv[:, None, :] * pr).sum(-1)) / 8.0
            out[q_row:q_row + T, c] = torch.softmax(s, -1) @ v
    return out


@pytest.mark.parametrize("heads,seqs", [
    (2, [(0, 1, 1), (5, 25, 200), (40, 50, 77)]),
    (8, [(0, 50, 450), (60, 25, 25), (100, 300, 300), (420, 130, 731)]),
])
def test_relattn(heads, seqs):
    """Sequences (query row, T, K): single query / key, partial key tiles, several 128-query tiles, keys shuffled
    through the pool."""
    H, mf = heads * 64, 1024
    rows = max(r + T for r, T, _ in seqs) + 7
    qkv4 = torch.randn(rows, 4 * H, device="cuda").to(torch.bfloat16)
    n_keys = sum(K for *_, K in seqs)
    pool_rows = n_keys + 50
    pool = torch.randn(pool_rows, 2 * H, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(pool_rows)[:n_keys].tolist()
    pos = (torch.randn(2 * mf - 1, H, device="cuda") * 0.5).to(torch.bfloat16)
    out = torch.full((rows, H), 3.0, device="cuda").to(torch.bfloat16)
    offs, o = [], 0
    for *_, K in seqs:
        offs.append(o)
        o += K
    L.call("t2w_enc_relattn", P(qkv4), rows, heads, P(pool), pool_rows, P(pos), mf, len(seqs),
           L.i32_array([s[0] for s in seqs]), L.i32_array([s[1] for s in seqs]), L.i32_array([s[2] for s in seqs]),
           L.i32_array(offs), L.i32_array(perm), len(perm), P(out), S())
    torch.cuda.synchronize()
    ref = relattn_ref(qkv4, pool, pos, mf, [(r, T, K, off) for (r, T, K), off in zip(seqs, offs)], perm, heads)
    for r, T, K in seqs:
        e = rel(out[r:r + T], ref[r:r + T])
        print(f"relattn heads={heads} T={T} K={K}: rel-L2 {e:.2e}")
        assert e < TOL


def test_relattn_rejects_bad_args():
    H, heads, mf = 128, 2, 64
    qkv4 = torch.zeros(64, 4 * H, dtype=torch.bfloat16, device="cuda")
    pool = torch.zeros(16, 2 * H, dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(2 * mf - 1, H, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(64, H, dtype=torch.bfloat16, device="cuda")
    args = lambda q_row, T, K, idx: (P(qkv4), 64, heads, P(pool), 16, P(pos), mf, 1, L.i32_array([q_row]),  # noqa
                                     L.i32_array([T]), L.i32_array([K]), L.i32_array([0]), L.i32_array(idx), len(idx),
                                     P(out), S())
    lib = L.load()
    assert lib.t2w_enc_relattn(*args(60, 8, 8, list(range(8)))) == -1   # queries past the buffer
    assert lib.t2w_enc_relattn(*args(0, 8, 4, list(range(4)))) == -1    # fewer keys than queries
    assert lib.t2w_enc_relattn(*args(0, 4, 4, [0, 1, 2, 16])) == -1     # a key outside the pool
    assert lib.t2w_enc_relattn(*args(0, 4, 65, list(range(65)))) == -1  # more keys than the table spans


# ---------------------------------------------------------------- whole encoder


def build(cfg, **kw):
    flow = eo.build_flow(cfg, seed=0)
    return flow, B200FlowEncoder.from_flow(flow, device="cuda", **kw)


@pytest.mark.parametrize("name,cfg", [("encoder_tiny", ENCODER_TINY), ("encoder_reference", ENCODER)])
def test_encoder_vs_reference_driver_golden(golden_dir, name, cfg):
    """Every prompt setup and window of the fixture (calls mixing cache lengths, trims, a final merged into a steady
    call, a final call) against the reference driver's mu; cache lengths against the oracle's after every call."""
    rec = torch.load(os.path.join(golden_dir, f"{name}.pt"))
    flow, enc = build(cfg, max_frames=1024, n_slots1=4096, n_slots2=8192, n_streams=16)
    assert eo.EncoderConfig(**rec["config"]) == cfg
    handles, mus = enc.setup([p["tokens"] for p in rec["prompts"]])
    sts = []
    for i, (p, mu) in enumerate(zip(rec["prompts"], mus)):
        e = rel(mu, p["mu"])
        print(f"{name} prompt {i}: rel-L2 {e:.2e}")
        assert mu.shape == p["mu"].shape and e < TOL
        sts.append(eo.encode_prompt(flow, p["tokens"])[1])
    for c, call in enumerate(rec["calls"]):
        ws = call["windows"]
        finals = [call["last"] or w["final"] for w in ws]
        got = enc.encode([handles[w["stream"]] for w in ws], [w["tokens"] for w in ws], finals)
        for w, mu, fin in zip(ws, got, finals):
            e = rel(mu, w["mu"])
            print(f"{name} call {c} stream {w['stream']} final={fin}: rel-L2 {e:.2e}")
            assert mu.shape == w["mu"].shape and e < TOL
            st = sts[w["stream"]]
            eo.encode_window(flow, st, w["tokens"], fin)
            k1, k2, _ = enc.stream_info(handles[w["stream"]])
            assert (k1, k2) == (st.att.shape[3] // 2, st.att.shape[3]), (k1, k2, st.att.shape)
    enc.check()
    for h in handles:
        enc.release(h)
    assert enc.usage() == (0, 0, 0)


def test_encoder_ragged_batches_vs_oracle():
    """Reference config: 12 streams with ragged prompts, steady windows of different streams in shared calls (some
    calls skip streams), then finals of different lengths in one call; every window against the fp32 oracle."""
    torch.manual_seed(7)
    flow, enc = build(ENCODER, max_frames=1536, n_slots1=16384, n_slots2=32768, n_streams=64)
    cfg = ENCODER
    lens = [int(x) for x in torch.randint(20, 260, (12,))]
    prompts = [torch.randint(0, cfg.vocab, (n,)) for n in lens]
    handles, mus = enc.setup(prompts)
    sts = []
    for p, mu in zip(prompts, mus):
        ref, st = eo.encode_prompt(flow, p)
        sts.append(st)
        assert rel(mu, ref) < TOL
    worst = 0.0
    for r in range(6):
        idx = [i for i in range(12) if (i + r) % 4 != 3]
        wins = [torch.randint(0, cfg.vocab, (28,)) for _ in idx]
        got = enc.encode([handles[i] for i in idx], wins, [False] * len(idx))
        for i, w, mu in zip(idx, wins, got):
            ref = eo.encode_window(flow, sts[i], w, False)
            e = rel(mu, ref)
            worst = max(worst, e)
            assert e < TOL, (r, i, e)
            k1, k2, _ = enc.stream_info(handles[i])
            assert (k1, k2) == (sts[i].att.shape[3] // 2, sts[i].att.shape[3])
    fin_lens = [int(x) for x in torch.randint(1, 29, (12,))]
    wins = [torch.randint(0, cfg.vocab, (n,)) for n in fin_lens]
    got = enc.encode(handles, wins, [True] * 12)
    for i, (w, mu) in enumerate(zip(wins, got)):
        ref = eo.encode_window(flow, sts[i], w, True)
        e = rel(mu, ref)
        worst = max(worst, e)
        assert mu.shape == ref.shape and e < TOL
    print(f"ragged batches: worst window rel-L2 {worst:.2e}")
    enc.check()


def test_encoder_rejects_bad_calls():
    flow, enc = build(ENCODER_TINY, max_frames=256, n_slots1=512, n_slots2=1024, n_streams=2)
    h = enc.new_stream(40)
    with pytest.raises(L.T2WError):  # a kept window needs 2 frames
        enc.encode([h], [[1, 2, 3, 4]], [False])
    with pytest.raises(L.T2WError):  # token out of range
        enc.encode([h], [[1, 2, 3, 4, ENCODER_TINY.vocab]], [False])
    with pytest.raises(L.T2WError):  # the same stream twice
        enc.encode([h, h], [[1] * 8, [1] * 8], [False, False])
    with pytest.raises(L.T2WError):  # more upsampled frames than max_frames
        enc.encode([h], [[1] * 200], [False])
    h2 = enc.new_stream(40)
    with pytest.raises(L.T2WError):  # stream handles exhausted
        enc.new_stream(40)
    enc.release(h2)
    with pytest.raises(L.T2WError):  # released handle
        enc.encode([h2], [[1] * 8], [False])
    enc.encode([h], [[1] * 8], [False])  # still usable
    enc.check()


def test_encoder_graph_replay_equals_eager():
    """Steady windows through CUDA-graph replay (one graph per launch structure, captured on its second sight) give
    the eager calls' mu bit for bit; finals and calls of other structures fall back to eager calls."""
    torch.manual_seed(3)
    flow = eo.build_flow(ENCODER_TINY, seed=0)
    kw = dict(max_frames=512, n_slots1=2048, n_slots2=4096, n_streams=8)
    eager = B200FlowEncoder.from_flow(flow, device="cuda", **kw)
    graph = B200FlowEncoder.from_flow(flow, device="cuda", use_graphs=True, **kw)
    prompts = [torch.randint(0, ENCODER_TINY.vocab, (n,)) for n in (30, 45, 52, 61)]
    he, _ = eager.setup(prompts)
    hg, _ = graph.setup(prompts)
    out_e = torch.empty(4 * 50, ENCODER_TINY.mel, device="cuda")
    out_g = torch.empty_like(out_e)
    for r in range(8):
        wins = [torch.randint(0, ENCODER_TINY.vocab, (28,)) for _ in range(4)]
        eager.encode_packed(he, wins, [False] * 4, out=out_e)
        graph.encode_packed(hg, wins, [False] * 4, out=out_g)
        torch.cuda.synchronize()
        assert torch.equal(out_e, out_g), r
    fins = [torch.randint(0, ENCODER_TINY.vocab, (n,)) for n in (5, 9, 13, 20)]
    a = eager.encode(he, fins, [True] * 4)
    b = graph.encode(hg, fins, [True] * 4)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    c = graph.counts
    print("graph encoder calls:", c)
    assert c["replays"] >= 3 and c["captures"] >= 1
    graph.check()


def test_encode_op_equals_ctypes():
    """``torch.ops.b200t2w.encode`` (what ``B200FlowEncoder`` calls) against the same C-ABI call made through ctypes,
    on two encoders fed the same prompts and windows: bit for bit."""
    torch.manual_seed(5)
    flow = eo.build_flow(ENCODER_TINY, seed=0)
    kw = dict(max_frames=512, n_slots1=2048, n_slots2=4096, n_streams=4)
    a = B200FlowEncoder.from_flow(flow, device="cuda", **kw)
    b = B200FlowEncoder.from_flow(flow, device="cuda", **kw)
    prompts = [torch.randint(0, ENCODER_TINY.vocab, (n,)) for n in (25, 40)]
    ha, _ = a.setup(prompts)
    hb, _ = b.setup(prompts)
    lib = L.load()
    for r in range(3):
        wins = [torch.randint(0, ENCODER_TINY.vocab, (28,)).tolist() for _ in range(2)]
        out_a = a.encode_packed(ha, wins, [False, False])
        out_b = torch.empty_like(out_a)
        flat = [t for w in wins for t in w]
        batch = L.EncBatch(2, L.i32_array(hb), L.i32_array([28, 28]), (ctypes.c_uint8 * 2)(0, 0), L.i32_array(flat),
                           P(out_b))
        need = lib.t2w_enc_workspace_bytes(b.handle, ctypes.byref(batch))
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        L.call("t2w_encode", b.handle, ctypes.byref(batch), P(ws), ctypes.c_size_t(need), 0, S())
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b), r


def test_stream_clone():
    """A cloned stream (a request's copy of its prompt's encoder caches) encodes the same windows as the stream it was
    copied from, bit for bit, and both advance independently; releasing both returns every slot."""
    torch.manual_seed(8)
    flow, enc = build(ENCODER_TINY, max_frames=512, n_slots1=2048, n_slots2=4096, n_streams=4)
    (h,), _ = enc.setup([torch.randint(0, ENCODER_TINY.vocab, (70,))])
    c = enc.clone(h)
    assert enc.stream_info(c) == enc.stream_info(h)
    for r in range(4):
        w = torch.randint(0, ENCODER_TINY.vocab, (28,))
        a, b = enc.encode([h, c], [w, w], [False, False])
        assert torch.equal(a, b), r
    w2 = torch.randint(0, ENCODER_TINY.vocab, (28,))
    a = enc.encode([h], [w2], [False])[0]
    b = enc.encode([c], [torch.randint(0, ENCODER_TINY.vocab, (28,))], [False])[0]
    assert not torch.equal(a, b)
    enc.release(h)
    enc.release(c)
    assert enc.usage() == (0, 0, 0)
