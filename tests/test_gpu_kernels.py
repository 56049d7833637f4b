"""GPU: each CUDA kernel through the C ABI against a plain fp32 PyTorch statement of the same op on the same
(bf16-rounded) inputs.  Tolerances: fp32 outputs rel-L2 <= 1e-5; bf16 outputs rel-L2 <= 5e-3 (one bf16 rounding);
attention rel-L2 <= 1e-2 (P is rounded to bf16 before the PV product)."""

import ctypes

import pytest
import torch
import torch.nn.functional as F

from b200t2w import lib as L

pytestmark = pytest.mark.gpu


def P(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def S():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


@pytest.fixture(scope="module", autouse=True)
def _dev():
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    L.load()
    assert L.load().t2w_device_ok(torch.cuda.current_device()) == 1
    torch.manual_seed(0)


def gemm(A, W, bias, M, N, K, epi, out=None, ldo=0, taps=1, tap_row0=0, qk=None, qk_eps=1e-5):
    qk_arr = (ctypes.c_void_p * 4)(*[t.data_ptr() for t in qk]) if qk is not None else None
    L.call("t2w_gemm", P(A), A.shape[1], A.shape[0], P(W), P(bias), M, N, K, taps, tap_row0, L.EPI[epi], P(out), ldo,
           qk_arr, ctypes.c_float(qk_eps), S())
    torch.cuda.synchronize()


def rand_bf16(*s, scale=1.0):
    return (torch.randn(*s, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("C,rows", [(512, 300), (128, 77)])
def test_ln_mod(C, rows):
    h = torch.randn(rows, C, device="cuda") * 3 + 1
    sh, sc = torch.randn(C, device="cuda"), 1 + 0.3 * torch.randn(C, device="cuda")
    pad = (torch.rand(rows, device="cuda") < 0.1).to(torch.uint8)
    out = torch.full((rows, C), 7.0, device="cuda").to(torch.bfloat16)
    L.call("t2w_ln_mod", P(h), C, P(sh), P(sc), ctypes.c_float(1e-6), rows, C, P(out), C, P(pad), S())
    torch.cuda.synchronize()
    ref = F.layer_norm(h, (C,), eps=1e-6) * sc + sh
    ref[pad.bool()] = 0
    assert rel(out, ref) < 5e-3
    assert (out[pad.bool()] == 0).all()


@pytest.mark.parametrize("with_y", [True, False])
def test_add_ln_mod(with_y):
    rows, C = 333, 512
    h = torch.randn(rows, C, device="cuda") * 2
    y = rand_bf16(rows, C) if with_y else None
    g = torch.randn(C, device="cuda")
    sh, sc = torch.randn(C, device="cuda"), 1 + 0.3 * torch.randn(C, device="cuda")
    pad = torch.zeros(rows, dtype=torch.uint8, device="cuda")
    pad[5::40] = 1
    out = torch.empty(rows, C, device="cuda", dtype=torch.bfloat16)
    h_ref = h + g * y.float() if with_y else h.clone()
    L.call("t2w_add_ln_mod", P(h), P(y), P(g), P(sh), P(sc), ctypes.c_float(1e-6), rows, C, P(out), P(pad), S())
    torch.cuda.synchronize()
    assert rel(h, h_ref) < 1e-6
    ref = F.layer_norm(h_ref, (C,), eps=1e-6) * sc + sh
    ref[pad.bool()] = 0
    assert rel(out, ref) < 5e-3 and (out[pad.bool()] == 0).all()


def test_ln_mish():
    rows, C = 257, 512
    x = rand_bf16(rows, C, scale=2.0)
    w, b = 1 + 0.1 * torch.randn(C, device="cuda"), 0.1 * torch.randn(C, device="cuda")
    pad = torch.zeros(rows, dtype=torch.uint8, device="cuda")
    pad[::17] = 1
    out = torch.empty(rows, C, device="cuda", dtype=torch.bfloat16)
    L.call("t2w_ln_mish", P(x), P(w), P(b), ctypes.c_float(1e-5), rows, C, P(out), P(pad), S())
    torch.cuda.synchronize()
    ref = F.mish(F.layer_norm(x.float(), (C,), w, b, eps=1e-5))
    ref[pad.bool()] = 0
    assert rel(out, ref) < 5e-3


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (384, 512, 512), (256, 80, 512), (256, 384, 128), (1280, 2048, 192)])
def test_gemm_f32(M, N, K):
    A, W, b = rand_bf16(M, K), rand_bf16(N, K, scale=0.05), torch.randn(N, device="cuda")
    out = torch.zeros(M, N, device="cuda")
    gemm(A, W, b, M, N, K, "f32", out, N)
    ref = A.float() @ W.float().t() + b
    assert rel(out, ref) < 1e-5, rel(out, ref)


@pytest.mark.parametrize("M,N,K", [(384, 2048, 512), (512, 384, 2048)])
def test_gemm_bf16_and_gelu(M, N, K):
    A, W, b = rand_bf16(M, K), rand_bf16(N, K, scale=0.05), torch.randn(N, device="cuda") * 0.1
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    gemm(A, W, b, M, N, K, "bf16", out, N)
    ref = A.float() @ W.float().t() + b
    assert rel(out, ref) < 5e-3
    gemm(A, W, b, M, N, K, "gelu", out, N)
    assert rel(out, F.gelu(ref, approximate="tanh")) < 5e-3


@pytest.mark.parametrize("H", [512, 128])
def test_gemm_qkv_head_norms(H):
    M, N, K = 256, 3 * H, H
    A, W, b = rand_bf16(M, K), rand_bf16(N, K, scale=0.05), torch.randn(N, device="cuda") * 0.1
    qn = [1 + 0.1 * torch.randn(64, device="cuda"), 0.1 * torch.randn(64, device="cuda")]
    kn = [1 + 0.1 * torch.randn(64, device="cuda"), 0.1 * torch.randn(64, device="cuda")]
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    gemm(A, W, b, M, N, K, "qkv", out, N, qk=qn + kn, qk_eps=1e-5)
    y = A.float() @ W.float().t() + b
    q, k, v = y.split(H, dim=1)
    q = F.layer_norm(q.view(M, -1, 64), (64,), qn[0], qn[1], eps=1e-5).view(M, H)
    k = F.layer_norm(k.view(M, -1, 64), (64,), kn[0], kn[1], eps=1e-5).view(M, H)
    ref = torch.cat([q, k, v], dim=1)
    assert rel(out, ref) < 5e-3


def test_gemm_causal_conv_taps():
    """taps = 3, tap_row0 = -2: row m sums A[m - 2 + t] . W_t (rows before 0 read as zero): a kernel-3 causal conv."""
    M, H = 384, 512
    A = rand_bf16(M, H)
    W, b = rand_bf16(H, 3 * H, scale=0.03), torch.randn(H, device="cuda") * 0.1
    out = torch.empty(M, H, device="cuda")
    gemm(A, W, b, M, H, H, "f32", out, H, taps=3, tap_row0=-2)
    Ap = torch.cat([torch.zeros(2, H, device="cuda"), A.float()])
    im2col = torch.cat([Ap[0:M], Ap[1:M + 1], Ap[2:M + 2]], dim=1)
    ref = im2col @ W.float().t() + b
    assert rel(out, ref) < 1e-5
    # the same through Conv1d with weight [out, in, k] laid out tap-major
    w = W.float().view(H, 3, H).permute(0, 2, 1)
    conv = F.conv1d(F.pad(A.float().t()[None], (2, 0)), w, b)[0].t()
    assert rel(out, conv) < 1e-5


@pytest.mark.parametrize("M,N,K,taps,epi", [
    (11264, 512, 320, 1, "f32"),    # the solve's in_proj at config 2: 176 tiles on 148 SMs (a partial second wave)
    (11264, 512, 512, 3, "bf16"),   # causal conv: 24 k blocks per tile
    (11264, 512, 2048, 1, "bf16"),  # fc2
    (2560, 2048, 512, 1, "gelu"),   # 160 tiles
    (6400, 384, 256, 1, "bf16"),    # 128-column tiles: 150 tiles
    (11264, 1536, 512, 1, "qkv"),   # 528 tiles: 3-4 tiles per CTA through both TMEM accumulators
    (45056, 512, 512, 3, "bf16"),   # long K with many rounds: the CTA-pair (cta_group::2) 256 x 256 kernel
    (45184, 512, 2048, 1, "bf16"),  # CTA pairs with M % 256 == 128 (the last pair's second CTA has no rows)
])
def test_gemm_full_size(M, N, K, taps, epi):
    """The solve's GEMM shapes at config-2 size (11264 packed rows) and tile counts that are not a multiple of the SM
    count, checked whole and per 128-row block (a wrong tile shows up as one bad block)."""
    A = rand_bf16(M, K)
    W, b = rand_bf16(N, taps * K, scale=0.03), torch.randn(N, device="cuda") * 0.1
    f32 = epi == "f32"
    out = torch.empty(M, N, device="cuda", dtype=torch.float32 if f32 else torch.bfloat16)
    qk = None
    if epi == "qkv":
        qk = [1 + 0.1 * torch.randn(64, device="cuda"), 0.1 * torch.randn(64, device="cuda"),
              1 + 0.1 * torch.randn(64, device="cuda"), 0.1 * torch.randn(64, device="cuda")]
    outs = []
    for _ in range(2):  # two launches: bitwise identical (no atomics or order-dependent sums)
        out.fill_(float("nan"))
        gemm(A, W, b, M, N, K, epi, out, N, taps=taps, tap_row0=-2 if taps == 3 else 0, qk=qk)
        outs.append(out.clone())
    assert torch.equal(outs[0], outs[1])
    if taps == 3:
        Ap = torch.cat([torch.zeros(2, K, device="cuda"), A.float()])
        ref = torch.cat([Ap[0:M], Ap[1:M + 1], Ap[2:M + 2]], dim=1) @ W.float().t() + b
    else:
        ref = A.float() @ W.float().t() + b
    if epi == "gelu":
        ref = F.gelu(ref, approximate="tanh")
    elif epi == "qkv":
        H = N // 3
        q, k, v = ref.split(H, dim=1)
        q = F.layer_norm(q.reshape(M, -1, 64), (64,), qk[0], qk[1], eps=1e-5).reshape(M, H)
        k = F.layer_norm(k.reshape(M, -1, 64), (64,), qk[2], qk[3], eps=1e-5).reshape(M, H)
        ref = torch.cat([q, k, v], dim=1)
    assert torch.isfinite(out).all()
    e = rel(out, ref)
    assert e < (1e-5 if f32 else 5e-3), e
    blk = (out.float() - ref).view(M // 128, 128, N).norm(dim=(1, 2)) / ref.view(M // 128, 128, N).norm(dim=(1, 2))
    assert float(blk.max()) < (1e-4 if f32 else 1e-2), float(blk.max())


@pytest.mark.parametrize("M,N,K,taps", [
    (384, 512, 512, 1),      # one partial round
    (11264, 512, 512, 1),    # proj at config 2: 176 tiles on 148 SMs
    (11264, 512, 512, 3),    # conv2 (causal taps) at config 2
    (11264, 512, 2048, 1),   # fc2 at config 2
    (512, 384, 256, 1),      # 128-column tiles
    (45184, 512, 2048, 1),   # CTA pairs, M % 256 == 128 (the last pair's second CTA has no rows)
])
def test_gemm_gated_residual(M, N, K, taps):
    """T2W_EPI_RESID: h += gate * (A W^T + bias) in place in fp32 (the solve's proj / conv2 / fc2 epilogue), checked
    whole and per 128-row block, with a row stride wider than N; two launches from the same h are bitwise equal."""
    A = rand_bf16(M, K)
    W, b = rand_bf16(N, taps * K, scale=0.03), torch.randn(N, device="cuda") * 0.1
    gate = torch.randn(N, device="cuda")
    ldo = N + 128
    h0 = torch.randn(M, ldo, device="cuda") * 2
    outs = []
    for _ in range(2):
        h = h0.clone()
        gemm(A, W, b, M, N, K, "resid", h, ldo, taps=taps, tap_row0=-2 if taps == 3 else 0, qk=[gate])
        outs.append(h)
    assert torch.equal(outs[0], outs[1])
    h = outs[0]
    if taps == 3:
        Ap = torch.cat([torch.zeros(2, K, device="cuda"), A.float()])
        y = torch.cat([Ap[0:M], Ap[1:M + 1], Ap[2:M + 2]], dim=1) @ W.float().t() + b
    else:
        y = A.float() @ W.float().t() + b
    ref = h0.clone()
    ref[:, :N] += gate * y
    assert torch.equal(h[:, N:], h0[:, N:])  # columns past N untouched
    e = rel(h[:, :N] - h0[:, :N], ref[:, :N] - h0[:, :N])  # error relative to the update itself
    assert e < 1e-5, e
    d = (h[:, :N] - ref[:, :N]).view(M // 128, 128, N).norm(dim=(1, 2))
    assert float((d / (gate * y).view(M // 128, 128, N).norm(dim=(1, 2))).max()) < 1e-4


def test_gemm_gated_residual_rejects_bad_args():
    A, W, b = rand_bf16(128, 64), rand_bf16(256, 64), torch.zeros(256, device="cuda")
    h = torch.zeros(128, 256, device="cuda")
    qk_arr = None
    rc = L.load().t2w_gemm(P(A), 64, 128, P(W), P(b), 128, 256, 64, 1, 0, L.EPI["resid"], P(h), 256, qk_arr,
                           ctypes.c_float(0.0), S())
    assert rc == -1  # T2W_ERR_INVALID: no gate


def _attn_ref(qkv, seqs, heads):
    H = heads * 64
    out = torch.zeros(qkv.shape[0], H, device="cuda")
    for row, Ls, Ps in seqs:
        x = qkv[row:row + Ls].float()
        q, k, v = (x[:, i * H:(i + 1) * H].view(Ls, heads, 64).transpose(0, 1) for i in range(3))
        lim = torch.where(torch.arange(Ls, device="cuda") < Ps, Ps, Ls)
        mask = torch.arange(Ls, device="cuda")[None, :] < lim[:, None]
        o = F.scaled_dot_product_attention(q[None], k[None], v[None], attn_mask=mask[None, None])[0]
        out[row:row + Ls] = o.transpose(0, 1).reshape(Ls, H)
    return out


@pytest.mark.parametrize("heads", [8, 2])
def test_attention_block_causal_varlen(heads):
    seqs = [(2, 350, 300), (356, 30, 30), (390, 260, 200), (652, 1, 1), (655, 129, 128), (790, 600, 500)]
    rows = 1400
    qkv = rand_bf16(rows, 3 * heads * 64, scale=2.0)
    out = torch.zeros(rows, heads * 64, device="cuda", dtype=torch.bfloat16)
    r, Ls, Ps = zip(*seqs)
    L.call("t2w_attn_varlen", P(qkv), rows, heads, len(seqs), L.i32_array(r), L.i32_array(Ls), L.i32_array(Ps), P(out), S())
    torch.cuda.synchronize()
    ref = _attn_ref(qkv, seqs, heads)
    for row, Ls_, _ in seqs:
        e = rel(out[row:row + Ls_], ref[row:row + Ls_])
        assert e < 1e-2, (row, Ls_, e)
    assert (out[0:2] == 0).all() and (out[386:390] == 0).all()  # rows outside every sequence are untouched


def test_euler_cfg():
    n_tok, mel, half = 300, 80, 400
    x = torch.randn(n_tok, mel, device="cuda")
    dphi = torch.randn(2 * half, mel, device="cuda")
    tok_row = torch.randperm(half, device="cuda")[:n_tok].int()
    hx = torch.zeros(2 * half, 320, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(n_tok, mel, device="cuda")
    x_ref = x.clone()
    L.call("t2w_euler_cfg", P(x), P(dphi), mel, P(tok_row), n_tok, mel, half, ctypes.c_float(0.05), ctypes.c_float(0.7),
           P(hx), 320, P(out), S())
    torch.cuda.synchronize()
    d, u = dphi[tok_row.long()], dphi[tok_row.long() + half]
    ref = x_ref + 0.05 * ((1 + 0.7) * d - 0.7 * u)
    assert rel(x, ref) < 1e-6 and torch.equal(out, x)
    assert torch.equal(hx[tok_row.long(), :mel], x.to(torch.bfloat16))
    assert torch.equal(hx[tok_row.long() + half, :mel], x.to(torch.bfloat16))
