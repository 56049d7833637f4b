"""GPU: the FP8 (e4m3, power-of-two block scales) path through the C ABI.

Quantisers are checked byte-exactly against the torch statement of the format in ``e4m3_ref``; the block-scaled GEMM
against an fp32 matmul of the dequantised operands (its only errors are fp32 summation order and the output rounding:
rel-L2 <= 5e-3 for bf16 outputs); the producers that quantise their own outputs against their fp32 statement within
e4m3's rounding (rel-L2 <= 4e-2); and the whole FP8 solve against the fp32 oracle within the north star's 3e-2.
"""

import ctypes

import pytest
import torch
import torch.nn.functional as F

import e4m3_ref as Q
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
    assert L.load().t2w_device_ok(torch.cuda.current_device()) == 1
    torch.manual_seed(0)


def sf_bytes(rows, C):
    return int(L.load().t2w_e4m3_sf_bytes(rows, C))


def quant_rows(x_bf16, n_layouts=1):
    rows, C = x_bf16.shape
    lb = sf_bytes(rows + 128, C)
    q = torch.empty(rows, C, dtype=torch.uint8, device="cuda")
    sf = torch.full((n_layouts * lb,), 127, dtype=torch.uint8, device="cuda")
    L.call("t2w_quant_e4m3", P(x_bf16), rows, C, P(q), P(sf), n_layouts, lb, S())
    torch.cuda.synchronize()
    return q, sf, lb


def test_quant_rows_bytes_exact():
    rows, C = 300, 512
    x = torch.randn(rows, C, device="cuda") * torch.logspace(-6, 3, rows, device="cuda")[:, None]
    x[7] = 0                    # all-zero row: scale byte 127, zero values
    x[11, :32] = 448.0          # exactly the e4m3 maximum at scale 1
    x[12, :32] = 1.75 * 2 ** 9  # mantissa 1.75: still inside the smaller power of two
    x[13, :32] = 900.0          # 0.8789 * 2^10: the next power of two
    xb = x.to(torch.bfloat16)
    q, sf, lb = quant_rows(xb, n_layouts=3)
    qr, er = Q.quant_blocks(xb.float(), 32)
    assert torch.equal(q, qr.view(torch.uint8))
    for d in range(3):
        assert torch.equal(Q.bytes_from_atoms(sf[d * lb:(d + 1) * lb], rows, C, shift=d), er), d
    assert int(er[7].unique().item()) == 127 and int(er[11, 0]) == 127 and int(er[12, 0]) == 128 and int(er[13, 0]) == 129


def test_quant_weight_bytes_exact():
    N, Kt = 768, 1536
    w = torch.randn(N, Kt, device="cuda") * torch.logspace(-3, 1, N, device="cuda")[:, None]
    q = torch.empty(N, Kt, dtype=torch.uint8, device="cuda")
    sf = torch.empty(N * Kt // 32, dtype=torch.uint8, device="cuda")
    L.call("t2w_quant_weight_e4m3", P(w), N, Kt, P(q), P(sf), S())
    torch.cuda.synchronize()
    qr, atoms, _ = Q.quant_weight(w)
    assert torch.equal(q, qr.view(torch.uint8))
    assert torch.equal(sf, atoms)


def _weights(N, Kt, scale=0.05):
    w = torch.randn(N, Kt, device="cuda") * scale
    w *= torch.exp(torch.randn(N, Kt // 128, device="cuda")).repeat_interleave(128, dim=1)  # varied block scales
    q, atoms, e32 = Q.quant_weight(w)
    return q, atoms, Q.dequant(q, e32, 32)


def gemm8(A8, lda, rows_a, sfa, layouts, lb, W8, sfw, bias, M, N, K, taps, tap_row0, epi, out, ldo, out_sf=None, qk=None):
    qk_arr = (ctypes.c_void_p * 4)(*[t.data_ptr() for t in qk]) if qk is not None else None
    L.call("t2w_gemm_e4m3", P(A8), lda, rows_a, P(sfa), layouts, lb, P(W8), P(sfw), P(bias), M, N, K, taps, tap_row0,
           L.EPI[epi], P(out), ldo, P(out_sf), qk_arr, ctypes.c_float(1e-5), S())
    torch.cuda.synchronize()


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (1280, 512, 512), (11264, 512, 2048), (384, 1536, 512)])
def test_gemm_e4m3_bf16_out(M, N, K):
    x = (torch.randn(M, K, device="cuda") * torch.exp(torch.randn(M, 1, device="cuda"))).to(torch.bfloat16)
    A8, sfa, lb = quant_rows(x)
    W8, sfw, Wd = _weights(N, K)
    bias = torch.randn(N, device="cuda") * 0.1
    out = torch.full((M, N), float("nan"), device="cuda").to(torch.bfloat16)
    gemm8(A8, K, M, sfa, 1, lb, W8, sfw, bias, M, N, K, 1, 0, "bf16", out, N)
    Ad = Q.dequant(A8.view(torch.float8_e4m3fn), Q.bytes_from_atoms(sfa[:lb], M, K), 32)
    ref = Ad @ Wd.t() + bias
    assert torch.isfinite(out.float()).all()
    assert rel(out, ref) < 5e-3, rel(out, ref)
    blk = (out.float() - ref).view(M // 128, 128, N).norm(dim=(1, 2)) / ref.view(M // 128, 128, N).norm(dim=(1, 2))
    assert float(blk.max()) < 1e-2


def test_gemm_e4m3_causal_conv_taps():
    """taps = 3, tap_row0 = -2 over row-shifted scale layouts 0, 1, 2 (rows before 0 read as zero)."""
    M, H = 640, 512
    x = (torch.randn(M, H, device="cuda") * torch.exp(torch.randn(M, 1, device="cuda"))).to(torch.bfloat16)
    A8, sfa, lb = quant_rows(x, n_layouts=3)
    W8, sfw, Wd = _weights(H, 3 * H, scale=0.03)
    bias = torch.randn(H, device="cuda") * 0.1
    out = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    gemm8(A8, H, M, sfa, 3, lb, W8, sfw, bias, M, H, H, 3, -2, "bf16", out, H)
    Ad = Q.dequant(A8.view(torch.float8_e4m3fn), Q.bytes_from_atoms(sfa[:lb], M, H), 32)
    Ap = torch.cat([torch.zeros(2, H, device="cuda"), Ad])
    ref = torch.cat([Ap[0:M], Ap[1:M + 1], Ap[2:M + 2]], dim=1) @ Wd.t() + bias
    assert rel(out, ref) < 5e-3, rel(out, ref)


def test_gemm_e4m3_qkv_and_gelu_epilogues():
    M, H = 512, 512
    x = torch.randn(M, H, device="cuda").to(torch.bfloat16)
    A8, sfa, lb = quant_rows(x)
    Ad = Q.dequant(A8.view(torch.float8_e4m3fn), Q.bytes_from_atoms(sfa[:lb], M, H), 32)
    # QKV with per-head q / k LayerNorm
    W8, sfw, Wd = _weights(3 * H, H)
    b = torch.randn(3 * H, device="cuda") * 0.1
    qk = [1 + 0.1 * torch.randn(64, device="cuda"), 0.1 * torch.randn(64, device="cuda"),
          1 + 0.1 * torch.randn(64, device="cuda"), 0.1 * torch.randn(64, device="cuda")]
    out = torch.empty(M, 3 * H, device="cuda", dtype=torch.bfloat16)
    gemm8(A8, H, M, sfa, 1, lb, W8, sfw, b, M, 3 * H, H, 1, 0, "qkv", out, 3 * H, qk=qk)
    y = Ad @ Wd.t() + b
    q, k, v = y.split(H, dim=1)
    q = F.layer_norm(q.reshape(M, -1, 64), (64,), qk[0], qk[1], eps=1e-5).reshape(M, H)
    k = F.layer_norm(k.reshape(M, -1, 64), (64,), qk[2], qk[3], eps=1e-5).reshape(M, H)
    assert rel(out, torch.cat([q, k, v], dim=1)) < 5e-3
    # fc1 with GELU, e4m3 output and its scale atoms (fc2's operand)
    Fd = 2048
    W8, sfw, Wd = _weights(Fd, H)
    b = torch.randn(Fd, device="cuda") * 0.1
    f8 = torch.empty(M, Fd, dtype=torch.uint8, device="cuda")
    sff = torch.full((sf_bytes(M + 128, Fd),), 127, dtype=torch.uint8, device="cuda")
    gemm8(A8, H, M, sfa, 1, lb, W8, sfw, b, M, Fd, H, 1, 0, "gelu_fp8", f8, Fd, out_sf=sff)
    ref = F.gelu(Ad @ Wd.t() + b, approximate="tanh")
    e = Q.bytes_from_atoms(sff, M, Fd)
    deq = Q.dequant(f8.view(torch.float8_e4m3fn), e, 32)
    assert rel(deq, ref) < 4e-2, rel(deq, ref)
    # each block's scale is the rule's scale for the block's own maximum (fp32 rounding may move a borderline block)
    er = Q.ue8m0(ref.view(M, Fd // 32, 32).abs().amax(dim=2))
    assert float((e - er).abs().float().mean()) < 0.02 and int((e - er).abs().max()) <= 1


def test_add_ln_mod_and_ln_mish_e4m3():
    rows, C = 333, 512
    h = torch.randn(rows, C, device="cuda") * 2
    y = torch.randn(rows, C, device="cuda").to(torch.bfloat16)
    g, sh, sc = torch.randn(C, device="cuda"), torch.randn(C, device="cuda"), 1 + 0.3 * torch.randn(C, device="cuda")
    pad = torch.zeros(rows, dtype=torch.uint8, device="cuda")
    pad[5::40] = 1
    lb = sf_bytes(rows + 128, C)
    out = torch.empty(rows, C, dtype=torch.uint8, device="cuda")
    sf = torch.full((3 * lb,), 127, dtype=torch.uint8, device="cuda")
    h_ref = h + g * y.float()
    L.call("t2w_add_ln_mod_e4m3", P(h), P(y), P(g), P(sh), P(sc), ctypes.c_float(1e-6), rows, C, P(out), P(sf), 3, lb,
           P(pad), S())
    torch.cuda.synchronize()
    assert rel(h, h_ref) < 1e-6
    ref = F.layer_norm(h_ref, (C,), eps=1e-6) * sc + sh
    ref[pad.bool()] = 0
    for d in range(3):
        e = Q.bytes_from_atoms(sf[d * lb:(d + 1) * lb], rows, C, shift=d)
        deq = Q.dequant(out.view(torch.float8_e4m3fn), e, 32)
        assert rel(deq, ref) < 4e-2, (d, rel(deq, ref))
    assert (out[pad.bool()] == 0).all()
    # LN(affine) + Mish
    x = (torch.randn(rows, C, device="cuda") * 2).to(torch.bfloat16)
    w, b = 1 + 0.1 * torch.randn(C, device="cuda"), 0.1 * torch.randn(C, device="cuda")
    sf.fill_(127)
    L.call("t2w_ln_mish_e4m3", P(x), P(w), P(b), ctypes.c_float(1e-5), rows, C, P(out), P(sf), 3, lb, P(pad), S())
    torch.cuda.synchronize()
    ref = F.mish(F.layer_norm(x.float(), (C,), w, b, eps=1e-5))
    ref[pad.bool()] = 0
    deq = Q.dequant(out.view(torch.float8_e4m3fn), Q.bytes_from_atoms(sf[:lb], rows, C), 32)
    assert rel(deq, ref) < 4e-2


def test_attention_e4m3_output():
    heads = 8
    seqs = [(2, 350, 300), (356, 30, 30), (390, 260, 200), (655, 129, 128)]
    rows = 896
    qkv = (torch.randn(rows, 3 * heads * 64, device="cuda") * 2).to(torch.bfloat16)
    ref_out = torch.zeros(rows, heads * 64, device="cuda", dtype=torch.bfloat16)
    r, Ls, Ps = zip(*seqs)
    args = (P(qkv), rows, heads, len(seqs), L.i32_array(r), L.i32_array(Ls), L.i32_array(Ps))
    L.call("t2w_attn_varlen", *args, P(ref_out), S())
    o8 = torch.zeros(rows, heads * 64, dtype=torch.uint8, device="cuda")
    sf = torch.full((sf_bytes(rows + 128, heads * 64),), 127, dtype=torch.uint8, device="cuda")
    L.call("t2w_attn_varlen_e4m3", *args, P(o8), P(sf), S())
    torch.cuda.synchronize()
    deq = Q.dequant(o8.view(torch.float8_e4m3fn), Q.bytes_from_atoms(sf, rows, heads * 64), 32)
    for row, Ls_, _ in seqs:
        e = rel(deq[row:row + Ls_], ref_out[row:row + Ls_])
        assert e < 4e-2, (row, e)
