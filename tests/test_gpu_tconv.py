"""GPU: the vocoder's tensor-core convolution (``t2w_test_tconv``) against a plain fp64 convolution.

Every epilogue (bias, Snake, residual update with the next Snake, ELU), the transposed-convolution phase form (output row
row_mul m + row_add), every column tile (32, 64, 128, 256), padding rows, taps past either end of A, and the split form
(3xTF32: hi / lo operand pairs of TF32 values) in and out.  Tolerances: TF32 operands rel-L2 <= 3e-3 (10-bit
mantissas); the split form rel-L2 <= 2e-5 (fp32-level: the lo x lo term and the pairs' rounding, about 3 x 2^-24 per
product, are all it loses)."""

import ctypes

import pytest
import torch

from b200t2w import lib as L

pytestmark = pytest.mark.gpu
BIAS, SNAKE, RESID, ELU = 0, 1, 2, 3


@pytest.fixture(scope="module", autouse=True)
def _dev():
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    assert L.load().t2w_device_ok(torch.cuda.current_device()) == 1


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def tf32_rn(x):
    """Nearest TF32 value: half of the dropped unit added to the bit pattern, then the 13 low mantissa bits cleared."""
    return ((x.contiguous().view(torch.int32) + 0x1000) & -8192).view(torch.float32)


def split_rows(a):
    """[rows, C] -> [rows, 2 C] = [hi | lo], both TF32 values."""
    h = tf32_rn(a)
    return torch.cat([h, tf32_rn(a - h)], dim=1).contiguous()


def split_weight(w, taps, cin):
    """[N, taps Cin] -> [N, taps 3 Cin] = per tap [W_hi | W_lo | W_hi]."""
    w3 = w.view(w.shape[0], taps, cin)
    h = tf32_rn(w3)
    return torch.cat([h, tf32_rn(w3 - h), h], dim=2).reshape(w.shape[0], taps * 3 * cin).contiguous()


def conv_ref(a, w, bias, M, taps, tap_row0, dil):
    """fp64: y[m, n] = bias[n] + sum_t sum_c a[m + tap_row0 + t dil, c] w[n, t Cin + c] (rows outside a read as 0)."""
    rows, cin = a.shape
    idx = torch.arange(M, device=a.device)[:, None] + tap_row0 + dil * torch.arange(taps, device=a.device)[None, :]
    ok = (idx >= 0) & (idx < rows)
    g = a.double()[idx.clamp(0, rows - 1)] * ok[..., None]  # [M, taps, Cin]
    return torch.einsum("mtc,ntc->mn", g, w.double().view(w.shape[0], taps, cin)) + bias.double()


def snake(x, a, inv):
    return x + inv * torch.sin(x * a) ** 2


def run(A, lda, rows_a, W, bias, M, N, Cin, taps, tap_row0, dil, out, ldo, pad, epi=BIAS, row_mul=1, row_add=0,
        alpha=None, inv=None, out2=None, split_in=0, split_out=0, resid_in=None):
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    args = L.TConvArgs(ptr(A), lda, rows_a, ptr(W), ptr(bias), M, N, Cin, taps, tap_row0, dil, ptr(out), ldo, row_mul,
                       row_add, ptr(pad), epi, ptr(alpha), ptr(inv), ptr(out2), split_in, split_out, ptr(err),
                       ptr(resid_in))
    L.call("t2w_test_tconv", ctypes.byref(args), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def case(M, N, Cin, taps, dil, seed, pad_frac=0.1, rows_extra=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rows_a = M + rows_extra
    a = torch.randn(rows_a, Cin, device="cuda", generator=g)
    w = torch.randn(N, taps * Cin, device="cuda", generator=g) / (taps * Cin) ** 0.5
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    pad = (torch.rand(M, device="cuda", generator=g) < pad_frac).to(torch.uint8)
    return a, w, b, pad


@pytest.mark.parametrize("N", [32, 64, 128, 256])
@pytest.mark.parametrize("split", [False, True], ids=["tf32", "split"])
def test_bias_epilogue_tiles_and_taps(N, split):
    """Bias epilogue over every column tile (256 needs enough 128 x 256 tiles for every SM: M = 19200), taps reaching
    past both ends of A (tap_row0 < 0, rows_a = M), dilation 3."""
    M = 19200 if N == 256 else 2048
    Cin, taps, dil, r0 = 64, 5, 3, -6
    a, w, b, pad = case(M, N, Cin, taps, dil, seed=N + split)
    out = torch.full((M, N), 7.0, device="cuda")
    A, W = (split_rows(a), split_weight(w, taps, Cin)) if split else (a, w)
    run(A, A.shape[1], M, W, b, M, N, Cin, taps, r0, dil, out, N, pad, split_in=int(split))
    ref = conv_ref(a, w, b, M, taps, r0, dil)
    ref[pad.bool()] = 0
    e = rel(out, ref)
    print(f"N={N} split={split}: rel-L2 {e:.2e}")
    assert e < (2e-5 if split else 3e-3)
    assert torch.all(out[pad.bool()] == 0)


def test_snake_epilogue_transposed_phase():
    """Snake epilogue writing every 3rd row from row 1 (a transposed conv's output phase) of a 3 M-row layout; the rows
    of the other phases stay untouched."""
    M, N, Cin, taps = 1024, 128, 96, 3
    a, w, b, _ = case(M, N, Cin, taps, 1, seed=11)
    g = torch.Generator(device="cuda").manual_seed(12)
    pad3 = (torch.rand(3 * M, device="cuda", generator=g) < 0.1).to(torch.uint8)
    alpha = torch.rand(N, device="cuda", generator=g) + 0.5
    inv = 1.0 / (alpha + 1e-9)
    out = torch.full((3 * M, N), 5.0, device="cuda")
    run(a, Cin, M, w, b, M, N, Cin, taps, -1, 1, out, N, pad3, epi=SNAKE, row_mul=3, row_add=1, alpha=alpha, inv=inv)
    ref = snake(conv_ref(a, w, b, M, taps, -1, 1), alpha.double(), inv.double())
    ref[pad3[1::3].bool()] = 0
    e = rel(out[1::3], ref)
    print(f"snake, phase 1 of 3: rel-L2 {e:.2e}")
    assert e < 3e-3
    assert torch.all(out[0::3] == 5.0) and torch.all(out[2::3] == 5.0)


@pytest.mark.parametrize("oop", [False, True], ids=["in_place", "out_of_place"])
@pytest.mark.parametrize("N", [64, 128, 256])
def test_residual_epilogue_with_next_snake(N, oop):
    """out += bias + conv and out2 = Snake(out), padding rows of both untouched: conv2 of a ResBlock.  Out of place:
    out = resid_in + bias + conv with resid_in's (zero) padding rows copied (a ResBlock's first update of the stage's
    common input)."""
    M = 19200 if N == 256 else 4096
    Cin, taps, dil = N, 3, 1
    a, w, b, pad = case(M, N, Cin, taps, dil, seed=21 + N)
    g = torch.Generator(device="cuda").manual_seed(22)
    x0 = torch.randn(M, N, device="cuda", generator=g)
    x0[pad.bool()] = 0
    alpha = torch.rand(N, device="cuda", generator=g) + 0.5
    inv = 1.0 / (alpha + 1e-9)
    out = torch.full((M, N), 6.0, device="cuda") if oop else x0.clone()
    out2 = torch.full((M, N), 3.0, device="cuda")
    run(a, Cin, M, w, b, M, N, Cin, taps, -1, dil, out, N, pad, epi=RESID, alpha=alpha, inv=inv, out2=out2,
        resid_in=x0 if oop else None)
    y = x0.double() + conv_ref(a, w, b, M, taps, -1, dil)
    y[pad.bool()] = 0
    s = snake(y, alpha.double(), inv.double())
    s[pad.bool()] = 3.0
    e1, e2 = rel(out, y), rel(out2, s)
    print(f"resid N={N}: out rel-L2 {e1:.2e}, out2 rel-L2 {e2:.2e}")
    assert e1 < 3e-3 and e2 < 3e-3
    assert torch.all(out[pad.bool()] == 0) and torch.all(out2[pad.bool()] == 3.0)


@pytest.mark.parametrize("M,taps,dil", [(2048, 11, 5), (2176, 3, 1), (2048, 11, 7), (2048, 1, 1), (2304, 7, 3)],
                         ids=["two_halves", "one_half_odd_M", "one_half_wide_halo", "per_tap", "two_halves_9x256"])
@pytest.mark.parametrize("N", [64, 128])
def test_tile_forms(M, taps, dil, N):
    """The kernel's tile forms at the vocoder's widths: 256-row tiles of two halves sharing each W box (M a multiple
    of 256, 128 + (taps - 1) dil <= 192), one 128-row half in the tap-reuse form (M not a multiple of 256, or a wider
    halo), one A box per tap (a single tap); residual update with the next Snake, padding rows."""
    Cin = N
    r0 = -((taps - 1) * dil) // 2
    a, w, b, pad = case(M, N, Cin, taps, dil, seed=60 + taps + N)
    g = torch.Generator(device="cuda").manual_seed(61)
    x0 = torch.randn(M, N, device="cuda", generator=g)
    x0[pad.bool()] = 0
    alpha = torch.rand(N, device="cuda", generator=g) + 0.5
    inv = 1.0 / (alpha + 1e-9)
    out = x0.clone()
    out2 = torch.full((M, N), 3.0, device="cuda")
    run(a, Cin, M, w, b, M, N, Cin, taps, r0, dil, out, N, pad, epi=RESID, alpha=alpha, inv=inv, out2=out2)
    y = x0.double() + conv_ref(a, w, b, M, taps, r0, dil)
    y[pad.bool()] = 0
    s = snake(y, alpha.double(), inv.double())
    s[pad.bool()] = 3.0
    e1, e2 = rel(out, y), rel(out2, s)
    print(f"M={M} taps={taps} dil={dil} N={N}: out rel-L2 {e1:.2e}, out2 rel-L2 {e2:.2e}")
    assert e1 < 3e-3 and e2 < 3e-3
    assert torch.all(out[pad.bool()] == 0) and torch.all(out2[pad.bool()] == 3.0)


@pytest.mark.parametrize("split_out", [False, True])
def test_split_elu_layer(split_out):
    """The f0 predictor's middle layer: split-form input, ELU, output plain or as [hi | lo] pairs (hi TF32-exact)."""
    M, N, Cin, taps = 4224, 512, 512, 3
    a, w, b, pad = case(M, N, Cin, taps, 1, seed=31)
    ldo = 2 * N if split_out else N
    out = torch.full((M, ldo), 9.0, device="cuda")
    run(split_rows(a), 2 * Cin, M, split_weight(w, taps, Cin), b, M, N, Cin, taps, -1, 1, out, ldo, pad, epi=ELU,
        split_in=1, split_out=int(split_out))
    ref = torch.nn.functional.elu(conv_ref(a, w, b, M, taps, -1, 1))
    ref[pad.bool()] = 0
    if split_out:
        hi, lo = out[:, :N], out[:, N:]
        assert torch.equal(hi, tf32_rn(hi)) and torch.equal(lo, tf32_rn(lo))
        got = hi.double() + lo.double()
    else:
        got = out
    e = rel(got, ref)
    print(f"split ELU layer, split_out={split_out}: rel-L2 {e:.2e}")
    assert e < 2e-5


def test_rejects_bad_shapes():
    M, N, Cin = 256, 64, 64
    a, w, b, pad = case(M, N, Cin, 1, 1, seed=41)
    out = torch.zeros(M, N, device="cuda")
    lib = L.load()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for kw in ({"M": 200}, {"Cin": 50}, {"N": 96}, {"ldo": 32}, {"row_add": 1}):
        p = dict(M=M, N=N, Cin=Cin, ldo=N, row_add=0)
        p.update(kw)
        args = L.TConvArgs(ctypes.c_void_p(a.data_ptr()), Cin, M, ctypes.c_void_p(w.data_ptr()),
                           ctypes.c_void_p(b.data_ptr()), p["M"], p["N"], p["Cin"], 1, 0, 1,
                           ctypes.c_void_p(out.data_ptr()), p["ldo"], 1, p["row_add"], ctypes.c_void_p(pad.data_ptr()),
                           BIAS, None, None, None, 0, 0, None, None)
        assert lib.t2w_test_tconv(ctypes.byref(args), st) == -1, kw


@pytest.mark.parametrize("cin", [20, 60, 300])
def test_narrow_input_bias_with_next_snake(cin):
    """Inputs whose channel count is not a multiple of 32 (the STFT rows grouped by the source_down strides: 20, 3 x 20,
    15 x 20 floats), W padded per tap to a multiple of 32 columns; bias epilogue with Snake(out) into out2."""
    M, N, taps = 2048, 128, 3
    cp = (cin + 31) // 32 * 32
    a, w, b, pad = case(M, N, cin, taps, 1, seed=50 + cin)
    wp = torch.zeros(N, taps, cp, device="cuda")
    wp[:, :, :cin] = w.view(N, taps, cin)
    g = torch.Generator(device="cuda").manual_seed(51)
    alpha = torch.rand(N, device="cuda", generator=g) + 0.5
    inv = 1.0 / (alpha + 1e-9)
    out = torch.full((M, N), 4.0, device="cuda")
    out2 = torch.full((M, N), 4.0, device="cuda")
    run(a, cin, M, wp.reshape(N, taps * cp).contiguous(), b, M, N, cin, taps, -1, 1, out, N, pad, alpha=alpha, inv=inv,
        out2=out2)
    ref = conv_ref(a, w, b, M, taps, -1, 1)
    ref[pad.bool()] = 0
    s = snake(ref, alpha.double(), inv.double())
    e1, e2 = rel(out, ref), rel(out2, s)
    print(f"Cin={cin}: out rel-L2 {e1:.2e}, out2 rel-L2 {e2:.2e}")
    assert e1 < 3e-3 and e2 < 3e-3
    assert torch.all(out[pad.bool()] == 0) and torch.all(out2[pad.bool()] == 0)
