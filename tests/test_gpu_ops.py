"""GPU: the torch custom ops (``torch.ops.b200t2w.*``) against the ctypes binding of the same C ABI, bit for bit.

Both routes end in the same ``t2w_*`` call, so the results must be identical: the whole packed solve, the
attention, a GEMM epilogue and the row kernels, each on the same inputs through both."""

import ctypes

import pytest
import torch

from b200t2w import lib as L
from b200t2w import ops as O
from b200t2w.config import TINY
from b200t2w.solver import B200Solver, Layout, state_dict_from_module
from b200t2w.workload import Workload, make_streams
from oracle import dit_oracle

pytestmark = pytest.mark.gpu


def P(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def S():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.fixture(scope="module")
def ns():
    assert torch.cuda.is_available()
    return O.load()


def test_solve_packed_op_equals_ctypes(ns):
    m = dit_oracle.build_model(TINY, seed=0)
    s = B200Solver(TINY, state_dict_from_module(m))
    streams = make_streams(Workload("ops", 3, ((30, 10), (12, 7))), TINY.mel)
    lay = Layout(tuple(x["P"] for x in streams), tuple(x["T"] for x in streams))
    b = s.static_buffers(lay)
    for k in ("x0", "mu", "cond"):
        b[k].copy_(torch.cat([x[k].t() for x in streams]))
    b["spk"].copy_(torch.stack([x["spk"] for x in streams]))
    out_op = torch.zeros_like(b["out"])
    ns.solve_packed(s._hid, list(lay.prompt), list(lay.chunk), b["x0"], b["mu"], b["cond"], b["spk"], out_op, b["ws"],
                    False)
    out_c = torch.zeros_like(b["out"])
    batch = L.Batch(lay.n_streams, L.i32_array(lay.prompt), L.i32_array(lay.chunk), b["x0"].data_ptr(),
                    b["mu"].data_ptr(), b["cond"].data_ptr(), b["spk"].data_ptr(), out_c.data_ptr())
    L.call("t2w_solve_packed", s._h, ctypes.byref(batch), P(b["ws"]), ctypes.c_size_t(b["ws"].numel()),
           ctypes.c_uint32(0), S())
    torch.cuda.synchronize()
    s.check()
    assert torch.equal(out_op, out_c)
    assert out_op.abs().sum() > 0
    s.close()


def test_kernel_ops_equal_ctypes(ns):
    g = torch.Generator(device="cuda").manual_seed(3)
    rows, C, heads = 384, 128, 2
    # attention
    qkv = torch.randn(rows, 3 * C, device="cuda", generator=g).to(torch.bfloat16)
    seqs = ([2, 200], [180, 150], [120, 150])
    a_op = torch.zeros(rows, C, device="cuda", dtype=torch.bfloat16)
    a_c = torch.zeros_like(a_op)
    ns.attn_varlen(qkv, heads, seqs[0], seqs[1], seqs[2], a_op)
    L.call("t2w_attn_varlen", P(qkv), rows, heads, 2, L.i32_array(seqs[0]), L.i32_array(seqs[1]),
           L.i32_array(seqs[2]), P(a_c), S())
    # GEMM with the GELU epilogue
    A = torch.randn(rows, C, device="cuda", generator=g).to(torch.bfloat16)
    W = torch.randn(256, C, device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(256, device="cuda", generator=g)
    g_op = torch.zeros(rows, 256, device="cuda", dtype=torch.bfloat16)
    g_c = torch.zeros_like(g_op)
    ns.gemm(A, W, bias, rows, 256, C, 1, 0, L.EPI["gelu"], g_op, 256, [], 0.0)
    L.call("t2w_gemm", P(A), C, rows, P(W), P(bias), rows, 256, C, 1, 0, L.EPI["gelu"], P(g_c), 256, None,
           ctypes.c_float(0.0), S())
    # add + LN + modulate (h updated in place: each route gets its own copy)
    h0 = torch.randn(rows, C, device="cuda", generator=g)
    y = torch.randn(rows, C, device="cuda", generator=g).to(torch.bfloat16)
    gate, sh, sc = (torch.randn(C, device="cuda", generator=g) for _ in range(3))
    h_op, h_c = h0.clone(), h0.clone()
    n_op = torch.zeros(rows, C, device="cuda", dtype=torch.bfloat16)
    n_c = torch.zeros_like(n_op)
    ns.add_ln_mod(h_op, y, gate, sh, sc, 1e-6, n_op, None)
    L.call("t2w_add_ln_mod", P(h_c), P(y), P(gate), P(sh), P(sc), ctypes.c_float(1e-6), rows, C, P(n_c), None, S())
    # LN (affine) + Mish
    w, bb = torch.randn(C, device="cuda", generator=g), torch.randn(C, device="cuda", generator=g)
    m_op = torch.zeros(rows, C, device="cuda", dtype=torch.bfloat16)
    m_c = torch.zeros_like(m_op)
    ns.ln_mish(y, w, bb, 1e-5, m_op, None)
    L.call("t2w_ln_mish", P(y), P(w), P(bb), ctypes.c_float(1e-5), rows, C, P(m_c), None, S())
    torch.cuda.synchronize()
    for a, b in ((a_op, a_c), (g_op, g_c), (h_op, h_c), (n_op, n_c), (m_op, m_c)):
        assert torch.equal(a, b)
        assert a.float().abs().sum() > 0


def test_op_failure_is_a_t2w_error(ns):
    m = dit_oracle.build_model(TINY, seed=0)
    s = B200Solver(TINY, state_dict_from_module(m))
    z = torch.zeros(8, TINY.mel, device="cuda")
    with pytest.raises(L.T2WError) as e:
        O.call("solve_packed", s._hid, [5], [3], z, z, z, torch.zeros(1, TINY.mel, device="cuda"), z,
               torch.empty(256, dtype=torch.uint8, device="cuda"), False)
    assert e.value.status == -6
    s.close()
