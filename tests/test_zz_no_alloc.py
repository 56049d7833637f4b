"""GPU: the allocation-free attention entry point (t2w_attn_varlen_noalloc) against the regular one.

Callers that cannot allocate device memory when they call in (a runtime that reserves the whole GPU for its own pool,
or a plugin running where the CUDA allocator must not be called) use the variant whose per-call work list lives in a
fixed device array of the library.  Two calls in a row, each on its own inputs and sequence layout, must match the
regular entry point within the attention tolerance of the kernel tests (rel-L2 <= 1e-2; the same kernel runs, so they
agree exactly in practice).  This file is collected last and passes alone in a fresh process as well."""

import ctypes

import pytest
import torch

from b200t2w import lib as L

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _attn(fn, qkv, rows, heads, seqs, out):
    r, Ls, Ps = zip(*seqs)
    L.call(fn, _ptr(qkv), rows, heads, len(seqs), L.i32_array(r), L.i32_array(Ls), L.i32_array(Ps), _ptr(out),
           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


@pytest.fixture(scope="module", autouse=True)
def _dev():
    assert torch.cuda.is_available()
    assert L.load().t2w_device_ok(torch.cuda.current_device()) == 1


def test_noalloc_matches_regular_entry_point_on_two_calls():
    g = torch.Generator(device="cuda").manual_seed(11)
    cases = [(8, [(2, 350, 300), (356, 30, 30), (390, 260, 200)], 700),
             (2, [(0, 129, 128), (130, 1, 1), (140, 600, 450)], 760)]
    for heads, seqs, rows in cases:
        qkv = (torch.randn(rows, 3 * heads * 64, device="cuda", generator=g) * 2).to(torch.bfloat16)
        ref = torch.zeros(rows, heads * 64, device="cuda", dtype=torch.bfloat16)
        got = torch.zeros_like(ref)
        _attn("t2w_attn_varlen", qkv, rows, heads, seqs, ref)
        _attn("t2w_attn_varlen_noalloc", qkv, rows, heads, seqs, got)
        torch.cuda.synchronize()
        for row, n, _ in seqs:
            assert _rel(got[row:row + n], ref[row:row + n]) <= TOL
        assert torch.equal(got, ref)


def test_noalloc_rejects_more_tiles_than_its_array():
    rows, heads = 128 * 8193, 1
    seqs = [(i * 128, 128, 128) for i in range(8193)]  # one more 128-query tile than the fixed array holds
    qkv = torch.zeros(1, device="cuda")  # never read: the size check comes first
    with pytest.raises(L.T2WError) as e:
        r, Ls, Ps = zip(*seqs)
        L.call("t2w_attn_varlen_noalloc", _ptr(qkv), rows, heads, len(seqs), L.i32_array(r), L.i32_array(Ls),
               L.i32_array(Ps), _ptr(qkv), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert e.value.status == -1


def test_noalloc_refuses_a_capturing_stream():
    """The work list is copied from host memory that lives only for the call, so a stream under capture is refused
    with T2W_ERR_INVALID; nothing is enqueued and the capture stays valid."""
    rows, heads = 256, 2
    qkv = torch.zeros(rows, 3 * heads * 64, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(rows, heads * 64, device="cuda", dtype=torch.bfloat16)
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        graph.capture_begin()
        try:
            rc = L.load().t2w_attn_varlen_noalloc(_ptr(qkv), rows, heads, 1, L.i32_array([0]), L.i32_array([200]),
                                                  L.i32_array([150]), _ptr(out), ctypes.c_void_p(side.cuda_stream))
            out.add_(0)  # the capture is still usable after the refusal
        finally:
            graph.capture_end()
    assert rc == -1
    graph.replay()
    torch.cuda.synchronize()
