"""GPU: the slot-pool attention of the steady-state solve (``t2w_test_attn_gathered``), single and paired form, against
a plain fp32 softmax attention over the same bf16 values.

The single form puts one (window, head) item in each 128-query tile; the paired form puts two items block-diagonally
into one tile (each with up to 64 queries and 32 of its keys per 64-key tile).  Cases: the steady windows' shapes (50
queries against 400 keys), full 64-query windows, one-query windows, key counts that are not multiples of 32 or 64,
items of one pair with different key counts, an odd head count (pairs that straddle two windows and a last pair with
one item), scores large enough to raise the running maximum.  Tolerance: rel-L2 <= 1e-2 per item (P is rounded to
bf16 before P V, as in the reference's FlashInfer fp16 path); rows outside every item's queries stay untouched."""

import ctypes

import pytest
import torch

from b200t2w import lib as L

pytestmark = pytest.mark.gpu
TOL = 1e-2
SENTINEL = 7.0


@pytest.fixture(scope="module", autouse=True)
def _dev():
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    assert L.load().t2w_device_ok(torch.cuda.current_device()) == 1


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def make_case(windows, heads, seed, n_slots=1024, q_scale=1.0):
    """windows: [(T, L)]; rows laid out as the slot solve does (two rows before each window)."""
    g = torch.Generator().manual_seed(seed)
    H = heads * 64
    work, idx, row = [], [], 0
    for T, Lk in windows:
        row += 2
        work.append((row, len(idx), 0, T, Lk))
        idx.extend(torch.randint(0, n_slots, (Lk,), generator=g).tolist())
        row += T
    rows = row + 2
    qkv = (torch.randn(rows, 3 * H, generator=g) * q_scale).to(torch.bfloat16).cuda()
    pool = torch.randn(n_slots, 2 * H, generator=g).to(torch.bfloat16).cuda()
    return qkv, pool, work, idx


def reference(qkv, pool, work, idx, heads):
    H = heads * 64
    out = {}
    for i, (q_row, k_row, q_pos, P, Lk) in enumerate(work):
        sel = torch.tensor(idx[k_row:k_row + Lk], device="cuda")
        for h in range(heads):
            q = qkv[q_row:q_row + P - q_pos, h * 64:(h + 1) * 64].float()
            k = pool[sel, h * 64:(h + 1) * 64].float()
            v = pool[sel, H + h * 64:H + (h + 1) * 64].float()
            out[(i, h)] = torch.softmax(q @ k.t() / 8.0, dim=-1) @ v
    return out


def run(qkv, pool, work, idx, heads, pair):
    rows = qkv.shape[0]
    out = torch.full((rows, heads * 64), SENTINEL, dtype=torch.bfloat16, device="cuda")
    flat = [x for w in work for x in w]
    w_arr = (ctypes.c_int32 * len(flat))(*flat)
    i_arr = (ctypes.c_int32 * len(idx))(*idx)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = L.load().t2w_test_attn_gathered(qkv.data_ptr(), rows, heads, len(work), w_arr, pool.data_ptr(), pool.shape[0],
                                         pool.shape[1], i_arr, len(idx), int(pair), out.data_ptr(), err.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream)
    return rc, out, int(err.item())


CASES = {
    "steady_windows": ([(50, 400)] * 6, 8, 1.0),
    "ragged": ([(50, 400), (64, 64), (1, 1), (33, 97), (17, 350), (64, 129), (2, 31)], 8, 1.0),
    "odd_heads": ([(50, 400), (40, 333), (64, 65)], 3, 1.0),
    "large_scores": ([(50, 400), (30, 250), (64, 200)], 8, 4.0),
}


@pytest.mark.parametrize("name", list(CASES))
def test_gathered_single_and_paired_vs_fp32(name):
    windows, heads, q_scale = CASES[name]
    qkv, pool, work, idx = make_case(windows, heads, seed=11 + list(CASES).index(name), q_scale=q_scale)
    ref = reference(qkv, pool, work, idx, heads)
    outs = {}
    for pair in (False, True):
        rc, out, err = run(qkv, pool, work, idx, heads, pair)
        assert rc == 0 and err == 0, (pair, rc, err)
        covered = torch.zeros(qkv.shape[0], dtype=torch.bool)
        worst = 0.0
        for (i, h), r in ref.items():
            q_row, _, q_pos, P, _ = work[i]
            got = out[q_row:q_row + P - q_pos, h * 64:(h + 1) * 64]
            worst = max(worst, rel(got, r))
            covered[q_row:q_row + P - q_pos] = True
        print(f"{name} pair={pair}: worst item rel-L2 {worst:.2e}")
        assert worst <= TOL
        assert bool((out[~covered.cuda()] == SENTINEL).all()), "rows outside the items' queries were written"
        outs[pair] = out
    assert rel(outs[True], outs[False]) <= TOL


def test_paired_rejects_windows_past_64_queries():
    qkv, pool, work, idx = make_case([(50, 100), (65, 100)], 8, seed=3)
    rc, out, _ = run(qkv, pool, work, idx, 8, True)
    assert rc != 0
    assert bool((out == SENTINEL).all())
    rc, _, err = run(qkv, pool, work, idx, 8, False)  # the single form takes it
    assert rc == 0 and err == 0
