"""GPU: a bounded wait that runs out.

Every device wait of the library gives up after a limit, records T2W_ERR_TIMEOUT in the solver's error word and lets
its kernel return, so a lost arrival never hangs the GPU.  ``t2w_test_wait_timeout`` launches the row kernel in its
early-start mode on scratch rows whose block counter nothing publishes, with a 1 ms limit: the kernel must end on its
own, ``t2w_check`` must report the timeout once (and clear it), and the next solve on the same solver must be
unchanged (bit for bit against the solve before the timeout, within the bf16 tolerance of the oracle)."""

import ctypes
import time

import pytest
import torch

from b200t2w import lib as L
from b200t2w.config import TINY
from b200t2w.solver import B200Solver, state_dict_from_module
from b200t2w.workload import Workload, make_streams
from oracle import dit_oracle

pytestmark = pytest.mark.gpu


def test_wait_runs_out_and_the_solver_recovers():
    m = dit_oracle.build_model(TINY, seed=0)
    s = B200Solver(TINY, state_dict_from_module(m))
    streams = make_streams(Workload("timeout", 4, ((40, 12), (9, 5))), TINY.mel)
    before = [o.clone() for o in s.solve_streams(streams)]
    s.check()
    lib = L.load()
    t0 = time.perf_counter()
    L.call("t2w_test_wait_timeout", s._h, ctypes.c_int64(1_000_000),
           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 1.0, elapsed  # 1 ms limit per warp: the kernel returned on its own
    assert lib.t2w_check(s._h) == -4  # T2W_ERR_TIMEOUT, reported once
    assert lib.t2w_check(s._h) == 0  # and cleared
    after = s.solve_streams(streams)
    s.check()
    for st, a, b in zip(streams, before, after):
        assert torch.equal(a, b)
        ref = dit_oracle.solve_packed(m, st["x0"], st["mu"], st["cond"], st["spk"], st["P"], st["T"])
        assert float((b.cpu() - ref).norm() / ref.norm()) < 1e-2
    s.close()


def test_wait_limit_outside_its_range_is_refused():
    m = dit_oracle.build_model(TINY, seed=0)
    s = B200Solver(TINY, state_dict_from_module(m))
    lib = L.load()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.t2w_test_wait_timeout(s._h, ctypes.c_int64(10), st) == -1
    assert lib.t2w_test_wait_timeout(s._h, ctypes.c_int64(10 ** 10), st) == -1
    assert lib.t2w_check(s._h) == 0
    s.close()
