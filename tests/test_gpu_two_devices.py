"""GPU, two devices in one process: a solver per GPU (what a process driving several GPUs from threads does).  The
kernels' launch attributes (the dynamic shared-memory limit of each kernel) are per device, so the second GPU's first
launches must set them too.  Both solvers run the same streams: their outputs are equal bit for bit (the same kernels
on the same inputs) and within the bf16 tolerance of the oracle.  Skipped with fewer than two GPUs."""

import pytest
import torch

from b200t2w.config import TINY
from b200t2w.solver import B200Solver, state_dict_from_module
from b200t2w.workload import Workload, make_streams
from oracle import dit_oracle

pytestmark = pytest.mark.gpu
TOL_BF16 = 1e-2


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_solvers_on_two_devices_in_one_process():
    model = dit_oracle.build_model(TINY, seed=0)
    sd = state_dict_from_module(model)
    streams = make_streams(Workload("two_devices", 5, ((48, 16), (20, 9), (130, 40))), TINY.mel)
    outs = []
    for d in (0, 1):
        s = B200Solver(TINY, sd, device=f"cuda:{d}")
        for graph in (False, True):
            o = s.solve_streams(streams, graph=graph)
            s.check()
            assert all(x.device == torch.device("cuda", d) for x in o)
            outs.append([x.cpu() for x in o])
        s.close()
    for o in outs[1:]:
        assert all(torch.equal(a, b) for a, b in zip(outs[0], o))
    for st, o in zip(streams, outs[0]):
        ref = dit_oracle.solve_packed(model, st["x0"], st["mu"], st["cond"], st["spk"], st["P"], st["T"])
        e = float((o - ref).norm() / ref.norm())
        assert e < TOL_BF16, e
