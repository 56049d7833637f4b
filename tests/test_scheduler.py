"""CPU: per-GPU stream placement / sharding / EDF order, and the multi-rank sharded solve as ``bench.py --gpus N`` runs
it (world_size 2, gloo, each rank solving its shard with the oracle; no data-path collective, only gathering results
for the check and the max of the timed region)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from b200t2w.config import TINY
from b200t2w.scheduler import GpuPlacement, edf_windows, shard_streams
from b200t2w.workload import C3, Workload, make_streams


def test_placement_is_sticky_and_least_loaded():
    p = GpuPlacement(3)
    assert [p.open(s, 100) for s in "abc"] == [0, 1, 2]
    assert p.open("a", 999) == 0  # sticky: already placed
    p.add("b", 500)
    assert p.open("d", 10) == 0  # devices 0 and 2 tie at 100; lowest index
    p.done("b", 600)
    assert p.load[1] == 0 and p.open("e", 1) == 1
    p.close("a")
    assert "a" not in p.where
    with pytest.raises(ValueError):
        GpuPlacement(0)


@pytest.mark.parametrize("n_gpus", [1, 2, 4, 8])
def test_shards_cover_every_stream_once_and_balance(n_gpus):
    lengths = list(C3.lengths)
    parts = shard_streams(lengths, n_gpus)
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(len(lengths)))
    loads = [sum(lengths[i][0] + lengths[i][1] for i in p) for p in parts]
    biggest = max(p + t for p, t in lengths)
    assert max(loads) - min(loads) <= biggest  # greedy longest-first bound
    cont = shard_streams([(300, 50)] * 1024, n_gpus, contiguous=True)
    assert [len(p) for p in cont] == [1024 // n_gpus] * n_gpus and cont[0][0] == 0


def test_edf_order_and_row_cap():
    ready = [(3.0, "c"), (1.0, "a"), (2.0, "b"), (0.5, "z")]
    assert edf_windows(ready) == ["z", "a", "b", "c"]
    assert edf_windows(ready, max_rows=2) == ["z", "a"]


def _rank(rank: int, world: int, port: int, q) -> None:
    from oracle import dit_oracle

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    wl = Workload("shard", 9, ((6, 3), (4, 5), (7, 2), (3, 3)))
    parts = shard_streams(list(wl.lengths), world, contiguous=True)
    model = dit_oracle.build_model(TINY, seed=0)
    mine = {}
    for i in parts[rank]:
        s = make_streams(wl, TINY.mel, first=i, count=1)[0]
        mine[i] = dit_oracle.solve_packed(model, s["x0"], s["mu"], s["cond"], s["spk"], s["P"], s["T"])
    t = torch.tensor([float(10 + rank)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    if rank == 0:
        q.put((float(t), {k: v for d in gathered for k, v in d.items()}))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sharded_solve_matches_single_process():
    from oracle import dit_oracle

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    tmax, results = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert tmax == 11.0
    wl = Workload("shard", 9, ((6, 3), (4, 5), (7, 2), (3, 3)))
    model = dit_oracle.build_model(TINY, seed=0)
    assert sorted(results) == [0, 1, 2, 3]
    for s in make_streams(wl, TINY.mel):
        ref = dit_oracle.solve_packed(model, s["x0"], s["mu"], s["cond"], s["spk"], s["P"], s["T"])
        assert torch.equal(results[s["index"]], ref)
