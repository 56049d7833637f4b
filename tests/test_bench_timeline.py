"""CPU: bench.py's per-position timeline of a solve (names kernels by their place in a DiT block and attributes the
solve's span to the kernels that extend it), on a hand-made event list shaped like one block."""

import importlib.util
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_for_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    try:
        sys.argv = ["bench.py"]
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


def g(bn, epi):
    return f"void t2w::(anonymous namespace)::k_gemm<{bn}, {epi}, true>(CUtensorMap_st, CUtensorMap_st, DevArgs)"


def test_timeline_names_and_exposed_span():
    b = load_bench()
    row = "void t2w::(anonymous namespace)::k_add_ln_mod<4, false>(float*, ...)"
    mish = "void t2w::(anonymous namespace)::k_ln_mish<4, false>(...)"
    attn = "void t2w::(anonymous namespace)::k_attn<false, false>(...)"
    # one block: qkv, attn, proj, aln, conv1, ln_mish, conv2, aln, fc1, fc2, aln (overlapping starts)
    seq = [(g(256, 4), 0, 20), (attn, 15, 45), (g(256, 1), 40, 60), (row, 55, 70), (g(256, 1), 69, 95),
           (mish, 90, 99), (g(256, 1), 98, 125), (row, 120, 130), (g(256, 2), 129, 155), (g(256, 1), 154, 185),
           (row, 180, 190)]
    t = b.timeline_from_events(seq)
    assert t["kernels"] == 11
    assert abs(t["solve_ms"] - 0.190) < 1e-9
    assert abs(sum(t["exposed_ms"].values()) - t["solve_ms"]) < 1e-6
    assert set(t["exposed_ms"]) == {"qkv", "attn", "proj", "add_ln_mod after proj", "conv1", "ln_mish after conv1",
                                    "conv2", "add_ln_mod after conv2", "fc1", "fc2", "add_ln_mod after fc2"}
    assert abs(t["exposed_ms"]["attn"] - 0.025) < 1e-9  # ends 25 us after QKV
    assert abs(t["kernel_ms"]["proj"] - 0.020) < 1e-9
    assert b.timeline_from_events([]) == {}
    # the CTA-pair and FP8 GEMMs carry only their epilogue as a template argument
    pair = "void t2w::(anonymous namespace)::k_gemm_pair<1>(CUtensorMap_st, CUtensorMap_st, CUtensorMap_st, DevArgs)"
    fp8 = "void t2w::(anonymous namespace)::k_gemm8<2>(...)"
    t = b.timeline_from_events([(attn, 0, 10), (pair, 5, 20), (fp8, 19, 30)])
    assert set(t["kernel_ms"]) == {"attn", "proj", "fc1"}


def test_timeline_slot_solve_scatter_kernels():
    """The slot-pool solve puts k_kv_scatter after QKV and k_conv_cache after the norms before each conv: the GEMMs
    after them keep their block positions (conv2 after ln_mish, not conv1)."""
    b = load_bench()
    row = "void t2w::(anonymous namespace)::k_add_ln_mod<4, false>(float*, ...)"
    mish = "void t2w::(anonymous namespace)::k_ln_mish<4, false>(...)"
    attn = "void t2w::(anonymous namespace)::k_attn<false, true>(...)"
    scat = "void t2w::(anonymous namespace)::k_kv_scatter(...)"
    cc = "void t2w::(anonymous namespace)::k_conv_cache(...)"
    seq = [(g(256, 4), 0, 10), (scat, 10, 11), (attn, 11, 20), (g(256, 3), 20, 30), (row, 29, 32), (cc, 32, 33),
           (g(256, 1), 33, 40), (mish, 39, 42), (cc, 42, 43), (g(256, 1), 43, 50)]
    t = b.timeline_from_events(seq)
    assert set(t["kernel_ms"]) == {"qkv", "kv_scatter", "attn", "proj", "add_ln_mod after proj", "conv_cache",
                                   "conv1", "ln_mish after conv1", "conv2"}


def test_c5_ranks_partition_the_1024_streams_through_the_scheduler():
    """bench.py's default job: config 5's 1024 streams split by the product's scheduler, contiguous and equal per rank,
    every stream on exactly one rank at N = 1, 2, 4, 8 (strong scaling)."""
    for world in (1, 2, 4, 8):
        bench = load_bench()
        parts = [bench.rank_streams("c5", r, world)[1] for r in range(world)]
        assert sorted(i for p in parts for i in p) == list(range(1024))
        assert all(len(p) == 1024 // world for p in parts)
        assert all(p == list(range(p[0], p[0] + len(p))) for p in parts)
