"""Generate the golden fixtures that pin the CPU oracle (``oracle/dit_oracle.py``) to the reference's own solver code.

Run in a container that has the reference checkout (it is read-only and never needed at test time)::

    python tests/golden/make_golden.py --reference /path/to/reference

What it does, per fixture stream ``(P, T)``:

1. Builds the restated estimator (``oracle.dit_oracle.build_model``) and installs a ``stepaudio2.cosyvoice2.flow.
   decoder_dit`` shim module exposing ``modulate`` (the one symbol the reference driver imports).
2. Runs the reference's two-stage solve with its OWN code, ``engine.runtime.token2wav_batch.BatchedToken2Wav._solve``
   (which calls ``_estimator_temb`` / ``_block_chunk`` / ``_conv_block_chunk``): first the prompt setup (prompt mel as
   condition, empty caches, ``keep_cache=True``), then the chunk against the caches it left (``cond=None``).  The fixed
   noise is read from ``cfm.rand_noise`` at offset 0 for the prompt and at the cache length P for the chunk, exactly as
   the reference does, so ``rand_noise[:, :P + T]`` is the packed stream's x0.
3. Runs the oracle's packed solve ``solve_packed`` over ``[prompt | chunk]`` and asserts both agree (fp32, CPU).
4. Writes ``tests/golden/*.pt``: the reference driver's outputs (prompt and chunk mel), the inputs' and weights'
   digests, and for the tiny config the inputs themselves.

``steady_tiny.pt`` pins the steady-state form: per stream, the prompt setup and then a run of windows through the
reference's ``_solve`` with ``keep_cache`` (and, for a final flush, without), trimming the estimator's key cache after
every kept window with the reference's own ``_trim`` (``token2wav_batch.py:36-39``, as ``_flow_finish`` does with the
prompt's mel frames as ``keep``).  The windows are long enough for the trim to evict keys.  The oracle's
``solve_window`` is checked against it.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import types
from types import SimpleNamespace

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "minicpm-o-4.5-single-gpu-engine_b200"))

from b200t2w.config import REFERENCE, TINY  # noqa: E402
from b200t2w.workload import C1, Workload, make_streams  # noqa: E402
from oracle import dit_oracle  # noqa: E402


def digest(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()[:32]


def weights_digest(model) -> str:
    sd = dit_oracle.state_dict_np(model)
    return digest(*[sd[k] for k in sorted(sd)])


def install_shim() -> None:
    names = ["stepaudio2", "stepaudio2.cosyvoice2", "stepaudio2.cosyvoice2.flow", "stepaudio2.cosyvoice2.flow.decoder_dit"]
    for n in names:
        sys.modules.setdefault(n, types.ModuleType(n))
    sys.modules["stepaudio2.cosyvoice2.flow.decoder_dit"].modulate = dit_oracle.modulate


def reference_two_stage(model, s: dict) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference driver's setup solve then chunk solve; returns (prompt mel [mel, P], chunk mel [mel, T])."""
    from engine.models.token2wav import StreamState
    from engine.runtime.token2wav_batch import BatchedToken2Wav

    cfg = model.estimator.cfg
    P, T = s["P"], s["T"]
    bt = BatchedToken2Wav.__new__(BatchedToken2Wav)
    bt.flow = SimpleNamespace(decoder=model)
    bt.t2w = SimpleNamespace(n_timesteps=cfg.steps)
    bt.graphs = bt.euler = None
    with torch.no_grad():
        model.rand_noise.zero_()
        model.rand_noise[0, :, :P + T] = s["x0"]
    st = StreamState(prompt=None, flow_cache={
        "estimator_cnn_cache": torch.zeros(cfg.steps, cfg.depth, 2, 2 * cfg.hidden, 2),
        "estimator_att_cache": torch.zeros(cfg.steps, cfg.depth, 2, cfg.heads, 0, 2 * cfg.head_dim)}, hift_cache={})
    with torch.inference_mode():
        mel_p = bt._solve([st], s["mu"][None, :, :P].contiguous(), s["spk"][None], cond=s["cond"][None, :, :P].contiguous(),
                          keep_cache=True)
        assert st.flow_cache["estimator_att_cache"].shape[4] == P
        mel_c = bt._solve([st], s["mu"][None, :, P:].contiguous(), s["spk"][None], cond=None, keep_cache=True)
    return mel_p[0], mel_c[0]


def rel(a, b) -> float:
    return float((a - b).norm() / b.norm())


def make(cfg, workload: Workload, name: str, keep_inputs: bool) -> None:
    model = dit_oracle.build_model(cfg, seed=0, noise_frames=max(p + t for p, t in workload.lengths) + 8)
    streams = make_streams(workload, cfg.mel)
    rec = {"config": cfg.to_dict(), "workload": {"name": workload.name, "seed": workload.seed, "lengths": list(workload.lengths)},
           "weights_digest": weights_digest(model), "streams": []}
    for s in streams:
        mel_p, mel_c = reference_two_stage(model, s)
        packed = dit_oracle.solve_packed(model, s["x0"], s["mu"], s["cond"], s["spk"], s["P"], s["T"])
        ep, ec = rel(packed[:, :s["P"]], mel_p), rel(packed[:, s["P"]:], mel_c)
        print(f"{name} stream {s['index']} P={s['P']} T={s['T']}: packed vs reference two-stage rel-L2 prompt {ep:.2e} chunk {ec:.2e}")
        assert ep < 1e-5 and ec < 1e-5, (ep, ec)
        item = {"P": s["P"], "T": s["T"], "index": s["index"], "inputs_digest": digest(s["x0"], s["mu"], s["cond"], s["spk"]),
                "ref_prompt_mel": mel_p.clone(), "ref_chunk_mel": mel_c.clone(), "packed_vs_ref_rel": max(ep, ec)}
        if keep_inputs:
            item.update({k: s[k].clone() for k in ("x0", "mu", "cond", "spk")})
        rec["streams"].append(item)
    torch.save(rec, os.path.join(HERE, f"{name}.pt"))


def reference_windows(model, P: int, windows: list, seed: int) -> dict:
    """One stream through the reference driver: setup over the prompt, then ``windows`` = [(T, keep_cache), ...]."""
    from engine.models.token2wav import StreamState
    from engine.runtime.token2wav_batch import BatchedToken2Wav, _trim

    cfg = model.estimator.cfg
    g = torch.Generator().manual_seed(seed)
    bt = BatchedToken2Wav.__new__(BatchedToken2Wav)
    bt.flow = SimpleNamespace(decoder=model)
    bt.t2w = SimpleNamespace(n_timesteps=cfg.steps)
    bt.graphs = bt.euler = None
    st = StreamState(prompt=None, flow_cache={
        "estimator_cnn_cache": torch.zeros(cfg.steps, cfg.depth, 2, 2 * cfg.hidden, 2),
        "estimator_att_cache": torch.zeros(cfg.steps, cfg.depth, 2, cfg.heads, 0, 2 * cfg.head_dim)}, hift_cache={})
    spk = torch.randn(cfg.mel, generator=g)
    out = {"P": P, "spk": spk, "windows": []}
    for wi, (T, keep) in enumerate([(P, True)] + list(windows)):
        mu = torch.randn(cfg.mel, T, generator=g)
        cond = torch.randn(cfg.mel, T, generator=g) if wi == 0 else None
        o = st.flow_cache["estimator_att_cache"].shape[4]
        x0 = model.rand_noise[0, :, o:o + T].clone()
        with torch.inference_mode():
            mel = bt._solve([st], mu[None].contiguous(), spk[None], cond=None if cond is None else cond[None].contiguous(),
                            keep_cache=keep)[0]
            if keep:
                st.flow_cache["estimator_att_cache"] = _trim(st.flow_cache["estimator_att_cache"], P, 4)
        out["windows"].append({"T": T, "keep": keep, "offset": o, "x0": x0, "mu": mu, "cond": cond, "ref_mel": mel.clone(),
                               "cache_len_after": st.flow_cache["estimator_att_cache"].shape[4]})
    return out


def make_steady() -> None:
    cfg = TINY
    model = dit_oracle.build_model(cfg, seed=0, noise_frames=2048)
    plans = [(20, [(12, True), (30, True), (41, True), (7, True), (25, False)], 11),
             (9, [(5, True), (1, True), (33, True), (40, True), (50, True), (2, False)], 12),
             (64, [(50, True), (50, True), (3, True)], 13)]
    rec = {"config": cfg.to_dict(), "weights_digest": weights_digest(model), "streams": []}
    for P, windows, seed in plans:
        s = reference_windows(model, P, windows, seed)
        cache = dit_oracle.StreamCache(cfg, keep=P)
        for w in s["windows"]:
            mel = dit_oracle.solve_window(model, cache, w["x0"], w["mu"], s["spk"], w["cond"], keep_cache=w["keep"])
            e = rel(mel, w["ref_mel"])
            print(f"steady P={P} T={w['T']} keep={w['keep']} offset={w['offset']} cache after={w['cache_len_after']}: "
                  f"oracle vs reference rel-L2 {e:.2e}")
            assert e < 1e-5 and cache.length == w["cache_len_after"], (e, cache.length)
        rec["streams"].append(s)
    torch.save(rec, os.path.join(HERE, "steady_tiny.pt"))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("T2W_REFERENCE", "/root/reference"))
    ap.add_argument("--skip-full", action="store_true")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    install_shim()
    torch.set_num_threads(os.cpu_count() or 1)
    make(TINY, Workload("tiny_ragged", 7, ((24, 10), (17, 13), (3, 1), (1, 6))), "tiny_ragged", keep_inputs=True)
    make_steady()
    if not a.skip_full:
        make(REFERENCE, C1, "c1_reference", keep_inputs=False)


if __name__ == "__main__":
    main()
