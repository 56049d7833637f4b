"""Generate the golden fixtures that pin the flow-encoder oracle (``oracle/encoder_oracle.py``) to the reference's own
encoder driver code.

Run in a container that has the reference checkout (read-only; never needed at test time)::

    python tests/golden/make_encoder_golden.py --reference /path/to/reference

What it does, per fixture (a few streams with different prompt lengths):

1. Builds the restated flow encoder (``encoder_oracle.build_flow``) and a reference ``BatchedToken2Wav`` around it
   (``flow`` only; no fast DiT, no graphs, per-stream cache I/O).
2. Prompt setups with the reference's ``_setup_encoder_batched`` (``engine/runtime/token2wav_batch.py:566-616``: one
   right-padded batch of every prompt plus 3 silence tokens, conv caches gathered at each prompt's real end, attention
   caches cut to its length) and ``flow.encoder_proj``.
3. Windows with the reference's ``_encoder`` (``:402-445``: caches left-padded to the call's longest, key masks, the
   padded ``_encoder_core``, the new caches split back per stream), ``flow.encoder_proj``, and ``_flow_finish``'s trim of
   the attention cache (``:395``, the reference's ``_trim`` with the prompt's mel frames as ``keep``).  The calls mix
   streams of different cache lengths, run long enough for the trim to cut, and end with a final window
   (``last=True``: 3 zero look-ahead frames) and a merged call where one stream's final window rides in a steady call
   (``valid``: its frames after its tokens are padding, ``:363-371``).
4. Checks the oracle's unpadded per-stream restatement (``encode_prompt`` / ``encode_window``) against every output
   (fp32, CPU) and writes ``tests/golden/encoder_*.pt``: the tokens, the reference driver's mu per call and stream, and
   the weights' digest (weights are rebuilt from the seed).
"""

from __future__ import annotations

import argparse
import dataclasses
import hashlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "minicpm-o-4.5-single-gpu-engine_b200"))

from b200t2w.config import ENCODER, ENCODER_TINY  # noqa: E402
from oracle import encoder_oracle as eo  # noqa: E402

CHUNK, LOOK = 25, 3  # engine/token2wav_chunker.py:20-21


def digest(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()[:32]


def weights_digest(flow) -> str:
    sd = eo.state_dict_np(flow)
    return digest(*[torch.from_numpy(sd[k]) for k in sorted(sd)])


def rel(a, b) -> float:
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


class _St:
    """The parts of ``StreamState`` the encoder driver reads."""

    def __init__(self, cnn, att, keep, cfg):
        self.flow_cache = {"conformer_cnn_cache": cnn, "conformer_att_cache": att}
        self.prompt = type("P", (), {"mels": torch.zeros(1, keep, cfg.mel)})()


def plan_calls(n_streams: int, gen: torch.Generator) -> list:
    """Calls of (stream indices, window token counts, final flags, call last flag): steady windows of CHUNK + LOOK
    tokens over subsets of the streams, then finals."""
    calls = []
    for r in range(4):  # 4 steady rounds: enough for 2 * 25 frames per window to pass the keep + 100 trim
        idx = [i for i in range(n_streams) if (r + i) % 3 != 2 or r == 0]
        calls.append((idx, [CHUNK + LOOK] * len(idx), [False] * len(idx), False))
    # a merged call: stream 0's final window (17 tokens) rides with the others' steady windows
    calls.append((list(range(n_streams)), [17] + [CHUNK + LOOK] * (n_streams - 1), [True] + [False] * (n_streams - 1), False))
    # a final call of the other streams (last=True: 3 zero look-ahead frames, 20 tokens each)
    calls.append((list(range(1, n_streams)), [20] * (n_streams - 1), [True] * (n_streams - 1), True))
    return calls


def make(cfg, prompt_lens: list, name: str, seed: int) -> None:
    from engine.runtime import token2wav_batch as tb

    flow = eo.build_flow(cfg, seed=0)
    gen = torch.Generator().manual_seed(seed)
    bt = tb.BatchedToken2Wav.__new__(tb.BatchedToken2Wav)
    bt.flow = flow
    bt.fast = None
    bt.enc_graphs = None
    bt.encoder_batched_io = False
    bt.profile = bt.trace = None
    rec = {"config": dataclasses.asdict(cfg), "weights_digest": weights_digest(flow),
           "prompts": [], "calls": []}
    prompts = [torch.randint(0, cfg.vocab, (1, n), generator=gen) for n in prompt_lens]
    with torch.inference_mode():
        feats = [(p, None, torch.zeros(1, cfg.spk_dim), torch.zeros(1, 2 * p.shape[1], cfg.mel), None) for p in prompts]
        encs = bt._setup_encoder_batched(feats)
        sts_ref, sts_or = [], []
        for p, (h, cnn, att) in zip(prompts, encs):
            mu_ref = h[0].t().contiguous()
            mu_or, st = eo.encode_prompt(flow, p[0])
            e = rel(mu_or, mu_ref)
            print(f"{name} prompt n={p.shape[1]}: oracle vs reference setup rel-L2 {e:.2e}")
            assert e < 1e-5 and rel(st.att, att) < 1e-5 and rel(st.cnn, cnn) < 1e-5, e
            sts_ref.append(_St(cnn.clone(), att.clone(), st.keep, cfg))
            sts_or.append(st)
            rec["prompts"].append({"tokens": p[0].clone(), "mu": mu_ref.clone()})
        for idx, ntok, fins, last in plan_calls(len(prompts), gen):
            L = max(ntok)
            wins = [torch.randint(0, cfg.vocab, (n,), generator=gen) for n in ntok]
            tok = torch.stack([torch.cat([w, w.new_zeros(L - len(w))]) for w in wins])
            merged = any(fins) and not last
            vl = ntok if merged else None
            valid = torch.tensor(ntok) if merged else None
            sts = [sts_ref[i] for i in idx]
            xs = bt._encoder(sts, flow.input_embedding(tok), last, valid, vl)
            h = flow.encoder_proj(xs)
            out = []
            for j, i in enumerate(idx):
                T = 2 * ntok[j] if (merged and fins[j]) else h.shape[1]
                mu_ref = h[j, :T].t().contiguous()
                c = sts[j].flow_cache
                c["conformer_att_cache"] = tb._trim(c["conformer_att_cache"], sts[j].prompt.mels.shape[1], 3)
                mu_or = eo.encode_window(flow, sts_or[i], wins[j], last or fins[j])[:, :T] if not (merged and fins[j]) else \
                    _oracle_final_in_merged(flow, sts_or[i], wins[j])
                e = rel(mu_or, mu_ref)
                assert e < 1e-5, (name, idx, j, e)
                if not (merged and fins[j]):  # a final window's caches are never read again (garbage in a merged call)
                    ea = rel(sts_or[i].att, c["conformer_att_cache"])
                    assert sts_or[i].att.shape == c["conformer_att_cache"].shape and ea < 1e-5, (ea, sts_or[i].att.shape)
                out.append({"stream": i, "tokens": wins[j].clone(), "final": bool(fins[j]), "mu": mu_ref.clone()})
            print(f"{name} call streams={idx} tokens={ntok} last={last} merged={merged}: oracle matches (max cache "
                  f"{max(sts_ref[i].flow_cache['conformer_att_cache'].shape[3] for i in idx)} frames)")
            rec["calls"].append({"last": bool(last), "merged": bool(merged), "windows": out})
    torch.save(rec, os.path.join(HERE, f"{name}.pt"))


def _oracle_final_in_merged(flow, st, tokens) -> torch.Tensor:
    """A final window merged into a steady call equals the same window run alone as a final (``last=True``)."""
    import copy

    return eo.encode_window(flow, copy.deepcopy(st), tokens, True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    torch.set_num_threads(min(16, os.cpu_count() or 1))
    make(ENCODER_TINY, [20, 33, 47], "encoder_tiny", seed=5)
    make(ENCODER, [50, 61], "encoder_reference", seed=6)


if __name__ == "__main__":
    main()
