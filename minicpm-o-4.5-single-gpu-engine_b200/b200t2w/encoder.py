"""Host side of the B200 flow encoder (speech tokens -> mu), through the C ABI of ``libt2w_b200.so``.

The reference runs the flow module's encoder per decode call from ``BatchedToken2Wav._flow_encode`` / ``_encoder``
(``engine/runtime/token2wav_batch.py:365-478``) with the caches in each stream's ``flow_cache`` (tensors it left-pads
per call), and prompt setups through ``_setup_encoder_batched`` (``:566-616``).  ``B200FlowEncoder`` keeps the caches
in the library (a stream is a handle; keys live in per-layer pools), so a call passes only the windows' tokens:

* ``setup(prompts)``: each prompt (plus the look-ahead silence tokens) through a new stream with empty caches, trim
  length = its mu frames (``_setup_encoder_one``, ``:556-564``); returns the streams and their mu ``[mel, 2 n]``.
* ``encode(handles, windows, finals)``: one window per stream (``_flow_encode``'s ``mu`` entries ``[mel, 2 T]``); the
  caches advance and are trimmed as ``_flow_finish`` trims them (``:388-399``).

Calls go through the torch custom ops ``torch.ops.b200t2w.enc_workspace_bytes`` / ``encode`` on the current torch
stream; the encoder object and its streams through the ctypes binding.  All arithmetic runs in the CUDA library; a
missing library or a non-sm_100 device raises.
"""

from __future__ import annotations

import ctypes
from dataclasses import replace

import torch

from . import lib as L
from . import ops as O
from .config import ENCODER, EncoderConfig

SILENCE_TOKEN = 4218  # engine/models/token2wav.py:39: the look-ahead tokens that close a prompt


def flow_state_dict(flow) -> dict:
    """fp32 weights of a flow module (``input_embedding``, ``encoder``, ``encoder_proj``), keyed by state-dict path."""
    return {k: v.detach().float() for k, v in flow.state_dict().items()}


def encoder_config_from_flow(flow, base: EncoderConfig = ENCODER) -> EncoderConfig:
    """The ``EncoderConfig`` of a loaded flow module, read off the attributes the reference's encoder driver reads
    (``token2wav_batch.py:408-418``: ``len(enc.encoders)``, ``len(enc.up_encoders)``, ``enc.up_layer.stride``,
    ``enc.pre_lookahead_layer.pre_lookahead_len``) and the layers' shapes and LayerNorm eps.  The leaky-ReLU slope and
    the sinusoid's max period are not module attributes and come from ``base``."""
    enc = flow.encoder
    a = enc.encoders[0].self_attn
    return replace(
        base, vocab=int(flow.input_embedding.num_embeddings), hidden=int(flow.input_embedding.embedding_dim),
        heads=int(a.h), head_dim=int(a.d_k), ffn=int(enc.encoders[0].feed_forward.w_1.out_features),
        blocks1=len(enc.encoders), blocks2=len(enc.up_encoders), stride=int(enc.up_layer.stride),
        lookahead=int(enc.pre_lookahead_layer.pre_lookahead_len), mel=int(flow.encoder_proj.out_features),
        spk_dim=int(flow.spk_embed_affine_layer.in_features), eps_layer=float(enc.encoders[0].norm_mha.eps),
        eps_embed=float(enc.embed.out[1].eps), eps_after=float(enc.after_norm.eps))


class B200FlowEncoder:
    """The flow encoder's chunk forward on one sm_100 GPU.

    ``weights``: fp32 state dict of the flow module (``flow_state_dict``).  ``max_frames`` bounds a window's upsampled
    frames and every attention's keys; ``n_slots1`` / ``n_slots2`` are the key slots of each first- / second-stack
    layer's pool (a steady stream holds about (keep + 100) / 2 and keep + 100 of them), ``n_streams`` the live streams.
    """

    def __init__(self, cfg: EncoderConfig, weights: dict, device="cuda", max_frames: int = 2048,
                 n_slots1: int = 1 << 16, n_slots2: int = 1 << 17, n_streams: int = 1024, use_graphs: bool = False):
        cfg.validate_for_kernels()
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("B200FlowEncoder needs a CUDA device (no CPU fallback)")
        self.lib = L.load()
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", idx)
        if not self.lib.t2w_device_ok(idx):
            raise RuntimeError(f"cuda:{idx} is not an sm_100 GPU: the B200 kernels cannot run there")
        names = list(L.E_GLOBAL)
        for l in range(cfg.blocks1 + cfg.blocks2):
            p = f"encoder.encoders.{l}." if l < cfg.blocks1 else f"encoder.up_encoders.{l - cfg.blocks1}."
            names += [p + n for n in L.E_LAYER]
        missing = [n for n in names if n not in weights]
        if missing:
            raise KeyError(f"flow weights lack {missing[:4]}{'...' if len(missing) > 4 else ''}")
        with torch.cuda.device(self.device):
            self._w = [weights[n].detach().to(self.device, torch.float32).contiguous() for n in names]
            ptrs = (ctypes.c_void_p * len(self._w))(*[t.data_ptr() for t in self._w])
            c = L.EncConfig(cfg.vocab, cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn, cfg.blocks1, cfg.blocks2,
                            cfg.stride, cfg.lookahead, cfg.mel, cfg.eps_layer, cfg.eps_embed, cfg.eps_after,
                            cfg.leaky_slope, cfg.max_period)
            h = ctypes.c_void_p()
            L.call("t2w_encoder_create", ctypes.byref(c), ptrs, len(self._w), max_frames, n_slots1, n_slots2,
                   n_streams, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(h))
        self._w = None  # the library holds its own copies
        self.handle = h
        self.max_frames = max_frames
        self.use_graphs = use_graphs
        self._ws = None

    @classmethod
    def from_flow(cls, flow, device="cuda", **kw) -> "B200FlowEncoder":
        """Built from a loaded flow module (config read off its attributes, weights from its state dict)."""
        return cls(encoder_config_from_flow(flow), flow_state_dict(flow), device=device, **kw)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.t2w_encoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- streams
    def new_stream(self, keep: int) -> int:
        """A stream with empty caches (a prompt setup's state) whose attention caches trim to ``keep`` + 100 frames."""
        h = ctypes.c_int32()
        with torch.cuda.device(self.device):
            L.call("t2w_enc_stream_new", self.handle, int(keep),
                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(h))
        return h.value

    def clone(self, handle: int) -> int:
        """A new stream with a copy of ``handle``'s caches (a request's stream from a prompt it does not adopt)."""
        h = ctypes.c_int32()
        with torch.cuda.device(self.device):
            L.call("t2w_enc_stream_clone", self.handle, int(handle),
                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(h))
        return h.value

    def release(self, handle: int) -> None:
        L.call("t2w_enc_stream_release", self.handle, int(handle))

    def stream_info(self, handle: int) -> tuple:
        """(first-stack keys, second-stack keys, keep) of a stream."""
        k1, k2, keep = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        L.call("t2w_enc_stream_get", self.handle, int(handle), ctypes.byref(k1), ctypes.byref(k2), ctypes.byref(keep))
        return k1.value, k2.value, keep.value

    def usage(self) -> tuple:
        """(first-stack slots in use, second-stack slots in use, live streams)."""
        a, b, c = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        L.call("t2w_enc_usage", self.handle, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    # ---- calls
    def frames(self, n_tokens: int, final: bool) -> int:
        return n_tokens if final else n_tokens - self.cfg.lookahead

    def encode_packed(self, handles, windows, finals, out: torch.Tensor | None = None) -> torch.Tensor:
        """One window per stream; returns mu token-major ``[sum stride * T_i, mel]`` fp32 on the device (windows in
        order): the layout ``t2w_solve_cached`` takes.  ``windows``: token lists or int tensors (look-ahead tokens
        included unless final)."""
        toks = [w.tolist() if isinstance(w, torch.Tensor) else list(w) for w in windows]
        n = len(toks)
        if n == 0 or len(handles) != n or len(finals) != n:
            raise ValueError("one handle, window and final flag per stream")
        flat = [int(t) for w in toks for t in w]
        n_out = sum(self.cfg.stride * self.frames(len(w), bool(f)) for w, f in zip(toks, finals))
        if out is None:
            out = torch.empty(n_out, self.cfg.mel, dtype=torch.float32, device=self.device)
        elif out.shape != (n_out, self.cfg.mel) or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous fp32 [{n_out}, {self.cfg.mel}] tensor")
        h = int(self.handle.value)
        hs = [int(x) for x in handles]
        nt = [len(w) for w in toks]
        fin = [1 if f else 0 for f in finals]
        with torch.cuda.device(self.device):
            need = O.call("enc_workspace_bytes", h, hs, nt, fin, flat)
            if need == 0:
                raise L.T2WError("t2w_enc_workspace_bytes", -1)
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty(need + need // 4, dtype=torch.uint8, device=self.device)
            O.call("encode", h, hs, nt, fin, flat, out, self._ws, bool(self.use_graphs))
        return out

    def encode(self, handles, windows, finals) -> list:
        """``encode_packed`` split per stream as the reference's ``_flow_encode`` returns mu: ``[mel, stride T_i]``."""
        flat = self.encode_packed(handles, windows, finals)
        out, o = [], 0
        for w, f in zip(windows, finals):
            n = self.cfg.stride * self.frames(len(w), bool(f))
            out.append(flat[o:o + n].t())
            o += n
        return out

    def setup(self, prompts) -> tuple:
        """Prompt setups: each prompt's tokens plus ``lookahead`` silence tokens through a new stream with empty caches
        (trim length = its mu frames, stride * its tokens).  Returns (handles, mu per prompt ``[mel, stride n]``)."""
        handles = []
        try:
            for p in prompts:
                handles.append(self.new_stream(self.cfg.stride * len(p)))
            wins = [(p.tolist() if isinstance(p, torch.Tensor) else list(p)) + [SILENCE_TOKEN] * self.cfg.lookahead
                    for p in prompts]
            mus = self.encode(handles, wins, [False] * len(wins))
        except Exception:
            for h in handles:
                self.release(h)
            raise
        return handles, mus

    @property
    def counts(self) -> dict:
        """Calls so far: graph replays, graph captures, eager calls."""
        r, c, e = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        L.call("t2w_enc_counts", self.handle, ctypes.byref(r), ctypes.byref(c), ctypes.byref(e))
        return {"replays": r.value, "captures": c.value, "eager": e.value}

    def check(self) -> None:
        L.check("t2w_enc_check", self.lib.t2w_enc_check(self.handle))
