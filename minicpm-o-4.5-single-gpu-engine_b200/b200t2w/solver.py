"""Host side of the B200 Token2Wav flow-matching solve: weights in, mel out, through the C ABI of ``libt2w_b200.so``.

``B200Solver`` plays the role of the reference's ``FastDiT`` (``engine/runtime/dit_fast.py:99-155``): it owns the
weights (cast once), the adaLN modulation tables and the solve's CUDA graphs.  Its packed entry point takes requests
as ``[prompt | chunk]`` streams (see ``b200t2w.workload``) and returns every frame's final mel; ``forward_chunk`` keeps
the reference's ``CausalConditionalCFM.forward_chunk`` argument meaning for one request.  All arithmetic runs in the
CUDA library; a missing library or a non-sm_100 device raises.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import lib as L
from . import ops as O
from .config import DiTConfig, t_schedule
from .staging import HostStaging


def state_dict_from_module(cfm) -> dict:
    """fp32 weights of a ``CausalConditionalCFM``-like module (``cfm.estimator`` with the stepaudio2 DiT attribute
    layout the reference engine reads: ``dit_fast.py:107-145``), keyed ``estimator.<path>``."""
    return {f"estimator.{k}": v.detach().float() for k, v in cfm.estimator.state_dict().items()}


@dataclass
class Layout:
    """The packed layout of one solve call: per-stream prompt / chunk frames."""
    prompt: tuple
    chunk: tuple

    @property
    def n_streams(self) -> int:
        return len(self.prompt)

    @property
    def lengths(self) -> list:
        return [p + t for p, t in zip(self.prompt, self.chunk)]

    @property
    def n_tok(self) -> int:
        return sum(self.lengths)

    def offsets(self) -> list:
        out, o = [], 0
        for n in self.lengths:
            out.append(o)
            o += n
        return out


class B200Solver:
    """The CFG Euler solve of the DiT estimator on one sm_100 GPU.

    ``weights``: fp32 state dict keyed like ``estimator.blocks.0.attn.to_q.weight`` (``state_dict_from_module``).
    ``cfg``: the hyper-parameters (``b200t2w.config``).  ``device``: a CUDA device."""

    def __init__(self, cfg: DiTConfig, weights: dict, precision: str = "bf16", device=None):
        cfg.validate_for_kernels()
        self.cfg = cfg
        self.precision = precision
        dev = torch.device(device) if device is not None else torch.device("cuda")
        self.device = dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())
        self._lib = L.load()
        if not self._lib.t2w_device_ok(self.device.index):
            raise L.T2WError("t2w_device_ok", -5)
        names = L.W_GLOBAL + [f"estimator.blocks.{b}.{n}" for b in range(cfg.depth) for n in L.W_BLOCK]
        missing = [n for n in names if n not in weights]
        if missing:
            raise KeyError(f"weights missing {len(missing)} entries, e.g. {missing[:3]}")
        with torch.cuda.device(self.device):
            dev_w = [weights[n].detach().to(self.device, torch.float32).contiguous() for n in names]
            ts, dts = t_schedule(cfg.steps)
            cfg_i = [cfg.mel, cfg.hidden, cfg.depth, cfg.heads, cfg.head_dim, cfg.ffn, cfg.steps, cfg.freq_dim]
            cfg_f = [cfg.cfg_rate, cfg.t_scale, cfg.max_period, cfg.eps_block, cfg.eps_final, cfg.eps_qk, cfg.eps_conv]
            hid = O.call("create", cfg_i, cfg_f, [v for pair in zip(ts, dts) for v in pair], dev_w, L.PREC[precision])
            del dev_w
        self._hid = int(hid)  # the solver handle as the torch ops take it
        self._h = ctypes.c_void_p(self._hid)  # and as the ctypes binding takes it
        self._ws: dict = {}
        self._bufs: dict = {}
        self._staging: dict = {}

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            O.call("destroy", self._hid)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------------------------------------ introspection
    def mods(self) -> tuple:
        """(mods [S, depth, 9, H], final [S, 2, H], dts [S]) as the solver computed them (scales stored as 1 + scale)."""
        c = self.cfg
        m = torch.empty(c.steps, c.depth, 9, c.hidden, device=self.device)
        f = torch.empty(c.steps, 2, c.hidden, device=self.device)
        d = torch.empty(c.steps, device=self.device)
        L.call("t2w_mods", self._h, ctypes.c_void_p(m.data_ptr()), ctypes.c_void_p(f.data_ptr()),
               ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        return m, f, d

    def counts(self) -> dict:
        r, c, e = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        L.call("t2w_counts", self._h, ctypes.byref(r), ctypes.byref(c), ctypes.byref(e))
        return {"graph": r.value, "captures": c.value, "eager": e.value}

    def check(self) -> None:
        """Synchronise and raise if any kernel of an earlier solve gave up on a bounded wait."""
        L.call("t2w_check", self._h)

    # ------------------------------------------------------------------------------------------------ packed solve
    def workspace_bytes(self, layout: Layout) -> int:
        n = O.call("workspace_bytes", self._hid, list(layout.prompt), list(layout.chunk))
        if not n:
            raise L.T2WError("t2w_workspace_bytes", -1)
        return int(n)

    def workspace(self, layout: Layout, key=None) -> torch.Tensor:
        """A device workspace for ``layout`` (kept per key so CUDA-graph replays see the same buffers)."""
        need = self.workspace_bytes(layout)
        k = key if key is not None else need
        ws = self._ws.get(k)
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self._ws[k] = ws
        return ws

    def solve_packed_dev(self, layout: Layout, x0, mu, cond, spk, out, workspace=None, graph: bool = True,
                         stream=None) -> torch.Tensor:
        """Enqueue one solve on device tensors: x0 / mu / cond / out [n_tok, mel] fp32 (token-major, streams
        concatenated), spk [n_streams, mel].  Asynchronous on ``stream`` (default: the current stream)."""
        c = self.cfg
        for name, t, shape in (("x0", x0, (layout.n_tok, c.mel)), ("mu", mu, (layout.n_tok, c.mel)),
                               ("cond", cond, (layout.n_tok, c.mel)), ("out", out, (layout.n_tok, c.mel)),
                               ("spk", spk, (layout.n_streams, c.mel))):
            if tuple(t.shape) != shape or t.dtype != torch.float32 or not t.is_contiguous() or t.device != self.device:
                raise ValueError(f"{name}: expected contiguous fp32 {shape} on {self.device}, got {tuple(t.shape)} "
                                 f"{t.dtype} on {t.device}")
        ws = workspace if workspace is not None else self.workspace(layout, key=(layout.prompt, layout.chunk))
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        with torch.cuda.stream(st):  # the op enqueues on the current stream of the tensors' device
            O.call("solve_packed", self._hid, list(layout.prompt), list(layout.chunk), x0, mu, cond, spk, out, ws,
                   bool(graph))
        return out

    def profile(self, layout: Layout, bufs: dict | None = None) -> dict:
        """One eager solve of ``layout`` with CUDA events between launches: {kernel class: (ms, launches)}."""
        b = bufs if bufs is not None else self.static_buffers(layout)
        P, T = L.i32_array(layout.prompt), L.i32_array(layout.chunk)
        batch = L.Batch(layout.n_streams, P, T, b["x0"].data_ptr(), b["mu"].data_ptr(), b["cond"].data_ptr(),
                        b["spk"].data_ptr(), b["out"].data_ptr())
        n = len(L.KERNEL_CLASSES)
        ms, cnt = (ctypes.c_float * n)(), (ctypes.c_int32 * n)()
        st = torch.cuda.current_stream(self.device)
        L.call("t2w_profile_solve", self._h, ctypes.byref(batch), ctypes.c_void_p(b["ws"].data_ptr()),
               ctypes.c_size_t(b["ws"].numel()), ctypes.c_void_p(st.cuda_stream), ms, cnt)
        return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(L.KERNEL_CLASSES)}

    def static_buffers(self, layout: Layout) -> dict:
        """Per-layout static input / output buffers (CUDA-graph replays hit the same pointers)."""
        key = (layout.prompt, layout.chunk)
        b = self._bufs.get(key)
        if b is None:
            n, m = layout.n_tok, self.cfg.mel
            z = lambda *s: torch.zeros(*s, dtype=torch.float32, device=self.device)  # noqa: E731
            b = {"x0": z(n, m), "mu": z(n, m), "cond": z(n, m), "spk": z(layout.n_streams, m), "out": z(n, m),
                 "ws": self.workspace(layout, key=key)}
            self._bufs[key] = b
        return b

    def solve_streams(self, streams: list, graph: bool = True) -> list:
        """Solve packed streams (dicts with x0 / mu / cond [mel, L], spk [mel], P, T; host or device tensors) and return
        each stream's final x [mel, L] fp32 on the solver's device (the chunk mel is ``[:, P:]``; views of one fresh
        tensor).  Host inputs are gathered into pinned mirrors of the static buffers and moved by one asynchronous copy
        per input, so the host can prepare the next call while this one runs."""
        layout = Layout(tuple(int(s["P"]) for s in streams), tuple(int(s["T"]) for s in streams))
        b = self.static_buffers(layout)
        st = torch.cuda.current_stream(self.device)
        key = (layout.prompt, layout.chunk)
        for k in ("x0", "mu", "cond", "spk"):
            parts = [s[k] if k == "spk" else s[k].t() for s in streams]
            if all(p.device == self.device for p in parts):
                if k == "spk":
                    torch.stack([p.to(torch.float32) for p in parts], out=b[k])
                else:
                    torch.cat([p.to(torch.float32) for p in parts], out=b[k])
                continue
            host = torch.stack([p.to("cpu", torch.float32) for p in parts]) if k == "spk" else \
                torch.cat([p.to("cpu", torch.float32) for p in parts])
            stg = self._staging.get((key, k))
            if stg is None:
                stg = self._staging[(key, k)] = HostStaging(b[k])
            stg.copy(b[k], host, st)
        self.solve_packed_dev(layout, b["x0"], b["mu"], b["cond"], b["spk"], b["out"], workspace=b["ws"], graph=graph)
        out = b["out"].clone()  # the static buffer is rewritten by the next call
        return [out[o:o + n].t() for o, n in zip(layout.offsets(), layout.lengths)]

    # ------------------------------------------------------------------------------------------------ reference API
    def forward_chunk(self, mu, spks, cond, n_timesteps: int = 10, temperature: float = 1.0, x0=None, prompt_len: int = 0):
        """``CausalConditionalCFM.forward_chunk`` argument meaning for one request in packed form: ``mu`` [1, mel, L]
        conditioning over prompt + chunk, ``spks`` [1, mel] (post-affine), ``cond`` [1, mel, L] (prompt mel, zeros over
        the chunk), ``x0`` [1, mel, L] fixed noise (the reference reads ``rand_noise`` at the cache offset) scaled by
        ``temperature``.  Returns the chunk mel [1, mel, L - prompt_len] fp32.  The solver's step count is fixed at
        construction and must equal ``n_timesteps``."""
        if n_timesteps != self.cfg.steps:
            raise ValueError(f"solver built for {self.cfg.steps} steps, asked for {n_timesteps}")
        Lf = mu.shape[2]
        if x0 is None:
            raise ValueError("x0 (the fixed noise window) is required")
        s = {"x0": x0[0].float() * temperature, "mu": mu[0].float(), "cond": cond[0].float(), "spk": spks[0].float(),
             "P": int(prompt_len), "T": int(Lf - prompt_len)}
        return self.solve_streams([s])[0][:, prompt_len:][None]
