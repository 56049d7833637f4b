"""Steady-state Token2Wav solve on B200: the drop-in for the reference's ``FastDiT`` (engine/runtime/dit_fast.py).

The reference keeps every CFG row's cached key frames in a slot pool (FlashInfer paged K/V, page size 1) and its two
conv-cache frames per (step, block) in a row-slot pool; a call solves one window per request against those caches,
appends the window's keys (``[new, cache]`` order) and trims the cache to the prompt's frames plus the last 100
(``dit_fast.py:58-97,432-495``, ``token2wav_batch.py:33-39``).  ``B200FastDiT`` keeps that host bookkeeping (slot ids,
the reference's key order, the trim) in Python, as the reference does, and runs the solve in the CUDA library
(``t2w_solve_slots``): pools on the device, attention gathering each row's key list, conv caches filled in front of
each window.  Method names and argument meaning follow ``FastDiT``: ``new_cache``, ``release``, ``clone``, ``solve``,
``counts``, ``pool.in_use()``.  With ``use_graphs`` the solve replays a CUDA graph per call structure (sizes of the
window and key lists), as ``FastDiT.capture`` does per bucket (``dit_fast.py:347-428``): inputs are copied into
static buffers first (``dit_fast.py:463-469``), and a structure is captured the second time it is seen.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import lib as L
from .solver import B200Solver

TRIM_SUFFIX = 100


class SlotIds:
    """Host free list of pool slot ids (the reference's ``SlotPool`` bookkeeping, ``dit_fast.py:58-78``)."""

    def __init__(self, n: int):
        self.n = n
        self.free = list(range(n - 1, -1, -1))

    def alloc(self, k: int) -> list:
        if k > len(self.free):
            raise RuntimeError(f"Token2Wav cache pool exhausted ({k} slots wanted, {len(self.free)} free of {self.n})")
        out = self.free[len(self.free) - k:][::-1] if k else []
        del self.free[len(self.free) - k:]
        return out

    def release(self, ids: list) -> None:
        self.free.extend(ids)

    def in_use(self) -> int:
        return self.n - len(self.free)


@dataclass
class FastRow:
    """One CFG row's caches: key slots in the reference's tensor order and its conv-cache row slot."""
    order: list = field(default_factory=list)
    cnn: int = -1


@dataclass
class FastCache:
    """A request's estimator caches (conditional and unconditional rows) and its trim length (prompt mel frames)."""
    rows: tuple
    keep: int = 0

    @property
    def length(self) -> int:
        return len(self.rows[0].order)


class _DeviceArray:
    """A device buffer handed to torch through the CUDA array interface (no copy; the owner keeps it alive)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "strides": None, "version": 2}


class B200FastDiT:
    """``FastDiT`` on the B200 kernels.

    ``solver``: a bf16 ``B200Solver`` (weights, modulation tables).  ``noise``: the flow's fixed noise [mel, frames]
    (``cfm.rand_noise[0]``), read at each request's cache length.  ``n_slots``: key slots (each holds K and V of every
    (step, block) of one frame: steps * depth * 4 * hidden bytes).  ``max_streams``: concurrent requests (two
    conv-cache row slots each)."""

    def __init__(self, solver: B200Solver, noise: torch.Tensor, n_slots: int = 32768, max_streams: int = 96,
                 use_graphs: bool = True):
        if solver.precision != "bf16":
            raise ValueError("the slot-pool solve runs the bf16 path")
        self.solver, self.cfg, self.device = solver, solver.cfg, solver.device
        self.noise = noise.detach().to(self.device, torch.float32).contiguous()
        self._lib = L.load()
        n_rs = 2 * max_streams + 1  # + one scratch row slot: the write target of rows that keep nothing
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            L.call("t2w_slots_create", solver._h, n_slots, n_rs, ctypes.byref(h))
        self._p = h
        self.pool = SlotIds(n_slots)
        self.cnn_free = list(range(n_rs - 1, 0, -1))
        self.cnn_scratch = 0
        self._ws = None
        self.use_graphs = use_graphs
        self._static = {}  # (tokens, requests, has cond) -> static input / output buffers of the graph path
        self.counts = {"graph": 0, "eager": 0}
        self.scratch = 0  # pool slots reserved for pad rows: none (pad rows never reach the pool here)

    @classmethod
    def from_cfm(cls, cfm, steps: int, n_slots: int = 32768, max_streams: int = 96, device="cuda",
                 use_graphs: bool = False, setup_tokens: int = 0, fused_residual: bool = False,
                 fused_conv: bool = False) -> "B200FastDiT":
        """Built as the reference builds ``FastDiT(cfm, steps, ...)`` (``engine/runtime/dit_fast.py:99-146``): the
        config read off ``cfm.estimator`` (``config_from_module``), the weights packed to bf16 from the module's own
        parameters, the fixed noise ``cfm.rand_noise[0]``.  ``setup_tokens``, ``fused_residual`` and ``fused_conv``
        select graph-bucket padding and kernel fusions inside the reference's solve; this solve has no row buckets and
        always runs its fused residual / norm / conv-gather kernels, so they are accepted and change nothing (the
        reference's own check that ``fused_conv`` needs ``fused_residual`` is kept)."""
        from .config import config_from_module
        from .solver import state_dict_from_module

        if fused_conv and not fused_residual:
            raise ValueError("fused_conv is a fused_residual option")
        if int(setup_tokens) < 0:
            raise ValueError("setup_tokens must be >= 0")
        cfg = config_from_module(cfm, steps=steps)
        solver = B200Solver(cfg, state_dict_from_module(cfm), precision="bf16", device=device)
        return cls(solver, cfm.rand_noise[0], n_slots=n_slots, max_streams=max_streams, use_graphs=use_graphs)

    def capture_all(self, row_buckets=None) -> int:
        """The reference captures one graph per row bucket up front (``dit_fast.py:347-428``).  Here a graph is keyed
        by the call's exact structure and captured the second time that structure is solved, so nothing is captured
        ahead; returns 0 (graphs captured now)."""
        return 0

    def close(self) -> None:
        if getattr(self, "_p", None) is not None and self._p.value:
            self._lib.t2w_slots_destroy(self._p)
            self._p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    # --- caches -------------------------------------------------------------------------------------------------------
    def new_cache(self) -> FastCache:
        if len(self.cnn_free) < 2:
            raise RuntimeError("Token2Wav conv-cache row slots exhausted")
        rows = (FastRow(cnn=self.cnn_free.pop()), FastRow(cnn=self.cnn_free.pop()))
        for r in rows:
            L.call("t2w_slots_copy_row", self._p, -1, r.cnn, self._stream())
        return FastCache(rows)

    def release(self, c: FastCache) -> None:
        for r in c.rows:
            self.pool.release(r.order)
            r.order = []
            if r.cnn >= 0:
                self.cnn_free.append(r.cnn)
                r.cnn = -1

    def clone(self, c: FastCache) -> FastCache:
        """An independent copy (new slots holding the same keys and values, copied conv caches)."""
        out = self.new_cache()
        out.keep = c.keep
        for src, dst in zip(c.rows, out.rows):
            L.call("t2w_slots_copy_row", self._p, src.cnn, dst.cnn, self._stream())
            dst.order = self.pool.alloc(len(src.order))
            if src.order:
                L.call("t2w_slots_copy", self._p, L.i32_array(src.order), L.i32_array(dst.order), len(src.order),
                       self._stream())
        return out

    # --- caches as tensors (the module-level forward_chunk adapter) ---------------------------------------------------
    def pools(self) -> tuple:
        """The slot pools as torch views (no copy): K/V [steps * depth, n_slots, 2H] (K heads, then V heads) and conv
        caches [steps * depth, n_rowslots, 2 convs, 2 frames (oldest first), H], bf16."""
        if getattr(self, "_pool_views", None) is None:
            kv, cn = ctypes.c_void_p(), ctypes.c_void_p()
            n_sb, n_slots, n_rs, H = (ctypes.c_int32() for _ in range(4))
            L.call("t2w_slots_pools", self._p, ctypes.byref(kv), ctypes.byref(cn), ctypes.byref(n_sb),
                   ctypes.byref(n_slots), ctypes.byref(n_rs), ctypes.byref(H))
            with torch.cuda.device(self.device):
                k = torch.as_tensor(_DeviceArray(kv.value, (n_sb.value, n_slots.value, 2 * H.value), "<i2"),
                                    device=self.device).view(torch.bfloat16)
                c = torch.as_tensor(_DeviceArray(cn.value, (n_sb.value, n_rs.value, 2, 2, H.value), "<i2"),
                                    device=self.device).view(torch.bfloat16)
            self._pool_views = (k, c)
        return self._pool_views

    def load_cache(self, att: torch.Tensor, cnn: torch.Tensor, keep: int = 0) -> FastCache:
        """A cache holding the reference's tensors (``token2wav_batch.py:643-644``): ``att`` [steps, depth, 2, heads,
        L, 2 * 64] (K then V of each head, keys in the reference's order), ``cnn`` [steps, depth, 2, 2H, 2] (each
        conv's last two input frames, conv 1 then conv 2).  Values are stored in bf16."""
        c = self.cfg
        S, D, H, nh = c.steps, c.depth, c.hidden, c.heads
        Lk = int(att.shape[4])
        if tuple(att.shape) != (S, D, 2, nh, Lk, 2 * c.head_dim) or tuple(cnn.shape) != (S, D, 2, 2 * H, 2):
            raise ValueError(f"caches: expected att [{S}, {D}, 2, {nh}, L, {2 * c.head_dim}] and cnn [{S}, {D}, 2, "
                             f"{2 * H}, 2], got {tuple(att.shape)} and {tuple(cnn.shape)}")
        kv, cn = self.pools()
        fc = self.new_cache()
        fc.keep = keep
        a = att.to(self.device, torch.bfloat16)
        cc = cnn.to(self.device, torch.bfloat16)
        for half, row in enumerate(fc.rows):
            row.order = self.pool.alloc(Lk)
            if Lk:
                x = a[:, :, half]  # [S, D, heads, L, 128]
                k = x[..., :c.head_dim].permute(0, 1, 3, 2, 4).reshape(S * D, Lk, H)
                v = x[..., c.head_dim:].permute(0, 1, 3, 2, 4).reshape(S * D, Lk, H)
                kv[:, torch.tensor(row.order, device=self.device)] = torch.cat([k, v], dim=2)
            cn[:, row.cnn] = cc[:, :, half].reshape(S * D, 2, H, 2).permute(0, 1, 3, 2)
        return fc

    def export_cache(self, fc: FastCache, dtype=torch.float32) -> tuple:
        """``fc``'s caches as the reference's tensors ``(att, cnn)`` (layouts of ``load_cache``)."""
        c = self.cfg
        S, D, H, nh, hd = c.steps, c.depth, c.hidden, c.heads, c.head_dim
        kv, cn = self.pools()
        Lk = fc.length
        att = torch.empty(S, D, 2, nh, Lk, 2 * hd, dtype=dtype, device=self.device)
        cnn = torch.empty(S, D, 2, 2 * H, 2, dtype=dtype, device=self.device)
        for half, row in enumerate(fc.rows):
            if Lk:
                x = kv[:, torch.tensor(row.order, device=self.device)]  # [S * D, L, 2H]
                k = x[..., :H].reshape(S, D, Lk, nh, hd).permute(0, 1, 3, 2, 4)
                v = x[..., H:].reshape(S, D, Lk, nh, hd).permute(0, 1, 3, 2, 4)
                att[:, :, half] = torch.cat([k, v], dim=-1).to(dtype)
            cnn[:, :, half] = cn[:, row.cnn].permute(0, 1, 3, 2).reshape(S, D, 2 * H, 2).to(dtype)
        return att, cnn

    @torch.inference_mode()
    def forward_chunk(self, mu, spks, cond, n_timesteps: int = 10, temperature: float = 1.0, cnn_cache=None,
                      att_cache=None):
        """``CausalConditionalCFM.forward_chunk(mu, spks, cond, n_timesteps, temperature, cnn_cache, att_cache)`` for
        one request (``tools/spike/t2w_profile.py:63-64``): ``mu`` / ``cond`` [1, mel, T], ``spks`` [1, mel] (after
        the affine layer), caches as in ``load_cache`` (None: empty).  The noise is the flow's fixed noise at the
        cache length, times ``temperature``.  Returns ``(mel [1, mel, T] fp32, new_cnn, new_att)`` with the new keys
        in front of the old ones and nothing trimmed (the caller trims, as the reference's callers do); caches come
        back in ``att_cache``'s dtype (fp32 when None)."""
        c = self.cfg
        if n_timesteps != c.steps:
            raise ValueError(f"solver built for {c.steps} steps, asked for {n_timesteps}")
        T = int(mu.shape[2])
        dtype = att_cache.dtype if att_cache is not None else torch.float32
        if att_cache is None:
            att_cache = torch.zeros(c.steps, c.depth, 2, c.heads, 0, 2 * c.head_dim)
        if cnn_cache is None:
            cnn_cache = torch.zeros(c.steps, c.depth, 2, 2 * c.hidden, 2)
        fc = self.load_cache(att_cache, cnn_cache, keep=int(att_cache.shape[4]) + T)  # nothing to trim
        try:
            mel = self.solve([fc], [mu[0]], spks.reshape(1, -1), [cond[0]] if cond is not None else None, [True],
                             temperature=temperature)[0]
            new_att, new_cnn = self.export_cache(fc, dtype)
        finally:
            self.release(fc)
        return mel[None], new_cnn, new_att

    # --- solve --------------------------------------------------------------------------------------------------------
    @torch.inference_mode()
    def solve(self, caches: list, mu: list, spks: torch.Tensor, cond: list | None, keep: list,
              temperature: float = 1.0) -> list:
        """One window per request (``FastDiT.solve``): ``mu[i]`` [mel, T_i], ``spks`` [n, mel] (after the affine
        layer), ``cond[i]`` [mel, T_i] or None (zeros; ``cond`` None: zeros for all).  Requests with ``keep[i]`` keep
        the window's keys and conv caches, trimmed as the reference trims them; the others (final flushes) leave their
        caches untouched.  Returns each request's mel [mel, T_i] fp32."""
        n = len(caches)
        mel = self.cfg.mel
        Ts = [int(m.shape[1]) for m in mu]
        lens = [c.length for c in caches]
        rows = [c.rows[0] for c in caches] + [c.rows[1] for c in caches]
        new = [self.pool.alloc(t) for t in Ts + Ts]
        kv_len, kv_idx, rd, wr = [], [], [], []
        for r in range(2 * n):
            i = r % n
            lst = rows[r].order + new[r]  # attention depends on the key set; the window's slots go last
            kv_len.append(len(lst))
            kv_idx += lst
            rd.append(rows[r].cnn)
            wr.append(rows[r].cnn if keep[i] else self.cnn_scratch)
        dev = self.device
        n_tok = sum(Ts)
        key = (n_tok, n, cond is not None)
        bufs = self._static.get(key)
        if bufs is None:
            z = lambda *sh: torch.zeros(*sh, dtype=torch.float32, device=dev)  # noqa: E731
            bufs = {"x0": z(n_tok, mel), "mu": z(n_tok, mel), "cond": z(n_tok, mel) if cond is not None else None,
                    "spk": z(n, mel), "out": z(n_tok, mel)}
            self._static[key] = bufs
        torch.cat([self.noise[:, o:o + t].t() for o, t in zip(lens, Ts)], out=bufs["x0"])
        if temperature != 1.0:  # the fixed noise scaled as CausalConditionalCFM.forward_chunk scales it
            bufs["x0"].mul_(temperature)
        # inputs in pinned host memory are copied without stalling the host (pageable ones copy synchronously)
        torch.cat([m.t().to(dev, torch.float32, non_blocking=True) for m in mu], out=bufs["mu"])
        if cond is not None:
            torch.cat([(c.t() if c is not None else torch.zeros(t, mel)).to(dev, torch.float32, non_blocking=True)
                       for c, t in zip(cond, Ts)], out=bufs["cond"])
        bufs["spk"].copy_(spks.to(dev, torch.float32, non_blocking=True))
        out = bufs["out"]
        P = lambda t: ctypes.c_void_p(t.data_ptr() if t is not None else 0)  # noqa: E731
        arrs = [L.i32_array(a) for a in (Ts, kv_len, kv_idx, rd, wr)]  # alive until the call returns
        ip = [ctypes.cast(a, ctypes.POINTER(ctypes.c_int32)) for a in arrs]
        b = L.SlotBatch(n, *ip, P(bufs["x0"]), P(bufs["mu"]), P(bufs["cond"]), P(bufs["spk"]), P(out))
        need = int(self._lib.t2w_slot_workspace_bytes(self.solver._h, self._p, ctypes.byref(b)))
        if not need:
            raise L.T2WError("t2w_slot_workspace_bytes", -1)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=dev)
        before = self.solver.counts()["graph"]
        L.call("t2w_solve_slots", self.solver._h, self._p, ctypes.byref(b), P(self._ws), self._ws.numel(),
               L.FLAG_GRAPH if self.use_graphs else 0, self._stream())
        self.counts["graph" if self.solver.counts()["graph"] > before else "eager"] += 1
        # the reference's cache order and trim (dit_fast.py:482-490)
        for i, c in enumerate(caches):
            for r, nw in ((rows[i], new[i]), (rows[n + i], new[n + i])):
                if keep[i]:
                    order = nw + r.order
                    if len(order) > c.keep + TRIM_SUFFIX:
                        self.pool.release(order[c.keep:len(order) - TRIM_SUFFIX])
                        order = order[:c.keep] + order[len(order) - TRIM_SUFFIX:]
                    r.order = order
                else:
                    self.pool.release(nw)
        res, o = [], 0
        for t in Ts:
            res.append(out[o:o + t].t().clone())  # the static buffer is rewritten by the next call
            o += t
        return res
