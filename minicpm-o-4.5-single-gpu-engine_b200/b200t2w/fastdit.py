"""Steady-state Token2Wav solve on B200: the drop-in for the reference's ``FastDiT`` (engine/runtime/dit_fast.py).

The reference keeps every CFG row's cached key frames in a slot pool (FlashInfer paged K/V, page size 1) and its two
conv-cache frames per (step, block) in a row-slot pool; a call solves one window per request against those caches,
appends the window's keys (``[new, cache]`` order) and trims the cache to the prompt's frames plus the last 100
(``dit_fast.py:58-97,432-495``, ``token2wav_batch.py:33-39``).  Here the pools, the caches' key orders, slot allocation
and the trim all live in the CUDA library (``t2w_cache_*``, ``t2w_solve_cached``): a ``FastCache`` is a handle, and a
call hands the library the handles, window lengths and inputs; the library builds every CFG row's key list, gathers
x0 from the flow's fixed noise at each cache length, runs the solve (attention gathering each row's key list, conv
caches filled in front of each window) and updates the orders.  Method names and argument meaning follow ``FastDiT``:
``new_cache``, ``release``, ``clone``, ``solve``, ``counts``, ``pool.in_use()``, ``cnn_free``.  With ``use_graphs`` the
solve replays a CUDA graph per call structure (sizes of the window and key lists), as ``FastDiT.capture`` does per
bucket (``dit_fast.py:347-428``): inputs are copied into static buffers first (``dit_fast.py:463-469``), and a
structure is captured the second time it is seen.
"""

from __future__ import annotations

import ctypes

import torch

from . import lib as L
from . import ops as O
from .solver import B200Solver
from .staging import HostStaging

TRIM_SUFFIX = 100  # keys kept after the first ``keep`` (the library applies the trim)
_WORKSPACE_TOO_SMALL = -6


class FastCache:
    """A request's estimator caches (both CFG rows), held by the library: a handle plus the two attributes the engine
    reads and sets, ``length`` (cached keys per CFG row) and ``keep`` (the trim length: the prompt's mel frames)."""

    __slots__ = ("_fd", "handle")

    def __init__(self, fd: "B200FastDiT", handle: int):
        self._fd, self.handle = fd, handle

    def _info(self) -> L.CacheInfo:
        info = L.CacheInfo()
        L.call("t2w_cache_get", self._fd._p, self.handle, ctypes.byref(info))
        return info

    @property
    def length(self) -> int:
        return self._info().length if self.handle >= 0 else 0

    @property
    def keep(self) -> int:
        return self._info().keep if self.handle >= 0 else 0

    @keep.setter
    def keep(self, v: int) -> None:
        L.call("t2w_cache_set_keep", self._fd._p, self.handle, int(v))


class _PoolUsage:
    """``pool.in_use()``: key slots handed out (both CFG rows count)."""

    def __init__(self, fd: "B200FastDiT"):
        self._fd = fd

    def in_use(self) -> int:
        return self._fd._usage()[0]


class _FreeRowSlots:
    """``len(cnn_free)``: conv-cache row slots still free (two per new cache)."""

    def __init__(self, fd: "B200FastDiT"):
        self._fd = fd

    def __len__(self) -> int:
        return self._fd._usage()[1]


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
        with torch.cuda.device(self.device):
            self._pid = int(O.call("slots_create", solver._hid, n_slots, n_rs))
        self._p = ctypes.c_void_p(self._pid)
        self.pool = _PoolUsage(self)
        self.cnn_free = _FreeRowSlots(self)
        self._ws = None
        self.use_graphs = use_graphs
        self._static = {}  # (tokens, requests, has cond) -> static input / output buffers of the graph path
        self._staging = {}
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
            O.call("slots_destroy", self._pid)
            self._p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _usage(self) -> tuple:
        used, free, live = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        L.call("t2w_slots_usage", self._p, ctypes.byref(used), ctypes.byref(free), ctypes.byref(live))
        return used.value, free.value, live.value

    # --- caches -------------------------------------------------------------------------------------------------------
    def new_cache(self) -> FastCache:
        h = ctypes.c_int32()
        L.call("t2w_cache_new", self._p, 0, self._stream(), ctypes.byref(h))
        return FastCache(self, h.value)

    def release(self, c: FastCache) -> None:
        if c.handle >= 0:
            L.call("t2w_cache_release", self._p, c.handle)
            c.handle = -1

    def clone(self, c: FastCache) -> FastCache:
        """An independent copy (new slots holding the same keys and values, copied conv caches)."""
        h = ctypes.c_int32()
        L.call("t2w_cache_clone", self._p, c.handle, self._stream(), ctypes.byref(h))
        return FastCache(self, h.value)

    def _keys(self, c: FastCache, half: int) -> list:
        n = c.length
        arr = (ctypes.c_int32 * max(n, 1))()
        L.call("t2w_cache_keys", self._p, c.handle, half, arr, n)
        return list(arr[:n])

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
        slots = (ctypes.c_int32 * max(2 * Lk, 1))()
        L.call("t2w_cache_reserve", self._p, fc.handle, Lk, slots)
        rowslots = fc._info().rowslot
        a = att.to(self.device, torch.bfloat16)
        cc = cnn.to(self.device, torch.bfloat16)
        for half in range(2):
            if Lk:
                x = a[:, :, half]  # [S, D, heads, L, 128]
                k = x[..., :c.head_dim].permute(0, 1, 3, 2, 4).reshape(S * D, Lk, H)
                v = x[..., c.head_dim:].permute(0, 1, 3, 2, 4).reshape(S * D, Lk, H)
                idx = torch.tensor(list(slots[half * Lk:(half + 1) * Lk]), device=self.device)
                kv[:, idx] = torch.cat([k, v], dim=2)
            cn[:, rowslots[half]] = cc[:, :, half].reshape(S * D, 2, H, 2).permute(0, 1, 3, 2)
        return fc

    def export_cache(self, fc: FastCache, dtype=torch.float32) -> tuple:
        """``fc``'s caches as the reference's tensors ``(att, cnn)`` (layouts of ``load_cache``)."""
        c = self.cfg
        S, D, H, nh, hd = c.steps, c.depth, c.hidden, c.heads, c.head_dim
        kv, cn = self.pools()
        Lk = fc.length
        att = torch.empty(S, D, 2, nh, Lk, 2 * hd, dtype=dtype, device=self.device)
        cnn = torch.empty(S, D, 2, 2 * H, 2, dtype=dtype, device=self.device)
        rowslots = fc._info().rowslot
        for half in range(2):
            if Lk:
                x = kv[:, torch.tensor(self._keys(fc, half), device=self.device)]  # [S * D, L, 2H]
                k = x[..., :H].reshape(S, D, Lk, nh, hd).permute(0, 1, 3, 2, 4)
                v = x[..., H:].reshape(S, D, Lk, nh, hd).permute(0, 1, 3, 2, 4)
                att[:, :, half] = torch.cat([k, v], dim=-1).to(dtype)
            cnn[:, :, half] = cn[:, rowslots[half]].permute(0, 1, 3, 2).reshape(S, D, 2 * H, 2).to(dtype)
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
    def _stage(self, key, name: str, dst: torch.Tensor, parts: list) -> None:
        """Concatenate ``parts`` ([T_i, mel] views, host or device) into the static device buffer ``dst``: on the
        device with one kernel when every part is there, else on the host into a pinned mirror and one copy."""
        if all(t.device == self.device for t in parts):
            torch.cat([t.to(torch.float32) for t in parts], out=dst)
            return
        host = torch.cat([t.detach().to("cpu", torch.float32) for t in parts])
        st = self._staging.get((key, name))
        if st is None:
            st = self._staging[(key, name)] = HostStaging(dst)
        st.copy(dst, host, torch.cuda.current_stream(self.device))

    @torch.inference_mode()
    def solve(self, caches: list, mu: list, spks: torch.Tensor, cond: list | None, keep: list,
              temperature: float = 1.0) -> list:
        """One window per request (``FastDiT.solve``): ``mu[i]`` [mel, T_i], ``spks`` [n, mel] (after the affine
        layer), ``cond[i]`` [mel, T_i] or None (zeros; ``cond`` None: zeros for all).  Requests with ``keep[i]`` keep
        the window's keys and conv caches, trimmed as the reference trims them; the others (final flushes) leave their
        caches untouched.  Returns each request's mel [mel, T_i] fp32 (views of one fresh tensor, as the reference
        returns views of its output)."""
        n = len(caches)
        mel = self.cfg.mel
        Ts = [int(m.shape[1]) for m in mu]
        dev = self.device
        n_tok = sum(Ts)
        key = (n_tok, n, cond is not None)
        bufs = self._static.get(key)
        if bufs is None:
            z = lambda *sh: torch.zeros(*sh, dtype=torch.float32, device=dev)  # noqa: E731
            bufs = {"mu": z(n_tok, mel), "cond": z(n_tok, mel) if cond is not None else None, "spk": z(n, mel),
                    "out": z(n_tok, mel)}
            self._static[key] = bufs
        self._stage(key, "mu", bufs["mu"], [m.t() for m in mu])
        if cond is not None:
            self._stage(key, "cond", bufs["cond"],
                        [c.t() if c is not None else torch.zeros(t, mel, device=mu[i].device) for i, (c, t)
                         in enumerate(zip(cond, Ts))])
        self._stage(key, "spk", bufs["spk"], [spks.reshape(n, mel)])
        handles = [c.handle for c in caches]
        kp = [1 if k else 0 for k in keep]
        before = self.solver.counts()["graph"]
        if self._ws is None:
            self._ws = torch.empty(256, dtype=torch.uint8, device=dev)
        args = (self.solver._hid, self._pid, handles, Ts, kp, self.noise, float(temperature), bufs["mu"], bufs["cond"],
                bufs["spk"], bufs["out"])
        try:
            O.call("solve_cached", *args, self._ws, bool(self.use_graphs))
        except L.T2WError as e:
            if e.status != _WORKSPACE_TOO_SMALL:
                raise
            need = int(O.call("cached_workspace_bytes", *args[:6]))
            if not need:
                raise L.T2WError("t2w_cached_workspace_bytes", -1) from e
            self._ws = torch.empty(need + need // 4, dtype=torch.uint8, device=dev)
            O.call("solve_cached", *args, self._ws, bool(self.use_graphs))
        self.counts["graph" if self.solver.counts()["graph"] > before else "eager"] += 1
        out = bufs["out"].clone()  # the static buffer is rewritten by the next call
        res, o = [], 0
        for t in Ts:
            res.append(out[o:o + t].t())
            o += t
        return res
