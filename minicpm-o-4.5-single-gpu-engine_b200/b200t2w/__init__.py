"""B200-native Token2Wav flow-matching solve (DiT velocity estimator + CFG Euler ODE) behind the reference engine's
solver interface.  The arithmetic lives in ``libt2w_b200.so`` (hand-written sm_100a CUDA, C ABI in
``include/t2w_b200.h``); this package plans, binds and schedules."""

from .config import REFERENCE, TINY, DiTConfig, t_schedule  # noqa: F401

__all__ = ["DiTConfig", "REFERENCE", "TINY", "t_schedule", "B200Solver", "Layout", "state_dict_from_module",
           "B200FastDiT", "FastCache"]


def __getattr__(name):
    if name in ("B200Solver", "Layout", "state_dict_from_module"):
        from . import solver

        return getattr(solver, name)
    if name in ("B200FastDiT", "FastCache"):
        from . import fastdit

        return getattr(fastdit, name)
    raise AttributeError(name)
