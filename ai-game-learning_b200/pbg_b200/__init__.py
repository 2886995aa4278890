"""pbg_b200: the B200-native data-parallel hot path of pbg.

Submodules mirror the reference's interfaces for the path:
rng (core/rollout.py RNG), poker (queued/hooks.py state machine),
policy (queued/policy.py), rollout (fused sampled step), loss (fused PPO
backward), optim (flat Adam), distributed (gradient SUM).  All compute runs
in libpbgb200.so (sm_100a); there is no CPU fallback.
"""

from ._native import LIB_PATH, NativeError, lib  # noqa: F401

__all__ = ["LIB_PATH", "NativeError", "lib"]
