"""bozo_b200 — B200-native (sm_100a) sigmoid-tension operator for TensionLM.

Public API:
  causal_tension(Q, K, V, window, scale, return_tau=False, bias=None)
      drop-in for ``triton_tension.causal_tension`` (BoggersTheFish/bozo).
  tension(q, k, v, *, window, ...)
      fused RoPE + local/global tension + normalisation (+ τ export).
  install_as_triton_tension()
      registers this package under the module name ``triton_tension`` so the
      reference's model.py / train.py / generate.py import it unchanged.
"""
from __future__ import annotations

import sys
import types

from .ops import (causal_tension, check_device_error, last_launches, last_path,
                  poll_device_error, rope_tables, set_kernel_path, tension)

__all__ = ["causal_tension", "tension", "install_as_triton_tension", "set_kernel_path",
           "last_path", "last_launches", "poll_device_error", "check_device_error",
           "rope_tables"]


def install_as_triton_tension() -> types.ModuleType:
    """Make ``from triton_tension import causal_tension`` (model.py:248) and
    ``from triton_tension.ops import causal_tension`` resolve to this build."""
    from . import ops as _ops
    pkg = types.ModuleType("triton_tension")
    pkg.causal_tension = _ops.causal_tension
    pkg.__all__ = ["causal_tension"]
    pkg.__path__ = []  # mark as a package
    pkg.ops = _ops
    sys.modules["triton_tension"] = pkg
    sys.modules["triton_tension.ops"] = _ops
    return pkg
