"""CPU oracle for the device graph bias — TEST INFRASTRUCTURE ONLY.

Only ``tests/`` import it; ``bozo_b200.graph_bias`` builds the bias on the
GPU and never routes through this file.  It restates ts_bridge/bias.py's
``GraphBias.local_bias`` (bias.py:125-170) and ``global_bias``
(bias.py:172-233): per context token its content (``id_to_token`` or
``"<id>"``), then α · edge_weight(content[s] → content[t]) for every key s of
the local window (slot w ↔ s = t − (W − w) ≥ 0) or of the causal triangle
(s < t) whose weight is positive, with the count, max and mean of those
weights.  Pinned by ``tests/test_oracle_golden.py`` against
``tests/golden/golden_bias.npz`` (the reference class itself,
``tests/golden/make_golden_bias.py``).
"""
from __future__ import annotations

import numpy as np


def _contents(ctx_ids, tokenizer):
    return [tokenizer.id_to_token(int(t)) or f"<{int(t)}>" for t in ctx_ids]


def _finish(bias, weights):
    hits = len(weights)
    return bias, (hits, max(weights) if weights else 0.0, sum(weights) / hits if hits else 0.0)


def local_bias(edge_map, alpha, ctx_ids, tokenizer, window):
    """[T, W] float32 and (pairs, max weight, mean weight)."""
    c = _contents(ctx_ids, tokenizer)
    T, W = len(c), window
    bias = np.zeros((T, W), dtype=np.float32)
    used = []
    for t in range(T):
        for w in range(W):
            s = t - (W - w)
            if s < 0:
                continue
            wt = edge_map.get((c[s], c[t]), 0.0)
            if wt > 0.0:
                bias[t, w] = alpha * wt
                used.append(wt)
    return _finish(bias, used)


def global_bias(edge_map, alpha, ctx_ids, tokenizer):
    """[T, T] float32 and (pairs, max weight, mean weight)."""
    c = _contents(ctx_ids, tokenizer)
    T = len(c)
    bias = np.zeros((T, T), dtype=np.float32)
    used = []
    for t in range(T):
        for s in range(t):
            wt = edge_map.get((c[s], c[t]), 0.0)
            if wt > 0.0:
                bias[t, s] = alpha * wt
                used.append(wt)
    return _finish(bias, used)
