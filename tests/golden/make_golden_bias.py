"""Golden vectors for the device graph bias (``bozo_b200/graph_bias.py``),
made by the REFERENCE ``GraphBias`` (ts_bridge/bias.py:81-233) on the CPU.

Run once in a container that has the reference checkout, passing its path
with ``--ref PATH`` or the ``BOZO_REFERENCE`` environment variable::

    python tests/golden/make_golden_bias.py

It writes ``tests/golden/golden_bias.npz``: a seeded edge map over a small
content vocabulary (some weights ≤ 0, which the reference skips), a
tokenizer whose ``id_to_token`` returns ``None`` for some ids (the ``"<id>"``
fallback), two contexts with repeated tokens, and for each the reference's
``local_bias`` (W = 8) and ``global_bias`` tensors (batch 2) with their
``BiasStats``.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
VOCAB = 24         # token ids 0..23
N_CONTENT = 18     # ids ≥ 18 decode to None → "<id>"
ALPHA = 0.7
W = 8


class FixedTokenizer:
    """id_to_token: ``tok{i}`` for i < N_CONTENT, else None."""

    def id_to_token(self, i):
        return f"tok{i}" if i < N_CONTENT else None


def make_edge_map(seed):
    rng = np.random.default_rng(seed)
    names = [f"tok{i}" for i in range(N_CONTENT)] + ["<20>", "<22>"]
    edges = {}
    for _ in range(150):
        a, b = rng.choice(len(names), 2)
        edges[(names[a], names[b])] = float(np.round(rng.uniform(-0.3, 1.0), 6))
    return edges


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BOZO_REFERENCE"),
                    required="BOZO_REFERENCE" not in os.environ,
                    help="path of the reference checkout (or set BOZO_REFERENCE)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from ts_bridge.bias import GraphBias  # the reference class

    edges = make_edge_map(41)
    gb = GraphBias(edge_map=edges, alpha=ALPHA)
    tok = FixedTokenizer()
    rng = np.random.default_rng(42)
    out = {"edges": np.asarray(json.dumps([[s, d, w] for (s, d), w in edges.items()])),
           "alpha": np.asarray(ALPHA), "W": np.asarray(W)}
    for name, T in (("ctx_a", 40), ("ctx_b", 17)):
        ids = rng.integers(0, VOCAB, T)
        out[f"{name}_ids"] = ids
        lb, ls = gb.local_bias(ids.tolist(), tok, W, batch=2)
        gbias, gs = gb.global_bias(ids.tolist(), tok, batch=2)
        out[f"{name}_local"] = lb.numpy()
        out[f"{name}_local_stats"] = np.array([ls.nonzero_pairs, ls.max_weight, ls.mean_weight])
        out[f"{name}_global"] = gbias.numpy()
        out[f"{name}_global_stats"] = np.array([gs.nonzero_pairs, gs.max_weight, gs.mean_weight])
        print(name, "local pairs", ls.nonzero_pairs, "global pairs", gs.nonzero_pairs)
    path = os.path.join(HERE, "golden_bias.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


if __name__ == "__main__":
    main()
