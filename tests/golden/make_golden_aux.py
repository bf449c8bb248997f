"""Golden vectors for the fused τ consumer (``bozo_b200/aux.py``), made by the
REFERENCE loss functions on the CPU.

Run once in a container that has the reference checkout, passing its path
with ``--ref PATH`` or the ``BOZO_REFERENCE`` environment variable::

    python tests/golden/make_golden_aux.py

It writes ``tests/golden/golden_aux.npz``: for a few sets of seeded fp32 τ
fields, the masks of the reference ``uncertainty_gate`` (train.py:411-447)
at the thresholds ``GATE_THRESHOLDS``, and the values of the reference
``tension_diversity_loss``
(model.py:498-532), ``constraint_consistency_loss`` (model.py:535-577) and
``tension_entropy_loss`` (model.py:580-611), and the gradients w.r.t. every
field of ``W_DIV·div + W_CONS·cons + W_ENT·ent`` (all weights non-zero, so
every term's backward is pinned, unlike train.py's defaults).  The fields
mimic exported τ: sigmoid values with the slots before the sequence start
zeroed, and rows pushed towards 0 or 1 so both relu branches of the entropy
regulariser and the transitivity hinge are live.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (shape [B,T,H,W], layers, window_groups or None, seed)
CASES = {
    # local layers plus one wider-keyed group, as TensionLM.window_groups has it
    "grouped": ((2, 40, 3, 16), 4, {16: [0, 1, 2], 40: [3]}, 31),
    # odd width (scalar path of the kernels), m = 3
    "odd_w": ((1, 12, 2, 5), 2, None, 32),
    # W = 3 → one transitivity slot
    "w3": ((2, 9, 2, 3), 2, None, 33),
    # T too short for any slot: consistency skips every layer
    "short_t": ((2, 4, 2, 8), 2, None, 34),
    # fp32 vector path with W = 8: slot 4 in the second lane of a row
    "w8": ((2, 24, 2, 8), 3, {8: [0, 1, 2]}, 35),
}
W_DIV, W_CONS, W_ENT = 1.0, 0.7, 0.3
GATE_THRESHOLDS = (0.15, 1.0, 2.0)


def make_fields(shape, n, seed):
    B, T, H, W = shape
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        x = torch.randn(B, T, H, W, generator=g) * 1.5
        # per-row offsets push some rows towards 0 or 1 (mean-τ band penalties)
        off = torch.randint(-1, 2, (B, T, H, 1), generator=g).float() * 4.0
        tau = torch.sigmoid(x + off)
        # slot w of query t sees key t − (W − w): zero before the sequence start
        t = torch.arange(T).view(1, T, 1, 1)
        w = torch.arange(W).view(1, 1, 1, W)
        tau = tau * ((t - (W - w)) >= 0).float()
        out.append(tau)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BOZO_REFERENCE"),
                    required="BOZO_REFERENCE" not in os.environ,
                    help="path of the reference checkout (or set BOZO_REFERENCE)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import model as M  # the reference's model.py
    import train as TR  # the reference's train.py (uncertainty_gate)

    out = {}
    for name, (shape, n, groups, seed) in CASES.items():
        fields = [t.clone().requires_grad_(True) for t in make_fields(shape, n, seed)]
        div = M.tension_diversity_loss(fields, groups)
        cons = M.constraint_consistency_loss(fields)
        ent = M.tension_entropy_loss(fields)
        total = W_DIV * div + W_CONS * cons + W_ENT * ent
        total.backward()
        for k, th in enumerate(GATE_THRESHOLDS):
            out[f"{name}/gate{k}"] = TR.uncertainty_gate([t.detach() for t in fields], th).numpy()
        for i, t in enumerate(fields):
            out[f"{name}/tau{i}"] = t.detach().numpy()
            out[f"{name}/grad{i}"] = t.grad.numpy()
        out[f"{name}/diversity"] = np.asarray(float(div))
        out[f"{name}/consistency"] = np.asarray(float(cons))
        out[f"{name}/entropy"] = np.asarray(float(ent))
        out[f"{name}/groups"] = np.asarray(repr(groups))
        print(name, "div", float(div), "cons", float(cons), "ent", float(ent))
    path = os.path.join(HERE, "golden_aux.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path) // 1024, "KiB")


if __name__ == "__main__":
    main()
