"""Golden vectors for the TensionLM harness (``bozo_b200/lm.py``), made by the
REFERENCE model on the CPU.

Run once in a container that has the reference checkout, passing its path
with ``--ref PATH`` or the ``BOZO_REFERENCE`` environment variable::

    python tests/golden/make_golden_lm.py

It writes ``tests/golden/golden_lm.npz``: for two small configurations, the
reference ``model.TensionLM`` (model.py:391-480) in float32 with dropout 0,
its parameters (``state_dict``), seeded token ids, and the outputs of the
aux-loss training forward (``return_all=True``, model.py:461-480): logits,
final hidden state, the per-layer τ, the CE loss and the four aux losses
(model.py:487-611), and the gradients of train.py's default total loss
(train.py:1122-1128, w_closure 0.01, w_diversity 0.02) for a few
parameters.  Local layers take the reference's unfold path on the CPU
(model.py:266-283) and global layers the einsum path (model.py:217-237).

* ``rope_global``: RoPE, no oscillation, global layer every 2nd block,
  head_dim 64 and W 64 — the 117M preset's structure at toy width.
* ``norope_osc``: fused ``wkv`` projection, learned positions, oscillatory
  modulation, head_dim 16 — the 1.1M CPU configuration's structure.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))

CONFIGS = {
    "rope_global": dict(cfg=dict(vocab_size=97, dim=128, num_layers=4, num_heads=2, window=64,
                                 ffn_mult=3, max_seq_len=192, dropout=0.0, use_oscillation=False,
                                 use_rope=True, use_triton=False, global_every=2),
                        B=2, T=160, seed=21),
    "norope_osc": dict(cfg=dict(vocab_size=97, dim=64, num_layers=2, num_heads=4, window=8,
                                ffn_mult=3, max_seq_len=48, dropout=0.0, use_oscillation=True,
                                use_rope=False, use_triton=False, global_every=0),
                       B=2, T=40, seed=22),
}

# parameters whose gradients are recorded
GRAD_PARAMS = ("embedding.weight", "blocks.0.tension.wq.weight", "blocks.1.tension.wo.weight",
               "blocks.0.ffn.gate.weight", "final_norm.scale")

W_CLOSURE, W_DIVERSITY, W_CONSISTENCY, W_ENTROPY = 0.01, 0.02, 0.0, 0.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BOZO_REFERENCE"),
                    required="BOZO_REFERENCE" not in os.environ,
                    help="path of the reference checkout (or set BOZO_REFERENCE)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import model as M  # the reference's model.py

    out = {}
    for name, c in CONFIGS.items():
        torch.manual_seed(c["seed"])
        cfg = M.TensionConfig(**c["cfg"])
        lm = M.TensionLM(cfg).float().eval()
        g = torch.Generator().manual_seed(c["seed"] + 1000)
        ids = torch.randint(0, cfg.vocab_size, (c["B"], c["T"] + 1), generator=g)
        inputs, targets = ids[:, :-1], ids[:, 1:]
        logits, hidden, tensions = lm(inputs, return_all=True)
        ce = F.cross_entropy(logits.reshape(-1, cfg.vocab_size), targets.reshape(-1))
        mcl = M.manifold_closure_loss(hidden)
        div = M.tension_diversity_loss(tensions, lm.window_groups)
        cons = M.constraint_consistency_loss(tensions)
        ent = M.tension_entropy_loss(tensions)
        loss = (ce + W_CLOSURE * mcl + W_DIVERSITY * div + W_CONSISTENCY * cons
                + W_ENTROPY * ent)
        loss.backward()
        params = dict(lm.named_parameters())
        for k, v in lm.state_dict().items():
            out[f"{name}/sd.{k}"] = v.detach().cpu().numpy()
        out[f"{name}/inputs"] = inputs.numpy()
        out[f"{name}/targets"] = targets.numpy()
        out[f"{name}/logits"] = logits.detach().numpy()
        out[f"{name}/hidden"] = hidden.detach().numpy()
        for i, t in enumerate(tensions):
            out[f"{name}/tau{i}"] = t.detach().numpy()
        for k, v in (("ce", ce), ("closure", mcl), ("diversity", div), ("consistency", cons),
                     ("entropy", ent), ("loss", loss)):
            out[f"{name}/{k}"] = np.asarray(float(v.detach()))
        for p in GRAD_PARAMS:
            out[f"{name}/grad.{p}"] = params[p].grad.detach().numpy()
        print(name, "params", lm.num_params, "loss", float(loss))
    path = os.path.join(HERE, "golden_lm.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path) // 1024, "KiB")


if __name__ == "__main__":
    main()
