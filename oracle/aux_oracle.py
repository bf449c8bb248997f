"""CPU oracle for the fused τ-field consumer — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/`` import it.
The shipped consumer (``bozo_b200.aux``) runs on the GPU and raises on CPU
tensors; it never routes through this file.

It restates, in plain PyTorch on the CPU (float64), the reference's three τ
regularisers of BoggersTheFish/bozo as train.py:1083-1087 calls them:

* ``diversity``   — ``model.py:498-532`` (``tension_diversity_loss``): per
  window group, ``relu(log W − mean_r ent_r)`` with ``ent_r`` the entropy of
  the row normalised by ``Σ + 1e-8`` (``+1e-8`` inside the log), averaged
  over groups; groups are the given ``{W: [layer, …]}`` map or, without one,
  the fields' last dimension.
* ``consistency`` — ``model.py:535-577``: mean over ``i < m = min(W−2, 4)``
  and ``t ∈ [i+2, i+2+T−m−1)`` of ``relu(τ[t,i]·τ[t−1,0] − τ[t,i+1])``,
  averaged over the layers with ``W ≥ 3``, ``T ≥ 3`` and ``m+1 < T``.
* ``entropy``     — ``model.py:580-611``: ``relu(0.05 − μ) + relu(μ − 0.8)``
  of the row means ``μ``, averaged over rows, then over layers.
* ``uncertainty_gate`` — ``train.py:411-447``: 1 where the mean over layers
  and heads of the row entropy (first min W slots) exceeds the threshold.

``losses_and_grads`` returns the three values and the gradients of a
weighted sum w.r.t. every field (autograd of these formulas).  Parity is
pinned by ``tests/test_oracle_golden.py`` against ``tests/golden/golden_aux.npz``
(the reference functions themselves, ``tests/golden/make_golden_aux.py``).
"""
from __future__ import annotations

import math
from collections import defaultdict
from typing import Dict, List, Optional, Sequence, Tuple

import torch

EPS = 1e-8  # model.py:527-528


def _groups(taus: Sequence[torch.Tensor], window_groups: Optional[dict]) -> Dict[int, List[int]]:
    if window_groups is not None:
        return {int(W): list(idx) for W, idx in window_groups.items()}
    g: Dict[int, List[int]] = defaultdict(list)
    for i, t in enumerate(taus):
        g[int(t.shape[-1])].append(i)
    return dict(g)


def diversity(taus: Sequence[torch.Tensor], window_groups: Optional[dict] = None) -> torch.Tensor:
    """model.py:498-532."""
    total = taus[0].new_zeros(())
    groups = _groups(taus, window_groups)
    for W, idx in groups.items():
        ents = []
        for i in idx:
            x = taus[i]
            p = x / (x.sum(-1, keepdim=True) + EPS)
            ents.append(-(p * torch.log(p + EPS)).sum(-1).reshape(-1))
        total = total + torch.relu(math.log(W) - torch.cat(ents).mean())
    return total / max(len(groups), 1)


def consistency(taus: Sequence[torch.Tensor]) -> torch.Tensor:
    """model.py:535-577."""
    total = taus[0].new_zeros(())
    count = 0
    for x in taus:
        B, T, H, W = x.shape
        if W < 3 or T < 3:
            continue
        m = min(W - 2, 4)
        if m + 1 >= T:
            continue
        n = T - (m + 1)
        terms = []
        for i in range(m):
            leg1 = x[:, i + 2:i + 2 + n, :, i]
            leg2 = x[:, i + 1:i + 1 + n, :, 0]
            comb = x[:, i + 2:i + 2 + n, :, i + 1]
            terms.append(torch.relu(leg1 * leg2 - comb).reshape(-1))
        total = total + torch.cat(terms).mean()
        count += 1
    return total / max(count, 1)


def entropy(taus: Sequence[torch.Tensor]) -> torch.Tensor:
    """model.py:580-611."""
    total = taus[0].new_zeros(())
    for x in taus:
        mu = x.mean(-1)
        total = total + torch.relu(0.05 - mu).mean() + torch.relu(mu - 0.80).mean()
    return total / len(taus)


def losses_and_grads(taus: Sequence[torch.Tensor], window_groups: Optional[dict] = None,
                     weights: Tuple[float, float, float] = (1.0, 1.0, 1.0),
                     dtype=torch.float64):
    """((diversity, consistency, entropy), [d(w·losses)/dτ_l]) in ``dtype``."""
    xs = [t.detach().to("cpu", dtype).requires_grad_(True) for t in taus]
    d, c, e = diversity(xs, window_groups), consistency(xs), entropy(xs)
    total = weights[0] * d + weights[1] * c + weights[2] * e
    grads = torch.autograd.grad(total, xs, allow_unused=True)
    grads = [g if g is not None else torch.zeros_like(x) for g, x in zip(grads, xs)]
    return (float(d.detach()), float(c.detach()), float(e.detach())), grads


def row_entropy_mean(taus: Sequence[torch.Tensor]) -> torch.Tensor:
    """train.py:431-445: mean over layers and heads of the row entropies of
    the first min W slots, [B, T] float64."""
    min_w = min(t.shape[-1] for t in taus)
    acc = None
    for t in taus:
        x = t[..., :min_w].detach().to("cpu", torch.float64)
        p = x / (x.sum(-1, keepdim=True) + EPS)
        ent = -(p * torch.log(p + EPS)).sum(-1).mean(-1)
        acc = ent if acc is None else acc + ent
    return acc / len(taus)


def uncertainty_gate(taus: Sequence[torch.Tensor], threshold: float = 0.15) -> torch.Tensor:
    """train.py:411-447."""
    return (row_entropy_mean(taus) > threshold).double()
