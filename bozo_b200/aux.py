"""Fused τ-field consumer: the reference's three τ regularisers from one pass
over the exported τ fields.

``tension_aux_losses(all_tensions, window_groups)`` returns the values of
``tension_diversity_loss`` (model.py:498-532), ``constraint_consistency_loss``
(model.py:535-577) and ``tension_entropy_loss`` (model.py:580-611) for the
list of per-layer τ fields a ``return_all`` forward yields, with gradients
w.r.t. every field.  The per-row work — row sums, entropies of the
normalised rows, the transitivity hinges, the mean-τ band penalties — runs in
``bozo_tau_aux_fwd`` (one read of every field, per-layer statistics) and
its cotangent in ``bozo_tau_aux_bwd`` (one read and one write per field,
``include/bozo_tau_aux.h``); ``uncertainty_gate`` (train.py:411-447) reads
the per-row entropies of the same pass.  What remains here are the reference's scalar
tails over those statistics (group means, ``relu(log W − ·)``, the averages),
so their gradient flows back through ordinary autograd into the statistics'
cotangent, which the backward kernel reads on the device.

The statistics are accumulated in fp32/fp64 from the stored τ values; the
reference's framework ops round some intermediates to bf16 under autocast,
so bf16 results agree within bf16 rounding and fp32 results within fp32
summation-order rounding.  CUDA tensors only: there is no CPU path here.
"""
from __future__ import annotations

import math
from collections import defaultdict
from typing import Dict, List, Optional, Sequence, Tuple

import torch
from torch import Tensor

from . import _capi

__all__ = ["tau_field_stats", "tension_aux_losses", "uncertainty_gate"]


class _TauStatsFn(torch.autograd.Function):
    """[L, 3] fp32 statistics of L equally shaped τ fields (see the header).

    Backward: fields that carry a ``_bozo_tau_slot`` (exported by a tension
    call whose backward can form the cotangent itself, ``ops._TauSlot``) get
    their cotangent as per-query-row coefficients in that slot — row mode of
    ``bozo_tau_aux_bwd``, allowed only when the consistency statistic takes
    no gradient (``row_ok``) — and ``None`` here; the others get a
    materialised cotangent."""

    @staticmethod
    def forward(ctx, row_ok: bool, *taus: Tensor) -> Tensor:
        ctx.save_for_backward(*taus)
        ctx.slots = [getattr(t, "_bozo_tau_slot", None) if row_ok else None for t in taus]
        return _capi.ext().tau_aux_fwd(list(taus))

    @staticmethod
    def backward(ctx, d_stats: Tensor):
        taus = ctx.saved_tensors
        d_stats = d_stats.float().contiguous()
        grads: List[Optional[Tensor]] = [None] * len(taus)
        rows = [i for i, sl in enumerate(ctx.slots) if sl is not None]
        mats = [i for i, sl in enumerate(ctx.slots) if sl is None]
        if rows:
            coef = _capi.ext().tau_aux_rowcoef([taus[i] for i in rows],
                                               _take(d_stats, rows).contiguous())
            for j, i in enumerate(rows):
                ctx.slots[i].add(coef[j])
        if mats:
            sub = mats if len(mats) < len(taus) else None
            dts = _capi.ext().tau_aux_bwd([taus[i] for i in mats],
                                          _take(d_stats, sub).contiguous() if sub else d_stats)
            for j, i in enumerate(mats):
                grads[i] = dts[j]
        return (None, *grads)


def tau_field_stats(taus: Sequence[Tensor], row_ok: bool = False) -> Tensor:
    """Per-layer statistics ``[L, 3]``: mean row entropy of ``τ/(Στ+1e-8)``,
    mean transitivity hinge, mean-τ band penalty (``bozo_tau_aux_fwd``).
    Fields of different shapes or dtypes are batched per shape.  ``row_ok``:
    the caller takes no gradient through column 1 (consistency), so fields
    exported with a slot may receive their cotangent per row."""
    if not taus:
        raise ValueError("tau_field_stats: no τ fields")
    for t in taus:
        if not t.is_cuda:
            raise RuntimeError("tau_field_stats: τ fields must be CUDA tensors "
                               "(the fused τ consumer has no CPU path)")
    by_kind: Dict[tuple, List[int]] = defaultdict(list)
    for i, t in enumerate(taus):
        by_kind[(tuple(t.shape), t.dtype)].append(i)
    if len(by_kind) == 1:
        return _TauStatsFn.apply(row_ok, *[t.contiguous() for t in taus])
    rows: List[Optional[Tensor]] = [None] * len(taus)
    for idx in by_kind.values():
        st = _TauStatsFn.apply(row_ok, *[taus[i].contiguous() for i in idx])
        for j, i in enumerate(idx):
            rows[i] = st[j]
    return torch.stack(rows)


def _consistency_applies(shape: torch.Size) -> bool:
    """model.py:551-562: layers with W < 3, T < 3 or no live slot are skipped."""
    _, T, _, W = shape
    if W < 3 or T < 3:
        return False
    return min(W - 2, 4) + 1 < T


_index_cache: Dict[tuple, Tensor] = {}


def _take(col: Tensor, idx: List[int]) -> Tensor:
    """``col[idx]`` without copying a host index list to the device on every
    call (a pageable copy per loss term, and one a CUDA graph cannot hold): a
    slice when ``idx`` is a contiguous run, else an index tensor made once
    per (device, idx)."""
    idx = list(idx)
    if idx == list(range(idx[0], idx[0] + len(idx))):
        return col[idx[0]:idx[0] + len(idx)]
    key = (col.device, tuple(idx))
    ix = _index_cache.get(key)
    if ix is None:
        ix = _index_cache[key] = torch.tensor(idx, dtype=torch.long, device=col.device)
    return col.index_select(0, ix)


def tension_aux_losses(all_tensions: Sequence[Tensor], window_groups: Optional[dict] = None,
                       grad_consistency: bool = True) -> Tuple[Tensor, Tensor, Tensor]:
    """(diversity, consistency, entropy) of model.py:498-611 for the per-layer
    τ fields, as fp32 scalars with gradients w.r.t. every field.

    ``grad_consistency=False`` (a caller whose consistency weight is 0, as
    train.py's default): the consistency value is returned without a
    gradient, which is what a zero weight makes of it anyway, and fields
    exported by the local tensor-core kernels then receive the diversity and
    entropy cotangents per query row, formed inside the tension backward
    instead of being written out and read back."""
    if not all_tensions:
        z = torch.tensor(0.0)
        return z, z, z
    stats = tau_field_stats(all_tensions, row_ok=not grad_consistency)
    # diversity (model.py:511-532): per window group, relu(log W − mean entropy)
    if window_groups is not None:
        groups = {W: list(idx) for W, idx in window_groups.items()}
    else:
        groups = defaultdict(list)
        for i, t in enumerate(all_tensions):
            groups[t.shape[-1]].append(i)
    div = stats.new_zeros(())
    for W, idx in groups.items():
        # every field of a group has N = B·T·H rows, so the mean of the
        # per-layer means is the mean over the stacked rows
        ent = _take(stats[:, 0], idx).mean()
        div = div + torch.relu(math.log(W) - ent)
    div = div / max(len(groups), 1)
    # consistency (model.py:548-577): average over the layers that apply
    live = [i for i, t in enumerate(all_tensions) if _consistency_applies(t.shape)]
    cons_col = stats[:, 1] if grad_consistency else stats[:, 1].detach()
    cons = _take(cons_col, live).sum() / max(len(live), 1) if live else stats.new_zeros(())
    # entropy regulariser (model.py:597-611): average over all layers
    ent_loss = stats[:, 2].sum() / len(all_tensions)
    return div, cons, ent_loss


def uncertainty_gate(tensions: Sequence[Tensor], threshold: float = 0.15) -> Tensor:
    """train.py:411-447: [B, T] float mask, 1 where the mean over layers and
    heads of the row entropy of ``τ/(Στ+1e-8)`` (over the first min W slots)
    exceeds ``threshold``.  The entropies come from the statistics pass
    (``bozo_tau_aux_fwd`` with ``row_ent``), one read of every field; fields
    wider than the narrowest are cut to its width first, as the reference
    does.  No gradient (the reference computes it under ``no_grad``)."""
    if not tensions:
        raise ValueError("uncertainty_gate: no τ fields")
    with torch.no_grad():
        min_w = min(t.shape[-1] for t in tensions)
        fields = [t if t.shape[-1] == min_w else t[..., :min_w] for t in tensions]
        for t in fields:
            if not t.is_cuda:
                raise RuntimeError("uncertainty_gate: τ fields must be CUDA tensors")
        B, T, H, _ = fields[0].shape
        by_kind: Dict[tuple, List[int]] = defaultdict(list)
        for i, t in enumerate(fields):
            by_kind[(tuple(t.shape), t.dtype)].append(i)
        sum_ent = torch.zeros(B, T, device=fields[0].device, dtype=torch.float32)
        for idx in by_kind.values():
            ent = _capi.ext().tau_row_entropy([fields[i].contiguous() for i in idx])
            sum_ent += ent.view(len(idx), B, T, H).mean(-1).sum(0)
        mean_ent = sum_ent / len(fields)
        return (mean_ent > threshold).float()
