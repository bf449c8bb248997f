"""Fused elementwise work around the tension operator in a TensionLM block
(``include/bozo_block_ops.h``): residual add + RMSNorm and SwiGLU, forward
and backward, as autograd functions.

* ``add_rms_norm(x, y, scale, eps)`` = ``rms_norm(x + y)`` (model.py:86-98
  after the residual adds of model.py:259, 283, 330; ``y=None`` for the
  pre-norm and the final norm): one kernel reads x and y and writes the
  output and a per-row rstd; the backward recomputes x + y and writes dx,
  dy and the scale's gradient (fixed-order partial sums).  Output in x's
  dtype — fp32 for the model's fp32 residual stream, as ``rms_norm`` gives
  under bf16 autocast.
* ``swiglu(g, v)`` = ``silu(g) * v`` (model.py:328-329): one pass each way.
* ``cross_entropy(logits, targets)`` = ``F.cross_entropy`` (train.py:920,
  mean over targets ≠ −100) from the logits in their own dtype: one pass
  for the per-row logsumexp, one for the gradient, no fp32 copy.

``applies(...)`` says whether a call can take the kernels (CUDA tensors,
contiguous rows of width 128·{1, 2, 4, 6, 8} for the norm, a multiple of 4
elements for SwiGLU, fp32/bf16); ``bozo_b200.lm`` uses them where they apply
and the framework ops elsewhere (CPU runs of the harness, other widths).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import _capi

__all__ = ["add_rms_norm", "swiglu", "cross_entropy", "norm_applies", "swiglu_applies",
           "xent_applies"]

_WIDTHS = {128, 256, 512, 768, 1024}
_DTYPES = (torch.float32, torch.bfloat16)


def norm_applies(x: Tensor, y: Optional[Tensor]) -> bool:
    if not x.is_cuda or x.shape[-1] not in _WIDTHS or x.dtype not in _DTYPES:
        return False
    if y is not None:
        if y.shape != x.shape or y.dtype not in _DTYPES or y.device != x.device:
            return False
        if x.dtype == torch.bfloat16 and y.dtype != torch.bfloat16:
            return False
    return True


def swiglu_applies(g: Tensor, v: Tensor) -> bool:
    return (g.is_cuda and g.shape == v.shape and g.dtype == v.dtype and g.dtype in _DTYPES
            and g.numel() % 4 == 0)


class _AddRMSNormFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, x, y, scale, eps):
        D = x.shape[-1]
        x2 = x.reshape(-1, D).contiguous()
        y2 = y.reshape(-1, D).contiguous() if y is not None else None
        out, rstd = _capi.ext().add_rmsnorm_fwd(x2, y2, scale.contiguous(), float(eps))
        ctx.save_for_backward(x2, y2, scale, rstd)
        ctx.has_y = y is not None
        ctx.shape = x.shape
        return out.view(x.shape)

    @staticmethod
    def backward(ctx, d_out):
        x2, y2, scale, rstd = ctx.saved_tensors
        D = x2.shape[-1]
        dx, dy, dscale = _capi.ext().add_rmsnorm_bwd(d_out.reshape(-1, D).contiguous().to(x2.dtype),
                                                     x2, y2 if ctx.has_y else None,
                                                     scale.contiguous(), rstd)
        return (dx.view(ctx.shape), dy.view(ctx.shape) if ctx.has_y else None,
                dscale.to(scale.dtype), None)


class _SwiGLUFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, g, v):
        g2, v2 = g.contiguous(), v.contiguous()
        ctx.save_for_backward(g2, v2)
        return _capi.ext().swiglu_fwd(g2, v2)

    @staticmethod
    def backward(ctx, dh):
        g2, v2 = ctx.saved_tensors
        dg, dv = _capi.ext().swiglu_bwd(dh.contiguous().to(g2.dtype), g2, v2)
        return dg, dv


def add_rms_norm(x: Tensor, y: Optional[Tensor], scale: Tensor, eps: float) -> Tensor:
    """``rms_norm(x + y)`` (or ``rms_norm(x)``) through the fused kernels."""
    if scale.dtype != x.dtype:
        scale = scale.to(x.dtype)
    return _AddRMSNormFn.apply(x, y, scale, eps)


def swiglu(g: Tensor, v: Tensor) -> Tensor:
    """``silu(g) * v`` through the fused kernels."""
    return _SwiGLUFn.apply(g, v)


def xent_applies(logits: Tensor, targets: Tensor) -> bool:
    return (logits.is_cuda and logits.dim() == 2 and logits.dtype in _DTYPES
            and logits.shape[1] % (8 if logits.dtype == torch.bfloat16 else 4) == 0
            and targets.dtype == torch.long and targets.shape == logits.shape[:1])


class _CrossEntropyFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, logits, targets):
        lg, tg = logits.contiguous(), targets.contiguous()
        row_loss, lse = _capi.ext().cross_entropy_fwd(lg, tg)
        live = (tg != -100).sum().clamp(min=1).float()
        ctx.save_for_backward(lg, tg, lse, live)
        return row_loss.sum() / live

    @staticmethod
    def backward(ctx, d_mean):
        lg, tg, lse, live = ctx.saved_tensors
        g = (d_mean.float() / live).reshape(1).contiguous()
        return _capi.ext().cross_entropy_bwd(lg, tg, lse, g), None


def cross_entropy(logits: Tensor, targets: Tensor) -> Tensor:
    """Mean cross-entropy of ``logits [R, V]`` against ``targets [R]`` (fp32)."""
    return _CrossEntropyFn.apply(logits, targets)
