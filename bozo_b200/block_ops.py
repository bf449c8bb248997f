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
* ``wo_add_rms_norm(x, msg, wo_weight, scale, eps)`` = ``rms_norm(x +
  wo(msg))`` with a bf16 projection (model.py:259, 283 under bf16 autocast),
  forward only: one tensor-core kernel per 128 rows computes the projection
  and applies the add and the norm to its accumulator, so the projection's
  output never goes through device memory.  For prefill, decoding and
  evaluation (no gradients); ``wo_norm_applies`` says when it can be used.
  Off in the model unless ``FUSED_WO_NORM`` is set: on B200 it is still
  slower than the library GEMM followed by ``add_rms_norm`` at every
  measured size (one 128-row tile pulls the whole weight through at most
  eight SMs), so the model keeps the two-kernel path by default.
* ``add_rms_norm_lp(x, y, scale, eps)``: the same for an fp32 stream, also
  returning the output rounded to bf16 — the operand bf16 autocast would
  cast it to for every projection that reads it, made once by the same
  kernel; the backward takes that copy's bf16 cotangent into the kernel
  instead of an fp32 cast and add per projection.
* ``swiglu(g, v)`` = ``silu(g) * v`` (model.py:328-329): one pass each way;
  ``swiglu_packed(gv)`` takes one GEMM's packed ``[g | v]`` rows and returns
  the cotangent in that layout.
* ``embedding(ids, weight)`` = ``F.embedding`` (the token embedding, tied
  to the output head) whose weight gradient is one pass over the sorted ids
  — every vocabulary row written once, each the sum of its tokens' rows in
  position order — instead of the framework's sort-and-scatter kernels.
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

__all__ = ["add_rms_norm", "add_rms_norm_lp", "swiglu", "swiglu_packed", "cross_entropy",
           "norm_applies", "swiglu_applies", "swiglu_packed_applies", "xent_applies",
           "wo_add_rms_norm", "wo_norm_applies", "embedding", "embedding_applies"]

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


def swiglu_packed_applies(gv: Tensor) -> bool:
    return (gv.is_cuda and gv.dtype in _DTYPES and gv.shape[-1] % 8 == 0 and gv.is_contiguous()
            and gv.numel() > 0)


def swiglu_applies(g: Tensor, v: Tensor) -> bool:
    return (g.is_cuda and g.shape == v.shape and g.dtype == v.dtype and g.dtype in _DTYPES
            and g.numel() % 4 == 0)


class _AddRMSNormFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, x, y, scale, eps):
        D = x.shape[-1]
        x2 = x.reshape(-1, D).contiguous()
        y2 = y.reshape(-1, D).contiguous() if y is not None else None
        out, rstd, _ = _capi.ext().add_rmsnorm_fwd(x2, y2, scale.contiguous(), float(eps), False)
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
                                                     scale.contiguous(), rstd, None)
        return (dx.view(ctx.shape), dy.view(ctx.shape) if ctx.has_y else None,
                dscale.to(scale.dtype), None)


class _AddRMSNormLPFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, x, y, scale, eps):
        D = x.shape[-1]
        x2 = x.reshape(-1, D).contiguous()
        y2 = y.reshape(-1, D).contiguous() if y is not None else None
        out, rstd, out_lp = _capi.ext().add_rmsnorm_fwd(x2, y2, scale.contiguous(), float(eps), True)
        ctx.save_for_backward(x2, y2, scale, rstd)
        ctx.has_y = y is not None
        ctx.shape = x.shape
        return out.view(x.shape), out_lp.view(x.shape)

    @staticmethod
    def backward(ctx, d_out, d_out_lp):
        x2, y2, scale, rstd = ctx.saved_tensors
        D = x2.shape[-1]
        d_out = torch.zeros_like(x2) if d_out is None else d_out.reshape(-1, D).contiguous().to(x2.dtype)
        if d_out_lp is not None:
            d_out_lp = d_out_lp.reshape(-1, D).contiguous().to(torch.bfloat16)
        dx, dy, dscale = _capi.ext().add_rmsnorm_bwd(d_out, x2, y2 if ctx.has_y else None,
                                                     scale.contiguous(), rstd, d_out_lp)
        return (dx.view(ctx.shape), dy.view(ctx.shape) if ctx.has_y else None,
                dscale.to(scale.dtype), None)


class _SwiGLUPackedFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, gv):
        shape = gv.shape
        gv2 = gv.reshape(-1, shape[-1])
        ctx.save_for_backward(gv2)
        ctx.shape = shape
        return _capi.ext().swiglu_packed_fwd(gv2).view(*shape[:-1], shape[-1] // 2)

    @staticmethod
    def backward(ctx, dh):
        (gv2,) = ctx.saved_tensors
        dh2 = dh.reshape(gv2.shape[0], -1).contiguous().to(gv2.dtype)
        return _capi.ext().swiglu_packed_bwd(dh2, gv2).view(ctx.shape)


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


_WO_OK = {}
FUSED_WO_NORM = False  # route the model's no-grad wo + add + norm through the fused kernel


def _wo_width_ok(D: int, dtype: torch.dtype) -> bool:
    """Whether the library's kernel takes this width for x of this dtype."""
    key = (D, dtype)
    if key not in _WO_OK:
        code = 1 if dtype == torch.bfloat16 else 0
        _WO_OK[key] = bool(_capi.lib().bozo_wo_add_rmsnorm_supported(D, code))
    return _WO_OK[key]


def wo_norm_applies(x: Tensor, msg: Tensor, weight: Tensor) -> bool:
    """Whether the model routes this call to ``wo_add_rms_norm``:
    ``FUSED_WO_NORM`` set, no gradient wanted, CUDA
    tensors, a supported width, and a projection that would run in bf16 (bf16
    autocast, or bf16 operands)."""
    if not FUSED_WO_NORM:
        return False
    if torch.is_grad_enabled() and (x.requires_grad or msg.requires_grad or weight.requires_grad):
        return False
    if not (x.is_cuda and msg.is_cuda and weight.is_cuda) or x.dtype not in _DTYPES:
        return False
    D = x.shape[-1]
    if msg.shape != x.shape or tuple(weight.shape) != (D, D) or not _wo_width_ok(D, x.dtype):
        return False
    if torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda") == torch.bfloat16
    return msg.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16


def _bf16_weight(weight: Tensor) -> Tensor:
    """A contiguous bf16 copy of ``weight``, kept on the tensor until the
    weight changes (its version counter moves), as autocast keeps its casts."""
    if weight.dtype == torch.bfloat16 and weight.is_contiguous():
        return weight
    key = (weight.data_ptr(), weight._version)
    cached = getattr(weight, "_bozo_bf16", None)
    if cached is None or cached[0] != key:
        with torch.no_grad():
            cached = (key, weight.detach().to(torch.bfloat16).contiguous())
        weight._bozo_bf16 = cached
    return cached[1]


def wo_add_rms_norm(x: Tensor, msg: Tensor, weight: Tensor, scale: Tensor, eps: float) -> Tensor:
    """``rms_norm(x + bf16(msg)·bf16(weight)ᵀ)`` in one kernel, forward only."""
    D = x.shape[-1]
    if x.numel() == 0:
        return torch.empty_like(x)
    x2 = x.reshape(-1, D).contiguous()
    m2 = msg.reshape(-1, D).to(torch.bfloat16).contiguous()
    w2 = _bf16_weight(weight)
    sc = scale.to(x.dtype).contiguous()
    out, _ = _capi.ext().wo_add_rmsnorm_fwd(m2, w2, x2, sc, float(eps))
    return out.view(x.shape)


def add_rms_norm_lp(x: Tensor, y: Optional[Tensor], scale: Tensor, eps: float):
    """``(rms_norm(x + y), rms_norm(x + y).to(bf16))`` for an fp32 stream,
    both from one kernel; gradients flow through both."""
    if scale.dtype != x.dtype:
        scale = scale.to(x.dtype)
    return _AddRMSNormLPFn.apply(x, y, scale, eps)


def swiglu_packed(gv: Tensor) -> Tensor:
    """``silu(g) * v`` for ``g, v = gv.chunk(2, -1)``, without splitting gv."""
    return _SwiGLUPackedFn.apply(gv)


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


def embedding_applies(ids: Tensor, weight: Tensor) -> bool:
    return (weight.is_cuda and weight.dim() == 2 and weight.dtype == torch.float32
            and weight.shape[1] % 4 == 0 and ids.device == weight.device
            and ids.dtype in (torch.long, torch.int) and 0 < ids.numel() < 2 ** 31)


class _EmbeddingFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, ids, weight):
        ctx.save_for_backward(ids)
        ctx.vocab = weight.shape[0]
        return torch.nn.functional.embedding(ids, weight)

    @staticmethod
    def backward(ctx, d_out):
        (ids,) = ctx.saved_tensors
        # stable: equal ids keep increasing positions, the order the rows are summed in
        keys, order = torch.sort(ids.reshape(-1).to(torch.int32), stable=True)
        dim = d_out.shape[-1]
        dw = _capi.ext().embedding_bwd(keys, order, d_out.reshape(-1, dim).float().contiguous(),
                                       ctx.vocab)
        return None, dw


def embedding(ids: Tensor, weight: Tensor) -> Tensor:
    """``weight[ids]`` with the weight gradient of ``bozo_embedding_bwd``."""
    return _EmbeddingFn.apply(ids, weight)
