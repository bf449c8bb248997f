"""Autograd front-ends of the B200 tension operator.

* ``causal_tension`` — drop-in for ``triton_tension.causal_tension``
  (reference triton_tension/ops.py:192-224): same signature, same raw
  (unnormalised) Σ τ·V output, same optional ``[B,T,H,W]`` τ, same bias
  contract (``[B,T,W]``, fp32, no gradient; ops.py:90-100, 184-187), outputs
  in ``Q.dtype`` and gradients in each input's dtype (ops.py:122-124,
  186-187).  Unlike the reference there is no CPU/float64 branch
  (ops.py:217-219): such inputs raise.
* ``tension`` — the fused entry point: RoPE on Q/K (model.py:200-204), local
  window or global full-causal mode (model.py:217-237), the model's τ-mass
  (model.py:257-258) or position-count (model.py:261-264) normalisation and
  optional τ export, in one forward and one backward kernel family.

Both call the C ABI (``include/bozo_tension.h``) through ``_capi`` on the
caller's current CUDA stream.
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Optional, Tuple

import torch
from torch import Tensor

from . import _capi

_DT = {torch.float32: _capi.DT_F32, torch.bfloat16: _capi.DT_BF16,
       torch.float16: _capi.DT_F16}
_NORM = {None: _capi.NORM_NONE, "none": _capi.NORM_NONE, "mass": _capi.NORM_MASS,
         "count": _capi.NORM_COUNT}
_PATH = {"auto": _capi.PATH_AUTO, "simt": _capi.PATH_SIMT, "tcgen05": _capi.PATH_TCGEN05}

# Kernel-path override for tests and benchmarks ("auto", "simt", "tcgen05").
_path_override = "auto"


def set_kernel_path(path: str) -> None:
    """Select the kernel family: "auto" (default), "simt" or "tcgen05"."""
    global _path_override
    if path not in _PATH:
        raise ValueError(f"unknown kernel path {path!r}")
    _path_override = path


def _dt(t) -> int:
    """ABI dtype code of a tensor or a torch.dtype (TypeError if unsupported)."""
    dtype = t if isinstance(t, torch.dtype) else t.dtype
    try:
        return _DT[dtype]
    except KeyError:
        raise TypeError(f"bozo tension: unsupported dtype {dtype} "
                        "(float32, bfloat16 and float16 are supported)") from None


def _t4(t: Optional[Tensor]) -> _capi.Tensor4:
    s = _capi.Tensor4()
    if t is None:
        return s
    s.ptr = t.data_ptr()
    s.dtype = _dt(t)
    for i in range(4):
        s.stride[i] = t.stride(i)
    return s


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _require_cuda(*ts: Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("bozo tension runs on CUDA only (no CPU fallback); "
                               f"got a tensor on {t.device}")
        if t.dim() != 4:
            raise ValueError(f"expected a 4-D [B,T,H,HD] tensor, got shape {tuple(t.shape)}")
    dev = ts[0].device
    for t in ts[1:]:
        if t.device != dev:
            raise RuntimeError("bozo tension: all tensors must be on one device")


_rope_cache: dict = {}


def rope_tables(head_dim: int, length: int, base: float, device):
    """fp32 (cos, sin) ``[length, HD/2]`` and θ ``[HD/2]`` built exactly as
    model.py:66-73 does (cos[t][i] = cos(fl(t·θ_i)))."""
    key = (head_dim, length, float(base), str(device))
    tab = _rope_cache.get(key)
    if tab is None:
        half = head_dim // 2
        theta = 1.0 / (base ** (torch.arange(0, half).float() / half))
        freqs = torch.outer(torch.arange(length).float(), theta)
        tab = (freqs.cos().contiguous().to(device), freqs.sin().contiguous().to(device),
               theta.contiguous().to(device))
        _rope_cache[key] = tab
    return tab


def _fill_common(a, B, T, H, HD, mode, window, norm, scale, rope):
    a.B, a.T, a.H, a.HD = B, T, H, HD
    a.mode, a.window, a.normalize = mode, window, norm
    a.path = _PATH[_path_override]
    a.scale = float(scale)
    if rope is not None:
        cos, sin, theta = rope
        a.rope_len = cos.shape[0]
        a.rope_cos, a.rope_sin, a.rope_theta = cos.data_ptr(), sin.data_ptr(), theta.data_ptr()
    else:
        a.rope_len = 0


def _bias_arg(a, bias: Optional[Tensor]):
    if bias is not None:
        a.bias = bias.data_ptr()
        for i in range(3):
            a.bias_stride[i] = bias.stride(i)


def _rope_args(rope):
    return rope if rope is not None else (None, None, None)


def _launch_fwd(q, k, v, *, mode, window, norm, scale, rope, bias, tau_width,
                out_dtype, tau_dtype, want_mass, want_rotated=False, want_lp=False):
    """One forward through the C ABI (via the C++ extension); returns
    (out, tau, row_mass, q_rot, k_rot) with None for outputs not asked for,
    and with ``want_lp`` also (q_lp, k_lp): the bf16 operand copies of fp32
    q/k the tensor-core path computed from (None when it did not)."""
    cos, sin, theta = _rope_args(rope)
    res = _capi.ext().tension_fwd(
        q, k, v, mode, window, norm, float(scale), _PATH[_path_override], cos, sin, theta,
        bias, tau_width or 0, _dt(out_dtype), _dt(tau_dtype), bool(want_mass),
        bool(want_rotated), bool(want_lp))
    return tuple(res) if want_lp else tuple(res[:5])


def _launch_bwd(q, k, v, d_out, *, mode, window, norm, scale, rope, bias, out,
                mass, d_tau, qk_rotated=False, aux_row=None, grad_dtypes=None):
    """One backward through the C ABI (via the C++ extension); returns
    (dq, dk, dv) in the dtypes of q, k, v, or dq/dk in ``grad_dtypes``
    (used when q, k are the forward's bf16 copies of fp32 inputs).
    ``aux_row`` ([3, B·H·T] fp32): a per-query-row cotangent of τ the
    tensor-core kernel forms itself (``bozo_tension_bwd_args.aux_row``)."""
    cos, sin, theta = _rope_args(rope)
    gq, gk = ((_dt(grad_dtypes[0]), _dt(grad_dtypes[1])) if grad_dtypes is not None
              else (-1, -1))
    dq, dk, dv = _capi.ext().tension_bwd(
        q, k, v, d_out, mode, window, norm, float(scale), _PATH[_path_override], cos, sin,
        theta, bias, out, mass, d_tau, bool(qk_rotated), aux_row, gq, gk)
    return dq, dk, dv


class _TauSlot:
    """Per-query-row cotangent of an exported τ field ([a1 | a0 | 1/D] planes
    over B·H·T rows), left by the fused τ consumer's backward
    (``bozo_b200.aux``) for the backward of the tension call that exported
    the field, which forms the per-element cotangent itself instead of
    reading a materialised one.  Attached to the τ tensor as
    ``_bozo_tau_slot``."""

    __slots__ = ("row",)

    def __init__(self):
        self.row = None

    def add(self, coef: Tensor) -> None:
        # a second consumer of the same field: the a1 and a0 planes add, 1/D is shared
        if self.row is None:
            self.row = coef
        else:
            self.row = torch.cat([self.row[:2] + coef[:2], self.row[2:]])

    def take(self) -> Optional[Tensor]:
        row, self.row = self.row, None
        return row


def _row_cotangent_ok(q: Tensor, k: Tensor, v: Tensor, mode: int, window: int) -> bool:
    """The exported τ of this call can take its consumer's cotangent per row:
    local window on the tensor-core band kernels (bf16, HD 64) with a width
    the row-mode consumer serves (W = 32, 64, 128)."""
    return (mode == _capi.MODE_LOCAL and window in (32, 64, 128) and q.shape[3] == 64
            and q.dtype == k.dtype == v.dtype == torch.bfloat16
            and _path_override != "simt")


def _prep_bias(bias: Optional[Tensor], shape: tuple) -> Optional[Tensor]:
    if bias is None:
        return None
    b = bias.to(torch.float32)
    # same contract and message as triton_tension/ops.py:93-97
    assert b.ndim == 3 and tuple(b.shape) == shape, (
        f"bias must be [B, T, W]=[{shape[0]}, {shape[1]}, {shape[2]}], got {tuple(b.shape)}")
    return b


# ───────────────────────── drop-in raw operator ─────────────────────────
#
# The forward and backward launches are torch.library custom ops with fake
# (shape-only) implementations, so torch.compile (train.py:776-780 compiles
# model.py, whose local layers call this op) traces through the autograd
# function instead of breaking the graph at it.  Absent outputs are empty
# tensors: an op returns tensors only.

def _wants_lp(Q: Tensor, K: Tensor, V: Tensor) -> bool:
    """fp32 Q/K with bf16 V (model.py's autocast call): the forward makes bf16
    operand copies of Q/K, which the tensor cores compute from and the
    backward takes as its Q/K."""
    return Q.dtype == torch.float32 and K.dtype == torch.float32 and V.dtype == torch.bfloat16


@torch.library.custom_op("bozo::causal_tension_fwd", mutates_args=(), device_types="cuda")
def _causal_fwd_op(Q: Tensor, K: Tensor, V: Tensor, W: int, scale: float, return_tau: bool,
                   bias: Optional[Tensor], path: int) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    cos = sin = theta = None
    out, tau, _, _, _, q_lp, k_lp = _capi.ext().tension_fwd(
        Q, K, V, _capi.MODE_LOCAL, W, _capi.NORM_NONE, float(scale), path, cos, sin, theta, bias,
        W if return_tau else 0, _dt(Q), _dt(Q), False, False, _wants_lp(Q, K, V))
    none_f = Q.new_empty(0)
    none_b = Q.new_empty(0, dtype=torch.bfloat16)
    return (out, tau if tau is not None else none_f, q_lp if q_lp is not None else none_b,
            k_lp if k_lp is not None else none_b.clone())


@_causal_fwd_op.register_fake
def _(Q, K, V, W, scale, return_tau, bias, path):
    B, T, H, HD = Q.shape
    out = Q.new_empty((B, T, H, HD))
    tau = Q.new_empty((B, T, H, W)) if return_tau else Q.new_empty(0)
    lp = _wants_lp(Q, K, V)
    q_lp = Q.new_empty((B, T, H, HD) if lp else (0,), dtype=torch.bfloat16)
    k_lp = Q.new_empty((B, T, H, HD) if lp else (0,), dtype=torch.bfloat16)
    return out, tau, q_lp, k_lp


@torch.library.custom_op("bozo::causal_tension_bwd", mutates_args=(), device_types="cuda")
def _causal_bwd_op(Q: Tensor, K: Tensor, V: Tensor, d_out: Tensor, d_tau: Optional[Tensor], W: int,
                   scale: float, bias: Optional[Tensor], path: int, dq_dtype: int,
                   dk_dtype: int) -> Tuple[Tensor, Tensor, Tensor]:
    dq, dk, dv = _capi.ext().tension_bwd(
        Q, K, V, d_out, _capi.MODE_LOCAL, W, _capi.NORM_NONE, float(scale), path, None, None,
        None, bias, None, None, d_tau, False, None, dq_dtype, dk_dtype)
    return dq, dk, dv


_DT_BACK = {v: k for k, v in _DT.items()}


@_causal_bwd_op.register_fake
def _(Q, K, V, d_out, d_tau, W, scale, bias, path, dq_dtype, dk_dtype):
    dq = Q.new_empty(Q.shape, dtype=_DT_BACK[dq_dtype] if dq_dtype >= 0 else Q.dtype)
    dk = K.new_empty(K.shape, dtype=_DT_BACK[dk_dtype] if dk_dtype >= 0 else K.dtype)
    return dq, dk, V.new_empty(V.shape)


class _CausalTensionFn(torch.autograd.Function):
    """Mirror of triton_tension/ops.py:73-187 over the C ABI.

    model.py's call under bf16 autocast (fp32 RoPE-promoted Q/K, bf16 V;
    model.py:200-204, 248-264) runs on the tensor cores: the forward makes
    bf16 operand copies of Q and K, returns fp32 out and τ, and keeps the
    copies for the backward, which returns fp32 dQ/dK and bf16 dV."""

    @staticmethod
    def forward(ctx, Q, K, V, W: int, scale: float, return_tau: bool, bias):
        B, T, H, HD = Q.shape
        Bias = _prep_bias(bias, (B, T, W))
        path = _PATH[_path_override]
        out, tau, q_lp, k_lp = _causal_fwd_op(Q, K, V, W, float(scale), bool(return_tau), Bias, path)
        ctx.grad_dtypes = (-1, -1)
        if _wants_lp(Q, K, V):
            ctx.save_for_backward(q_lp, k_lp, V, Bias)
            ctx.grad_dtypes = (_dt(Q), _dt(K))
        else:
            ctx.save_for_backward(Q, K, V, Bias)
        ctx.W, ctx.scale, ctx.return_tau, ctx.path = W, scale, return_tau, path
        if return_tau:
            return out, tau
        return out

    @staticmethod
    def backward(ctx, *grads):
        Q, K, V, Bias = ctx.saved_tensors
        d_out = grads[0]
        d_tau = grads[1] if ctx.return_tau else None
        if d_out is None:
            d_out = torch.zeros_like(Q)
        if d_tau is not None:
            d_tau = d_tau.contiguous()
        dq, dk, dv = _causal_bwd_op(Q, K, V, d_out, d_tau, ctx.W, float(ctx.scale), Bias,
                                    ctx.path, ctx.grad_dtypes[0], ctx.grad_dtypes[1])
        return dq, dk, dv, None, None, None, None


def causal_tension(Q: Tensor, K: Tensor, V: Tensor, window: int, scale: float,
                   return_tau: bool = False, bias: Tensor | None = None):
    """Fused causal sigmoid tension — drop-in for triton_tension.causal_tension.

    Q, K, V : [B, T, H, HD] CUDA tensors (float32 / bfloat16 / float16, any
              strides, dtypes may differ).
    window  : causal look-back W (self excluded).
    scale   : dot-product divisor (√HD in model.py).
    return_tau : also return τ [B, T, H, W] (dtype of Q).
    bias    : optional [B, T, W] pre-sigmoid bias, broadcast over heads.

    Returns raw out [B, T, H, HD] = Σ τ·V (dtype of Q) or (out, tau).
    """
    _require_cuda(Q, K, V)
    if int(window) < 1:
        raise ValueError("window must be >= 1")
    return _CausalTensionFn.apply(Q, K, V, int(window), float(scale), bool(return_tau), bias)


# ───────────────────────── fused entry point ─────────────────────────

class _TensionFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, q, k, v, mode, window, tau_width, norm, scale, rope_base,
                rope_len, bias, return_tau):
        B, T, H, HD = q.shape
        rope = (rope_tables(HD, rope_len, rope_base, q.device)
                if rope_base is not None else None)
        if bias is not None:
            shape = (B, T, T) if mode == _capi.MODE_GLOBAL else (B, T, window)
            bias = _prep_bias(bias, shape)
        w_arg = window if mode == _capi.MODE_LOCAL else (tau_width or 0)
        # for training the forward also writes RoPE(q), RoPE(k); the backward
        # then reads the rotated tiles instead of rotating them again.  The
        # key-tile streaming forward (global block, windows over 128 keys)
        # always reads rotated copies.
        rotated = rope is not None and (any(ctx.needs_input_grad[:3])
                                        or mode == _capi.MODE_GLOBAL or window > 128)
        out, tau, mass, q_rot, k_rot = _launch_fwd(
            q, k, v, mode=mode, window=w_arg, norm=norm, scale=scale, rope=rope,
            bias=bias, tau_width=(w_arg if return_tau else None), out_dtype=q.dtype,
            tau_dtype=q.dtype, want_mass=True, want_rotated=rotated)
        if q_rot is not None:
            ctx.save_for_backward(q_rot, k_rot, v, out, mass, bias)
        else:
            ctx.save_for_backward(q, k, v, out, mass, bias)
        ctx.qk_rotated = q_rot is not None
        ctx.cfg = (mode, w_arg, norm, scale, rope_base, rope_len, return_tau)
        ctx.mark_non_differentiable(mass)
        # an unused τ (or out) arrives as None in the backward, not as zeros
        ctx.set_materialize_grads(False)
        ctx.tau_slot = None
        if return_tau and _row_cotangent_ok(q, k, v, mode, w_arg):
            ctx.tau_slot = tau._bozo_tau_slot = _TauSlot()
        if return_tau:
            return out, tau
        return out

    @staticmethod
    def backward(ctx, *grads):
        q, k, v, out, mass, bias = ctx.saved_tensors
        mode, w_arg, norm, scale, rope_base, rope_len, return_tau = ctx.cfg
        d_out = grads[0]
        if d_out is None:
            d_out = torch.zeros_like(out)
        d_tau = grads[1] if return_tau else None
        if d_tau is not None:
            d_tau = d_tau.contiguous()
        aux_row = ctx.tau_slot.take() if ctx.tau_slot is not None else None
        if aux_row is not None:
            d_out = d_out.contiguous()  # the tensor-core kernel's TMA view
        rope = (rope_tables(q.shape[3], rope_len, rope_base, q.device)
                if rope_base is not None else None)
        dq, dk, dv = _launch_bwd(q, k, v, d_out, mode=mode, window=w_arg, norm=norm,
                                 scale=scale, rope=rope, bias=bias, out=out, mass=mass,
                                 d_tau=d_tau, qk_rotated=ctx.qk_rotated, aux_row=aux_row)
        return dq, dk, dv, None, None, None, None, None, None, None, None, None


@torch._dynamo.disable
def tension(q: Tensor, k: Tensor, v: Tensor, *, window: Optional[int],
            scale: Optional[float] = None, rope_base: Optional[float] = 10_000.0,
            rope_len: Optional[int] = None, bias: Optional[Tensor] = None,
            return_tau: bool = False, normalize: Optional[str] = "mass",
            tau_window: Optional[int] = None):
    """Fused tension layer core: RoPE → tension → normalisation (+ τ export).

    q, k, v    : [B, T, H, HD] pre-RoPE projections (CUDA).
    window     : local look-back W, or ``None`` for the global full-causal mode
                 (self included, model.py:217-237).
    scale      : dot divisor, default √HD (model.py:122).
    rope_base  : RoPE base (model.py:66) or ``None`` for no rotation.
    rope_len   : rows of the RoPE table (model.py uses max_seq_len; only rows
                 < T are read), default T.
    bias       : [B, T, W] (local) / [B, T, T] (global) pre-sigmoid bias.
    normalize  : "mass" (model.py:257-258), "count" (model.py:261-264, local
                 only) or None (raw Σ τ·V).
    return_tau : also return τ; local → [B,T,H,W], global → the reference's
                 exported window [B,T,H,min(tau_window,T)] (model.py:235-236).
    tau_window : global mode only — the model's local W that sizes the
                 exported τ window (required with return_tau).
    """
    _require_cuda(q, k, v)
    B, T, H, HD = q.shape
    if scale is None:
        scale = math.sqrt(HD)
    if window is None:
        mode = _capi.MODE_GLOBAL
        if normalize == "count":
            raise ValueError("normalize='count' is defined for local windows only")
        if return_tau and not tau_window:
            raise ValueError("global mode exports τ over the model's local window: "
                             "pass tau_window (model.py:235 uses min(window, T))")
        tw = min(int(tau_window), T) if tau_window else 0
        win = 0
    else:
        mode, win, tw = _capi.MODE_LOCAL, int(window), None
        if win < 1:
            raise ValueError("window must be >= 1")
    return _TensionFn.apply(q, k, v, mode, win, tw, _NORM[normalize], float(scale),
                            rope_base, int(rope_len or T), bias, bool(return_tau))


def last_path() -> str:
    """Kernel family of the last call on this thread ("simt"/"tcgen05")."""
    return {0: "none", 1: "simt", 2: "tcgen05"}[_capi.lib().bozo_tension_last_path()]


def last_launches() -> int:
    return _capi.lib().bozo_tension_last_launches()


def poll_device_error(device=None) -> None:
    """Synchronise and raise if a bounded device-side wait timed out (the
    error word is cleared by the read)."""
    dev = torch.device(device) if device is not None else torch.device("cuda")
    with torch.cuda.device(dev):
        code = _capi.lib().bozo_tension_poll_error(_stream(dev))
    _capi.check(code, "device error poll")


class _ErrorWatch:
    """Per-device state of ``check_device_error``: a pinned host word the
    error word is copied into, and the event that marks the copy."""

    def __init__(self):
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = None


_watch: dict = {}


def check_device_error(device=None) -> None:
    """Non-blocking check of the device error word, for once-per-step use.

    Reads the word copied by the previous call if that copy has completed
    (no synchronisation), raises through ``poll_device_error`` when a bounded
    wait gave up in some earlier launch, then enqueues the next asynchronous
    copy on the current stream.  A timeout is thus reported at most one step
    late instead of never; nothing is enqueued while the stream is capturing
    a CUDA graph."""
    if torch.cuda.is_current_stream_capturing():
        return  # no event query or copy may join a graph capture
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    w = _watch.get(dev.index)
    if w is None:
        w = _watch[dev.index] = _ErrorWatch()
    if w.event is not None and w.event.query() and int(w.host[0]) != 0:
        w.host.zero_()
        w.event = None
        poll_device_error(dev)  # raises BOZO_ERR_DEVICE_TIMEOUT and clears the word
    with torch.cuda.device(dev):
        code = _capi.lib().bozo_tension_error_async(w.host.data_ptr(), _stream(dev))
    _capi.check(code, "device error copy")
    if w.event is None:
        w.event = torch.cuda.Event()
    w.event.record(torch.cuda.current_stream(dev))
