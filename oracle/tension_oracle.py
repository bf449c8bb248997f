"""CPU oracle for the sigmoid-tension operator — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it.
The shipped operator (``bozo_b200``) runs on the GPU and raises when its
CUDA library is missing; it never routes through this file.

It restates, in plain PyTorch on the CPU (float64 by default, float32 for the
timed CPU baseline), the reference algorithm of BoggersTheFish/bozo:

* ``local_tension_raw``   — ``triton_tension/ops.py:29-63`` (``_ref_forward``):
  unfold-gather the W keys before each query (self excluded), sigmoid of the
  scaled dot plus optional head-agnostic bias, raw Σ τ·V.
* ``local_tension_norm``  — ``model.py:271-283`` (τ-mass normalisation,
  unfold path) and ``model.py:257-258`` (same normalisation on the fused path);
  ``normalize="count"`` restates the divergent ``model.py:261-264`` branch.
* ``global_tension``      — ``model.py:217-237``: full-causal (self included)
  sigmoid tension, τ-mass normalisation, optional ``[B,T,T]`` bias and the
  flipped/downsampled τ export.
* ``rope``                — ``model.py:66-81``: half-split rotary embedding.

Parity is pinned by ``tests/test_oracle_golden.py`` against fixtures produced
by running the reference's own code (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

MASS_EPS = 1e-6  # model.py:227, 257, 281 — clamp(min=1e-6) on the τ-mass


def rope_tables(head_dim: int, max_seq_len: int, base: float = 10_000.0,
                dtype=torch.float32):
    """cos/sin tables ``[S, HD/2]`` — model.py:66-73 (θ_i = base^(−i/half))."""
    half = head_dim // 2
    theta = 1.0 / (base ** (torch.arange(0, half).float() / half))
    pos = torch.arange(max_seq_len).float()
    freqs = torch.outer(pos, theta)
    return freqs.cos().to(dtype), freqs.sin().to(dtype)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half-split rotation of ``x [B,T,H,HD]`` at positions 0..T−1 — model.py:75-81."""
    T = x.shape[1]
    c = cos[:T].to(x.dtype).unsqueeze(0).unsqueeze(2)
    s = sin[:T].to(x.dtype).unsqueeze(0).unsqueeze(2)
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


def _gather_window(z: torch.Tensor, W: int) -> torch.Tensor:
    """``z [B,T,H,C] → [B,T,H,W,C]``, slot w holds position t−(W−w), zero if
    negative — model.py:165-179 / ops.py:43-48."""
    T = z.shape[1]
    zt = z.permute(0, 2, 3, 1)
    zp = F.pad(zt, (W, 0), value=0.0)
    nb = zp.unfold(-1, W, 1)[:, :, :, :T, :]
    return nb.permute(0, 3, 1, 4, 2)


def window_mask(T: int, W: int, dtype=torch.float64) -> torch.Tensor:
    """Validity of slot (t, w): t + w ≥ W — model.py:150-156, ops.py:50-52."""
    t_idx = torch.arange(T).unsqueeze(1)
    w_idx = torch.arange(W).unsqueeze(0)
    return (t_idx + w_idx >= W).to(dtype)


def local_tension_raw(Q, K, V, W: int, scale: float, bias=None,
                      return_tau: bool = False):
    """Raw windowed tension, the drop-in op's semantics — ops.py:29-63.

    ``Q,K,V [B,T,H,HD]``; ``bias [B,T,W]`` (broadcast over heads).
    Returns ``S [B,T,H,HD] = Σ_w τ·V`` and optionally ``τ [B,T,H,W]``.
    All arithmetic happens in ``Q.dtype`` (pass float64 for a tight oracle).
    """
    B, T, H, HD = Q.shape
    nb_k = _gather_window(K.to(Q.dtype), W)
    nb_v = _gather_window(V.to(Q.dtype), W)
    mask = window_mask(T, W, Q.dtype)
    dots = (Q.unsqueeze(3) * nb_k).sum(-1) / scale
    if bias is not None:
        dots = dots + bias.unsqueeze(2).to(dots.dtype)
    tau = torch.sigmoid(dots) * mask.unsqueeze(0).unsqueeze(2)
    msg = (tau.unsqueeze(-1) * nb_v).sum(3)
    if return_tau:
        return msg, tau
    return msg


def valid_count(T: int, W: int, dtype=torch.float64) -> torch.Tensor:
    """Per-query count of valid window slots, clamped ≥ 1 — model.py:158-163."""
    return window_mask(T, W, dtype).sum(-1).clamp(min=1)


def local_tension_norm(Q, K, V, W: int, scale: float, bias=None,
                       normalize: str = "mass"):
    """Normalised local tension as the model consumes it.

    ``normalize="mass"``: out = S / clamp(Σ_w τ, 1e-6) — model.py:257-258,
    280-282.  ``normalize="count"``: out = S / valid_count — model.py:261-264.
    Returns ``(out, tau)``.
    """
    msg, tau = local_tension_raw(Q, K, V, W, scale, bias, return_tau=True)
    if normalize == "mass":
        mass = tau.sum(-1).clamp(min=MASS_EPS)
        return msg / mass.unsqueeze(-1), tau
    if normalize == "count":
        T = Q.shape[1]
        return msg / valid_count(T, W, msg.dtype)[:T, None, None], tau
    if normalize in (None, "none"):
        return msg, tau
    raise ValueError(f"unknown normalize={normalize!r}")


def global_tension(Q, K, V, scale: float, bias=None, local_window: int = 64):
    """Full-causal (self-inclusive) tension — model.py:217-237.

    ``bias [B,T,T]`` indexed by absolute key position.  Returns
    ``(out, tau_full, tau_local)`` where ``out`` is τ-mass normalised,
    ``tau_full [B,T,H,T]`` and ``tau_local [B,T,H,min(local_window,T)]`` is
    the reference's export ``tau[..., :T].flip(-1)[..., :W]`` (column j holds
    key position T−1−j).
    """
    B, T, H, HD = Q.shape
    scores = torch.einsum("bthd,bshd->bths", Q, K.to(Q.dtype)) / scale
    causal = torch.tril(torch.ones(T, T, dtype=scores.dtype))
    if bias is not None:
        scores = scores + bias.unsqueeze(2).to(scores.dtype)
    tau = torch.sigmoid(scores) * causal.unsqueeze(0).unsqueeze(2)
    mass = tau.sum(-1).clamp(min=MASS_EPS)
    msg = torch.einsum("bths,bshd->bthd", tau, V.to(Q.dtype))
    out = msg / mass.unsqueeze(-1)
    W_eff = min(local_window, T)
    tau_local = tau[:, :, :, :T].flip(-1)[:, :, :, :W_eff]
    return out, tau, tau_local


def tension_with_grads(fn, inputs, d_outputs):
    """Run ``fn(*inputs)`` (tuple of outputs) and return (outputs, grads) via
    autograd with the given output cotangents (``None`` entries skipped)."""
    leaves = [x.detach().clone().requires_grad_(True) for x in inputs]
    outs = fn(*leaves)
    if not isinstance(outs, (tuple, list)):
        outs = (outs,)
    pairs = [(o, d) for o, d in zip(outs, d_outputs) if d is not None]
    grads = torch.autograd.grad([o for o, _ in pairs], leaves,
                                [d.to(o.dtype) for o, d in pairs],
                                allow_unused=True)
    grads = [torch.zeros_like(x) if g is None else g for x, g in zip(leaves, grads)]
    return [o.detach() for o in outs], [g.detach() for g in grads]


def fused_reference(q_raw, k_raw, v, *, window: int | None, scale: float,
                    rope_base: float | None = 10_000.0, bias=None,
                    normalize: str = "mass", local_window: int = 64,
                    max_seq_len: int | None = None):
    """Reference composition for the fused entry point: RoPE(Q), RoPE(K) as in
    model.py:200-204, then the local (``window`` int) or global
    (``window=None``) tension with the model's normalisation.  Returns
    ``(out, tau)`` where for the global mode ``tau`` is the exported window."""
    T, HD = q_raw.shape[1], q_raw.shape[3]
    if rope_base is not None:
        cos, sin = rope_tables(HD, max_seq_len or T, rope_base, torch.float64)
        q = rope(q_raw, cos, sin)
        k = rope(k_raw, cos, sin)
    else:
        q, k = q_raw, k_raw
    if window is None:
        out, _, tau_local = global_tension(q, k, v, scale, bias, local_window)
        return out, tau_local
    return local_tension_norm(q, k, v, window, scale, bias, normalize)


def algorithmic_pairs(B: int, H: int, T: int, W: int | None) -> int:
    """Valid (query, key) pairs: B·H·(T·W − W(W+1)/2) local (T ≥ W),
    B·H·T(T+1)/2 global."""
    if W is None:
        return B * H * T * (T + 1) // 2
    # Σ_{t<T} min(t, W)
    per = T * W - W * (W + 1) // 2 if T >= W else T * (T - 1) // 2
    return B * H * per


def flops_fwd_bwd(B, H, T, HD, W) -> int:
    """4·P·HD forward + 8·P·HD backward (no credit for recompute)."""
    return 12 * algorithmic_pairs(B, H, T, W) * HD


def bytes_fwd_bwd(B, H, T, HD, elem_bytes: int = 2) -> int:
    """fwd: read Q,K,V + write O (+4 B row mass); bwd: read Q,K,V,dO,O + write
    dQ,dK,dV (+4 B row mass) — N_rows·(12·HD·e + 8)."""
    n = B * H * T
    return n * (4 * HD * elem_bytes + 4) + n * (8 * HD * elem_bytes + 4)


def cpu_fwd_bwd_sample(B=1, H=12, T=2048, HD=64, W=64, seed=0, threads=None,
                       dtype=torch.float32):
    """One fwd+bwd of the reference CPU path (unfold + autograd, fp32) at the
    given shape, with RoPE and τ-mass normalisation as model.py does.  Used
    as the timed CPU baseline; returns the loss so work cannot be skipped."""
    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, HD, generator=g, dtype=dtype, requires_grad=True)
    k = torch.randn(B, T, H, HD, generator=g, dtype=dtype, requires_grad=True)
    v = torch.randn(B, T, H, HD, generator=g, dtype=dtype, requires_grad=True)
    d = torch.randn(B, T, H, HD, generator=g, dtype=dtype)
    cos, sin = rope_tables(HD, T, 10_000.0, dtype)
    out, _ = local_tension_norm(rope(q, cos, sin), rope(k, cos, sin), v, W,
                                math.sqrt(HD), None, "mass")
    (out * d).sum().backward()
    return float(q.grad.sum() + k.grad.sum() + v.grad.sum())
