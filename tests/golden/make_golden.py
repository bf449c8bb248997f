"""Generate golden vectors by running the REFERENCE implementation on the CPU.

Run once in a container that has the reference checkout, passing its path
with ``--ref PATH`` or the ``BOZO_REFERENCE`` environment variable::

    python tests/golden/make_golden.py

It writes ``tests/golden/golden_op.npz`` and ``tests/golden/golden_layer.npz``.
The GPU box never runs this script; tests only read the committed ``.npz``.

* ``golden_op``: the raw drop-in operator, computed by the reference's own
  ``triton_tension/ops.py::_ref_forward`` (the path ``causal_tension`` takes for
  CPU / float64 inputs, ops.py:217-219), differentiated by autograd.  Shapes
  and seeds follow the reference's script tests (triton_tension/test.py:59,
  95, 131, 175; triton_tension/test_tau.py:28, 63) plus edge cases (T < W,
  ragged T, W = 1, HD = 64).
* ``golden_layer``: ``model.py``'s ``MultiHeadCausalTensionLayer`` run in
  float64 with RoPE on and dropout 0 (unfold path for local layers,
  model.py:271-287; einsum path for global layers, model.py:217-237).  Forward
  hooks capture the pre-RoPE projections (q_raw, k_raw, v), the normalised
  message entering ``wo`` and the exported τ; autograd gives the gradients
  w.r.t. the pre-RoPE projections for seeded cotangents of (message, τ).
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    return t.detach().to(torch.float64).cpu().numpy()


def op_cases(ref_forward):
    """(name, B, T, H, HD, W, seed, bias_scale, dtau_scale)."""
    cases = [
        ("fwd_t32_w8_s0", 2, 32, 4, 16, 8, 0, None, None),        # test.py:59
        ("grad_t24_w8_s2", 2, 24, 4, 16, 8, 2, None, None),       # test.py:95
        ("bias_t32_w8_s10", 2, 32, 4, 16, 8, 10, 0.5, None),      # test.py:131
        ("biasgrad_t24_w8_s12", 2, 24, 4, 16, 8, 12, 0.5, None),  # test.py:175
        ("dtau_t24_w8_s2", 2, 24, 4, 16, 8, 2, None, 0.1),        # test_tau.py:63
        ("short_t5_w8_s3", 1, 5, 2, 16, 8, 3, None, 0.1),          # T < W
        ("w1_t17_s4", 1, 17, 2, 32, 1, 4, 0.3, 0.1),               # W = 1
        ("hd64_t160_w64_s5", 1, 160, 2, 64, 64, 5, 0.5, 0.1),      # ragged T
        ("hd64_t260_w128_s6", 1, 260, 1, 64, 128, 6, None, 0.1),
    ]
    out = {}
    for name, B, T, H, HD, W, seed, bscale, dscale in cases:
        g = torch.Generator().manual_seed(seed)
        # Inputs are drawn in float32 (as the reference tests do) and widened,
        # so they are stored exactly as float32; outputs stay float64.
        Q = torch.randn(B, T, H, HD, generator=g).double()
        K = torch.randn(B, T, H, HD, generator=g).double()
        V = torch.randn(B, T, H, HD, generator=g).double()
        dO = torch.randn(B, T, H, HD, generator=g).double()
        bias = ((torch.randn(B, T, W, generator=g) * bscale).double()
                if bscale is not None else None)
        dT = ((torch.randn(B, T, H, W, generator=g) * dscale).double()
              if dscale is not None else None)
        scale = math.sqrt(HD)
        Ql, Kl, Vl = [x.clone().requires_grad_(True) for x in (Q, K, V)]
        o, tau = ref_forward(Ql, Kl, Vl, W, scale, return_tau=True, bias=bias)
        loss = (o * dO).sum()
        if dT is not None:
            loss = loss + (tau * dT).sum()
        loss.backward()
        p = name + "/"
        out[p + "meta"] = np.array([B, T, H, HD, W], dtype=np.int64)
        out[p + "scale"] = np.array(scale)
        for k, v in (("q", Q), ("k", K), ("v", V), ("d_out", dO)):
            out[p + k] = _np(v).astype(np.float32)
        for k, v in (("out", o), ("tau", tau), ("dq", Ql.grad), ("dk", Kl.grad),
                     ("dv", Vl.grad)):
            out[p + k] = _np(v)
        if bias is not None:
            out[p + "bias"] = _np(bias).astype(np.float32)
        if dT is not None:
            out[p + "d_tau"] = _np(dT).astype(np.float32)
    return out


def layer_cases(model_mod):
    """Layer-level fixtures through model.py (RoPE, τ-mass, global path)."""
    cases = [
        # name, global, dim, heads, window, max_seq_len, B, T, seed, bias
        ("local_hd64_w16_t40", False, 128, 2, 16, 48, 1, 40, 20, False),
        ("local_bias_hd64_w16_t40", False, 128, 2, 16, 48, 1, 40, 21, True),
        ("local_hd32_w64_t100", False, 64, 2, 64, 128, 1, 100, 22, False),
        ("global_hd64_t40", True, 128, 2, 16, 48, 1, 40, 23, False),
        ("global_bias_hd64_t40", True, 128, 2, 16, 48, 1, 40, 24, True),
        ("global_hd64_t12_w16", True, 128, 2, 16, 48, 1, 12, 25, False),
    ]
    out = {}
    for name, is_global, dim, heads, window, msl, B, T, seed, with_bias in cases:
        torch.manual_seed(seed)
        cfg = model_mod.TensionConfig(
            vocab_size=64, dim=dim, num_layers=1, num_heads=heads,
            window=window, max_seq_len=msl, dropout=0.0, use_rope=True,
            use_oscillation=False, use_triton=False)
        layer = model_mod.MultiHeadCausalTensionLayer(cfg, global_layer=is_global)
        layer = layer.double().eval()
        cap = {}
        layer.wq.register_forward_hook(lambda m, i, o: cap.__setitem__("q_raw", o))
        layer.wk.register_forward_hook(lambda m, i, o: cap.__setitem__("k_raw", o))
        layer.wv.register_forward_hook(lambda m, i, o: cap.__setitem__("v", o))
        layer.wo.register_forward_pre_hook(lambda m, i: cap.__setitem__("msg", i[0]))
        g = torch.Generator().manual_seed(seed + 1000)
        x = torch.randn(B, T, dim, generator=g, dtype=torch.float64)
        HD = dim // heads
        bias = None
        if with_bias:
            shape = (B, T, T) if is_global else (B, T, window)
            bias = torch.randn(*shape, generator=g, dtype=torch.float64) * 0.5
        _, tau = layer(x, return_tensions=True, tau_bias=bias)
        msg = cap["msg"].view(B, T, heads, HD)
        d_out = torch.randn(B, T, heads, HD, generator=g, dtype=torch.float64)
        d_tau = torch.randn(*tau.shape, generator=g, dtype=torch.float64) * 0.1
        grads = torch.autograd.grad([cap["msg"], tau],
                                    [cap["q_raw"], cap["k_raw"], cap["v"]],
                                    [d_out.reshape(B, T, dim), d_tau])
        p = name + "/"
        out[p + "meta"] = np.array([B, T, heads, HD, -1 if is_global else window,
                                    window, msl], dtype=np.int64)
        out[p + "scale"] = np.array(math.sqrt(HD))
        sh = (B, T, heads, HD)
        out[p + "q_raw"] = _np(cap["q_raw"].reshape(sh))
        out[p + "k_raw"] = _np(cap["k_raw"].reshape(sh))
        out[p + "v"] = _np(cap["v"].reshape(sh))
        out[p + "out"] = _np(msg)
        out[p + "tau"] = _np(tau)
        out[p + "d_out"] = _np(d_out)
        out[p + "d_tau"] = _np(d_tau)
        out[p + "dq_raw"] = _np(grads[0].reshape(sh))
        out[p + "dk_raw"] = _np(grads[1].reshape(sh))
        out[p + "dv"] = _np(grads[2].reshape(sh))
        out[p + "rope_cos"] = _np(layer.rope.cos)
        out[p + "rope_sin"] = _np(layer.rope.sin)
        if not is_global:
            out[p + "valid_count"] = _np(layer.valid_count)
        if bias is not None:
            out[p + "bias"] = _np(bias)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BOZO_REFERENCE"),
                    required="BOZO_REFERENCE" not in os.environ,
                    help="path of the reference checkout (or set BOZO_REFERENCE)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import model as model_mod  # noqa: E402  (reference model.py)
    from triton_tension.ops import _ref_forward  # noqa: E402  (reference ops.py)

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    op = op_cases(_ref_forward)
    np.savez_compressed(os.path.join(HERE, "golden_op.npz"), **op)
    lay = layer_cases(model_mod)
    np.savez_compressed(os.path.join(HERE, "golden_layer.npz"), **lay)
    print("wrote", len(op), "op arrays and", len(lay), "layer arrays")


if __name__ == "__main__":
    main()
