"""Fused τ-field consumer (``bozo_b200.aux``, ``include/bozo_tau_aux.h``).

* GPU, fp32: the three losses and the gradients of their weighted sum match
  the reference functions' own outputs (``tests/golden/golden_aux.npz``).
* GPU, bf16 / fp32 at training widths and odd widths (vector and scalar
  kernel paths): against the float64 oracle on the same τ values.
* GPU: the statistics are bit-identical run to run (fixed-order reduction).
* CPU: CUDA-only — CPU fields raise instead of falling back.
"""
import numpy as np
import pytest
import torch

from oracle import aux_oracle
from tests.test_oracle_golden import AUX_WEIGHTS, _aux_case, _aux_names


def _close(got, ref, rtol, atol_rel, what):
    g = got.detach().double().cpu().numpy()
    r = np.asarray(ref, dtype=np.float64)
    scale = float(np.abs(r).max()) or 1.0
    np.testing.assert_allclose(g, r, rtol=rtol, atol=atol_rel * scale, err_msg=what)


def _fused(taus, groups, weights=AUX_WEIGHTS):
    from bozo_b200 import aux
    xs = [t.detach().clone().requires_grad_(True) for t in taus]
    d, c, e = aux.tension_aux_losses(xs, groups)
    total = weights[0] * d + weights[1] * c + weights[2] * e
    grads = torch.autograd.grad(total, xs)
    return (d, c, e), grads


@pytest.mark.gpu
@pytest.mark.parametrize("name", _aux_names())
def test_fused_matches_reference_golden_fp32(name):
    taus, grads, groups, vals = _aux_case(name)
    dev = torch.device("cuda:0")
    (d, c, e), got = _fused([t.to(dev) for t in taus], groups)
    _close(torch.stack([d, c, e]), vals, 1e-5, 1e-6, f"{name} losses")
    for i, (g, r) in enumerate(zip(got, grads)):
        assert g.dtype == torch.float32
        _close(g, r, 1e-4, 1e-5, f"{name} dτ{i}")


def _fields(shape, n, dtype, seed):
    B, T, H, W = shape
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        x = torch.randn(B, T, H, W, generator=g) * 1.5
        off = torch.randint(-1, 2, (B, T, H, 1), generator=g).float() * 4.0
        tau = torch.sigmoid(x + off)
        t = torch.arange(T).view(1, T, 1, 1)
        w = torch.arange(W).view(1, 1, 1, W)
        out.append((tau * ((t - (W - w)) >= 0).float()).to(dtype))
    return out


# (shape, layers): vector paths G = 1…32 for bf16 (W = 8…256) and fp32, the
# scalar path for widths that are not whole 16-byte vectors of a power-of-two
# lane count (W = 24, 37, 300)
SHAPES = [((2, 300, 4, 64), 3), ((1, 257, 3, 128), 2), ((2, 64, 2, 8), 2), ((1, 96, 2, 256), 2),
          ((2, 70, 3, 24), 2), ((1, 50, 2, 37), 2), ((1, 40, 2, 300), 1), ((3, 33, 2, 16), 3)]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("shape,n", SHAPES)
def test_fused_matches_oracle(shape, n, dtype):
    taus = _fields(shape, n, dtype, seed=shape[-1] * 7 + n)
    groups = {shape[-1]: list(range(n - 1)), 4 * shape[-1]: [n - 1]} if n > 1 else None
    w = (1.0, 0.5, 2.0)
    vals, ref = aux_oracle.losses_and_grads(taus, groups, w)
    dev = torch.device("cuda:0")
    (d, c, e), got = _fused([t.to(dev) for t in taus], groups, w)
    # statistics in fp32 from the stored values: fp32 round-off against float64
    _close(torch.stack([d, c, e]), vals, 2e-5, 1e-6, f"{shape} {dtype} losses")
    # dτ is stored in the fields' dtype: its rounding is the tolerance.  Rows
    # with no live slot (t = 0) have Σ = 0, so the reference's +1e-8
    # denominator gives their slots cotangents near −2e5, beyond fp16's range:
    # compare with the oracle rounded to the field dtype (−inf there)
    rtol = {torch.float32: 1e-4, torch.bfloat16: 1e-2, torch.float16: 2e-3}[dtype]
    for i, (g, r) in enumerate(zip(got, ref)):
        assert g.dtype == dtype and g.shape == taus[i].shape
        r = r.to(dtype).double()
        fin = torch.isfinite(r)
        assert torch.equal(torch.isfinite(g.cpu()), fin), f"{shape} {dtype} dτ{i}: overflow pattern"
        _close(g.cpu()[fin], r[fin].numpy(), rtol, rtol * 1e-1, f"{shape} {dtype} dτ{i}")


@pytest.mark.gpu
def test_fields_of_two_shapes_and_dtypes():
    """Fields of different widths (local and a different exported window) are
    batched per shape and still produce one statistics row each."""
    from bozo_b200 import aux
    a = _fields((2, 80, 3, 64), 2, torch.bfloat16, 5)
    b = _fields((2, 80, 3, 16), 1, torch.bfloat16, 6)
    taus = [a[0], b[0], a[1]]
    groups = {64: [0, 2], 1024: [1]}
    vals, ref = aux_oracle.losses_and_grads(taus, groups, (1.0, 1.0, 1.0))
    dev = torch.device("cuda:0")
    st = aux.tau_field_stats([t.to(dev) for t in taus])
    assert st.shape == (3, 3)
    (d, c, e), got = _fused([t.to(dev) for t in taus], groups, (1.0, 1.0, 1.0))
    _close(torch.stack([d, c, e]), vals, 2e-5, 1e-6, "mixed losses")
    for g, r in zip(got, ref):
        _close(g, r.numpy(), 1e-2, 1e-3, "mixed dτ")


@pytest.mark.gpu
def test_statistics_are_deterministic():
    from bozo_b200 import aux
    taus = [t.cuda() for t in _fields((4, 512, 6, 64), 4, torch.bfloat16, 9)]
    a = aux.tau_field_stats(taus)
    b = aux.tau_field_stats(taus)
    assert torch.equal(a, b)


def test_cpu_fields_raise():
    from bozo_b200 import aux
    with pytest.raises(RuntimeError, match="CUDA"):
        aux.tension_aux_losses([torch.rand(1, 8, 2, 4)], None)


# ───────────── row mode: the cotangent formed inside the tension backward ─────────────

def _op_with_aux(q, k, v, d_out, W, weights, grad_consistency):
    import bozo_b200
    from bozo_b200 import aux
    leaves = [x.detach().clone().requires_grad_(True) for x in (q, k, v)]
    out, tau = bozo_b200.tension(*leaves, window=W, scale=8.0, return_tau=True, normalize="mass")
    slot = getattr(tau, "_bozo_tau_slot", None)
    d, c, e = aux.tension_aux_losses([tau], None, grad_consistency=grad_consistency)
    loss = (out.float() * d_out.float()).sum() + weights[0] * d + weights[1] * c + weights[2] * e
    grads = torch.autograd.grad(loss, leaves)
    return grads, slot


@pytest.mark.gpu
@pytest.mark.parametrize("W", [32, 64, 128])
def test_row_mode_matches_materialised_cotangent_and_oracle(W):
    """With the consistency weight 0, the diversity/entropy cotangent of τ goes
    to the tension backward per query row (a1·(log2 q − 1e-8/(q·ln 2)) + a0 at
    the recomputed τ) instead of as a [B,T,H,W] tensor: dQ/dK/dV agree with
    the materialised path and with float64 autograd through the oracle
    tension and the oracle losses."""
    from oracle import tension_oracle as orc
    from tests._tol import assert_close
    g = torch.Generator().manual_seed(W)
    B, T, H, HD = 2, 320, 3, 64
    q, k, v, d_out = (torch.randn(B, T, H, HD, generator=g) for _ in range(4))
    # heavy aux weights so the τ cotangent matters next to the output's
    w = (400.0, 0.0, 200.0)
    dev = torch.device("cuda:0")
    qb, kb, vb, db = (x.to(dev, torch.bfloat16) for x in (q, k, v, d_out))
    row, slot = _op_with_aux(qb, kb, vb, db, W, w, grad_consistency=False)
    assert slot is not None and slot.row is None  # created, filled and consumed
    mat, _ = _op_with_aux(qb, kb, vb, db, W, w, grad_consistency=True)
    for name, a, b in zip(("dq", "dk", "dv"), row, mat):
        assert_close(a, b, torch.bfloat16, f"W{W} row vs materialised {name}")

    # float64 oracle on the same bf16-rounded inputs
    def fn(q_, k_, v_):
        out, tau = orc.fused_reference(q_, k_, v_, window=W, scale=8.0, normalize="mass")
        d = aux_oracle.diversity([tau])
        e = aux_oracle.entropy([tau])
        return (out, w[0] * d + w[2] * e)

    xs = [x.to(torch.bfloat16).double() for x in (q, k, v)]
    _, ref = orc.tension_with_grads(fn, xs, [d_out.to(torch.bfloat16).double(),
                                             torch.tensor(1.0, dtype=torch.float64)])
    for name, a, b in zip(("dq", "dk", "dv"), row, ref):
        assert_close(a, b, torch.bfloat16, f"W{W} row mode vs oracle {name}")


@pytest.mark.gpu
def test_row_cotangent_needs_the_tensor_core_band_path():
    """The C ABI refuses a per-row τ cotangent on the CUDA-core path."""
    from bozo_b200 import _capi, ops
    dev = torch.device("cuda:0")
    B, T, H, HD, W = 1, 64, 2, 64, 32
    q, k, v, d_out = (torch.randn(B, T, H, HD, device=dev) for _ in range(4))  # fp32: CUDA-core
    out, _, mass, _, _ = ops._launch_fwd(q, k, v, mode=_capi.MODE_LOCAL, window=W,
                                         norm=_capi.NORM_MASS, scale=8.0, rope=None, bias=None,
                                         tau_width=None, out_dtype=q.dtype, tau_dtype=q.dtype,
                                         want_mass=True)
    aux_row = torch.zeros(3, B * H * T, device=dev)
    with pytest.raises(RuntimeError, match="unsupported"):
        ops._launch_bwd(q, k, v, d_out, mode=_capi.MODE_LOCAL, window=W, norm=_capi.NORM_MASS,
                        scale=8.0, rope=None, bias=None, out=out, mass=mass, d_tau=None,
                        aux_row=aux_row)


# ───────────── uncertainty_gate (train.py:411-447) ─────────────

@pytest.mark.gpu
@pytest.mark.parametrize("name", _aux_names())
def test_uncertainty_gate_matches_reference_golden(name):
    from bozo_b200 import aux
    from tests.conftest import _load
    from tests.test_oracle_golden import GATE_THRESHOLDS
    c = _load("golden_aux.npz")[name]
    taus, _, _, _ = _aux_case(name)
    dev = torch.device("cuda:0")
    for k, th in enumerate(GATE_THRESHOLDS):
        got = aux.uncertainty_gate([t.to(dev) for t in taus], th)
        assert got.shape == c[f"gate{k}"].shape and got.dtype == torch.float32
        np.testing.assert_array_equal(got.cpu().numpy(), c[f"gate{k}"], err_msg=f"{name} th={th}")


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_uncertainty_gate_vs_oracle_mixed_widths(dtype):
    """Fields of two widths (the reference cuts all to the narrowest) at a
    threshold near the median entropy: the masks agree except for rows whose
    mean entropy lies within fp32 round-off of the threshold."""
    from bozo_b200 import aux
    taus = _fields((2, 300, 4, 64), 3, dtype, 3) + _fields((2, 300, 4, 128), 1, dtype, 4)
    mean_ent = aux_oracle.row_entropy_mean(taus)
    th = float(mean_ent.median())
    ref = (mean_ent > th).double()
    got = aux.uncertainty_gate([t.cuda() for t in taus], th).double().cpu()
    near = (mean_ent - th).abs() < 1e-4
    assert torch.equal(got[~near], ref[~near])
    assert 0.3 < float(got.mean()) < 0.7
