"""Pin the CPU oracle against fixtures produced by the reference itself.

The fixtures (``tests/golden/*.npz``) come from running the reference's own
``triton_tension/ops.py::_ref_forward`` and ``model.py`` layer on the CPU
(``tests/golden/make_golden.py``).  Here the oracle restatement must
reproduce them to float64 round-off, forward and backward.
"""
import numpy as np
import pytest
import torch

from oracle import tension_oracle as orc

TOL = dict(rtol=1e-10, atol=1e-11)


def _t(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float64))


def _op_names():
    import os
    from tests.conftest import _load
    return sorted(_load("golden_op.npz"))


def _layer_names():
    from tests.conftest import _load
    return sorted(_load("golden_layer.npz"))


@pytest.mark.parametrize("name", _op_names())
def test_oracle_raw_op_matches_reference(golden_op, name):
    c = golden_op[name]
    B, T, H, HD, W = [int(x) for x in c["meta"]]
    scale = float(c["scale"])
    bias = _t(c["bias"]) if "bias" in c else None
    d_tau = _t(c["d_tau"]) if "d_tau" in c else None

    def fn(q, k, v):
        return orc.local_tension_raw(q, k, v, W, scale, bias, return_tau=True)

    (out, tau), (dq, dk, dv) = orc.tension_with_grads(
        fn, [_t(c["q"]), _t(c["k"]), _t(c["v"])], [_t(c["d_out"]), d_tau])
    for got, key in ((out, "out"), (tau, "tau"), (dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got.numpy(), c[key], err_msg=f"{name}:{key}", **TOL)


@pytest.mark.parametrize("name", _layer_names())
def test_oracle_layer_matches_reference(golden_layer, name):
    c = golden_layer[name]
    B, T, H, HD, W, Wl, msl = [int(x) for x in c["meta"]]
    scale = float(c["scale"])
    bias = _t(c["bias"]) if "bias" in c else None
    cos, sin = orc.rope_tables(HD, msl, 10_000.0, torch.float64)
    # the reference builds its tables in float32 then widens (model.py:69-73)
    np.testing.assert_allclose(cos.numpy(), c["rope_cos"], rtol=0, atol=0)
    np.testing.assert_allclose(sin.numpy(), c["rope_sin"], rtol=0, atol=0)

    def fn(q, k, v):
        out, tau = orc.fused_reference(q, k, v, window=None if W < 0 else W,
                                       scale=scale, bias=bias, local_window=Wl,
                                       max_seq_len=msl)
        return out, tau

    (out, tau), (dq, dk, dv) = orc.tension_with_grads(
        fn, [_t(c["q_raw"]), _t(c["k_raw"]), _t(c["v"])],
        [_t(c["d_out"]), _t(c["d_tau"])])
    for got, key in ((out, "out"), (tau, "tau"), (dq, "dq_raw"), (dk, "dk_raw"),
                     (dv, "dv")):
        np.testing.assert_allclose(got.numpy(), c[key], err_msg=f"{name}:{key}", **TOL)
    if "valid_count" in c:
        np.testing.assert_array_equal(orc.valid_count(msl, W).numpy(), c["valid_count"])


def test_algorithmic_pairs_matches_mask():
    for T, W in ((2048, 64), (5, 8), (100, 100), (300, 128), (1, 1)):
        m = orc.window_mask(T, W)
        assert int(m.sum()) == orc.algorithmic_pairs(1, 1, T, W)
    assert orc.algorithmic_pairs(1, 1, 7, None) == 28


# ───────────── τ-field consumer (model.py:498-611) ─────────────

def _aux_case(name):
    import ast
    from tests.conftest import _load
    c = _load("golden_aux.npz")[name]
    n = len([k for k in c if k.startswith("tau")])
    taus = [torch.from_numpy(c[f"tau{i}"]) for i in range(n)]
    grads = [c[f"grad{i}"] for i in range(n)]
    groups = ast.literal_eval(str(c["groups"]))
    vals = (float(c["diversity"]), float(c["consistency"]), float(c["entropy"]))
    return taus, grads, groups, vals


def _aux_names():
    from tests.conftest import _load
    return sorted(_load("golden_aux.npz"))


AUX_WEIGHTS = (1.0, 0.7, 0.3)  # tests/golden/make_golden_aux.py W_DIV, W_CONS, W_ENT


@pytest.mark.parametrize("name", _aux_names())
def test_aux_oracle_matches_reference(name):
    from oracle import aux_oracle
    taus, grads, groups, vals = _aux_case(name)
    got, got_grads = aux_oracle.losses_and_grads(taus, groups, AUX_WEIGHTS)
    # the reference ran in fp32: agree to fp32 round-off
    np.testing.assert_allclose(got, vals, rtol=2e-6, atol=1e-7)
    for g, r in zip(got_grads, grads):
        scale = float(np.abs(r).max()) or 1.0
        np.testing.assert_allclose(g.numpy(), r, rtol=1e-5, atol=1e-6 * scale)


GATE_THRESHOLDS = (0.15, 1.0, 2.0)  # tests/golden/make_golden_aux.py


@pytest.mark.parametrize("name", _aux_names())
def test_uncertainty_gate_oracle_matches_reference(name):
    from oracle import aux_oracle
    from tests.conftest import _load
    c = _load("golden_aux.npz")[name]
    taus, _, _, _ = _aux_case(name)
    for k, th in enumerate(GATE_THRESHOLDS):
        np.testing.assert_array_equal(aux_oracle.uncertainty_gate(taus, th).numpy(), c[f"gate{k}"])


# ───────────── graph bias (ts_bridge/bias.py:125-233) ─────────────

def _bias_golden():
    import json
    import os
    from tests.conftest import GOLDEN
    z = np.load(os.path.join(GOLDEN, "golden_bias.npz"))
    edges = {(s, d): w for s, d, w in json.loads(str(z["edges"]))}
    return z, edges


class _FixedTokenizer:
    """tests/golden/make_golden_bias.py's tokenizer: tok{i} for i < 18, else None."""

    def id_to_token(self, i):
        return f"tok{i}" if i < 18 else None


@pytest.mark.parametrize("ctx", ["ctx_a", "ctx_b"])
def test_bias_oracle_matches_reference(ctx):
    from oracle import bias_oracle
    z, edges = _bias_golden()
    ids, alpha, W = z[f"{ctx}_ids"].tolist(), float(z["alpha"]), int(z["W"])
    lb, ls = bias_oracle.local_bias(edges, alpha, ids, _FixedTokenizer(), W)
    gb, gs = bias_oracle.global_bias(edges, alpha, ids, _FixedTokenizer())
    for b in range(2):
        np.testing.assert_array_equal(lb, z[f"{ctx}_local"][b])
        np.testing.assert_array_equal(gb, z[f"{ctx}_global"][b])
    np.testing.assert_allclose(ls, z[f"{ctx}_local_stats"], rtol=1e-12)
    np.testing.assert_allclose(gs, z[f"{ctx}_global_stats"], rtol=1e-12)
