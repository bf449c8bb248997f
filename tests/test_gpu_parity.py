"""GPU parity of the tension operator against the reference (golden fixtures
made by the reference's own code) and the float64 CPU oracle.

Ports the intent of the reference's script tests — triton_tension/test.py
(forward, manual grads, bias variants, large bf16 spot check) and
triton_tension/test_tau.py (τ parity, Out bit-identical with/without τ,
backward through τ, τ-unused parity, memory bound) — with the stricter
tolerances of ``tests/_tol.py``.  Every call goes through the C ABI.
"""
import math

import numpy as np
import pytest
import torch

from oracle import tension_oracle as orc
from tests._tol import TOL, assert_close

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")


@pytest.fixture(scope="module")
def bz():
    import bozo_b200
    bozo_b200.set_kernel_path("auto")
    return bozo_b200


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    """Every test must leave the device error word clear (no bounded wait in
    a tensor-core kernel gave up)."""
    yield
    if torch.cuda.is_available():
        import bozo_b200
        bozo_b200.poll_device_error()


def _cu(a, dtype):
    return torch.from_numpy(np.asarray(a)).to("cuda").to(dtype)


def _run_raw(bz, c, dtype, with_tau=True):
    B, T, H, HD, W = [int(x) for x in c["meta"]]
    q, k, v = [_cu(c[n], dtype).requires_grad_(True) for n in ("q", "k", "v")]
    bias = _cu(c["bias"], torch.float32) if "bias" in c else None
    out, tau = bz.causal_tension(q, k, v, W, float(c["scale"]), return_tau=True, bias=bias)
    loss = (out.float() * _cu(c["d_out"], torch.float32)).sum()
    if "d_tau" in c:
        loss = loss + (tau.float() * _cu(c["d_tau"], torch.float32)).sum()
    loss.backward()
    return out, tau, q.grad, k.grad, v.grad


def _lp(xs):
    """Inputs or cotangents for the oracle run in bf16 arithmetic."""
    return [None if x is None else x.detach().to(torch.bfloat16) for x in xs]


def _oracle_raw(c, dtype, compute=torch.float64):
    """The oracle on the dtype-rounded inputs, in float64 (exact golden for
    fp32) or, with ``compute=torch.bfloat16``, in bf16 arithmetic — the
    reference path (ops.py:29-63) as torch runs it on bf16 tensors."""
    B, T, H, HD, W = [int(x) for x in c["meta"]]
    rd = lambda a: torch.from_numpy(np.asarray(a)).to(dtype).to(compute)
    bias = torch.from_numpy(np.asarray(c["bias"], np.float64)).to(compute) if "bias" in c else None
    d_tau = rd(c["d_tau"]) if "d_tau" in c else None

    def fn(q, k, v):
        return orc.local_tension_raw(q, k, v, W, float(c["scale"]), bias, return_tau=True)

    # autograd hands the op cotangents in the output dtype: round them too
    (o, t), (dq, dk, dv) = orc.tension_with_grads(
        fn, [rd(c["q"]), rd(c["k"]), rd(c["v"])], [rd(c["d_out"]), d_tau])
    return o, t, dq, dk, dv


@cuda
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_raw_op_matches_reference_golden(bz, golden_op, dtype):
    for name, c in sorted(golden_op.items()):
        got = _run_raw(bz, c, dtype)
        if dtype == torch.float32:
            ref = [c["out"], c["tau"], c["dq"], c["dk"], c["dv"]]
            ref_lp = [None] * 5
        else:
            ref = _oracle_raw(c, dtype)
            ref_lp = _oracle_raw(c, dtype, compute=torch.bfloat16)
        for g, r, rl, what in zip(got, ref, ref_lp, ("out", "tau", "dq", "dk", "dv")):
            assert_close(g, r, dtype, f"{name}/{dtype}/{what}", ref_lp=rl)


@cuda
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_layer_matches_reference_golden(bz, golden_layer, dtype):
    """RoPE + local/global tension + τ-mass normalisation + τ export vs
    model.py's own layer (golden), forward and backward."""
    for name, c in sorted(golden_layer.items()):
        B, T, H, HD, W, Wl, msl = [int(x) for x in c["meta"]]
        if dtype == torch.float32:
            qa, ka, va = c["q_raw"], c["k_raw"], c["v"]
        else:
            qa, ka, va = [torch.from_numpy(c[n]).to(dtype).double().numpy()
                          for n in ("q_raw", "k_raw", "v")]
        q, k, v = [_cu(a, dtype).requires_grad_(True) for a in (qa, ka, va)]
        bias = _cu(c["bias"], torch.float32) if "bias" in c else None
        out, tau = bz.tension(q, k, v, window=None if W < 0 else W,
                              scale=float(c["scale"]), rope_base=10_000.0, rope_len=msl,
                              bias=bias, return_tau=True, normalize="mass", tau_window=Wl)
        d_out = _cu(c["d_out"], torch.float32)
        d_tau = _cu(c["d_tau"], torch.float32)
        ((out.float() * d_out).sum() + (tau.float() * d_tau).sum()).backward()
        if dtype == torch.float32:
            ref = [c["out"], c["tau"], c["dq_raw"], c["dk_raw"], c["dv"]]
        else:
            bias64 = torch.from_numpy(c["bias"]) if "bias" in c else None

            def fn(q_, k_, v_):
                return orc.fused_reference(q_, k_, v_, window=None if W < 0 else W,
                                           scale=float(c["scale"]), bias=bias64,
                                           local_window=Wl, max_seq_len=msl)
            rd = lambda a: torch.from_numpy(a).to(dtype).double()
            (o, t), grads = orc.tension_with_grads(
                fn, [torch.from_numpy(a) for a in (qa, ka, va)],
                [rd(c["d_out"]), rd(c["d_tau"])])
            ref = [o, t, *grads]
        for g, r, what in zip((out, tau, q.grad, k.grad, v.grad), ref,
                              ("out", "tau", "dq", "dk", "dv")):
            assert_close(g, r, dtype, f"{name}/{dtype}/{what}")


@cuda
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_out_identical_with_and_without_tau(bz, dtype):
    """test_tau.py:47-60 — requesting τ must not change Out (bit-exact)."""
    torch.manual_seed(1)
    for (B, T, H, HD, W) in ((2, 16, 2, 16, 6), (2, 300, 3, 64, 64)):
        q, k, v = [torch.randn(B, T, H, HD, device="cuda", dtype=dtype) for _ in range(3)]
        a = bz.causal_tension(q, k, v, W, math.sqrt(HD))
        b, _ = bz.causal_tension(q, k, v, W, math.sqrt(HD), return_tau=True)
        assert torch.equal(a, b)


@cuda
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_backward_tau_unused_matches_no_tau(bz, dtype):
    """test_tau.py:102-127 — τ returned but unused gives the same grads."""
    torch.manual_seed(3)
    B, T, H, HD, W = 2, 200, 2, 64, 32
    base = [torch.randn(B, T, H, HD, device="cuda", dtype=dtype) for _ in range(3)]
    d_out = torch.randn(B, T, H, HD, device="cuda", dtype=dtype)
    qa, ka, va = [x.clone().requires_grad_(True) for x in base]
    (bz.causal_tension(qa, ka, va, W, 8.0) * d_out).sum().backward()
    qb, kb, vb = [x.clone().requires_grad_(True) for x in base]
    out_b, _ = bz.causal_tension(qb, kb, vb, W, 8.0, return_tau=True)
    (out_b * d_out).sum().backward()
    for ga, gb in ((qa.grad, qb.grad), (ka.grad, kb.grad), (va.grad, vb.grad)):
        assert (ga.float() - gb.float()).abs().max().item() <= 1e-5


@cuda
def test_zero_bias_equals_no_bias(bz):
    """ts_bridge/bias_smoke.py:10-25 — a zero bias is the unbiased op."""
    torch.manual_seed(5)
    B, T, H, HD, W = 2, 130, 2, 64, 16
    q, k, v = [torch.randn(B, T, H, HD, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    a = bz.causal_tension(q, k, v, W, 8.0)
    b = bz.causal_tension(q, k, v, W, 8.0, bias=torch.zeros(B, T, W, device="cuda"))
    assert torch.equal(a, b)


@cuda
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_prefix_rows_invariant_to_future(bz, dtype):
    """ts_bridge/streaming_parity.py:20-24 — by causality the τ rows and
    outputs of a prefix do not depend on later tokens (bit-identical)."""
    torch.manual_seed(6)
    B, T, H, HD, W = 1, 384, 2, 64, 64
    q, k, v = [torch.randn(B, T, H, HD, device="cuda", dtype=dtype) for _ in range(3)]
    full_o, full_t = bz.tension(q, k, v, window=W, return_tau=True)
    for Tp in (128, 200):
        o, t = bz.tension(q[:, :Tp].contiguous(), k[:, :Tp].contiguous(),
                          v[:, :Tp].contiguous(), window=W, return_tau=True)
        assert torch.equal(o, full_o[:, :Tp])
        assert torch.equal(t, full_t[:, :Tp])


@cuda
@pytest.mark.parametrize("W", [8, 32, 64, 100, 128, 129, 256])
@pytest.mark.parametrize("normalize", ["mass", "count", None])
def test_fused_local_bf16_vs_oracle(bz, W, normalize):
    """Fused local op at HD 64 (the tensor-core shape) across windows —
    the band kernels up to W 128, the key-tile streaming kernels above —
    normalisations, bias and τ cotangent, ragged T."""
    torch.manual_seed(100 + W)
    B, T, H, HD = 2, 333, 3, 64
    dt = torch.bfloat16
    q, k, v, d_out = [torch.randn(B, T, H, HD, dtype=dt) for _ in range(4)]
    bias = torch.randn(B, T, W) * 0.5
    d_tau = (torch.randn(B, T, H, W) * 0.1).to(dt)
    qg, kg, vg = [x.cuda().requires_grad_(True) for x in (q, k, v)]
    out, tau = bz.tension(qg, kg, vg, window=W, bias=bias.cuda(), return_tau=True,
                          normalize=normalize)
    assert bz.last_path() == "tcgen05"
    ((out.float() * d_out.cuda().float()).sum() + (tau.float() * d_tau.cuda().float()).sum()).backward()
    assert bz.last_path() == "tcgen05"

    def fn(q_, k_, v_):
        return orc.fused_reference(q_, k_, v_, window=W, scale=8.0, bias=bias.to(q_.dtype),
                                   normalize=normalize or "none")
    (o, t), grads = orc.tension_with_grads(fn, [x.double() for x in (q, k, v)],
                                           [d_out.double(), d_tau.double()])
    ref_lp = [None] * 5
    if normalize is None:  # raw Σ τ·V: the reference's own bf16 computation as the yardstick
        (ol, tl), gl = orc.tension_with_grads(fn, _lp((q, k, v)), _lp((d_out, d_tau)))
        ref_lp = [ol, tl, *gl]
    for g, r, rl, what in zip((out, tau, qg.grad, kg.grad, vg.grad), (o, t, *grads), ref_lp,
                              ("out", "tau", "dq", "dk", "dv")):
        assert_close(g, r, dt, f"W{W}/{normalize}/{what}", ref_lp=rl)


def _global_reference(q, k, v, scale, bias, tw, normalize):
    """RoPE + the global block (model.py:200-204, 217-237) in float64; raw
    Σ τ·V when ``normalize`` is None."""
    def fn(q_, k_, v_):
        T, HD = q_.shape[1], q_.shape[3]
        cos, sin = orc.rope_tables(HD, T, 10_000.0, q_.dtype)
        out, tau_full, tau_local = orc.global_tension(orc.rope(q_, cos, sin), orc.rope(k_, cos, sin),
                                                      v_, scale, bias, tw)
        if normalize is None:
            out = torch.einsum("bths,bshd->bthd", tau_full, v_)
        return out, tau_local
    return fn


@cuda
@pytest.mark.parametrize("T", [1, 100, 128, 300])
@pytest.mark.parametrize("normalize", ["mass", None])
def test_fused_global_bf16_vs_oracle(bz, T, normalize):
    """Global full-causal block on the tensor-core path (bf16, HD 64): RoPE,
    bias [B,T,T], the exported τ window and its cotangent, ragged T."""
    torch.manual_seed(200 + T)
    B, H, HD, tw = 2, 2, 64, min(64, T)
    dt = torch.bfloat16
    q, k, v, d_out = [torch.randn(B, T, H, HD, dtype=dt) for _ in range(4)]
    bias = torch.randn(B, T, T) * 0.5
    d_tau = (torch.randn(B, T, H, tw) * 0.1).to(dt)
    qg, kg, vg = [x.cuda().requires_grad_(True) for x in (q, k, v)]
    out, tau = bz.tension(qg, kg, vg, window=None, bias=bias.cuda(), return_tau=True,
                          normalize=normalize, tau_window=tw)
    assert bz.last_path() == "tcgen05"
    ((out.float() * d_out.cuda().float()).sum() + (tau.float() * d_tau.cuda().float()).sum()).backward()
    assert bz.last_path() == "tcgen05"
    fn = _global_reference(None, None, None, 8.0, bias.double(), tw, normalize)
    (o, t), grads = orc.tension_with_grads(fn, [x.double() for x in (q, k, v)],
                                           [d_out.double(), d_tau.double()])
    ref_lp = [None] * 5
    if normalize is None:  # raw Σ τ·V: the global einsum path in bf16 (model.py:217-229 under autocast)
        fl = _global_reference(None, None, None, 8.0, bias.bfloat16(), tw, normalize)
        (ol, tl), gl = orc.tension_with_grads(fl, _lp((q, k, v)), _lp((d_out, d_tau)))
        ref_lp = [ol, tl, *gl]
    for g, r, rl, what in zip((out, tau, qg.grad, kg.grad, vg.grad), (o, t, *grads), ref_lp,
                              ("out", "tau", "dq", "dk", "dv")):
        assert_close(g, r, dt, f"global T{T}/{normalize}/{what}", ref_lp=rl)


@cuda
def test_global_bf16_large_spot_check(bz):
    """Global block at T 1024 (the 117M layer's sequence), B1 H4: forward and
    all gradients against the float64 oracle."""
    torch.manual_seed(9)
    B, T, H, HD = 1, 1024, 4, 64
    dt = torch.bfloat16
    q, k, v, d_out = [torch.randn(B, T, H, HD, dtype=dt) for _ in range(4)]
    qg, kg, vg = [x.cuda().requires_grad_(True) for x in (q, k, v)]
    out = bz.tension(qg, kg, vg, window=None)
    assert bz.last_path() == "tcgen05"
    (out.float() * d_out.cuda().float()).sum().backward()
    fn = _global_reference(None, None, None, 8.0, None, 64, "mass")
    outs, grads = orc.tension_with_grads(lambda a, b, c: (fn(a, b, c)[0],),
                                         [x.double() for x in (q, k, v)], [d_out.double()])
    o = outs[0]
    for g, r, what in zip((out, qg.grad, kg.grad, vg.grad), (o, *grads), ("out", "dq", "dk", "dv")):
        assert_close(g, r, dt, f"global T1024/{what}")


@cuda
def test_large_bf16_spot_check(bz):
    """triton_tension/test.py:212-227 at B4 T512 H12 HD64 W64 (bf16)."""
    torch.manual_seed(3)
    B, T, H, HD, W = 4, 512, 12, 64, 64
    q, k, v = [torch.randn(B, T, H, HD, dtype=torch.bfloat16) for _ in range(3)]
    out = bz.causal_tension(q.cuda(), k.cuda(), v.cuda(), W, 8.0).float().cpu()
    ref = orc.local_tension_raw(q.double(), k.double(), v.double(), W, 8.0)
    rel = (out.double() - ref).abs() / (ref.abs() + 1e-6)
    assert rel.mean().item() < 0.02
    assert_close(out, ref, torch.bfloat16, "large",
                 ref_lp=orc.local_tension_raw(q, k, v, W, 8.0))


@cuda
def test_memory_vs_unfold(bz):
    """test_tau.py:130-159 — peak memory of the τ-returning op stays far
    below the unfold gather (B4 T1024 H16 HD64 W256 bf16)."""
    B, T, H, HD, W = 4, 1024, 16, 64, 256
    torch.manual_seed(4)
    q, k, v = [torch.randn(B, T, H, HD, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    before = torch.cuda.memory_allocated()
    out, tau = bz.causal_tension(q, k, v, W, 8.0, return_tau=True)
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated()
    unfold_bytes = B * T * H * W * HD * 2
    assert peak - before < unfold_bytes / 4


@cuda
def test_cpu_and_float64_inputs_raise(bz):
    q = torch.randn(1, 8, 1, 16)
    with pytest.raises(RuntimeError):
        bz.causal_tension(q, q, q, 4, 4.0)
    qd = q.double().cuda()
    with pytest.raises(TypeError):
        bz.causal_tension(qd, qd, qd, 4, 4.0)


@cuda
def test_bias_shape_assertion(bz):
    q = torch.randn(1, 8, 1, 16, device="cuda")
    with pytest.raises(AssertionError):
        bz.causal_tension(q, q, q, 4, 4.0, bias=torch.zeros(1, 8, 5, device="cuda"))


@cuda
@pytest.mark.parametrize("W,T,with_tau", [(16, 96, True), (64, 333, True), (128, 260, False)])
def test_mixed_dtype_model_call_site(bz, W, T, with_tau):
    """model.py under bf16 autocast feeds fp32 (RoPE-promoted) Q/K with bf16 V;
    the op returns Q.dtype and grads in each input's dtype (ops.py:122-124,
    186-187).  The call runs on the tensor cores from bf16 copies of Q/K, so
    it is held to the bf16 bound: out (and τ) and all gradients against the
    float64 oracle on the same inputs, with bias (and a τ cotangent).  fp32 τ
    export is served by the band kernel up to W 64 (its staging rows fit);
    W 128 is checked without τ."""
    torch.manual_seed(9 + W)
    B, H, HD = 2, 2, 64
    q = torch.randn(B, T, H, HD, device="cuda", requires_grad=True)
    k = torch.randn(B, T, H, HD, device="cuda", requires_grad=True)
    v = torch.randn(B, T, H, HD, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    bias = torch.randn(B, T, W, device="cuda") * 0.5
    d_out = torch.randn(B, T, H, HD, device="cuda")
    d_tau = torch.randn(B, T, H, W, device="cuda") * 0.1
    if with_tau:
        out, tau = bz.causal_tension(q, k, v, W, 8.0, return_tau=True, bias=bias)
        assert tau.dtype == torch.float32
    else:
        out = bz.causal_tension(q, k, v, W, 8.0, bias=bias)
        tau = torch.zeros(B, T, H, W, device="cuda")
        d_tau = torch.zeros_like(tau)
    assert bz.last_path() == "tcgen05"
    assert out.dtype == torch.float32
    ((out * d_out).sum() + (tau * d_tau).sum()).backward()
    assert bz.last_path() == "tcgen05"
    assert q.grad.dtype == torch.float32 and k.grad.dtype == torch.float32
    assert v.grad.dtype == torch.bfloat16

    def fn(q_, k_, v_):
        return orc.local_tension_raw(q_, k_, v_, W, 8.0, bias.to(q_.dtype).cpu(), return_tau=True)
    ins = [x.detach().cpu() for x in (q, k, v)]
    (o, t), grads = orc.tension_with_grads(fn, [x.double() for x in ins],
                                           [d_out.double().cpu(), d_tau.double().cpu()])
    (ol, tl), gl = orc.tension_with_grads(fn, _lp(ins), _lp((d_out.cpu(), d_tau.cpu())))
    for g, r, rl, what in zip((out, tau, q.grad, k.grad, v.grad), (o, t, *grads), (ol, tl, *gl),
                              ("out", "tau", "dq", "dk", "dv")):
        if what == "tau" and not with_tau:
            continue
        assert_close(g, r, torch.bfloat16, f"mixed W{W}/{what}", ref_lp=rl)


@cuda
def test_triton_tension_shim_model_call_site_117m_layer(bz):
    """The drop-in at model.py's own call site: ``install_as_triton_tension()``
    makes ``from triton_tension import causal_tension`` (model.py:248,
    triton_tension/__init__.py:1-3) and ``triton_tension.ops.causal_tension``
    resolve here; then model.py:250-258's sequence at the 117M layer shape
    (B16 T1024 H12 HD64 W64) under bf16 autocast — RoPE'd fp32 Q/K, bf16 V,
    τ returned, out = S / clamp(Στ, 1e-6) — forward and backward, on the
    tensor cores, against the float64 oracle on batch row 0, heads 0-1."""
    import importlib
    import sys
    saved = {n: sys.modules.get(n) for n in ("triton_tension", "triton_tension.ops")}
    try:
        bz.install_as_triton_tension()
        from triton_tension import causal_tension
        ops_mod = importlib.import_module("triton_tension.ops")
        assert causal_tension is bz.causal_tension and ops_mod.causal_tension is bz.causal_tension
        B, T, H, HD, W = 16, 1024, 12, 64, 64
        g = torch.Generator().manual_seed(21)
        q_raw, k_raw, v_raw, d = [torch.randn(B, T, H, HD, generator=g).to(torch.bfloat16) for _ in range(4)]
        cos, sin = [x.cuda() for x in orc.rope_tables(HD, T, 10_000.0, torch.float32)]

        def model_rope(x):  # model.py:75-81: fp32 table buffers, no cast
            c, s_ = cos[:T].unsqueeze(0).unsqueeze(2), sin[:T].unsqueeze(0).unsqueeze(2)
            x1, x2 = x[..., :HD // 2], x[..., HD // 2:]
            return torch.cat([x1 * c - x2 * s_, x1 * s_ + x2 * c], dim=-1)
        q_leaf, k_leaf, v_leaf = [x.cuda().requires_grad_(True) for x in (q_raw, k_raw, v_raw)]
        with torch.autocast("cuda", dtype=torch.bfloat16):
            # model.py:203-204: bf16 projections times fp32 tables → fp32 Q/K
            q = model_rope(q_leaf)
            k = model_rope(k_leaf)
            assert q.dtype == torch.float32 and v_leaf.dtype == torch.bfloat16
            msg, tau = causal_tension(q, k, v_leaf, W, 8.0, return_tau=True, bias=None)
            assert bz.last_path() == "tcgen05"
            out = msg / tau.sum(-1).clamp(min=1e-6).unsqueeze(-1)  # model.py:257-258
        gq, gk, gv = torch.autograd.grad(out, (q_leaf, k_leaf, v_leaf), d.cuda().float())
        assert bz.last_path() == "tcgen05"
        sl = lambda x: x[0:1, :, 0:2]

        def fn(a, b, c):
            return orc.fused_reference(a, b, c, window=W, scale=8.0)
        (o, t), grads = orc.tension_with_grads(fn, [sl(x).double() for x in (q_raw, k_raw, v_raw)],
                                               [sl(d).double(), None])
        for got, ref, what in zip((out, tau, gq, gk, gv), (o, t, *grads), ("out", "tau", "dq", "dk", "dv")):
            assert_close(sl(got), ref, torch.bfloat16, f"shim 117M layer/{what}")
    finally:
        for n, m in saved.items():
            if m is None:
                sys.modules.pop(n, None)
            else:
                sys.modules[n] = m


@cuda
@pytest.mark.parametrize("shape", [(1, 128, 1), (2, 128, 1), (1, 256, 2), (2, 130, 3)])
def test_backward_on_autograd_thread_small_shapes(bz, shape):
    """grad_outputs passed straight to autograd.grad: the backward runs on the
    autograd device thread, which must get the data's device and context
    bound before tensor maps are encoded."""
    B, T, H = shape
    torch.manual_seed(11)
    q, k, v, d = [torch.randn(B, T, H, 64, device="cuda", dtype=torch.bfloat16) for _ in range(4)]
    qg, kg, vg = [x.clone().requires_grad_(True) for x in (q, k, v)]
    out = bz.tension(qg, kg, vg, window=64)
    gq, gk, gv = torch.autograd.grad(out, (qg, kg, vg), d)

    def fn(a, b, c):
        return orc.fused_reference(a, b, c, window=64, scale=8.0)[0]
    (o,), grads = orc.tension_with_grads(fn, [x.double().cpu() for x in (q, k, v)],
                                         [d.double().cpu()])
    for g, r, what in zip((out, gq, gk, gv), (o, *grads), ("out", "dq", "dk", "dv")):
        assert_close(g, r, torch.bfloat16, f"{shape}/{what}")


@cuda
@pytest.mark.parametrize("W", [64, 256])
def test_bench_shape_parity(bz, W):
    """The benchmark's own step (B8 H12 T2048 HD64, RoPE,
    τ-mass) at full size: out and every gradient of batch row 0, heads 0-1,
    against the float64 oracle — W 64 on the band kernels, W 256 on the
    key-tile kernels."""
    B, H, T, HD = 8, 12, 2048, 64
    g = torch.Generator().manual_seed(1234)
    q, k, v, d = [torch.randn(B, T, H, HD, generator=g).to(torch.bfloat16) for _ in range(4)]
    qg, kg, vg = [x.cuda().requires_grad_(True) for x in (q, k, v)]
    out = bz.tension(qg, kg, vg, window=W, normalize="mass")
    gq, gk, gv = torch.autograd.grad(out, (qg, kg, vg), d.cuda())
    assert bz.last_path() == "tcgen05"
    sl = lambda x: x[0:1, :, 0:2]

    def fn(a, b, c):
        return orc.fused_reference(a, b, c, window=W, scale=8.0)[0]
    (o,), grads = orc.tension_with_grads(fn, [sl(x).double() for x in (q, k, v)], [sl(d).double()])
    for got, ref, what in zip((out, gq, gk, gv), (o, *grads), ("out", "dq", "dk", "dv")):
        assert_close(sl(got), ref, torch.bfloat16, f"bench shape W{W}/{what}")


@cuda
@pytest.mark.parametrize("window,T", [(64, 700), (200, 700), (None, 700)])
def test_tensor_core_paths_repeat_bit_identical(bz, window, T):
    """Every tensor-core kernel family gives bit-identical out, τ and grads
    over repeated calls on the same inputs (no atomics anywhere, so any
    difference would be a pipeline hand-off that depends on timing): the
    band kernels (W 64), the key-tile kernels for wide windows (W 200) and
    the global block, with bias and τ cotangent."""
    torch.manual_seed(300 + T)
    B, H, HD = 2, 4, 64
    q, k, v, d = [torch.randn(B, T, H, HD, dtype=torch.bfloat16, device="cuda") for _ in range(4)]
    W = window if window is not None else 64
    bias = torch.randn(B, T, W if window is not None else T, device="cuda") * 0.5
    d_tau = (torch.randn(B, T, H, W, device="cuda") * 0.1).to(torch.bfloat16)
    runs = []
    for _ in range(6):
        qg, kg, vg = [x.clone().requires_grad_(True) for x in (q, k, v)]
        out, tau = bz.tension(qg, kg, vg, window=window, bias=bias, return_tau=True,
                              tau_window=None if window is not None else W)
        ((out.float() * d.float()).sum() + (tau.float() * d_tau.float()).sum()).backward()
        assert bz.last_path() == "tcgen05"
        runs.append([x.detach().clone() for x in (out, tau, qg.grad, kg.grad, vg.grad)])
    for r in runs[1:]:
        for a, b, what in zip(runs[0], r, ("out", "tau", "dq", "dk", "dv")):
            assert torch.equal(a, b), f"{what} differs between identical calls"


@cuda
@pytest.mark.parametrize("mixed", [False, True])
def test_causal_tension_compiles_without_graph_breaks(bz, mixed):
    """train.py:776-780 wraps model.py in torch.compile; the drop-in op is a
    pair of torch.library custom ops with fake implementations, so the
    model.py use of it (model.py:248-258: τ returned, τ-mass division)
    compiles as one graph (fullgraph=True fails on any break) through
    AOTAutograd, and gives the eager values and gradients."""
    torch.manual_seed(31)
    B, T, H, HD, W = 2, 200, 3, 64, 64
    qd = torch.float32 if mixed else torch.bfloat16
    q0 = torch.randn(B, T, H, HD, device="cuda", dtype=qd)
    k0 = torch.randn(B, T, H, HD, device="cuda", dtype=qd)
    v0 = torch.randn(B, T, H, HD, device="cuda", dtype=torch.bfloat16)

    def f(q, k, v):
        msg, tau = bz.causal_tension(q, k, v, W, 8.0, return_tau=True)
        out = msg / tau.sum(-1).clamp(min=1e-6).unsqueeze(-1)
        return (out.float() ** 2).sum()

    def run(fn):
        q, k, v = [x.clone().requires_grad_(True) for x in (q0, k0, v0)]
        loss = fn(q, k, v)
        return (loss.detach(), *torch.autograd.grad(loss, (q, k, v)))

    torch._dynamo.reset()
    compiled = torch.compile(f, backend="aot_eager", fullgraph=True)
    got = run(compiled)
    want = run(f)
    for a, b, what in zip(got, want, ("loss", "dq", "dk", "dv")):
        assert a.dtype == b.dtype, what
        assert torch.allclose(a.float(), b.float(), rtol=1e-5, atol=1e-5), what
    torch._dynamo.reset()
