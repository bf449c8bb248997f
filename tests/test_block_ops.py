"""Fused residual add + RMSNorm and SwiGLU (``bozo_b200.block_ops``,
``include/bozo_block_ops.h``) against the framework ops they replace
(``F.rms_norm(x + y)``, ``F.silu(g) * v``), forward and backward, for the
dtype pairings of the model (fp32 stream + bf16 projection under autocast,
fp32 + fp32, bf16 + bf16) and every supported width; the scale gradient is
bit-identical run to run.  CPU: the kernels are not taken for CPU tensors.
"""
import pytest
import torch
import torch.nn.functional as F

from bozo_b200 import block_ops


def _ref_norm(x, y, scale, eps):
    s = x + y if y is not None else x
    return F.rms_norm(s, s.shape[-1:], scale, eps)


TOL = {torch.float32: dict(rtol=2e-5, atol=2e-5), torch.bfloat16: dict(rtol=1.6e-2, atol=1.6e-2)}


@pytest.mark.gpu
@pytest.mark.parametrize("D", [128, 768, 1024])
@pytest.mark.parametrize("xd,yd", [(torch.float32, torch.bfloat16), (torch.float32, torch.float32),
                                   (torch.bfloat16, torch.bfloat16), (torch.float32, None)])
def test_add_rms_norm_matches_framework(D, xd, yd):
    g = torch.Generator().manual_seed(D)
    dev = torch.device("cuda:0")
    x = (torch.randn(3, 333, D, generator=g) * 2).to(dev, xd)
    y = torch.randn(3, 333, D, generator=g).to(dev, yd) if yd is not None else None
    scale = (1 + 0.1 * torch.randn(D, generator=g)).to(dev, xd)
    dout = torch.randn(3, 333, D, generator=g).to(dev, xd)
    leaves = [t.clone().requires_grad_(True) if t is not None else None for t in (x, y, scale)]
    ref_leaves = [t.clone().requires_grad_(True) if t is not None else None for t in (x, y, scale)]
    assert block_ops.norm_applies(x, y)
    out = block_ops.add_rms_norm(leaves[0], leaves[1], leaves[2], 1e-6)
    ref = _ref_norm(ref_leaves[0], ref_leaves[1], ref_leaves[2], 1e-6)
    assert out.dtype == ref.dtype == xd
    torch.testing.assert_close(out, ref, **TOL[xd])
    out.backward(dout)
    ref.backward(dout)
    for name, a, b in zip(("dx", "dy", "dscale"), leaves, ref_leaves):
        if a is None:
            continue
        assert a.grad.dtype == b.grad.dtype
        scale_ = float(b.grad.abs().max())
        tol = dict(TOL[a.dtype])
        tol["atol"] = tol["atol"] * max(1.0, scale_)
        torch.testing.assert_close(a.grad, b.grad, **tol, msg=f"{name} D{D} {xd} {yd}")


@pytest.mark.gpu
def test_scale_gradient_is_deterministic():
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(1)
    x = torch.randn(16384, 768, generator=g).to(dev)
    y = torch.randn(16384, 768, generator=g).to(dev, torch.bfloat16)
    dout = torch.randn(16384, 768, generator=g).to(dev)
    grads = []
    for _ in range(2):
        s = torch.ones(768, device=dev, requires_grad=True)
        block_ops.add_rms_norm(x, y, s, 1e-6).backward(dout)
        grads.append(s.grad.clone())
    assert torch.equal(grads[0], grads[1])


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_swiglu_matches_framework(dtype):
    gen = torch.Generator().manual_seed(2)
    dev = torch.device("cuda:0")
    g = (torch.randn(4, 100, 2304, generator=gen) * 3).to(dev, dtype)
    v = torch.randn(4, 100, 2304, generator=gen).to(dev, dtype)
    dh = torch.randn(4, 100, 2304, generator=gen).to(dev, dtype)
    a = [g.clone().requires_grad_(True), v.clone().requires_grad_(True)]
    b = [g.clone().requires_grad_(True), v.clone().requires_grad_(True)]
    out = block_ops.swiglu(*a)
    ref = F.silu(b[0]) * b[1]
    tol = TOL[dtype] if dtype == torch.float32 else dict(rtol=1.6e-2, atol=2e-2)
    torch.testing.assert_close(out, ref, **tol)
    out.backward(dh)
    ref.backward(dh)
    for x, y in zip(a, b):
        torch.testing.assert_close(x.grad, y.grad, rtol=tol["rtol"], atol=tol["atol"] * 4)


def test_cpu_tensors_take_the_framework_ops():
    x = torch.randn(2, 4, 128)
    assert not block_ops.norm_applies(x, None)
    assert not block_ops.swiglu_applies(x, x)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,R,V", [(torch.bfloat16, 4096, 32768), (torch.float32, 1000, 1000),
                                       (torch.bfloat16, 77, 97 * 8)])
def test_cross_entropy_matches_framework(dtype, R, V):
    """Mean cross-entropy and its logits gradient against F.cross_entropy in
    fp32 on the same logits, the gradient rounded to the logits' dtype (the
    kernel's rounding point); some targets are the ignore index −100.  (The
    framework's own autocast path rounds each row's log-probabilities to
    bf16, so its loss differs from the fp32 value by ~1e-4 relative.)"""
    gen = torch.Generator().manual_seed(R)
    dev = torch.device("cuda:0")
    logits = (torch.randn(R, V, generator=gen) * 4).to(dev, dtype)
    targets = torch.randint(0, V, (R,), generator=gen)
    targets[::13] = -100
    targets = targets.to(dev)
    a = logits.clone().requires_grad_(True)
    b = logits.clone().requires_grad_(True)
    assert block_ops.xent_applies(a, targets)
    loss = block_ops.cross_entropy(a, targets)
    ref = F.cross_entropy(b.float(), targets)
    assert loss.dtype == torch.float32
    torch.testing.assert_close(loss, ref, rtol=1e-5, atol=1e-6)
    (loss * 3.0).backward()
    (ref * 3.0).backward()
    assert a.grad.dtype == b.grad.dtype == dtype
    tol = dict(rtol=1e-5, atol=1e-8) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-7)
    torch.testing.assert_close(a.grad, b.grad, **tol)
    assert float(a.grad[::13].abs().max()) == 0.0


def _ref_wo_norm(x, msg, w, scale, eps):
    """float64 restatement of rms_norm(x + wo(msg)) with the projection's
    output rounded to bf16 (model.py:259/283 under bf16 autocast) and the sum
    rounded to x's dtype."""
    y = (msg.to(torch.bfloat16).double() @ w.to(torch.bfloat16).double().T).to(torch.bfloat16)
    s = (x.double() + y.double()).to(x.dtype).double()
    rstd = torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps)
    return s * rstd * scale.to(x.dtype).double()


@pytest.mark.gpu
@pytest.mark.parametrize("D", [64, 128, 256, 384, 512, 768, 1024, 2048])
@pytest.mark.parametrize("rows", [1, 77, 999])
@pytest.mark.parametrize("xd", [torch.float32, torch.bfloat16])
def test_wo_add_rms_norm_matches_unfused(D, rows, xd):
    if D == 2048 and xd == torch.float32:
        pytest.skip("fp32 residual tile of a 2048-wide row share does not fit beside the ring")
    from tests._tol import assert_close
    g = torch.Generator().manual_seed(D * 7 + rows)
    dev = torch.device("cuda:0")
    x = (torch.randn(rows, D, generator=g) * 2).to(dev, xd)
    msg = torch.randn(rows, D, generator=g).to(dev, torch.bfloat16)
    w = (torch.randn(D, D, generator=g) / D ** 0.5).to(dev, torch.bfloat16)
    scale = (1 + 0.1 * torch.randn(D, generator=g)).to(dev, xd)
    out = block_ops.wo_add_rms_norm(x, msg, w, scale, 1e-6)
    assert out.dtype == xd and out.shape == x.shape
    assert_close(out, _ref_wo_norm(x, msg, w, scale, 1e-6), torch.bfloat16, f"D{D} rows{rows} {xd}")
    y = F.linear(msg, w)
    if block_ops.norm_applies(x, y):  # the unfused kernels' widths
        unfused = block_ops.add_rms_norm(x, y, scale, 1e-6)
        assert_close(out, unfused, torch.bfloat16, f"vs unfused D{D} rows{rows} {xd}")


@pytest.mark.gpu
def test_wo_add_rms_norm_at_prefill_size():
    # the 117M model's width over B8 x T2048 rows, fp32 residual stream under
    # autocast; fp32 weights go through the cached bf16 copy
    g = torch.Generator().manual_seed(5)
    dev = torch.device("cuda:0")
    R, D = 8 * 2048, 768
    x = torch.randn(R, D, generator=g).to(dev)
    msg = torch.randn(R, D, generator=g).to(dev)
    w = (torch.randn(D, D, generator=g) / D ** 0.5).to(dev)
    scale = (1 + 0.1 * torch.randn(D, generator=g)).to(dev)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        out = block_ops.wo_add_rms_norm(x, msg, w, scale, 1e-6)
        again = block_ops.wo_add_rms_norm(x, msg, w, scale, 1e-6)
    assert torch.equal(out, again)
    ref = _ref_wo_norm(x, msg, w, scale, 1e-6)
    from tests._tol import assert_close
    for lo in range(0, R, 4096):  # float64 reference in slices to bound host memory
        assert_close(out[lo:lo + 4096], ref[lo:lo + 4096], torch.bfloat16, f"rows {lo}+")
    # unit RMS of every normalised row (before the scale)
    rms = (out.double() / scale.double()).pow(2).mean(-1).sqrt()
    assert float((rms - 1).abs().max()) < 1e-3


@pytest.mark.gpu
def test_model_eval_takes_the_fused_projection(monkeypatch):
    from bozo_b200 import lm
    torch.manual_seed(0)
    cfg = lm.TensionConfig(vocab_size=512, dim=256, num_heads=4, num_layers=2, window=32,
                           max_seq_len=128)
    model = lm.TensionLM(cfg).cuda().eval()
    ids = torch.randint(0, 512, (2, 128), device="cuda")
    calls = []
    monkeypatch.setattr(block_ops, "FUSED_WO_NORM", True)
    real = block_ops.wo_add_rms_norm
    monkeypatch.setattr(block_ops, "wo_add_rms_norm",
                        lambda *a, **k: calls.append(1) or real(*a, **k))
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        fused = model(ids)
        assert len(calls) == cfg.num_layers
        monkeypatch.setattr(block_ops, "wo_norm_applies", lambda *a: False)
        unfused = model(ids)
    assert len(calls) == cfg.num_layers
    from tests._tol import assert_close
    assert_close(fused.float(), unfused.float(), torch.bfloat16, "logits")


def test_wo_norm_gating_on_cpu(monkeypatch):
    x = torch.randn(4, 128)
    w = torch.randn(128, 128)
    assert not block_ops.wo_norm_applies(x, x, w)
    monkeypatch.setattr(block_ops, "FUSED_WO_NORM", True)
    assert not block_ops.wo_norm_applies(x, x, w)
    f32, bf = torch.float32, torch.bfloat16
    for D in (64, 128, 256, 384, 512, 768, 1024):
        assert block_ops._wo_width_ok(D, f32) and block_ops._wo_width_ok(D, bf), D
    assert block_ops._wo_width_ok(2048, bf) and not block_ops._wo_width_ok(2048, f32)
    assert not block_ops._wo_width_ok(96, f32) and not block_ops._wo_width_ok(4096, bf)


@pytest.mark.gpu
@pytest.mark.parametrize("D", [768, 1024])
@pytest.mark.parametrize("with_y", [False, True])
def test_add_rms_norm_lp_is_the_norm_and_its_bf16_copy(D, with_y):
    g = torch.Generator().manual_seed(D + with_y)
    dev = torch.device("cuda:0")
    x = (torch.randn(2, 333, D, generator=g) * 2).to(dev)
    y = torch.randn(2, 333, D, generator=g).to(dev, torch.bfloat16) if with_y else None
    scale = (1 + 0.1 * torch.randn(D, generator=g)).to(dev)
    d_out = torch.randn(2, 333, D, generator=g).to(dev)
    d_lp = torch.randn(2, 333, D, generator=g).to(dev, torch.bfloat16)
    leaves = [t.clone().requires_grad_(True) if t is not None else None for t in (x, y, scale)]
    ref_leaves = [t.clone().requires_grad_(True) if t is not None else None for t in (x, y, scale)]
    out, out_lp = block_ops.add_rms_norm_lp(leaves[0], leaves[1], leaves[2], 1e-6)
    ref = block_ops.add_rms_norm(ref_leaves[0], ref_leaves[1], ref_leaves[2], 1e-6)
    assert torch.equal(out, ref)
    assert out_lp.dtype == torch.bfloat16 and torch.equal(out_lp, ref.to(torch.bfloat16))
    torch.autograd.backward((out, out_lp), (d_out, d_lp))
    ref.backward(d_out + d_lp.float())
    for a, b in zip(leaves, ref_leaves):
        if a is not None:
            assert torch.equal(a.grad, b.grad)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_swiglu_packed_matches_two_tensor_swiglu(dtype):
    g = torch.Generator().manual_seed(3)
    dev = torch.device("cuda:0")
    gv = torch.randn(4, 100, 2 * 2304, generator=g).to(dev, dtype)
    dh = torch.randn(4, 100, 2304, generator=g).to(dev, dtype)
    a = gv.clone().requires_grad_(True)
    gg, vv = (t.clone().requires_grad_(True) for t in gv.chunk(2, dim=-1))
    h = block_ops.swiglu_packed(a)
    ref = block_ops.swiglu(gg.contiguous(), vv.contiguous())
    assert torch.equal(h, ref)
    h.backward(dh)
    ref.backward(dh)
    assert torch.equal(a.grad, torch.cat([gg.grad, vv.grad], dim=-1))


def test_packed_swiglu_gating_on_cpu():
    assert not block_ops.swiglu_packed_applies(torch.randn(4, 16))


@pytest.mark.gpu
@pytest.mark.parametrize("V,D,n", [(32768, 768, 16384), (97, 1040, 600), (50, 36, 257)])
def test_embedding_weight_grad_matches_framework(V, D, n):
    """The fused embedding's weight gradient equals the framework's (sums of
    the same fp32 rows, possibly in another order), absent tokens get exact
    zero rows, and two calls give identical bits."""
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(V + D)
    ids = torch.randint(0, max(V // 2, 1), (n,), generator=g).to(dev)  # repeats, absent upper half
    w = torch.randn(V, D, generator=g).to(dev)
    dy = torch.randn(n, D, generator=g).to(dev)
    a = w.clone().requires_grad_(True)
    b = w.clone().requires_grad_(True)
    out = block_ops.embedding(ids, a)
    ref = F.embedding(ids, b)
    assert torch.equal(out, ref)
    (ga,) = torch.autograd.grad(out, a, dy)
    (gb,) = torch.autograd.grad(ref, b, dy)
    torch.testing.assert_close(ga, gb, rtol=1e-5, atol=1e-5)
    absent = torch.ones(V, dtype=torch.bool, device=dev)
    absent[ids] = False
    assert torch.count_nonzero(ga[absent]) == 0
    (ga2,) = torch.autograd.grad(block_ops.embedding(ids, a), a, dy)
    assert torch.equal(ga, ga2)


def test_embedding_gating_on_cpu():
    assert not block_ops.embedding_applies(torch.zeros(4, dtype=torch.long), torch.randn(8, 4))
