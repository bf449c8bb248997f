"""TensionLM harness (bozo_b200/lm.py) against the reference model.

* CPU: the harness with the oracle in place of the operator reproduces the
  reference model's aux-loss training forward and gradients
  (``tests/golden/golden_lm.npz``, made by ``make_golden_lm.py``).
* GPU: the same with the real operator — fp32 (exact CUDA-core path) and
  bf16 autocast (tensor-core path for the local layers).
* CPU, two gloo ranks: one DDP training step equals the single-process step
  with the two half-batch gradients averaged.
"""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from bozo_b200 import lm
from oracle import tension_oracle as orc
from tests.conftest import _load

CFGS = {
    "rope_global": dict(vocab_size=97, dim=128, num_layers=4, num_heads=2, window=64, ffn_mult=3,
                        max_seq_len=192, dropout=0.0, use_oscillation=False, use_rope=True,
                        global_every=2),
    "norope_osc": dict(vocab_size=97, dim=64, num_layers=2, num_heads=4, window=8, ffn_mult=3,
                       max_seq_len=48, dropout=0.0, use_oscillation=True, use_rope=False,
                       global_every=0),
}
WEIGHTS = lm.TrainWeights(w_closure=0.01, w_diversity=0.02, w_consistency=0.0, w_entropy=0.0)


def oracle_tension(q, k, v, *, window, scale, rope_base=10_000.0, rope_len=None, bias=None,
                   return_tau=False, normalize="mass", tau_window=None):
    """The oracle with ``bozo_b200.tension``'s keywords (test-only stand-in)."""
    out, tau = orc.fused_reference(q, k, v, window=window, scale=scale, rope_base=rope_base,
                                   bias=bias, normalize=normalize or "none",
                                   local_window=tau_window or 64, max_seq_len=rope_len)
    out = out.to(q.dtype)
    return (out, tau.to(q.dtype)) if return_tau else out


@pytest.fixture(scope="module")
def golden_lm():
    return _load("golden_lm.npz")


def _model(name, case, device):
    torch.manual_seed(0)
    m = lm.TensionLM(lm.TensionConfig(**CFGS[name]))
    sd = {k[3:]: torch.from_numpy(v) for k, v in case.items() if k.startswith("sd.")}
    missing, unexpected = m.load_state_dict(sd, strict=False)
    # the reference keeps the same parameters and persistent buffers
    assert not unexpected, unexpected
    assert not [k for k in missing if not k.endswith("lm_head.weight")], missing
    return m.to(device)


def _forward_losses(m, case, device, amp=False, fused_aux=False):
    inputs = torch.from_numpy(case["inputs"]).to(device)
    targets = torch.from_numpy(case["targets"]).to(device)
    V = m.cfg.vocab_size
    ctx = (torch.autocast(device_type=device.type, dtype=torch.bfloat16) if amp
           else torch.autocast(device_type=device.type, enabled=False))
    with ctx:
        logits, hidden, tensions = m(inputs, return_all=True)
        ce = torch.nn.functional.cross_entropy(logits.reshape(-1, V), targets.reshape(-1))
        if fused_aux:
            div, cons, ent = lm.aux_losses(tensions, m.window_groups)
        else:
            div = lm.tension_diversity_loss(tensions, m.window_groups)
            cons = lm.constraint_consistency_loss(tensions)
            ent = lm.tension_entropy_loss(tensions)
        parts = dict(ce=ce, closure=lm.manifold_closure_loss(hidden), diversity=div,
                     consistency=cons, entropy=ent)
        loss = (ce + WEIGHTS.w_closure * parts["closure"] + WEIGHTS.w_diversity * parts["diversity"]
                + WEIGHTS.w_consistency * parts["consistency"] + WEIGHTS.w_entropy * parts["entropy"])
    loss.backward()
    return logits, hidden, tensions, parts, loss


def _check(m, case, logits, hidden, tensions, parts, loss, rtol, atol, grad_rtol, grad_atol):
    def close(got, ref, what, rt=rtol, at=atol):
        g = got.detach().float().cpu().numpy()
        np.testing.assert_allclose(g, ref, rtol=rt, atol=at, err_msg=what)
    close(logits, case["logits"], "logits")
    close(hidden, case["hidden"], "hidden")
    for i, t in enumerate(tensions):
        close(t, case[f"tau{i}"], f"tau{i}")
    for k, v in parts.items():
        close(v, case[k], k)
    close(loss, case["loss"], "loss")
    params = dict(m.named_parameters())
    for k in case:
        if k.startswith("grad."):
            close(params[k[5:]].grad, case[k], k, grad_rtol, grad_atol)


@pytest.mark.parametrize("name", list(CFGS))
def test_harness_matches_reference_model_cpu(golden_lm, name):
    case = golden_lm[name]
    m = _model(name, case, torch.device("cpu"))
    m.set_tension_fn(oracle_tension)
    out = _forward_losses(m, case, torch.device("cpu"))
    _check(m, case, *out, rtol=1e-4, atol=1e-5, grad_rtol=1e-3, grad_atol=1e-6)


def test_117m_preset_parameter_count():
    m = lm.TensionLM(lm.preset_117m())
    assert m.num_params == 117_206_784
    assert m.window_groups == {64: [0, 1, 2, 4, 5, 6, 8, 9, 10], 1024: [3, 7, 11]}


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CFGS))
def test_harness_matches_reference_model_gpu_fp32(golden_lm, name):
    torch.backends.cuda.matmul.allow_tf32 = False
    case = golden_lm[name]
    m = _model(name, case, torch.device("cuda:0"))
    out = _forward_losses(m, case, torch.device("cuda:0"))
    _check(m, case, *out, rtol=1e-4, atol=1e-5, grad_rtol=1e-3, grad_atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CFGS))
def test_harness_fused_aux_losses_match_reference_model_gpu_fp32(golden_lm, name):
    """The fused τ consumer in the training loss: same losses and parameter
    gradients as the reference model's framework-op losses."""
    torch.backends.cuda.matmul.allow_tf32 = False
    case = golden_lm[name]
    m = _model(name, case, torch.device("cuda:0"))
    out = _forward_losses(m, case, torch.device("cuda:0"), fused_aux=True)
    _check(m, case, *out, rtol=1e-4, atol=1e-5, grad_rtol=1e-3, grad_atol=1e-6)


@pytest.mark.gpu
def test_harness_bf16_autocast_tensor_core_path(golden_lm):
    """bf16 autocast: local layers (HD 64, W 64) take the tcgen05 kernels."""
    from bozo_b200 import ops
    case = golden_lm["rope_global"]
    m = _model("rope_global", case, torch.device("cuda:0"))
    logits, hidden, tensions, parts, loss = _forward_losses(m, case, torch.device("cuda:0"),
                                                            amp=True)
    assert ops.last_path() in ("tcgen05", "simt")
    ref = case["logits"]
    g = logits.detach().float().cpu().numpy()
    # bf16 activations through 4 layers: relative error of the logits ~1e-2
    assert np.abs(g - ref).max() <= 3e-2 * max(1.0, np.abs(ref).max())
    assert abs(float(loss.detach()) - float(case["loss"])) < 2e-2
    for i, t in enumerate(tensions):
        assert np.abs(t.detach().float().cpu().numpy() - case[f"tau{i}"]).max() < 3e-2
    # gradients through the packed projections and the norms' bf16 side
    # outputs (their cotangents summed in the norm backward) against the
    # reference model's fp32 gradients, to bf16 accuracy
    params = dict(m.named_parameters())
    for k in case:
        if k.startswith("grad."):
            got = params[k[5:]].grad.detach().float().cpu().numpy()
            scale = np.abs(case[k]).max()
            assert np.abs(got - case[k]).max() <= 5e-2 * scale, k


@pytest.mark.gpu
def test_graphed_train_step_matches_eager():
    """``GraphedTrainStep`` (the step recorded as a CUDA graph, replayed per
    batch) leaves exactly the parameters and losses of the eager steps,
    including a batch copied in from pinned host memory."""
    dev = torch.device("cuda:0")
    cfg = lm.TensionConfig(**CFGS["rope_global"])
    g = torch.Generator().manual_seed(11)
    batches = [torch.randint(0, cfg.vocab_size, (2, 193), generator=g) for _ in range(2)]
    ids0 = batches[0].to(dev)
    ids1 = batches[1].pin_memory()

    def build():
        torch.manual_seed(0)
        base = lm.TensionLM(cfg).to(dev)
        return base, lm.make_optimizer(base, fused=True, capturable=True)

    base_e, opt_e = build()
    losses_e = []
    for ids in [ids0] * 5 + [ids1.to(dev)] * 2:
        losses_e.append(float(lm.train_step(base_e, base_e, opt_e, ids[:, :-1], ids[:, 1:])))
    base_g, opt_g = build()
    step = lm.GraphedTrainStep(base_g, base_g, opt_g, ids0, warmup=3)  # steps 1-3 eagerly
    losses_g = [float(step()), float(step())]
    losses_g += [float(step(ids1)), float(step())]
    step.release()
    assert losses_g == losses_e[3:]
    for (name, pe), pg in zip(base_e.named_parameters(), base_g.parameters()):
        assert torch.equal(pe, pg), name


@pytest.mark.gpu
def test_graphed_forward_matches_eager():
    """``GraphedForward`` (the no-grad forward replayed as CUDA graphs, two
    copies with their own outputs) returns exactly the eager forward's
    logits and τ fields for each batch it is given."""
    dev = torch.device("cuda:0")
    cfg = lm.TensionConfig(**CFGS["rope_global"])
    torch.manual_seed(0)
    model = lm.TensionLM(cfg).to(dev, torch.bfloat16).eval()
    g = torch.Generator().manual_seed(5)
    b0, b1 = (torch.randint(0, cfg.vocab_size, (2, 192), generator=g).to(dev) for _ in range(2))
    with torch.no_grad():
        ref0, ref1 = model(b0, return_all=True), model(b1, return_all=True)
    fw = lm.GraphedForward(model, b0, copies=2)
    out0 = fw(copy=0)
    out1 = fw(b1, copy=1)
    torch.cuda.synchronize()
    for ref, out in ((ref0, out0), (ref1, out1)):
        assert torch.equal(ref[0], out[0])
        assert len(ref[2]) == len(out[2])
        for a, b in zip(ref[2], out[2]):
            assert torch.equal(a, b)


# ───────────────────────── DDP over gloo (CPU) ─────────────────────────

TINY = dict(vocab_size=53, dim=32, num_layers=2, num_heads=2, window=4, ffn_mult=2,
            max_seq_len=24, dropout=0.0, use_oscillation=False, use_rope=True, global_every=2)


def _tiny_batch():
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, TINY["vocab_size"], (4, 17), generator=g)
    return ids[:, :-1], ids[:, 1:]


def _ddp_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        base = lm.TensionLM(lm.TensionConfig(**TINY))
        base.set_tension_fn(oracle_tension)
        model = lm.wrap_ddp(base)
        opt = lm.make_optimizer(base, fused=False)
        inputs, targets = _tiny_batch()
        half = inputs.shape[0] // world
        sl = slice(rank * half, (rank + 1) * half)
        lm.train_step(model, base, opt, inputs[sl], targets[sl], weights=WEIGHTS, amp=False)
        torch.save({k: v.detach().clone() for k, v in base.state_dict().items()},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ddp_step_equals_averaged_half_batch_gradients(tmp_path):
    world = 2
    mp.start_processes(_ddp_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    r0 = torch.load(tmp_path / "rank0.pt")
    r1 = torch.load(tmp_path / "rank1.pt")
    for k in r0:
        assert torch.equal(r0[k], r1[k]), f"ranks diverged at {k}"

    # single process: mean of the two half-batch gradients, then clip + AdamW
    torch.manual_seed(0)
    base = lm.TensionLM(lm.TensionConfig(**TINY))
    base.set_tension_fn(oracle_tension)
    opt = lm.make_optimizer(base, fused=False)
    inputs, targets = _tiny_batch()
    V = TINY["vocab_size"]
    for sl in (slice(0, 2), slice(2, 4)):
        logits, hidden, tensions = base(inputs[sl], return_all=True)
        loss = torch.nn.functional.cross_entropy(logits.reshape(-1, V), targets[sl].reshape(-1))
        loss = (loss + WEIGHTS.w_closure * lm.manifold_closure_loss(hidden)
                + WEIGHTS.w_diversity * lm.tension_diversity_loss(tensions, base.window_groups)
                + WEIGHTS.w_consistency * lm.constraint_consistency_loss(tensions)
                + WEIGHTS.w_entropy * lm.tension_entropy_loss(tensions))
        (loss / 2).backward()
    torch.nn.utils.clip_grad_norm_(base.parameters(), 1.0)
    opt.step()
    ref = base.state_dict()
    for k in r0:
        torch.testing.assert_close(r0[k], ref[k], rtol=1e-5, atol=1e-6, msg=k)
    assert not math.isnan(float(sum(v.float().sum() for v in r0.values())))


def _graphed_ddp_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg = lm.TensionConfig(**CFGS["rope_global"])
        g = torch.Generator().manual_seed(23 + rank)
        ids = torch.randint(0, cfg.vocab_size, (2, 193), generator=g).to(dev)
        finals = []
        for graphed in (False, True):
            torch.manual_seed(0)
            base = lm.TensionLM(cfg).to(dev)
            model = lm.wrap_ddp(base)
            opt = lm.make_optimizer(base, fused=True, capturable=True)
            if graphed:
                step = lm.GraphedTrainStep(model, base, opt, ids)  # 11 eager warm-up steps
                for _ in range(2):
                    step()
                step.release()
            else:
                for _ in range(13):
                    lm.train_step(model, base, opt, ids[:, :-1], ids[:, 1:])
            torch.cuda.synchronize()
            finals.append({k: v.detach().cpu().clone() for k, v in base.state_dict().items()})
            del model
        torch.save(finals, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_graphed_ddp_step_matches_eager_ddp(tmp_path):
    """The DDP step the multi-GPU bench replays — NCCL all-reduces with the
    averaging hook recorded inside ``GraphedTrainStep`` — leaves exactly the
    parameters of the same number of eager DDP steps (one NCCL rank here; the
    bench's two- and eight-rank runs use the same code)."""
    mp.start_processes(_graphed_ddp_worker, args=(1, _free_port(), str(tmp_path)), nprocs=1,
                       join=True, start_method="spawn")
    eager, graphed = torch.load(tmp_path / "rank0.pt")
    for k in eager:
        assert torch.equal(eager[k], graphed[k]), k


def test_packed_weight_cache_follows_the_weights():
    """Without autograd the concatenated projection weight is reused until a
    weight changes; with autograd it is built fresh (and differentiable)."""
    lin = torch.nn.Linear(4, 4, bias=False)
    owner = torch.nn.Module()
    ws = (lin.weight, lin.weight)
    with torch.no_grad():
        a = lm._packed_weight(owner, "_cat", ws)
        b = lm._packed_weight(owner, "_cat", ws)
        assert a is b and torch.equal(a, torch.cat(ws))
        lin.weight.add_(1.0)  # in-place update bumps the version counter
        c = lm._packed_weight(owner, "_cat", ws)
        assert c is not a and torch.equal(c, torch.cat(ws))
    d = lm._packed_weight(owner, "_cat", ws)
    assert d.requires_grad and d is not c
    assert "_cat" not in owner.state_dict()
