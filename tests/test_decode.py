"""Decode step (``bozo_tension_decode``, ``bozo_b200.decode``).

* GPU, kernel: a whole sequence fed one token at a time through the ring
  caches reproduces, row by row, the float64 oracle of the sequence operator
  (local W ∈ {16, 64} with τ-mass / count / raw normalisation, global with
  τ-mass) — outputs and the exported τ rows; a global ring shorter than the
  sequence keeps the last ``capacity`` keys; caches over 256 keys (the
  16-warp kernel) match too, wrapped or not.
* GPU, model: after a prefill, each decode step's logits equal the last row
  of a full forward of the harness over the same ids (plain forward: local
  count normalisation; export mode: the ``return_all`` forward, incl. its τ
  rows), for a RoPE + global-layer model and a learned-position +
  oscillation model; ``generate`` is reproducible under a seed.
* CPU: decoding needs a GPU model.
"""
import pytest
import torch

from bozo_b200 import _capi, lm
from oracle import tension_oracle as orc
from tests._tol import assert_close

SCALE = 8.0


def _seq(B, T, H, HD, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, T, H, HD, generator=g).to(dtype) for _ in range(3)]


def _decode_all(q, k, v, *, mode, W, norm, cap, tw, rope=True):
    """Feed positions 0..T−1 one at a time; returns per-step out and τ rows."""
    from bozo_b200 import ops
    B, T, H, HD = q.shape
    dev = torch.device("cuda:0")
    qd, kd, vd = (x.to(dev) for x in (q, k, v))
    kc = torch.zeros(B, cap, H, HD, device=dev, dtype=q.dtype)
    vc = torch.zeros_like(kc)
    pos = torch.zeros(1, dtype=torch.int32, device=dev)
    cos, sin, _ = ops.rope_tables(HD, T, 10_000.0, dev) if rope else (None, None, None)
    outs, taus = [], []
    for t in range(T):
        out, tau = _capi.ext().tension_decode(qd[:, t], kd[:, t], vd[:, t], kc, vc, pos, mode, W,
                                              norm, SCALE, cos, sin, tw, ops._dt(q.dtype),
                                              ops._dt(q.dtype))
        outs.append(out)
        taus.append(tau)
        pos += 1
    return torch.stack(outs, 1), (torch.stack(taus, 1) if tw else None)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("W,normalize", [(16, "mass"), (64, "mass"), (64, "count"), (16, None)])
def test_local_decode_matches_oracle_rows(dtype, W, normalize):
    q, k, v = _seq(2, 150, 3, 64, dtype, seed=W)
    norm = {"mass": _capi.NORM_MASS, "count": _capi.NORM_COUNT, None: _capi.NORM_NONE}[normalize]
    out, tau = _decode_all(q, k, v, mode=_capi.MODE_LOCAL, W=W, norm=norm, cap=W + 1, tw=W)
    ref_out, ref_tau = orc.fused_reference(*(x.double() for x in (q, k, v)), window=W, scale=SCALE,
                                           normalize=normalize or "none")
    assert_close(out, ref_out, dtype, f"local W{W} {normalize} out")
    assert_close(tau, ref_tau, dtype, f"local W{W} τ rows")


@pytest.mark.gpu
@pytest.mark.parametrize("HD", [32, 48, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_head_dims(HD, dtype):
    """HD 32 and 128 take the vector kernel, 48 the generic one."""
    q, k, v = _seq(1, 90, 2, HD, dtype, seed=HD)
    out, tau = _decode_all(q, k, v, mode=_capi.MODE_LOCAL, W=24, norm=_capi.NORM_MASS, cap=25, tw=24)
    ref_out, ref_tau = orc.fused_reference(*(x.double() for x in (q, k, v)), window=24,
                                           scale=SCALE, normalize="mass")
    assert_close(out, ref_out, dtype, f"HD{HD} out")
    assert_close(tau, ref_tau, dtype, f"HD{HD} τ rows")
    out, _ = _decode_all(q, k, v, mode=_capi.MODE_GLOBAL, W=0, norm=_capi.NORM_MASS, cap=90, tw=0)
    cos, sin = orc.rope_tables(HD, 90, 10_000.0, torch.float64)
    ref, _, _ = orc.global_tension(orc.rope(q.double(), cos, sin), orc.rope(k.double(), cos, sin),
                                   v.double(), SCALE)
    assert_close(out, ref, dtype, f"HD{HD} global out")


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_global_decode_matches_oracle_rows(dtype):
    W, T = 32, 130
    q, k, v = _seq(2, T, 2, 64, dtype, seed=3)
    out, tau = _decode_all(q, k, v, mode=_capi.MODE_GLOBAL, W=0, norm=_capi.NORM_MASS, cap=T, tw=W)
    cos, sin = orc.rope_tables(64, T, 10_000.0, torch.float64)
    qr, kr = orc.rope(q.double(), cos, sin), orc.rope(k.double(), cos, sin)
    ref_out, tau_full, _ = orc.global_tension(qr, kr, v.double(), SCALE, local_window=W)
    assert_close(out, ref_out, dtype, "global out")
    # row t of the field a forward over ids[:t+1] exports: column c ↔ key t − c
    ref_rows = torch.zeros(2, T, 2, W, dtype=torch.float64)
    for t in range(T):
        for c in range(min(W, t + 1)):
            ref_rows[:, t, :, c] = tau_full[:, t, :, t - c]
    assert_close(tau, ref_rows, dtype, "global τ rows")


@pytest.mark.gpu
def test_global_ring_keeps_last_capacity_keys():
    C, T, HD = 40, 100, 64
    q, k, v = _seq(1, T, 2, HD, torch.float32, seed=4)
    out, _ = _decode_all(q, k, v, mode=_capi.MODE_GLOBAL, W=0, norm=_capi.NORM_MASS, cap=C, tw=0)
    cos, sin = orc.rope_tables(HD, T, 10_000.0, torch.float64)
    qr, kr, vv = orc.rope(q.double(), cos, sin), orc.rope(k.double(), cos, sin), v.double()
    ref = torch.zeros(1, T, 2, HD, dtype=torch.float64)
    for t in range(T):
        s0 = max(0, t - C + 1)
        tau = torch.sigmoid(torch.einsum("bhd,bshd->bhs", qr[:, t], kr[:, s0:t + 1]) / SCALE)
        ref[:, t] = torch.einsum("bhs,bshd->bhd", tau, vv[:, s0:t + 1]) / tau.sum(-1, keepdim=True)
    assert_close(out, ref, torch.float32, "sliding global out")


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_long_caches_take_the_wide_kernel(dtype):
    """Caches over 256 keys (global layers, wide windows) run 16 warps per
    (b, h): global without and with the ring wrapping, and a local window of
    300."""
    T, HD = 420, 64
    q, k, v = _seq(1, T, 2, HD, dtype, seed=5)
    cos, sin = orc.rope_tables(HD, T, 10_000.0, torch.float64)
    qr, kr, vv = orc.rope(q.double(), cos, sin), orc.rope(k.double(), cos, sin), v.double()
    out, _ = _decode_all(q, k, v, mode=_capi.MODE_GLOBAL, W=0, norm=_capi.NORM_MASS, cap=T, tw=0)
    ref, _, _ = orc.global_tension(qr, kr, vv, SCALE)
    assert_close(out, ref, dtype, "global 420-key cache out")
    C = 300
    out, _ = _decode_all(q, k, v, mode=_capi.MODE_GLOBAL, W=0, norm=_capi.NORM_MASS, cap=C, tw=0)
    ref = torch.zeros(1, T, 2, HD, dtype=torch.float64)
    for t in range(T):
        s0 = max(0, t - C + 1)
        tau = torch.sigmoid(torch.einsum("bhd,bshd->bhs", qr[:, t], kr[:, s0:t + 1]) / SCALE)
        ref[:, t] = torch.einsum("bhs,bshd->bhd", tau, vv[:, s0:t + 1]) / tau.sum(-1, keepdim=True)
    assert_close(out, ref, dtype, "global ring of 300 out")
    out, tau = _decode_all(q, k, v, mode=_capi.MODE_LOCAL, W=300, norm=_capi.NORM_MASS, cap=301, tw=300)
    ref_out, ref_tau = orc.fused_reference(*(x.double() for x in (q, k, v)), window=300, scale=SCALE,
                                           normalize="mass")
    assert_close(out, ref_out, dtype, "local W300 out")
    assert_close(tau, ref_tau, dtype, "local W300 τ rows")


CFGS = {
    "rope_global": dict(vocab_size=97, dim=128, num_layers=4, num_heads=2, window=16, ffn_mult=3,
                        max_seq_len=192, dropout=0.0, use_oscillation=False, use_rope=True,
                        global_every=2),
    "norope_osc": dict(vocab_size=97, dim=64, num_layers=2, num_heads=4, window=8, ffn_mult=3,
                       max_seq_len=48, dropout=0.0, use_oscillation=True, use_rope=False,
                       global_every=0),
}


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CFGS))
@pytest.mark.parametrize("export", [False, True])
def test_decode_steps_match_full_forward(name, export):
    from bozo_b200 import decode
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(5)
    cfg = lm.TensionConfig(**CFGS[name])
    dev = torch.device("cuda:0")
    model = lm.TensionLM(cfg).to(dev).eval()
    T = min(cfg.max_seq_len, 90)
    P = T // 3
    g = torch.Generator().manual_seed(6)
    ids = torch.randint(0, cfg.vocab_size, (2, T), generator=g).to(dev)
    state = decode.DecodeState(model, 2, T)
    res = decode.prefill(state, ids[:, :P], export=export)
    logits = res[0] if export else res
    for t in range(P, T + 1):
        with torch.no_grad():
            full = model(ids[:, :t], return_all=export)
        ref_logits = full[0][:, -1] if export else full[:, -1]
        scale = float(ref_logits.abs().max())
        torch.testing.assert_close(logits, ref_logits, rtol=1e-4, atol=1e-4 * scale,
                                   msg=f"{name} export={export} logits at length {t}")
        if export and t > P:
            for li, (row, field) in enumerate(zip(rows, full[2])):
                torch.testing.assert_close(row, field[:, -1], rtol=1e-4, atol=1e-5,
                                           msg=f"{name} τ row layer {li} at length {t}")
        if t == T:
            break
        res = decode.step(state, ids[:, t], export=export)
        logits, rows = res if export else (res, None)


@pytest.mark.gpu
@pytest.mark.parametrize("export", [False, True])
def test_step_graph_replays_match_eager_steps(export):
    """A captured step replayed per token gives the eager steps' logits (and
    τ rows) and leaves the caches in the same state."""
    from bozo_b200 import decode
    torch.manual_seed(9)
    cfg = lm.TensionConfig(**CFGS["rope_global"])
    model = lm.TensionLM(cfg).to("cuda:0").eval()
    g = torch.Generator().manual_seed(10)
    ids = torch.randint(0, cfg.vocab_size, (2, 70), generator=g).to("cuda:0")
    states = [decode.DecodeState(model, 2, 70) for _ in range(2)]
    for st in states:
        decode.prefill(st, ids[:, :30])
    graph = decode.StepGraph(states[1], export=export)
    for t in range(30, 70):
        eager = decode.step(states[0], ids[:, t], export=export)
        replay = graph(ids[:, t])
        if export:
            torch.testing.assert_close(replay[0], eager[0], rtol=0, atol=0)
            for a, b in zip(replay[1], eager[1]):
                torch.testing.assert_close(a, b, rtol=0, atol=0)
        else:
            torch.testing.assert_close(replay, eager, rtol=0, atol=0)
    assert int(states[0].pos) == int(states[1].pos) == 70
    for a, b in zip(states[0].k_cache + states[0].v_cache, states[1].k_cache + states[1].v_cache):
        assert torch.equal(a, b)


@pytest.mark.gpu
def test_generate_is_seeded_and_sized():
    from bozo_b200 import decode
    torch.manual_seed(7)
    model = lm.TensionLM(lm.TensionConfig(**CFGS["rope_global"])).to("cuda:0")
    prompt = list(range(10, 30))
    torch.manual_seed(8)
    a = decode.generate(model, prompt, max_new=25)
    torch.manual_seed(8)
    b = decode.generate(model, prompt, max_new=25, graph=False)
    assert a == b and len(a) == len(prompt) + 25 and a[:len(prompt)] == prompt
    assert all(0 <= i < 97 for i in a)


def test_decode_state_needs_a_gpu_model():
    from bozo_b200 import decode
    model = lm.TensionLM(lm.TensionConfig(**CFGS["norope_osc"]))
    with pytest.raises(RuntimeError, match="GPU"):
        decode.DecodeState(model, 1, 16)
