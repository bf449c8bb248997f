"""Graph bias built on the device (``bozo_b200.graph_bias``,
``include/bozo_graph_bias.h``).

* GPU: ``local_bias`` / ``global_bias`` equal the reference ``GraphBias``'s
  tensors bit for bit and its ``BiasStats`` (``tests/golden/golden_bias.npz``),
  and the oracle's at a 2048-token context (W 64) and a 400-token global
  context over a random edge map; the batch-broadcast view feeds the
  operator exactly like a materialised bias.
* CPU: building on a CPU device raises.
"""
import numpy as np
import pytest
import torch

from oracle import bias_oracle
from tests.test_oracle_golden import _bias_golden, _FixedTokenizer


@pytest.mark.gpu
@pytest.mark.parametrize("ctx", ["ctx_a", "ctx_b"])
def test_device_bias_matches_reference(ctx):
    from bozo_b200.graph_bias import GraphBiasTable
    z, edges = _bias_golden()
    table = GraphBiasTable(edges, float(z["alpha"]))
    ids = z[f"{ctx}_ids"].tolist()
    lb, ls = table.local_bias(ids, _FixedTokenizer(), int(z["W"]), batch=2)
    gb, gs = table.global_bias(ids, _FixedTokenizer(), batch=2)
    assert lb.shape == z[f"{ctx}_local"].shape and gb.shape == z[f"{ctx}_global"].shape
    np.testing.assert_array_equal(lb.cpu().numpy(), z[f"{ctx}_local"])
    np.testing.assert_array_equal(gb.cpu().numpy(), z[f"{ctx}_global"])
    for st, ref in ((ls, z[f"{ctx}_local_stats"]), (gs, z[f"{ctx}_global_stats"])):
        assert st.nonzero_pairs == int(ref[0]) and st.max_weight == ref[1]
        assert st.mean_weight == pytest.approx(ref[2], rel=1e-12)


class _VocabTokenizer:
    def __init__(self, n):
        self.n = n

    def id_to_token(self, i):
        return f"w{i}" if i % 7 else None


def _random_edges(n_tokens, n_edges, seed):
    rng = np.random.default_rng(seed)
    names = [f"w{i}" for i in range(n_tokens)] + [f"<{i}>" for i in range(0, n_tokens, 7)]
    return {(names[a], names[b]): float(rng.uniform(-0.2, 1.0))
            for a, b in rng.integers(0, len(names), (n_edges, 2))}


@pytest.mark.gpu
@pytest.mark.parametrize("T,W", [(2048, 64), (400, 0)])
def test_device_bias_matches_oracle_at_size(T, W):
    from bozo_b200.graph_bias import GraphBiasTable
    edges = _random_edges(300, 20000, seed=T)
    ids = np.random.default_rng(T + 1).integers(0, 300, T).tolist()
    tok = _VocabTokenizer(300)
    table = GraphBiasTable(edges, 0.5)
    if W:
        got, st = table.local_bias(ids, tok, W)
        ref, rst = bias_oracle.local_bias(edges, 0.5, ids, tok, W)
    else:
        got, st = table.global_bias(ids, tok)
        ref, rst = bias_oracle.global_bias(edges, 0.5, ids, tok)
    np.testing.assert_array_equal(got[0].cpu().numpy(), ref)
    assert st.nonzero_pairs == rst[0] > 0 and st.max_weight == rst[1]
    assert st.mean_weight == pytest.approx(rst[2], rel=1e-12)


@pytest.mark.gpu
def test_broadcast_bias_feeds_the_operator():
    import bozo_b200
    from bozo_b200.graph_bias import GraphBiasTable
    edges = _random_edges(50, 2000, seed=3)
    ids = np.random.default_rng(4).integers(0, 50, 256).tolist()
    bias, _ = GraphBiasTable(edges, 0.8).local_bias(ids, _VocabTokenizer(50), 64, batch=2)
    assert bias.stride(0) == 0
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(2, 256, 2, 64, generator=g).cuda().to(torch.bfloat16) for _ in range(3))
    a = bozo_b200.tension(q, k, v, window=64, bias=bias)
    b = bozo_b200.tension(q, k, v, window=64, bias=bias.contiguous())
    assert torch.equal(a, b)


def test_device_bias_needs_cuda():
    from bozo_b200.graph_bias import GraphBiasTable
    try:
        table = GraphBiasTable({("a", "b"): 1.0}, 0.5, device="cpu")
    except Exception:
        pytest.skip("no torch CUDA build")
    with pytest.raises(RuntimeError, match="GPU"):
        table.local_bias([1, 2, 3], _VocabTokenizer(5), 2, device="cpu")
