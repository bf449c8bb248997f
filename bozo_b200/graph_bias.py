"""The graph bias built on the device (``include/bozo_graph_bias.h``).

``GraphBiasTable(edge_map, alpha)`` holds a ts_bridge ``GraphBias`` edge map
(``{(src_content, dst_content): weight}``, ts_bridge/bias.py:81-118) as a
device table: every content string that appears in an edge gets an integer
id, and each edge becomes a 64-bit key ``src_id << 32 | dst_id`` in a sorted
array with its weight (float64).  ``local_bias`` / ``global_bias`` have the
signatures of ``GraphBias.local_bias`` / ``global_bias`` (bias.py:125-233):
the host decodes each context token to its content once, as the reference
does, and one kernel (``bozo_graph_bias_build``) fills the whole ``[T, W]`` or
``[T, T]`` table by binary search, instead of the reference's O(T·W) /
O(T²) Python loops.  The ``[B, T, ·]`` result is a batch-broadcast view of
that table (every batch row of the reference's tensor is the same), which
the operator reads with a zero batch stride.  CUDA only.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Sequence, Tuple

import numpy as np
import torch
from torch import Tensor

from . import _capi

__all__ = ["BiasStats", "GraphBiasTable"]


@dataclass
class BiasStats:
    """bias.py:73-78: pairs with a positive weight, their max and mean weight."""
    nonzero_pairs: int
    max_weight: float
    mean_weight: float


class GraphBiasTable:
    """Device edge table of a ``GraphBias`` (same ``edge_map`` and ``alpha``)."""

    def __init__(self, edge_map: Dict[Tuple[str, str], float], alpha: float,
                 device: torch.device | str = "cuda"):
        self.alpha = float(alpha)
        self.device = torch.device(device)
        names = sorted({c for key in edge_map for c in key})
        self.content_id = {c: i for i, c in enumerate(names)}
        keys = np.array([(self.content_id[s] << 32) | self.content_id[d] for s, d in edge_map],
                        dtype=np.int64)
        weights = np.array(list(edge_map.values()), dtype=np.float64)
        order = np.argsort(keys, kind="stable")
        self.keys = torch.from_numpy(keys[order]).to(self.device)
        self.weights = torch.from_numpy(weights[order]).to(self.device)

    @classmethod
    def from_graph_bias(cls, gb, device: torch.device | str = "cuda") -> "GraphBiasTable":
        """From a ts_bridge ``GraphBias`` (its ``edge_map`` and ``alpha``)."""
        return cls(gb.edge_map, gb.alpha, device)

    def _content_ids(self, ctx_ids: Sequence[int], tokenizer) -> Tensor:
        # the token → content decoding of bias.py:146-149 / 205-208
        ids = [self.content_id.get(tokenizer.id_to_token(int(t)) or f"<{int(t)}>", -1)
               for t in ctx_ids]
        return torch.tensor(ids, dtype=torch.int32).to(self.device)

    def _build(self, ctx_ids, tokenizer, window: int, batch: int, device, dtype, with_stats):
        dev = torch.device(device) if device is not None else self.device
        if dev.type != "cuda":
            raise RuntimeError("GraphBiasTable builds the bias on the GPU (device must be CUDA)")
        cid = self._content_ids(ctx_ids, tokenizer).to(dev)
        keys, weights = self.keys.to(dev), self.weights.to(dev)
        table, stats = _capi.ext().graph_bias(cid, keys, weights, window, self.alpha)
        if dtype != torch.float32:
            table = table.to(dtype)
        bias = table.unsqueeze(0).expand(batch, *table.shape)
        if not with_stats:
            return bias, None
        hits, total, mx = stats.tolist()
        return bias, BiasStats(nonzero_pairs=int(hits), max_weight=mx,
                               mean_weight=total / hits if hits else 0.0)

    def local_bias(self, ctx_ids: Sequence[int], tokenizer, window: int, batch: int = 1,
                   device=None, dtype: torch.dtype = torch.float32, with_stats: bool = True):
        """bias.py:125-170: ``[B, T, W]``, slot w of query t ↔ key t − (W − w)."""
        if window < 1:
            raise ValueError("window must be >= 1")
        return self._build(ctx_ids, tokenizer, int(window), batch, device, dtype, with_stats)

    def global_bias(self, ctx_ids: Sequence[int], tokenizer, batch: int = 1, device=None,
                    dtype: torch.dtype = torch.float32, with_stats: bool = True):
        """bias.py:172-233: ``[B, T, T]``, key s < t."""
        return self._build(ctx_ids, tokenizer, 0, batch, device, dtype, with_stats)
