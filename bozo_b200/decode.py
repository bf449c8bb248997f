"""Token-by-token decoding of TensionLM with per-layer key/value ring caches.

model.py:718-768 (``generate_cached``) produces each new token by running
the whole model over the last ``max_seq_len`` tokens, so every token costs a
full forward of the context.  Here each tension layer keeps a ring cache of
RoPE-rotated keys and values — ``W + 1`` rows for a local layer, up to
``max_seq_len`` for a global one — and a new token costs one projection of
that token per layer plus ``bozo_tension_decode``: the new query against the
cached keys (O(W) per head for a local layer), with the new key and value
written into the ring by the same kernel.

* ``DecodeState``: the caches and the position of the next token (a device
  int32, read by the kernel, so a step does not depend on host state).
* ``prefill``: runs the model over a prompt with the fused sequence kernels
  (the same path as training and prefill) and fills the caches.
* ``step``: one token through every layer.  ``export=True`` follows the
  ``return_all`` forward (τ-mass normalisation in every layer, model.py:
  250-258) and returns each layer's τ row — what ts_bridge/streaming.py:
  100-194 (``ingest_step``) reads from a full forward; otherwise local
  layers use the valid-count normalisation of the plain forward
  (model.py:261-264), as ``generate_cached`` sees it.
* ``StepGraph``: ``step`` captured once as a CUDA graph and replayed per
  token (a step is a few hundred small launches; replaying them as one
  graph removes their host cost).
* ``generate``: the sampling loop of ``generate_cached`` (repetition
  penalty over the last 32 ids, temperature, nucleus sampling) on top.

Up to ``max_seq_len`` tokens a step's logits equal the full forward's last
row.  Past it, the reference re-runs a sliding window whose first tokens see
a truncated history; the caches instead keep every token's keys and values
as computed with its full history (the global ring keeps the last
``max_seq_len`` keys, so its reach matches the sliding window).  Learned
absolute positions (``use_rope=False``) and the oscillatory modulation index
positions below ``max_seq_len`` only.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _capi, ops

__all__ = ["DecodeState", "StepGraph", "prefill", "step", "generate"]


def _rotate(x: Tensor, cos: Tensor, sin: Tensor, t0: int) -> Tensor:
    """Half-split RoPE (model.py:75-81) of ``x [B, T, H, HD]`` at positions
    t0 … t0+T−1, in fp32."""
    T = x.shape[1]
    c = cos[t0:t0 + T].unsqueeze(0).unsqueeze(2)
    s = sin[t0:t0 + T].unsqueeze(0).unsqueeze(2)
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


class DecodeState:
    """Ring caches of one batch of sequences decoded in lock step.

    ``dtype``: dtype of the projections the model produces (the caches'
    dtype) — bf16 under bf16 autocast, else the parameters' dtype.
    ``max_len``: longest sequence (prompt + generated) the RoPE tables cover.
    """

    def __init__(self, model, batch: int, max_len: int, dtype: Optional[torch.dtype] = None):
        cfg = model.cfg
        dev = next(model.parameters()).device
        if dev.type != "cuda":
            raise RuntimeError("decoding runs on the CUDA decode kernel: move the model to a GPU")
        self.model = model
        self.dtype = dtype or next(model.parameters()).dtype
        H, HD = cfg.num_heads, cfg.head_dim
        self.k_cache: List[Tensor] = []
        self.v_cache: List[Tensor] = []
        for blk in model.blocks:
            cap = cfg.max_seq_len if blk.global_layer else cfg.window + 1
            self.k_cache.append(torch.zeros(batch, cap, H, HD, device=dev, dtype=self.dtype))
            self.v_cache.append(torch.zeros(batch, cap, H, HD, device=dev, dtype=self.dtype))
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)  # next token's position
        self.length = 0                                          # host copy (prefill only)
        self.batch = batch
        self.max_len = max_len
        self.rope = ops.rope_tables(HD, max_len, 10_000.0, dev) if cfg.use_rope else None

    def _fill(self, li: int, k: Tensor, v: Tensor) -> None:
        """Cache rows of prompt positions 0 … P−1 (the last ``capacity`` of them)."""
        P = k.shape[1]
        kc, vc = self.k_cache[li], self.v_cache[li]
        cap = kc.shape[1]
        lo = max(0, P - cap)
        idx = torch.arange(lo, P, device=kc.device) % cap
        kr = _rotate(k[:, lo:], self.rope[0], self.rope[1], lo) if self.rope is not None else k[:, lo:]
        kc[:, idx] = kr.to(kc.dtype)
        vc[:, idx] = v[:, lo:].to(vc.dtype)


@torch.no_grad()
def prefill(state: DecodeState, input_ids: Tensor, export: bool = False):
    """Run the model over ``input_ids [B, P]`` (P ≤ max_seq_len) with the
    sequence kernels, fill the caches and return the last position's logits
    ``[B, V]`` (and each layer's τ field when ``export``)."""
    model, cfg = state.model, state.model.cfg
    B, P = input_ids.shape
    if B != state.batch or P > min(cfg.max_seq_len, state.max_len):
        raise ValueError("prefill: batch or prompt length does not fit the decode state")
    x = model.embedding(input_ids)
    if model.pos_embedding is not None:
        x = x + model.pos_embedding(model.pos_buf[:, :P])
    taus = []
    for li, blk in enumerate(model.blocks):
        h = blk.pre_norm(x)
        _, k, v = blk.tension.project(h)
        state._fill(li, k, v)
        if export:
            hh, tau = blk.tension(h, return_tensions=True)
            taus.append(tau)
        else:
            hh = blk.tension(h)
        x = blk.ffn(blk._osc(hh))
    logits = model.lm_head(model.final_norm(x[:, -1:]))[:, 0]
    state.pos.fill_(P)
    state.length = P
    return (logits, taus) if export else logits


def _oscillate(osc, x: Tensor, pos: Tensor) -> Tensor:
    """model.py:303-310 for one token at the device position ``pos``."""
    mod = torch.sin(pos.float() * osc.freqs + osc.phases)
    return x * (1.0 + osc.amp * mod)


@torch.no_grad()
def step(state: DecodeState, tokens: Tensor, export: bool = False):
    """Feed one token per sequence (``tokens [B]``, at position ``state.pos``)
    through every layer; returns the logits ``[B, V]`` (and the layers' τ rows
    ``[B, H, W]`` when ``export``).  Uses only device state, so the step can
    be captured in a CUDA graph."""
    model, cfg = state.model, state.model.cfg
    B = tokens.shape[0]
    D, H, HD = cfg.dim, cfg.num_heads, cfg.head_dim
    x = model.embedding(tokens).unsqueeze(1)
    if model.pos_embedding is not None:
        x = x + model.pos_embedding(state.pos.long()).unsqueeze(0)
    cos, sin = (state.rope[0], state.rope[1]) if state.rope is not None else (None, None)
    rows = []
    for li, blk in enumerate(model.blocks):
        layer = blk.tension
        h = blk.pre_norm(x)
        q, k, v = layer.project(h)
        glob = layer.global_layer
        mode = _capi.MODE_GLOBAL if glob else _capi.MODE_LOCAL
        norm = _capi.NORM_MASS if (export or glob) else _capi.NORM_COUNT
        tw = cfg.window if export else 0
        out, tau = _capi.ext().tension_decode(
            q[:, 0], k[:, 0], v[:, 0], state.k_cache[li], state.v_cache[li], state.pos, mode,
            0 if glob else cfg.window, norm, float(layer.scale), cos, sin, tw, ops._dt(q.dtype),
            ops._dt(q.dtype))
        hh = layer.norm.wo_add_forward(h, out.view(B, 1, D), layer.wo, layer.dropout)
        if blk.oscillate is not None:
            hh = _oscillate(blk.oscillate, hh, state.pos)
        x = blk.ffn(hh)
        rows.append(tau)
    logits = model.lm_head(model.final_norm(x))[:, 0]
    state.pos += 1
    # a position outside the RoPE table sets the device error word: report it
    # (at most one step late, without a synchronisation; skipped in capture)
    ops.check_device_error(tokens.device)
    return (logits, rows) if export else logits


class StepGraph:
    """``step(state, tokens, export)`` captured as one CUDA graph.

    ``__call__(tokens)`` copies the tokens into the graph's input buffer and
    replays it; the returned logits (and τ rows) are the graph's output
    buffers, overwritten by the next call.  The position advances on the
    device inside the graph.  Capturing runs warm-up steps on a side stream
    first; the state's position is restored afterwards, and the cache rows
    those steps wrote are rewritten by the next real step before anything
    reads them (a step writes its own row first)."""

    def __init__(self, state: DecodeState, export: bool = False, warmup: int = 2):
        self.state = state
        dev = state.pos.device
        self.tokens = torch.zeros(state.batch, dtype=torch.long, device=dev)
        pos0 = state.pos.clone()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                step(state, self.tokens, export)
                state.pos.copy_(pos0)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = step(state, self.tokens, export)
        state.pos.copy_(pos0)  # capture recorded the increment without running it

    def __call__(self, tokens: Tensor):
        self.tokens.copy_(tokens)
        self.graph.replay()
        ops.check_device_error(self.tokens.device)
        return self.out


def _sample(logits: Tensor, recent: List[int], temp: float, top_p: float, rep_penalty: float) -> int:
    """Repetition penalty on the ids of ``recent``, temperature, nucleus
    sampling — the token choice of generate_cached (model.py:748-766)."""
    logits = logits.float().clone()
    for tok in set(recent):
        logits[tok] = logits[tok] / rep_penalty if logits[tok] > 0 else logits[tok] * rep_penalty
    probs = F.softmax(logits / max(temp, 1e-5), dim=-1)
    p_sorted, order = torch.sort(probs, descending=True)
    keep = (torch.cumsum(p_sorted, dim=-1) - p_sorted) < top_p
    p_sorted = torch.where(keep, p_sorted, torch.zeros_like(p_sorted))
    p_sorted = p_sorted / p_sorted.sum()
    return int(order[torch.multinomial(p_sorted, 1)].item())


@torch.no_grad()
def generate(model, input_ids: List[int], max_new: int = 200, temp: float = 0.8,
             top_p: float = 0.92, rep_penalty: float = 1.3,
             dtype: Optional[torch.dtype] = None, graph: bool = True) -> List[int]:
    """generate_cached (model.py:718-768) with O(W) tension work per token:
    the prompt (its last max_seq_len ids) is prefilled once, then every new
    id is one decode step (a replayed ``StepGraph`` unless ``graph=False``).
    Returns the prompt followed by the new ids."""
    model.eval()
    ids = list(input_ids)
    ctx = ids[-model.cfg.max_seq_len:]
    dev = next(model.parameters()).device
    state = DecodeState(model, 1, len(ctx) + max_new, dtype=dtype)
    logits = prefill(state, torch.tensor([ctx], dtype=torch.long, device=dev))[0]
    run = StepGraph(state) if graph and max_new > 1 else (lambda tok: step(state, tok))
    tok = torch.zeros(1, dtype=torch.long, device=dev)
    for i in range(max_new):
        nxt = _sample(logits, ids[-32:], temp, top_p, rep_penalty)
        ids.append(nxt)
        if i + 1 < max_new:
            tok.fill_(nxt)
            logits = run(tok)[0]
    return ids
