"""TensionLM on the B200 operator — the model the 117M training workload runs.

A restatement of the reference model (model.py:25-480) and of one training
step of train.py (train.py:1040-1150) with every tension layer on
``bozo_b200.tension``: RoPE, the local window or the global full-causal
block, the normalisation and the optional τ export happen inside the
operator's kernels instead of around ``causal_tension``.  Parameters, module
names and initialisation follow model.py, so a reference ``state_dict``
loads into it unchanged.

Where model.py has two local-layer branches (model.py:247-264), this one
keeps both: with ``return_tensions`` the τ-mass normalisation and τ export
(model.py:250-258), without it the position-count normalisation
(model.py:261-264).  Global layers use τ-mass and export the reference's
flipped τ window (model.py:217-237).
"""
from __future__ import annotations

import math
from collections import defaultdict
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from . import ops


@dataclass
class TensionConfig:
    """model.py:25-52 (same fields and defaults)."""
    vocab_size: int = 2048
    dim: int = 128
    num_layers: int = 4
    num_heads: int = 4
    window: int = 8
    ffn_mult: int = 3
    max_seq_len: int = 256
    dropout: float = 0.10
    use_grad_checkpoint: bool = False
    use_oscillation: bool = True
    use_rope: bool = False
    use_triton: bool = True  # kept for state compatibility; the operator is always used
    global_every: int = 0

    @property
    def head_dim(self) -> int:
        assert self.dim % self.num_heads == 0, "dim must be divisible by num_heads"
        return self.dim // self.num_heads


def preset_117m(**over) -> TensionConfig:
    """train.py:226-234 ``--preset large`` with the benchmark's
    ``--seq_len 1024 --max_seq_len 1024`` (117.2M parameters)."""
    cfg = dict(vocab_size=32768, dim=768, num_layers=12, num_heads=12, window=64, ffn_mult=3,
               max_seq_len=1024, dropout=0.0, use_oscillation=False, use_rope=True,
               global_every=4)
    cfg.update(over)
    return TensionConfig(**cfg)


def preset_13m(**over) -> TensionConfig:
    """dim 384, 6 layers, 6 heads (head_dim 64), vocab 8192,
    W 64, T 512, a global block every 4th layer (model.py:25-49 fields;
    train.py:219-258 presets span this size)."""
    cfg = dict(vocab_size=8192, dim=384, num_layers=6, num_heads=6, window=64, ffn_mult=3,
               max_seq_len=512, dropout=0.0, use_oscillation=False, use_rope=True,
               global_every=4)
    cfg.update(over)
    return TensionConfig(**cfg)


def preset_1m(**over) -> TensionConfig:
    """BASELINE configs[0], the reference's CPU-runnable case: dim 128, 4
    layers, 4 heads (head_dim 32), vocab 2048, W 64, T 256, RoPE, no
    oscillation, no global layer (1,115,776 parameters)."""
    cfg = dict(vocab_size=2048, dim=128, num_layers=4, num_heads=4, window=64, ffn_mult=3,
               max_seq_len=256, dropout=0.0, use_oscillation=False, use_rope=True,
               global_every=0)
    cfg.update(over)
    return TensionConfig(**cfg)


def preset_350m_prefill(**over) -> TensionConfig:
    """The 350M inference configuration: dim 1024, 24 layers, 16 heads,
    vocab 32768, W 128, T 2048, global layer every 3rd block (train.py:246-256
    ``--preset 350m`` with the benchmark's vocabulary and window)."""
    cfg = dict(vocab_size=32768, dim=1024, num_layers=24, num_heads=16, window=128, ffn_mult=3,
               max_seq_len=2048, dropout=0.0, use_oscillation=False, use_rope=True,
               global_every=3)
    cfg.update(over)
    return TensionConfig(**cfg)


def _packed_weight(owner: nn.Module, name: str, weights):
    """``torch.cat(weights)`` — the weight of one GEMM standing for several
    projections.  Without autograd (prefill, decoding, evaluation) the
    concatenation is kept on ``owner`` until one of the weights changes
    (storage or version counter), so a decode step does not re-copy it."""
    if torch.is_grad_enabled() and any(w.requires_grad for w in weights):
        return torch.cat(weights)
    key = tuple((w.data_ptr(), w._version, w.dtype) for w in weights)
    cached = owner.__dict__.get(name)
    if cached is None or cached[0] != key:
        cached = (key, torch.cat([w.detach() for w in weights]))
        owner.__dict__[name] = cached
    return cached[1]


class RMSNorm(nn.Module):
    """model.py:86-98."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        from . import block_ops
        if block_ops.norm_applies(x, None):
            return block_ops.add_rms_norm(x, None, self.scale, self.eps)
        return F.rms_norm(x, x.shape[-1:], self.scale, self.eps)

    def add_forward(self, x, y):
        """``self(x + y)`` — one fused kernel each way where it applies."""
        from . import block_ops
        if block_ops.norm_applies(x, y):
            return block_ops.add_rms_norm(x, y, self.scale, self.eps)
        return self(x + y)

    def forward_lin(self, x, y=None):
        """``(out, lin)``: ``out = self(x + y)`` and the operand the
        projections that read it take.  For an fp32 stream under bf16 autocast
        ``lin`` is out rounded to bf16 by the same kernel (autocast would cast
        it once per projection; its gradient returns into the kernel too);
        otherwise ``lin`` is out."""
        from . import block_ops
        if (x.is_cuda and x.dtype == torch.float32 and torch.is_autocast_enabled("cuda")
                and torch.get_autocast_dtype("cuda") == torch.bfloat16
                and block_ops.norm_applies(x, y)):
            return block_ops.add_rms_norm_lp(x, y, self.scale, self.eps)
        out = self(x) if y is None else self.add_forward(x, y)
        return out, out

    def wo_add_forward(self, x, msg, wo: nn.Linear, dropout: nn.Dropout):
        """``self(x + dropout(wo(msg)))``: without gradients and with an
        inactive dropout, one tensor-core kernel for the projection, the add
        and the norm together."""
        from . import block_ops
        if ((not dropout.training or dropout.p == 0.0)
                and block_ops.wo_norm_applies(x, msg, wo.weight)):
            return block_ops.wo_add_rms_norm(x, msg, wo.weight, self.scale, self.eps)
        return self.add_forward(x, dropout(wo(msg)))


class MultiHeadCausalTensionLayer(nn.Module):
    """model.py:103-283 with the tension core on the fused operator."""

    def __init__(self, cfg: TensionConfig, global_layer: bool = False):
        super().__init__()
        self.window = cfg.max_seq_len if global_layer else cfg.window
        self.local_window = cfg.window
        self.global_layer = global_layer
        self.num_heads = cfg.num_heads
        self.head_dim = cfg.head_dim
        self.scale = math.sqrt(self.head_dim)
        self.max_seq_len = cfg.max_seq_len
        D = cfg.dim
        self.wq = nn.Linear(D, D, bias=False)
        self.rope_enabled = cfg.use_rope
        if cfg.use_rope:
            self.wk = nn.Linear(D, D, bias=False)
            self.wv = nn.Linear(D, D, bias=False)
            self.wkv = None
        else:
            self.wkv = nn.Linear(D, 2 * D, bias=False)
            self.wk = self.wv = None
        self.wo = nn.Linear(D, D, bias=False)
        self.norm = RMSNorm(D)
        self.dropout = nn.Dropout(cfg.dropout)
        # the operator; tests may substitute a CPU restatement with the same keywords
        self.tension_fn: Callable = ops.tension

    def project(self, x):
        """q, k, v ``[B, T, H, HD]`` of ``x [B, T, D]`` (model.py:196-199).  On
        GPUs the projections run as one GEMM over the concatenated weights
        (q, k, v are views of its output; the input gradient is one GEMM that
        sums the three in its accumulator)."""
        B, T, D = x.shape
        H, HD = self.num_heads, self.head_dim
        if x.is_cuda:
            if self.rope_enabled:
                w = _packed_weight(self, "_qkv_cat", (self.wq.weight, self.wk.weight, self.wv.weight))
                q, k, v = F.linear(x, w).split(D, dim=-1)
                return q.view(B, T, H, HD), k.view(B, T, H, HD), v.view(B, T, H, HD)
            w = _packed_weight(self, "_qkv_cat", (self.wq.weight, self.wkv.weight))
            q, kv = F.linear(x, w).split([D, 2 * D], dim=-1)
            k, v = kv.view(B, T, H, 2 * HD).split(HD, dim=-1)
            return q.view(B, T, H, HD), k, v
        q = self.wq(x).view(B, T, H, HD)
        if self.rope_enabled:
            k = self.wk(x).view(B, T, H, HD)
            v = self.wv(x).view(B, T, H, HD)
        else:
            kv = self.wkv(x).view(B, T, H, 2 * HD)
            k, v = kv.split(HD, dim=-1)
        return q, k, v

    def forward(self, x, return_tensions: bool = False, tau_bias=None, x_lin=None,
                want_lin: bool = False):
        """``x_lin``: the operand the projections read (``RMSNorm.forward_lin``;
        default x).  ``want_lin``: the output is the pair ``(out, lin)`` of
        ``RMSNorm.forward_lin`` instead of out."""
        B, T, D = x.shape
        q, k, v = self.project(x if x_lin is None else x_lin)
        rope = 10_000.0 if self.rope_enabled else None
        tau = None
        if self.global_layer:
            res = self.tension_fn(q, k, v, window=None, scale=self.scale, rope_base=rope,
                                  rope_len=self.max_seq_len, bias=tau_bias,
                                  return_tau=return_tensions, normalize="mass",
                                  tau_window=self.local_window)
            msg, tau = res if return_tensions else (res, None)
            drop_first = False
        elif return_tensions:
            msg, tau = self.tension_fn(q, k, v, window=self.window, scale=self.scale,
                                       rope_base=rope, rope_len=self.max_seq_len,
                                       bias=tau_bias, return_tau=True, normalize="mass")
            drop_first = False
        else:
            msg = self.tension_fn(q, k, v, window=self.window, scale=self.scale, rope_base=rope,
                                  rope_len=self.max_seq_len, bias=tau_bias, normalize="count")
            drop_first = True  # model.py:261-263: dropout on msg, before wo
        out = self._residual(x, msg.reshape(B, T, D), drop_first, want_lin)
        return (out, tau) if return_tensions else out

    def _residual(self, x, msg, drop_first: bool, want_lin: bool):
        """norm(x + wo(msg)) with the branch's dropout placement."""
        if want_lin:
            y = self.wo(self.dropout(msg)) if drop_first else self.dropout(self.wo(msg))
            return self.norm.forward_lin(x, y)
        if drop_first and self.dropout.training and self.dropout.p > 0.0:
            return self.norm.add_forward(x, self.wo(self.dropout(msg)))
        return self.norm.wo_add_forward(x, msg, self.wo, self.dropout)


class OscillatoryModulation(nn.Module):
    """model.py:288-310."""

    def __init__(self, cfg: TensionConfig):
        super().__init__()
        self.freqs = nn.Parameter(torch.randn(cfg.dim) * 0.02)
        self.phases = nn.Parameter(torch.zeros(cfg.dim))
        self.amp = nn.Parameter(torch.full((1,), 0.1))
        pos = torch.arange(cfg.max_seq_len, dtype=torch.float).unsqueeze(-1)
        self.register_buffer("pos_buf", pos, persistent=False)

    def forward(self, x):
        T = x.shape[1]
        mod = torch.sin(self.pos_buf[:T] * self.freqs + self.phases)
        return x * (1.0 + self.amp * mod.unsqueeze(0))


class TensionFFN(nn.Module):
    """model.py:315-330 (SwiGLU)."""

    def __init__(self, cfg: TensionConfig):
        super().__init__()
        hidden = cfg.dim * cfg.ffn_mult
        self.gate = nn.Linear(cfg.dim, hidden, bias=False)
        self.val = nn.Linear(cfg.dim, hidden, bias=False)
        self.proj = nn.Linear(hidden, cfg.dim, bias=False)
        self.norm = RMSNorm(cfg.dim)
        self.dropout = nn.Dropout(cfg.dropout)

    def forward(self, x, x_lin=None):
        """``x_lin``: the operand the gate/value projections read (default x).
        On GPUs they run as one GEMM over the concatenated weights and SwiGLU
        reads its packed ``[g | v]`` rows."""
        from . import block_ops
        inp = x if x_lin is None else x_lin
        if inp.is_cuda:
            gv = F.linear(inp, _packed_weight(self, "_gv_cat", (self.gate.weight, self.val.weight)))
            if block_ops.swiglu_packed_applies(gv):
                h = block_ops.swiglu_packed(gv)
            else:
                g, v = gv.chunk(2, dim=-1)
                h = F.silu(g) * v
        else:
            g, v = self.gate(inp), self.val(inp)
            h = block_ops.swiglu(g, v) if block_ops.swiglu_applies(g, v) else F.silu(g) * v
        return self.norm.add_forward(x, self.dropout(self.proj(h)))


class TensionBlock(nn.Module):
    """model.py:335-386 (gradient checkpointing left out: the operator keeps no
    O(T·W·HD) intermediates, so there is nothing large to recompute)."""

    def __init__(self, cfg: TensionConfig, global_layer: bool = False):
        super().__init__()
        self.pre_norm = RMSNorm(cfg.dim)
        self.tension = MultiHeadCausalTensionLayer(cfg, global_layer=global_layer)
        self.oscillate = OscillatoryModulation(cfg) if cfg.use_oscillation else None
        self.ffn = TensionFFN(cfg)
        self.global_layer = global_layer

    def _osc(self, x):
        return self.oscillate(x) if self.oscillate is not None else x

    def forward(self, x, return_tensions: bool = False, tau_bias=None):
        h, h_lin = self.pre_norm.forward_lin(x)
        # the FFN's projections read a bf16 copy of the layer output unless the
        # oscillation sits between them
        want = self.oscillate is None
        res = self.tension(h, return_tensions=return_tensions, tau_bias=tau_bias, x_lin=h_lin,
                           want_lin=want)
        out, tau = res if return_tensions else (res, None)
        o, o_lin = out if want else (self._osc(out), None)
        y = self.ffn(o, x_lin=o_lin)
        return (y, tau) if return_tensions else y


class TensionLM(nn.Module):
    """model.py:391-480."""

    def __init__(self, cfg: TensionConfig):
        super().__init__()
        self.cfg = cfg
        self.embedding = nn.Embedding(cfg.vocab_size, cfg.dim)
        self.emb_drop = nn.Dropout(cfg.dropout)
        if not cfg.use_rope:
            self.pos_embedding = nn.Embedding(cfg.max_seq_len, cfg.dim)
            self.register_buffer("pos_buf", torch.arange(cfg.max_seq_len).unsqueeze(0),
                                 persistent=False)
        else:
            self.pos_embedding = None
        self.blocks = nn.ModuleList(
            TensionBlock(cfg, global_layer=cfg.global_every > 0 and (i + 1) % cfg.global_every == 0)
            for i in range(cfg.num_layers))
        groups = defaultdict(list)
        for i, b in enumerate(self.blocks):
            groups[b.tension.window].append(i)
        self.window_groups = dict(groups)
        self.final_norm = RMSNorm(cfg.dim)
        self.lm_head = nn.Linear(cfg.dim, cfg.vocab_size, bias=False)
        self.lm_head.weight = self.embedding.weight
        self._init_weights()

    def _init_weights(self):
        """model.py:412-424."""
        std, depth = 0.02, self.cfg.num_layers
        nn.init.normal_(self.embedding.weight, std=std)
        if self.pos_embedding is not None:
            nn.init.normal_(self.pos_embedding.weight, std=std)
        for name, m in self.named_modules():
            if isinstance(m, nn.Linear):
                if name.endswith(("wo", "proj")):
                    nn.init.normal_(m.weight, std=std / math.sqrt(2 * depth))
                else:
                    nn.init.normal_(m.weight, std=std / math.sqrt(depth))

    def set_tension_fn(self, fn: Callable) -> None:
        for b in self.blocks:
            b.tension.tension_fn = fn

    def forward(self, input_ids, return_all: bool = False, tau_bias=None, tau_bias_global=None):
        B, T = input_ids.shape
        assert T <= self.cfg.max_seq_len, \
            f"Sequence length {T} exceeds max_seq_len {self.cfg.max_seq_len}"
        from . import block_ops
        w = self.embedding.weight
        if w.requires_grad and torch.is_grad_enabled() and block_ops.embedding_applies(input_ids, w):
            x = block_ops.embedding(input_ids, w)  # fused weight gradient
        else:
            x = self.embedding(input_ids)
        if self.pos_embedding is not None:
            x = x + self.pos_embedding(self.pos_buf[:, :T])
        x = self.emb_drop(x)
        tensions = []
        for block in self.blocks:
            bias = tau_bias_global if block.global_layer else tau_bias
            if return_all:
                x, tau = block(x, return_tensions=True, tau_bias=bias)
                tensions.append(tau)
            else:
                x = block(x, tau_bias=bias)
        hidden, hidden_lin = self.final_norm.forward_lin(x)
        logits = self.lm_head(hidden_lin)
        if return_all:
            return logits, hidden, tensions
        return logits

    @property
    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())


# ── auxiliary losses (model.py:487-611) ──

def manifold_closure_loss(hidden):
    """model.py:487-494."""
    return F.mse_loss(hidden[:, -1], hidden[:, 0].detach())


def tension_diversity_loss(all_tensions, window_groups=None):
    """model.py:497-532."""
    if not all_tensions:
        return torch.tensor(0.0)
    if window_groups is not None:
        groups = {W: [all_tensions[i] for i in idx] for W, idx in window_groups.items()}
    else:
        groups = defaultdict(list)
        for t in all_tensions:
            groups[t.shape[-1]].append(t)
    total = torch.tensor(0.0, device=all_tensions[0].device)
    n = 0
    for W, ts in groups.items():
        tau = torch.stack(ts)
        p = tau / (tau.sum(-1, keepdim=True) + 1e-8)
        ent = -(p * torch.log(p + 1e-8)).sum(-1)
        total = total + F.relu(math.log(W) - ent.mean()).mean()
        n += 1
    return total / max(n, 1)


def constraint_consistency_loss(all_tensions):
    """model.py:535-577: tau[t,w1]·tau[t−w1,1] ≤ tau[t,w1+1] for w1 ∈ [1, min(W−2, 4)]."""
    if not all_tensions:
        return torch.tensor(0.0)
    total = torch.tensor(0.0, device=all_tensions[0].device)
    count = 0
    for tau in all_tensions:
        B, T, H, W = tau.shape
        if W < 3 or T < 3:
            continue
        m = min(W - 2, 4)
        last_start = m + 1
        if last_start >= T:
            continue
        n = T - last_start
        legs1 = torch.stack([tau[:, i + 2:i + 2 + n, :, i] for i in range(m)])
        legs2 = torch.stack([tau[:, i + 1:i + 1 + n, :, 0] for i in range(m)])
        comb = torch.stack([tau[:, i + 2:i + 2 + n, :, i + 1] for i in range(m)])
        total = total + F.relu(legs1 * legs2 - comb).mean()
        count += 1
    return total / max(count, 1)


def tension_entropy_loss(all_tensions):
    """model.py:580-611."""
    if not all_tensions:
        return torch.tensor(0.0)
    total = torch.tensor(0.0, device=all_tensions[0].device)
    for tau in all_tensions:
        mean_tau = tau.mean(-1)
        total = total + F.relu(0.05 - mean_tau).mean() + F.relu(mean_tau - 0.80).mean()
    return total / len(all_tensions)


def aux_losses(all_tensions, window_groups=None, grad_consistency=True):
    """(diversity, consistency, entropy) as train.py:1083-1087 computes them.
    CUDA τ fields go through the fused τ consumer (``bozo_b200.aux``: one
    kernel pass over every field, one for the cotangent — per query row,
    inside the tension backward, when the consistency term takes no
    gradient); the framework-op formulas above serve the harness when it
    runs on CPU tensors."""
    if all_tensions and all_tensions[0].is_cuda:
        from .aux import tension_aux_losses
        return tension_aux_losses(all_tensions, window_groups, grad_consistency)
    return (tension_diversity_loss(all_tensions, window_groups),
            constraint_consistency_loss(all_tensions), tension_entropy_loss(all_tensions))


@dataclass
class TrainWeights:
    """train.py:135-141 defaults (the large preset leaves them unchanged)."""
    w_closure: float = 0.01
    w_diversity: float = 0.02
    w_consistency: float = 0.0
    w_entropy: float = 0.0

    @property
    def aux_enabled(self) -> bool:
        return any(w > 0 for w in (self.w_closure, self.w_diversity, self.w_consistency,
                                   self.w_entropy))


def _avg_allreduce_hook(process_group, bucket):
    """DDP communication hook: one NCCL all-reduce with the AVG operator per
    gradient bucket.  Without a hook DDP divides every gradient by the world
    size as it becomes ready — one elementwise kernel per parameter on the
    compute stream (130 launches, 0.32 ms of device time per 117M step on
    B200) — while NCCL applies the 1/N inside the all-reduce."""
    group = process_group if process_group is not None else dist.group.WORLD
    fut = dist.all_reduce(bucket.buffer(), op=dist.ReduceOp.AVG, group=group,
                          async_op=True).get_future()
    return fut.then(lambda f: f.value()[0])


def wrap_ddp(model: nn.Module, compress: bool = False, bucket_cap_mb: float = 64.0):
    """train.py:789-797: DDP with static graph, no buffer broadcast; gradients
    are bucketed and all-reduced (NCCL on GPUs) while the backward runs, in
    64 MB buckets (DDP's default is 25 MB), averaged inside the all-reduce
    (``_avg_allreduce_hook``) on NCCL.  ``compress`` all-reduces the buckets
    in bf16 (the reference all-reduces fp32).  Measured on two B200s (117M
    model, batch 16 x 1024 per GPU, ms per step, max over ranks, before the
    averaging hook): fp32 25 MB 27.30, fp32 64 MB 27.16, fp32 128 MB 27.24,
    bf16 25 MB 31.14, bf16 64 MB 27.45, bf16 128 MB 27.80, no DDP 25.88 —
    over NVLink the casts of the compression hook cost more than the halved
    bytes save, so it is off by default."""
    from torch.nn.parallel import DistributedDataParallel as DDP
    dev = next(model.parameters()).device

    def make():
        return DDP(model, device_ids=[dev.index] if dev.type == "cuda" else None,
                   find_unused_parameters=False, broadcast_buffers=False, static_graph=True,
                   gradient_as_bucket_view=True, bucket_cap_mb=bucket_cap_mb)
    if dev.type == "cuda":
        # set up on a side stream, as a CUDA graph that records the step
        # (GraphedTrainStep) requires of DDP
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            ddp = make()
        torch.cuda.current_stream(dev).wait_stream(side)
    else:
        ddp = make()
    if compress and dev.type == "cuda":
        # gradients cross NVLink as bf16 (half the bytes of the fp32 all-reduce);
        # the averaged result is written back in fp32 before the optimiser step
        from torch.distributed.algorithms.ddp_comm_hooks import default_hooks
        ddp.register_comm_hook(state=None, hook=default_hooks.bf16_compress_hook)
    elif dev.type == "cuda" and dist.get_backend() == "nccl":
        ddp.register_comm_hook(state=None, hook=_avg_allreduce_hook)
    return ddp


def make_optimizer(model: nn.Module, lr: float = 3e-4, weight_decay: float = 0.10,
                   fused: Optional[bool] = None, capturable: bool = False):
    """train.py:893-901: AdamW, decay on ≥2-D parameters, betas (0.9, 0.95).
    ``capturable``: step counts kept on the device, so the step can be
    recorded in a CUDA graph (``GraphedTrainStep``)."""
    decay = [p for p in model.parameters() if p.requires_grad and p.dim() >= 2]
    nodecay = [p for p in model.parameters() if p.requires_grad and p.dim() < 2]
    return torch.optim.AdamW([{"params": decay, "weight_decay": weight_decay},
                              {"params": nodecay, "weight_decay": 0.0}],
                             lr=lr, betas=(0.9, 0.95), eps=1e-8, fused=fused,
                             capturable=capturable)


def train_step(model, base_model: TensionLM, optimizer, inputs, targets,
               weights: Optional[TrainWeights] = None, clip_grad: float = 1.0,
               amp: bool = True):
    """One optimiser step of train.py:1040-1150 with grad_accum 1: bf16
    autocast forward (τ returned when aux losses are on), CE + the four aux
    losses (the three τ terms through ``aux_losses``), backward, global-norm
    clip, AdamW step.  Returns the loss tensor
    (not synchronised)."""
    weights = weights or TrainWeights()
    V = base_model.cfg.vocab_size
    dev_type = inputs.device.type
    ctx = torch.autocast(device_type=dev_type, dtype=torch.bfloat16) if amp \
        else torch.autocast(device_type=dev_type, enabled=False)
    with ctx:
        if weights.aux_enabled:
            logits, hidden, tensions = model(inputs, return_all=True)
        else:
            logits, hidden, tensions = model(inputs), None, []
        from . import block_ops
        flat, tflat = logits.reshape(-1, V), targets.reshape(-1)
        if block_ops.xent_applies(flat, tflat):
            loss = block_ops.cross_entropy(flat, tflat)
        else:
            loss = F.cross_entropy(flat, tflat)
        if weights.aux_enabled and tensions:
            # a zero consistency weight gives that term no gradient
            div, cons, ent = aux_losses(tensions, base_model.window_groups,
                                        grad_consistency=weights.w_consistency != 0.0)
            loss = (loss
                    + weights.w_closure * manifold_closure_loss(hidden)
                    + weights.w_diversity * div
                    + weights.w_consistency * cons
                    + weights.w_entropy * ent)
    loss.backward()
    nn.utils.clip_grad_norm_(base_model.parameters(), clip_grad)
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    if inputs.is_cuda:
        # a bounded wait that gave up in this step's kernels raises here, at
        # most one step late (an asynchronous read of the device error word)
        from .ops import check_device_error
        check_device_error(inputs.device)
    return loss.detach()


class GraphedTrainStep:
    """``train_step`` recorded once as a CUDA graph and replayed per batch.

    The step (autocast forward, CE + aux losses, backward — with DDP's
    bucketed NCCL all-reduces when ``model`` is wrapped — global-norm clip,
    AdamW) launches several hundred kernels; eager, the host's launch and
    autograd work leaves the GPU idle between the short ones (one B200: the
    13.5M step 7.9 → 5.9 ms, the 117M step 19.9 → 19.5 ms).  Replay runs the
    same kernels on the same buffers and leaves bit-identical parameters:
    token ids are copied into a static ``[batch, seq + 1]`` buffer, and
    ``loss`` is the static result tensor of the recorded step.

    Requirements: a capturable optimiser (``make_optimizer(capturable=True)``),
    fixed shapes, a learning rate that does not change between steps.  The
    first ``warmup`` steps run eagerly on a side stream (DDP needs at least
    11 before its buckets are final).  Release the graph (``release()``)
    before destroying a process group whose all-reduces it holds."""

    def __init__(self, model, base_model: TensionLM, optimizer, ids: torch.Tensor,
                 weights: Optional[TrainWeights] = None, clip_grad: float = 1.0,
                 warmup: Optional[int] = None):
        if not ids.is_cuda:
            raise RuntimeError("GraphedTrainStep: token ids must be a CUDA tensor")
        if not all(g.get("capturable", False) for g in optimizer.param_groups):
            raise ValueError("GraphedTrainStep: the optimiser must be capturable")
        from torch.nn.parallel import DistributedDataParallel as DDP
        if warmup is None:
            warmup = 11 if isinstance(model, DDP) else 3
        self.device = ids.device
        self.ids = ids.detach().clone()
        inputs, targets = self.ids[:, :-1], self.ids[:, 1:]
        args = (model, base_model, optimizer, inputs, targets, weights, clip_grad)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                train_step(*args)
        torch.cuda.current_stream(self.device).wait_stream(side)
        optimizer.zero_grad(set_to_none=True)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.loss = train_step(*args)

    def __call__(self, ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One optimiser step on ``ids`` (copied into the static buffer; the
        previous batch again when None).  Returns the static loss tensor
        (not synchronised; the next replay overwrites it)."""
        if self.graph is None:
            raise RuntimeError("GraphedTrainStep: released")
        if ids is not None:
            self.ids.copy_(ids, non_blocking=True)
        self.graph.replay()
        from .ops import check_device_error
        check_device_error(self.device)
        return self.loss

    def release(self) -> None:
        """Drop the graph (and with it any NCCL calls it recorded)."""
        self.graph = None



class GraphedForward:
    """The no-grad forward ``model(ids, return_all=...)`` recorded as CUDA
    graphs and replayed per batch (inference prefill).

    ``copies`` graphs, each with its own static token buffer, outputs and
    memory pool: the outputs of one replay can be read out (τ export) while
    the next replay runs on the other copy.  The 350M prefill (batch 4 ×
    2048, τ from all 24 layers) replays in 8.07 ms against 8.50 ms eager on
    one B200, outputs bit-identical.  Weights must stay fixed (the packed
    projection weights are cached by the warm-up forwards)."""

    def __init__(self, model: nn.Module, ids: torch.Tensor, return_all: bool = True,
                 copies: int = 1, warmup: int = 2):
        if not ids.is_cuda:
            raise RuntimeError("GraphedForward: token ids must be a CUDA tensor")
        self.model, self.return_all = model, return_all
        dev = ids.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._fwd(ids)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.slots = []
        for _ in range(copies):
            buf = ids.detach().clone()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = self._fwd(buf)
            self.slots.append((g, buf, out))

    def _fwd(self, x):
        with torch.no_grad():
            return self.model(x, return_all=True) if self.return_all else self.model(x)

    def __call__(self, ids: Optional[torch.Tensor] = None, copy: int = 0):
        """Replay graph ``copy`` on ``ids`` (copied into its static buffer;
        its previous batch when None) and return its static outputs, which
        its next replay overwrites."""
        g, buf, out = self.slots[copy]
        if ids is not None:
            buf.copy_(ids, non_blocking=True)
        g.replay()
        return out
