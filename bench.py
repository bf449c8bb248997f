"""Benchmark of the B200 tension operator.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = forward + backward of the fused tension op (RoPE base 10000 on
Q/K, local window, τ-mass normalisation — the model.py call-site semantics)
on one synthetic batch B=8, H=12, T=2048, HD=64, W=64, bf16, Q/K/V/dOut ~
N(0,1) from seed 0 (+rank).  Per-rank work is fixed (weak scaling: every
rank runs its own batch, no data-path collective — the op shards by batch).

Printed JSON (one line, rank 0):
  value     algorithmic HBM GB/s of the whole job (bytes: N_rows·(24·HD+8)
            per step, N_rows = B·H·T), inputs resident in HBM, CUDA events on
            the launching stream, max over ranks;
  e2e       the same metric through the public API with pinned HOST inputs
            copied in and (out, dq, dk, dv) copied back every step;
  roofline  for the dominant phase (fwd or bwd kernels) vs MEASURED_PEAKS;
  cpu_baseline  the reference algorithm (CPU oracle port, fp32, all host
            threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

B, H, T, HD = 8, 12, 2048, 64
W_HEAD = 64
WINDOWS = (32, 64, 128, 256)
FALLBACK_HBM_GBS = 6650.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, 1590.0, "fallback"


def sustained_tflops():
    """Dense bf16 peak for work timed inside a long step (MEASURED_PEAKS.json
    bf16_tflops_sustained; the fallback's sustained figure otherwise)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured sustained"
    return 1400.0, "fallback sustained"


def bytes_fwd(b=B, h=H, t=T, hd=HD):
    return b * h * t * (4 * hd * 2 + 4)


def bytes_bwd(b=B, h=H, t=T, hd=HD):
    return b * h * t * (8 * hd * 2 + 4)


def pairs(b, h, t, w):
    return b * h * (t * w - w * (w + 1) // 2) if t >= w else b * h * t * (t - 1) // 2


def flops_fwd_bwd(b, h, t, hd, w):
    return 12 * pairs(b, h, t, w) * hd


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, fl in rows for i, v in enumerate(fl)
                          if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def make_inputs(device, seed, b=B, t=T, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    mk = lambda: torch.randn(b, t, H, HD, generator=g).to(dtype)
    return [mk() for _ in range(4)]  # q, k, v, d_out (host)


def run_ours(args, rank, world, local_rank):
    import torch.distributed as dist
    import bozo_b200
    from bozo_b200 import ops as bops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    hq, hk, hv, hdo = make_inputs(dev, 1234 + rank)
    q, k, v, d_out = [x.to(dev) for x in (hq, hk, hv, hdo)]
    q.requires_grad_(True); k.requires_grad_(True); v.requires_grad_(True)

    def fwd(W, qq=q, kk=k, vv=v):
        return bozo_b200.tension(qq, kk, vv, window=W, rope_base=10_000.0, normalize="mass")

    def step(W, qq=q, kk=k, vv=v, dd=d_out):
        out = fwd(W, qq, kk, vv)
        gq, gk, gv = torch.autograd.grad(out, (qq, kk, vv), dd)
        return out, gq, gk, gv

    def barrier():
        if world > 1:
            dist.barrier()

    def maxred(x):
        if world > 1:
            t_ = torch.tensor([x], device=dev, dtype=torch.float64)
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
            return float(t_.item())
        return x

    def capture_fn(fn):
        """fn (calls of the public API) as one CUDA graph: its kernel launches
        replay without host work between them."""
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            keep = fn()
        torch.cuda.synchronize()
        return graph, keep

    def capture(W):
        return capture_fn(lambda: step(W))

    def timed(run, n, clk=None):
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if clk:
            clk.__enter__()
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        for _ in range(n):
            run()
        e1.record(stream)
        torch.cuda.synchronize()
        if clk:
            clk.__exit__(None, None, None)
        return maxred(e0.elapsed_time(e1)) / n

    results = {}
    # Process-level warm-up before any timed block: the first timed block of a
    # fresh process otherwise runs slow (clock and power ramp, allocator and
    # module first use); at least the requested warm-up steps, and ~1 s of work.
    t_w = time.perf_counter()
    n_w = 0
    while n_w < args.warmup or time.perf_counter() - t_w < 1.0:
        step(W_HEAD)
        n_w += 1
        if n_w % 8 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    barrier()
    # kernels of our library per step (forward call + backward call)
    fwd(W_HEAD)
    fl = bops.last_launches()
    step(W_HEAD)
    launches_per_step = fl + bops.last_launches()
    # Device time of the forward alone (its own CUDA graph); the backward's is
    # the step's minus the forward's.  (A backward is never captured alone:
    # autograd would run it on the stream of a forward made outside the
    # capture.)  After a failed capture every later block runs eagerly.
    phase = {}
    can_capture = True
    try:
        gf, kf = capture_fn(lambda: fwd(W_HEAD))
        phase["fwd_ms"] = timed(gf.replay, args.steps)
        del gf, kf
    except Exception:
        can_capture = False
        phase["fwd_ms"] = timed(lambda: fwd(W_HEAD), args.steps)
    for W in args.windows:
        steps = args.steps if W == W_HEAD else max(3, args.steps // 4)
        graph = keep = None
        run, mode = (lambda W=W: step(W)), "eager (capture unavailable)"
        if can_capture:
            try:
                graph, keep = capture(W)
                run, mode = graph.replay, "cuda-graph replay of the fwd+bwd step"
            except Exception as ex:  # time the eager calls from here on
                can_capture = False
                graph = keep = None
                run, mode = (lambda W=W: step(W)), f"eager ({type(ex).__name__})"
        for _ in range(args.warmup):
            run()
        clk = Clocks(local_rank) if W == W_HEAD else None
        ms = timed(run, steps, clk)
        results[W] = dict(ms=ms, steps=steps, mode=mode, launches=launches_per_step * steps,
                          clocks=clk.summary() if clk else None, path=bops.last_path())
        del graph, keep
        barrier()
    results[W_HEAD].update(phase)
    results[W_HEAD]["bwd_ms"] = max(results[W_HEAD]["ms"] - phase["fwd_ms"], 1e-6)

    if args.no_e2e:
        return results, None, launches_per_step

    # ── e2e: public API, pinned host buffers in, results out, every step ──
    # Step i copies its inputs in on a copy stream (into one of two device
    # input sets) while the compute stream runs step i−1's fwd+bwd and reads
    # its results back; stream events order them, so each upload overlaps the
    # previous step's compute and read-out (the link is full duplex).  The
    # read-out is queued on the compute stream itself: the results' memory is
    # then free for the next step as soon as their copies are, with no
    # cross-stream hold on the allocator's blocks.
    hq, hk, hv, hdo = [x.pin_memory() for x in (hq, hk, hv, hdo)]
    outs_h = [[torch.empty(B, T, H, HD, dtype=torch.bfloat16).pin_memory() for _ in range(4)]
              for _ in range(2)]
    ins_d = [[torch.empty(B, T, H, HD, dtype=torch.bfloat16, device=dev) for _ in range(4)]
             for _ in range(2)]
    s_in = torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]   # compute done reading input set

    def e2e_step(i):
        sl = i & 1
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_used[sl])
            for dst, src in zip(ins_d[sl], (hq, hk, hv, hdo)):
                dst.copy_(src, non_blocking=True)
            ev_in[sl].record(s_in)
        stream.wait_event(ev_in[sl])
        qq, kk, vv, dd = [x.detach().requires_grad_(j < 3) for j, x in enumerate(ins_d[sl])]
        out, gq, gk, gv = step(W_HEAD, qq, kk, vv, dd)
        ev_used[sl].record(stream)
        for dst, src in zip(outs_h[sl], (out, gq, gk, gv)):
            dst.copy_(src.detach(), non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    s0 = torch.cuda.Event(enable_timing=True); s1 = torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    s_in.wait_stream(stream)
    for i in range(args.steps):
        e2e_step(i)
    s1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = maxred(s0.elapsed_time(s1)) / args.steps
    barrier()
    return results, e2e_ms, launches_per_step


TRAIN_B, TRAIN_T = 16, 1024  # per-GPU batch 16, seq 1024


def run_train(args, rank, world, local_rank, cfg=None, batch=TRAIN_B, seq=TRAIN_T,
              variants=("aux_on", "aux_off"), ddp=True):
    """TensionLM training steps through the harness bozo_b200.lm — by default
    the 117M model of BASELINE configs[3] (per-GPU batch 16 × 1024 tokens);
    also the 13.5M model of configs[2] (batch 32 × 512).  bf16 autocast, the
    operator in every tension layer, CE + train.py's default aux losses
    (w_closure 0.01, w_diversity 0.02, which put τ export and its cotangent
    in the loop; ``aux_off`` drops them), global-norm clip, fused AdamW; DDP
    over NCCL when world > 1 (fp32 gradient all-reduce in 64 MB buckets,
    averaged inside the all-reduce).  Each timed step is one replay of the
    whole optimiser step recorded as a CUDA graph (``lm.GraphedTrainStep``);
    the same step run eagerly is timed beside it (aux_on).  Uniform random
    token ids from a per-rank seed, random init.  Returns
    ({variant: (ms_per_step max over ranks, e2e ms_per_step, eager ms_per_step)},
    params)."""
    import torch.distributed as dist
    from bozo_b200 import lm
    dev = torch.device("cuda", local_rank)
    torch.manual_seed(0)  # identical init on every rank (DDP also broadcasts rank 0's)
    cfg = cfg or lm.preset_117m()
    base = lm.TensionLM(cfg).to(dev)
    model = lm.wrap_ddp(base) if (world > 1 and ddp) else base
    opt = lm.make_optimizer(base, fused=True, capturable=True)
    g = torch.Generator().manual_seed(4242 + rank)
    ids_h = torch.randint(0, cfg.vocab_size, (batch, seq + 1), generator=g).pin_memory()
    ids = ids_h.to(dev)
    inputs, targets = ids[:, :-1], ids[:, 1:]
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)

    def maxred(x):
        if world > 1:
            t_ = torch.tensor([x], device=dev, dtype=torch.float64)
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
            return float(t_.item())
        return x

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn, k):
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return maxred(e0.elapsed_time(e1)) / k

    out = {}
    weights = {"aux_on": lm.TrainWeights(), "aux_off": lm.TrainWeights(0.0, 0.0, 0.0, 0.0)}
    for name in variants:
        w = weights[name]
        eager = None
        if name == "aux_on":
            for _ in range(args.train_warmup):
                lm.train_step(model, base, opt, inputs, targets, weights=w)
            eager = timed(lambda: lm.train_step(model, base, opt, inputs, targets, weights=w),
                          args.train_steps)
        # the graph's own warm-up steps run eagerly first (11 under DDP)
        step = lm.GraphedTrainStep(model, base, opt, ids, weights=w)
        for _ in range(args.train_warmup):
            step()
        ms = timed(step, args.train_steps)
        e2e = None
        if name == "aux_on":
            # end to end: token ids copied in from pinned host memory and the
            # loss read back every step
            def e2e_step():
                loss_h.copy_(step(ids_h), non_blocking=True)
            e2e = timed(e2e_step, args.train_steps)
        step.release()  # before any process-group teardown: it holds NCCL calls
        del step
        out[name] = (ms, e2e, eager)
        barrier()
    params = base.num_params
    del model, base, opt
    torch.cuda.empty_cache()
    return out, params


def run_tau_consumer(local_rank, iters=20):
    """The fused τ consumer (bozo_b200.aux, csrc/tau_aux.cu) on the fields of
    the 117M training step: 12 τ fields [16,1024,12,64] bf16 (302 MB).  Device
    times (CUDA events over `iters` launches) of the statistics pass (one read
    of every field) and the cotangent pass (one read, one write), the fused
    losses fwd+bwd through autograd, and the framework-op formulation of the
    same three losses (model.py:498-611 restated in bozo_b200.lm, autocast)."""
    from bozo_b200 import _capi, aux, lm
    dev = torch.device("cuda", local_rank)
    g = torch.Generator(device=dev).manual_seed(77)
    taus = [torch.rand(TRAIN_B, TRAIN_T, 12, 64, device=dev, generator=g).to(torch.bfloat16)
            for _ in range(12)]
    groups = {64: [0, 1, 2, 4, 5, 6, 8, 9, 10], 1024: [3, 7, 11]}
    d_stats = torch.ones(12, 3, device=dev)
    leaves = [t.clone().requires_grad_(True) for t in taus]

    def fused_losses():
        d, c, e = aux.tension_aux_losses(leaves, groups)
        torch.autograd.grad(0.02 * d + 0.0 * c + 0.0 * e, leaves)

    def framework_losses():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            d = lm.tension_diversity_loss(leaves, groups)
            c = lm.constraint_consistency_loss(leaves)
            e = lm.tension_entropy_loss(leaves)
        torch.autograd.grad(0.02 * d + 0.0 * c + 0.0 * e, leaves)

    def timed(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n

    ms_stats = timed(lambda: aux.tau_field_stats(taus), iters)
    ms_cot = timed(lambda: _capi.ext().tau_aux_bwd(taus, d_stats), iters)
    ms_fused = timed(fused_losses, 10)
    ms_fw = timed(framework_losses, 3)
    field_bytes = 12 * TRAIN_B * TRAIN_T * 12 * 64 * 2
    hbm = peaks()[0]
    return {
        "fields": "12 x [16,1024,12,64] bf16 (the 117M step's tau fields)",
        "stats_us": round(ms_stats * 1e3, 1),
        "stats_gbs": round(field_bytes / (ms_stats * 1e-3) / 1e9, 1),
        "stats_frac_hbm": round(field_bytes / (ms_stats * 1e-3) / 1e9 / hbm, 4),
        "cotangent_us": round(ms_cot * 1e3, 1),
        "cotangent_gbs": round(2 * field_bytes / (ms_cot * 1e-3) / 1e9, 1),
        "cotangent_frac_hbm": round(2 * field_bytes / (ms_cot * 1e-3) / 1e9 / hbm, 4),
        "fused_losses_fwd_bwd_ms": round(ms_fused, 3),
        "framework_ops_fwd_bwd_ms": round(ms_fw, 3),
    }


GLOBAL_B, GLOBAL_T = 16, 1024  # the 117M model's global layer (configs[3] shape)


def run_global_block(local_rank, steps=20, warmup=5):
    """The global full-causal block (model.py:217-237) at the 117M layer
    shape B16 H12 T1024 HD64, bf16, RoPE, τ-mass: forward + backward of
    ``bozo_b200.tension(window=None)`` as one CUDA-graph replay, and the
    forward alone.  This block sits at the ridge (77.4 GFLOP against 303.6 MB
    per fwd+bwd), so both roofline fractions are reported."""
    import bozo_b200
    dev = torch.device("cuda", local_rank)
    g = torch.Generator().manual_seed(55)
    q, k, v, d = [torch.randn(GLOBAL_B, GLOBAL_T, H, HD, generator=g).to(dev, torch.bfloat16)
                  for _ in range(4)]
    for x in (q, k, v):
        x.requires_grad_(True)

    def fwd():
        return bozo_b200.tension(q, k, v, window=None, normalize="mass")

    def step():
        out = fwd()
        return torch.autograd.grad(out, (q, k, v), d)

    def graph_of(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            keep = fn()
        return gr, keep

    def timed(run):
        for _ in range(warmup):
            run()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            run()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps

    gs, ks = graph_of(step)
    ms_step = timed(gs.replay)
    path = bozo_b200.last_path()
    gf, kf = graph_of(fwd)
    ms_fwd = timed(gf.replay)
    del gs, ks, gf, kf
    hbm, tfl, kind = peaks()
    nbytes = bytes_fwd(GLOBAL_B, H, GLOBAL_T) + bytes_bwd(GLOBAL_B, H, GLOBAL_T)
    pairs_g = GLOBAL_B * H * GLOBAL_T * (GLOBAL_T + 1) // 2
    flops = 12 * pairs_g * HD
    gbs = nbytes / (ms_step * 1e-3) / 1e9
    tfs = flops / (ms_step * 1e-3) / 1e12
    ms_bwd = max(ms_step - ms_fwd, 1e-6)
    return {
        "workload": "global full-causal block fwd+bwd, B16 H12 T1024 HD64 bf16, RoPE, tau-mass "
                    "(the 117M model's global layer, model.py:217-237)",
        "ms_per_step": round(ms_step, 4), "fwd_ms": round(ms_fwd, 4), "bwd_ms": round(ms_bwd, 4),
        "kernel_path": path,
        "gbs": round(gbs, 1), "tflops": round(tfs, 1),
        "frac_hbm": round(gbs / hbm, 4), "frac_tensor": round(tfs / tfl, 4),
        "frac_roofline": round(max(nbytes / (hbm * 1e9), flops / (tfl * 1e12)) / (ms_step * 1e-3), 4),
        "fwd_tflops": round(4 * pairs_g * HD / (ms_fwd * 1e-3) / 1e12, 1),
        "bwd_tflops": round(8 * pairs_g * HD / (ms_bwd * 1e-3) / 1e12, 1),
        "algorithmic": {"bytes": nbytes, "flops": flops,
                        "hbm_floor_us": round(nbytes / (hbm * 1e9) * 1e6, 1),
                        "flop_floor_us": round(flops / (tfl * 1e12) * 1e6, 1)},
        "peaks": f"{hbm} GB/s, {tfl} TFLOP/s bf16 burst ({kind})",
    }


def run_drop_in_layer(local_rank, steps=20, warmup=5):
    """model.py's own call site at the 117M layer shape, through the drop-in
    ``causal_tension`` exactly as model.py:248-258 uses it under train.py's
    bf16 autocast: bf16 projections rotated by fp32 RoPE tables (fp32 Q/K,
    model.py:203-204), bf16 V, τ returned, out = S / clamp(Στ, 1e-6);
    forward + backward of ⟨out, dO⟩, B16 T1024 H12 HD64 W64.  Timed on the
    tensor cores (the default path) and, for context, forced onto the
    exact-fp32 CUDA-core kernels the same call would take without the
    bf16 operand copies."""
    import bozo_b200
    from bozo_b200 import ops as bops
    dev = torch.device("cuda", local_rank)
    Bq, Tq, W = TRAIN_B, TRAIN_T, 64
    g = torch.Generator().manual_seed(66)
    qr, kr, vr, d = [torch.randn(Bq, Tq, H, HD, generator=g).to(dev, torch.bfloat16) for _ in range(4)]
    for x in (qr, kr, vr):
        x.requires_grad_(True)
    cos, sin, _ = bops.rope_tables(HD, Tq, 10_000.0, dev)
    c_, s_ = cos.unsqueeze(0).unsqueeze(2), sin.unsqueeze(0).unsqueeze(2)

    def rope(x):  # model.py:75-81 with the fp32 table buffers
        x1, x2 = x[..., :HD // 2], x[..., HD // 2:]
        return torch.cat([x1 * c_ - x2 * s_, x1 * s_ + x2 * c_], dim=-1)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            msg, tau = bozo_b200.causal_tension(rope(qr), rope(kr), vr, W, 8.0, return_tau=True)
            out = msg / tau.sum(-1).clamp(min=1e-6).unsqueeze(-1)
        return torch.autograd.grad(out, (qr, kr, vr), d.float())

    def timed():
        for _ in range(warmup):
            step()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps

    ms_tc = timed()
    path_tc = bozo_b200.last_path()
    prev = bops._path_override
    bozo_b200.set_kernel_path("simt")
    try:
        steps_s, steps = steps, max(3, steps // 5)
        ms_simt = timed()
        steps = steps_s
    finally:
        bozo_b200.set_kernel_path(prev)
    tok = Bq * Tq
    return {
        "workload": "model.py call site via the drop-in causal_tension under bf16 autocast "
                    "(fp32 RoPE'd Q/K, bf16 V, tau returned, tau-mass division; model.py:248-258), "
                    "fwd+bwd incl. the RoPE and division ops, B16 T1024 H12 HD64 W64",
        "ms_per_step": round(ms_tc, 4), "tokens_per_s": round(tok / (ms_tc * 1e-3), 1),
        "kernel_path": path_tc,
        "cuda_core_fp32_ms_per_step": round(ms_simt, 4),
        "speedup_vs_cuda_core": round(ms_simt / ms_tc, 2),
        "timing": "eager calls, CUDA events",
    }


ONE_M_B, ONE_M_T = 8, 256  # the reference's CPU-runnable model


def _one_m_step(model, ids, targets):
    logits = model(ids)
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1))
    loss.backward()
    return loss


def run_1m_gpu(local_rank, steps=20):
    """configs[0] on the GPU: the 1.1M model (head_dim 32, fp32) forward +
    backward of the cross-entropy loss through the operator (the exact-fp32
    CUDA-core path serves HD 32 and fp32)."""
    import bozo_b200
    from bozo_b200 import lm
    dev = torch.device("cuda", local_rank)
    torch.manual_seed(0)
    model = lm.TensionLM(lm.preset_1m()).to(dev)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 2048, (ONE_M_B, ONE_M_T + 1), generator=g).to(dev)
    x, y = ids[:, :-1], ids[:, 1:]
    for _ in range(3):
        _one_m_step(model, x, y)
        model.zero_grad(set_to_none=True)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        _one_m_step(model, x, y)
        model.zero_grad(set_to_none=True)
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    return {"value": round(ONE_M_B * ONE_M_T / (ms * 1e-3), 1), "unit": "tokens/s",
            "ms_per_step": round(ms, 3), "kernel_path": bozo_b200.last_path(),
            "dtype": "fp32", "params": model.num_params}


def cpu_model_name() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_1m(budget_s=12.0):
    """configs[0] timed on the host cores: the same 1.1M model (the harness,
    model.py restated) with the oracle's unfold restatement of the tension
    op (ops.py:29-63, model.py:271-283) in place of the kernels, fp32
    forward + backward of the cross-entropy loss, all host threads."""
    from bozo_b200 import lm
    from oracle import tension_oracle as orc

    def oracle_tension(q, k, v, *, window, scale, rope_base=10_000.0, rope_len=None, bias=None,
                       return_tau=False, normalize="mass", tau_window=None):
        out, tau = orc.fused_reference(q, k, v, window=window, scale=scale, rope_base=rope_base,
                                       bias=bias, normalize=normalize or "none",
                                       local_window=tau_window or 64, max_seq_len=rope_len)
        return (out, tau) if return_tau else out

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    model = lm.TensionLM(lm.preset_1m())
    model.set_tension_fn(oracle_tension)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 2048, (ONE_M_B, ONE_M_T + 1), generator=g)
    x, y = ids[:, :-1], ids[:, 1:]
    _one_m_step(model, x, y)
    model.zero_grad(set_to_none=True)
    reps, t0 = 0, time.perf_counter()
    while True:
        _one_m_step(model, x, y)
        model.zero_grad(set_to_none=True)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 30:
            break
    ms = el * 1e3 / reps
    return {"value": round(ONE_M_B * ONE_M_T / (ms * 1e-3), 1), "unit": "tokens/s",
            "ms_per_step": round(ms, 2), "cores": threads, "cpu": cpu_model_name(),
            "kind": "port", "sample": f"{reps} fwd+bwd steps of B{ONE_M_B} T{ONE_M_T}, fp32"}


DECODE_B, DECODE_PROMPT, DECODE_NEW = 16, 960, 64


def run_decode(local_rank):
    """117M TensionLM decoding (the configs[3] model, bf16 weights): 16
    prompts of 960 tokens prefilled, then 64 tokens per sequence fed one at a
    time through the ring caches (bozo_b200.decode.StepGraph replays; CUDA
    events over the last 61 steps).  Beside it the reference's scheme
    (model.py:718-768 generate_cached: one full forward over the context per
    generated token), timed on the same model and batch at a 992-token
    context.  Returns a dict for the JSON line."""
    from bozo_b200 import decode, lm
    dev = torch.device("cuda", local_rank)
    torch.manual_seed(0)
    model = lm.TensionLM(lm.preset_117m()).to(dev).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(99)
    ids = torch.randint(0, 32768, (DECODE_B, DECODE_PROMPT + DECODE_NEW), generator=g).to(dev)
    state = decode.DecodeState(model, DECODE_B, DECODE_PROMPT + DECODE_NEW)
    decode.prefill(state, ids[:, :DECODE_PROMPT])
    graph = decode.StepGraph(state)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    warm = 3
    for t in range(DECODE_PROMPT, DECODE_PROMPT + warm):
        graph(ids[:, t])
    torch.cuda.synchronize(dev)
    e0.record()
    for t in range(DECODE_PROMPT + warm, DECODE_PROMPT + DECODE_NEW):
        graph(ids[:, t])
    e1.record()
    torch.cuda.synchronize(dev)
    ms_tok = e0.elapsed_time(e1) / (DECODE_NEW - warm)
    ctx = ids[:, :DECODE_PROMPT + 32]
    with torch.no_grad():
        for _ in range(2):
            model(ctx)
        torch.cuda.synchronize(dev)
        e0.record()
        for _ in range(5):
            model(ctx)
        e1.record()
        torch.cuda.synchronize(dev)
    ms_full = e0.elapsed_time(e1) / 5
    del graph, state, model
    return {
        "metric": "117M TensionLM decode tokens/s (batch of sequences, one token each per step)",
        "value": round(DECODE_B / (ms_tok * 1e-3), 1), "unit": "tokens/s",
        "ms_per_token_step": round(ms_tok, 4),
        "full_forward_per_token": {"value": round(DECODE_B / (ms_full * 1e-3), 1),
                                   "unit": "tokens/s", "ms_per_token_step": round(ms_full, 3),
                                   "scheme": "generate_cached: one forward over the context "
                                             "per generated token (992-token context)"},
        "speedup": round(ms_full / ms_tok, 1),
        "config": {"workload": "TensionLM 117M decode, ring caches + CUDA-graph step",
                   "batch": DECODE_B, "prompt": DECODE_PROMPT, "new_tokens": DECODE_NEW,
                   "dtype": "bf16 weights and caches",
                   "data": "uniform random token ids, random init"},
    }


PREFILL_B, PREFILL_T = 4, 2048  # batch 32 over 8 GPUs, seq 2048


def run_prefill(args, rank, world, local_rank):
    """350M TensionLM inference prefill with τ export:
    bf16 weights, no grad, every layer returns τ (local [B,T,H,W], global
    the exported window), batch 4 per GPU (32 over 8 GPUs), T 2048, random
    init, uniform token ids.  Pure replicas: no collective.  The timed
    forward is a CUDA-graph replay (``lm.GraphedForward``); the eager
    forward is timed beside it.  Returns (ms per forward max over ranks, e2e
    ms with token ids in and every layer's τ read back to pinned host
    memory, params, τ bytes, eager ms per forward)."""
    import torch.distributed as dist
    from bozo_b200 import lm
    dev = torch.device("cuda", local_rank)
    torch.manual_seed(0)
    cfg = lm.preset_350m_prefill()
    model = lm.TensionLM(cfg).to(dev, torch.bfloat16).eval()
    g = torch.Generator().manual_seed(777 + rank)
    ids_h = torch.randint(0, cfg.vocab_size, (PREFILL_B, PREFILL_T), generator=g).pin_memory()
    ids = ids_h.to(dev)
    stream = torch.cuda.current_stream(dev)

    def fwd(x):
        with torch.no_grad():
            return model(x, return_all=True)

    def maxred(x):
        if world > 1:
            t_ = torch.tensor([x], device=dev, dtype=torch.float64)
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
            return float(t_.item())
        return x

    _, _, taus = fwd(ids)
    tau_bytes = sum(t.numel() * t.element_size() for t in taus)
    del taus

    def timed(fn, k):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return maxred(e0.elapsed_time(e1)) / k

    for _ in range(args.train_warmup):
        fwd(ids)
    eager = timed(lambda: fwd(ids), args.train_steps)
    # the forward replayed as a CUDA graph: two copies with their own static
    # outputs, so one copy's τ can be read out while the other runs
    graphed = lm.GraphedForward(model, ids, copies=2)
    for _ in range(args.train_warmup):
        graphed()
    ms = timed(graphed, args.train_steps)
    # end to end: token ids in from pinned memory, every layer's τ out to
    # pinned memory each forward.  Forward i's τ read-out runs on a copy
    # stream while forward i+1 computes on the other graph copy; a copy is
    # replayed again only after the read-out of its previous τ finished.
    taus_hs = [[torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in graphed.slots[c][2][2]]
               for c in range(2)]
    s_out = torch.cuda.Stream(dev)
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]
    count = [0]

    def e2e_run(n):
        for _ in range(n):
            sl = count[0] & 1
            count[0] += 1
            if used[sl]:
                stream.wait_event(ev_out[sl])
            _, _, taus_i = graphed(ids_h, copy=sl)
            ev_done[sl].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[sl])
                for dst, src in zip(taus_hs[sl], taus_i):
                    dst.copy_(src, non_blocking=True)
                ev_out[sl].record(s_out)
            used[sl] = True
        stream.wait_stream(s_out)

    e2e_run(2)  # untimed
    e2e = timed(lambda: e2e_run(args.train_steps), 1) / args.train_steps
    params = model.num_params
    del model
    torch.cuda.empty_cache()
    del graphed
    return ms, e2e, params, tau_bytes, eager


def cpu_baseline(budget_s=12.0):
    """The reference CPU algorithm (oracle port of ops.py:29-63 + model.py
    τ-mass + RoPE, fp32 autograd) on B=1 slices of the workload."""
    from oracle import tension_oracle as orc
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    orc.cpu_fwd_bwd_sample(B=1, T=256, W=W_HEAD)  # warm the allocator
    reps, t0 = 0, time.perf_counter()
    while True:
        orc.cpu_fwd_bwd_sample(B=1, H=H, T=T, HD=HD, W=W_HEAD, seed=reps)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 8:
            break
    gbs = bytes_fwd(1) * reps / el / 1e9 + bytes_bwd(1) * reps / el / 1e9
    return dict(value=round(gbs, 4), unit="GB/s", cores=threads, cpu=cpu_model_name(), kind="port",
                sample=f"{reps} x B=1 slices (1/{B} of the batch each) of B{B} H{H} T{T} "
                       f"HD{HD} W{W_HEAD}, fp32 unfold+autograd, {el:.1f}s",
                tokens_per_s=round(reps * T / el, 1))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end leg (profiling runs)")
    ap.add_argument("--workload", default="all",
                    choices=["all", "op", "iso", "train", "prefill", "decode", "global"],
                    help="op: isolated operator (headline) + global block + drop-in call site; "
                         "iso: the isolated operator alone (profiling); train: 117M training step; "
                         "prefill: 350M inference prefill with tau export; "
                         "decode: 117M token-by-token decoding")
    ap.add_argument("--train-steps", type=int, default=10)
    ap.add_argument("--train-warmup", type=int, default=3)
    ap.add_argument("--windows", type=int, nargs="+", default=list(WINDOWS),
                    help="windows to time; the headline window is always included")
    args = ap.parse_args()
    # the headline window is timed first, the others follow
    args.windows = [W_HEAD] + [w for w in args.windows if w != W_HEAD]
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    hbm, tfl, peak_kind = peaks()
    per_step_bytes = bytes_fwd() + bytes_bwd()
    cfg = {"workload": "isolated tension op fwd+bwd (BASELINE configs[1])",
           "B": B, "H": H, "T": T, "HD": HD, "W": W_HEAD, "rope_base": 10000,
           "normalize": "mass", "tau_export": False, "per_rank_batch": B,
           "l2": "inputs+outputs 303.6 MB per step > 126 MB L2; no flush needed",
           "parallelism": f"batch-sharded replicas x{args.gpus}"}

    if args.impl == "reference":
        if rank != 0:
            return
        torch.set_num_threads(os.cpu_count() or 1)
        from oracle import tension_oracle as orc
        for _ in range(max(1, min(args.warmup, 1))):
            orc.cpu_fwd_bwd_sample(B=1, H=H, T=T, HD=HD, W=W_HEAD)
        t0 = time.perf_counter()
        for i in range(args.steps):
            orc.cpu_fwd_bwd_sample(B=1, H=H, T=T, HD=HD, W=W_HEAD, seed=i)
        el = time.perf_counter() - t0
        ms = el * 1e3 / args.steps
        val = (bytes_fwd(1) + bytes_bwd(1)) / (ms * 1e-3) / 1e9
        line = {"impl": "reference", "metric": "tension fwd+bwd algorithmic HBM GB/s",
                "value": round(val, 4), "unit": "GB/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic N(0,1)", "config": cfg,
                "cpu_baseline": {"value": round(val, 4), "unit": "GB/s",
                                 "cores": torch.get_num_threads(), "cpu": cpu_model_name(),
                                 "kind": "port",
                                 "sample": f"each step = one B=1 slice (1/{B} of the batch)"},
                "e2e": {"value": round(val, 4), "unit": "GB/s",
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    results = train = prefill = train13 = glob_obj = one_m = None
    if args.workload in ("all", "op", "iso"):
        results, e2e_ms, launches_per_step = run_ours(args, rank, world, local_rank)
    drop_in = None
    tau_consumer = None
    if args.workload in ("all", "train"):
        torch.cuda.empty_cache()
        train, n_params = run_train(args, rank, world, local_rank)
        torch.cuda.empty_cache()
        tau_consumer = run_tau_consumer(local_rank)
        torch.cuda.empty_cache()
        from bozo_b200 import lm as _lm
        # the 13.5M step is ≈ 6 ms: more steps for a stable figure (same
        # warm-up rule)
        a13 = argparse.Namespace(**vars(args))
        a13.train_steps, a13.train_warmup = max(args.train_steps, 30), max(args.train_warmup, 5)
        train13 = run_train(a13, rank, world, local_rank, cfg=_lm.preset_13m(), batch=32,
                            seq=512, variants=("aux_on",))
        torch.cuda.empty_cache()
        one_m = {"gpu": run_1m_gpu(local_rank)}
    # the single-layer measurements run after the training steps: those
    # (host-launch-heavy at 13.5M) read slower after them in one process
    if args.workload in ("all", "op", "global"):
        torch.cuda.empty_cache()
        glob_obj = run_global_block(local_rank)
    if args.workload in ("all", "op"):
        torch.cuda.empty_cache()
        drop_in = run_drop_in_layer(local_rank)
    if args.workload in ("all", "prefill"):
        torch.cuda.empty_cache()
        prefill = run_prefill(args, rank, world, local_rank)
    decode_obj = None
    if args.workload in ("all", "decode"):
        torch.cuda.empty_cache()
        decode_obj = run_decode(local_rank)
        decode_obj["n_gpus_running"] = 1  # each rank decodes its own batch; rank 0 reports
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return
    train_obj = None
    if train is not None:
        n = args.gpus
        tok = n * TRAIN_B * TRAIN_T
        ms_on, e2e_on, eager_on = train["aux_on"]
        ms_off, _, _ = train["aux_off"]
        flop_tok = 6 * n_params + 12 * 64 * 12 * (9 * 64 + 3 * (TRAIN_T + 1) / 2)
        tflops = tok * flop_tok / (ms_on * 1e-3) / 1e12
        train_obj = {
            "metric": "117M TensionLM train tokens/s (whole job)",
            "value": round(tok / (ms_on * 1e-3), 1), "unit": "tokens/s",
            "ms_per_step": round(ms_on, 3), "eager_ms_per_step": round(eager_on, 3),
            "steps": args.train_steps,
            "warmup": args.train_warmup, "n_gpus": n,
            "aux_losses": "on (train.py defaults w_closure 0.01, w_diversity 0.02)",
            "aux_off": {"value": round(tok / (ms_off * 1e-3), 1), "unit": "tokens/s",
                        "ms_per_step": round(ms_off, 3)},
            "model_tflops": round(tflops, 1),
            "mfu": round(tflops / (n * sustained_tflops()[0]), 4),
            "mfu_peak": f"{sustained_tflops()[0]} TFLOP/s bf16 per GPU ({sustained_tflops()[1]})",
            "flops_per_token": int(flop_tok),
            "e2e": {"value": round(tok / (e2e_on * 1e-3), 1), "unit": "tokens/s",
                    "ms_per_step": round(e2e_on, 3),
                    "h2d_bytes_per_step": TRAIN_B * (TRAIN_T + 1) * 8,
                    "d2h_bytes_per_step": 4},
            "config": {"workload": "TensionLM 117M training step (BASELINE configs[3])",
                       "params": n_params, "dim": 768, "layers": 12, "heads": 12,
                       "vocab": 32768, "W": 64, "global_every": 4, "seq_len": TRAIN_T,
                       "per_gpu_batch": TRAIN_B, "global_batch": TRAIN_B * n,
                       "dtype": "bf16 autocast, fp32 master weights", "optimizer": "AdamW (fused)",
                       "execution": ("whole optimiser step replayed as one CUDA graph "
                                     "(lm.GraphedTrainStep); eager_ms_per_step: the same step "
                                     "launched op by op"),
                       "parallelism": f"ddp{n}" if n > 1 else "single GPU",
                       "gradient_allreduce": ("NCCL, fp32, averaged in the all-reduce, 64 MB "
                                              "buckets overlapped with the "
                                              "backward (static graph)") if n > 1 else None,
                       "data": "uniform random token ids, random init"},
            "tau_consumer": tau_consumer,
        }
    train13_obj = None
    if train13 is not None:
        n = args.gpus
        (ms13, e2e13, eager13), p13 = train13[0]["aux_on"], train13[1]
        tok13 = n * 32 * 512
        train13_obj = {
            "metric": "13.5M TensionLM train tokens/s (whole job)",
            "value": round(tok13 / (ms13 * 1e-3), 1), "unit": "tokens/s",
            "ms_per_step": round(ms13, 3), "eager_ms_per_step": round(eager13, 3),
            "steps": max(args.train_steps, 30),
            "warmup": max(args.train_warmup, 5), "n_gpus": n,
            "e2e": {"value": round(tok13 / (e2e13 * 1e-3), 1), "unit": "tokens/s",
                    "ms_per_step": round(e2e13, 3), "h2d_bytes_per_step": 32 * 513 * 8,
                    "d2h_bytes_per_step": 4},
            "config": {"workload": "TensionLM 13.5M training step (BASELINE configs[2])",
                       "params": p13, "dim": 384, "layers": 6, "heads": 6, "vocab": 8192,
                       "W": 64, "global_every": 4, "seq_len": 512, "per_gpu_batch": 32,
                       "dtype": "bf16 autocast, fp32 master weights",
                       "aux_losses": "on (train.py defaults)", "optimizer": "AdamW (fused)",
                       "execution": "whole optimiser step replayed as one CUDA graph",
                       "parallelism": f"ddp{n}" if n > 1 else "single GPU",
                       "data": "uniform random token ids, random init"},
        }
    if one_m is not None and rank == 0 and args.gpus == 1 and not args.no_cpu_baseline:
        one_m["cpu"] = cpu_1m()
        one_m["config"] = {"workload": "TensionLM 1.1M fwd+bwd of the CE loss (BASELINE configs[0])",
                           "dim": 128, "layers": 4, "heads": 4, "head_dim": 32, "vocab": 2048,
                           "W": 64, "seq_len": ONE_M_T, "batch": ONE_M_B, "dtype": "fp32",
                           "data": "uniform random token ids (seed 0), random init"}
    prefill_obj = None
    if prefill is not None:
        n = args.gpus
        ms_p, e2e_p, p_params, tau_bytes, eager_p = prefill
        tok = n * PREFILL_B * PREFILL_T
        prefill_obj = {
            "metric": "350M TensionLM prefill tokens/s with tau export (whole job)",
            "value": round(tok / (ms_p * 1e-3), 1), "unit": "tokens/s",
            "ms_per_step": round(ms_p, 3), "eager_ms_per_step": round(eager_p, 3),
            "steps": args.train_steps, "n_gpus": n,
            "model_tflops": round(tok * 2 * p_params / (ms_p * 1e-3) / 1e12, 1),
            "e2e": {"value": round(tok / (e2e_p * 1e-3), 1), "unit": "tokens/s",
                    "ms_per_step": round(e2e_p, 3),
                    "h2d_bytes_per_step": PREFILL_B * PREFILL_T * 8,
                    "d2h_bytes_per_step": tau_bytes},
            "config": {"workload": "TensionLM 350M prefill, every layer's tau exported "
                                   "(BASELINE configs[4])",
                       "params": p_params, "dim": 1024, "layers": 24, "heads": 16,
                       "vocab": 32768, "W": 128, "global_every": 3, "seq_len": PREFILL_T,
                       "per_gpu_batch": PREFILL_B, "global_batch": PREFILL_B * n,
                       "dtype": "bf16 weights, no grad", "tau_bytes_per_gpu": tau_bytes,
                       "execution": ("forward replayed as a CUDA graph (lm.GraphedForward, two "
                                     "copies so one copy's tau read-out overlaps the next "
                                     "forward); eager_ms_per_step: launched op by op"),
                       "parallelism": f"batch-sharded replicas x{n}",
                       "data": "uniform random token ids, random init"},
        }
    if results is None:
        if train_obj is None and prefill_obj is None:
            solo = decode_obj if decode_obj is not None else dict(
                glob_obj, metric="global block fwd+bwd algorithmic GB/s", value=glob_obj["gbs"],
                unit="GB/s")
            print(json.dumps(dict(solo, higher_is_better=True, scaling="weak",
                                  vs_baseline=None, dtype="bf16", data="synthetic",
                                  n_gpus=args.gpus)))
            return
        line = dict(train_obj or prefill_obj)
        line.update({"higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                     "dtype": "bf16", "data": "synthetic"})
        line["config"] = (train_obj or prefill_obj)["config"]
        if train13_obj is not None:
            line["train_13m"] = train13_obj
        if one_m is not None:
            line["config0_1m"] = one_m
        if train_obj is not None and prefill_obj is not None:
            line["prefill_350m"] = prefill_obj
        if decode_obj is not None:
            line["decode_117m"] = decode_obj
        print(json.dumps(line))
        return

    head = results[W_HEAD]
    n = args.gpus
    value = n * per_step_bytes / (head["ms"] * 1e-3) / 1e9
    fwd_gbs = bytes_fwd() / (head["fwd_ms"] * 1e-3) / 1e9
    bwd_gbs = bytes_bwd() / (head["bwd_ms"] * 1e-3) / 1e9
    dom = "bwd" if head["bwd_ms"] >= head["fwd_ms"] else "fwd"
    ach = bwd_gbs if dom == "bwd" else fwd_gbs
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        traffic = json.load(open(tp)).get(f"{dom}_bytes_per_launch")
    h2d = 4 * B * T * H * HD * 2
    d2h = 4 * B * T * H * HD * 2
    line = {
        "metric": "tension fwd+bwd algorithmic HBM GB/s", "value": round(value, 2),
        "unit": "GB/s", "n_gpus": n, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(head["ms"], 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seed 1234+rank",
        "config": cfg,
        "tflops": round(n * flops_fwd_bwd(B, H, T, HD, W_HEAD) / (head["ms"] * 1e-3) / 1e12, 3),
        "kernel_path": head["path"],
        "timing": head["mode"],
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(ach, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(ach / hbm, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "fwd_gbs": round(fwd_gbs, 1), "bwd_gbs": round(bwd_gbs, 1),
                     "fwd_ms": round(head["fwd_ms"], 4), "bwd_ms": round(head["bwd_ms"], 4)},
        "per_window": {str(W): {"ms_per_step": round(r["ms"], 4), "timing": r["mode"],
                                "gbs": round(per_step_bytes / (r["ms"] * 1e-3) / 1e9, 1),
                                "tflops": round(flops_fwd_bwd(B, H, T, HD, W) / (r["ms"] * 1e-3) / 1e12, 3),
                                "frac_of_roofline": round(max(per_step_bytes / (hbm * 1e9),
                                                              flops_fwd_bwd(B, H, T, HD, W) / (tfl * 1e12))
                                                          / (r["ms"] * 1e-3), 4)}
                       for W, r in results.items()},
        "e2e": None if e2e_ms is None else {
            "value": round(n * per_step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h},
        "gpu_launches": head["launches"],
        "launches_per_step": launches_per_step,
        "clocks": head["clocks"],
    }
    if glob_obj is not None:
        line["global_block"] = glob_obj
    if drop_in is not None:
        line["drop_in_117m_layer"] = drop_in
    if train_obj is not None:
        line["train_117m"] = train_obj
    if train13_obj is not None:
        line["train_13m"] = train13_obj
    if one_m is not None:
        line["config0_1m"] = one_m
    if prefill_obj is not None:
        line["prefill_350m"] = prefill_obj
    if decode_obj is not None:
        line["decode_117m"] = decode_obj
    if n == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    # the headline figures once more, last on the line (a reader that keeps
    # only the tail of a long line still sees every workload's number)
    summ = {"op_gbs": line["value"], "op_frac": line["roofline"]["frac"],
            "op_ms": line["ms_per_step"]}
    if glob_obj is not None:
        summ.update(global_ms=glob_obj["ms_per_step"], global_frac_hbm=glob_obj["frac_hbm"],
                    global_frac_tensor=glob_obj["frac_tensor"])
    if drop_in is not None:
        summ.update(drop_in_ms=drop_in["ms_per_step"], drop_in_path=drop_in["kernel_path"])
    if train_obj is not None:
        summ.update(train_117m_tokens_per_s=train_obj["value"],
                    train_117m_ms=train_obj["ms_per_step"],
                    train_117m_aux_off_tokens_per_s=train_obj["aux_off"]["value"],
                    train_117m_mfu=train_obj["mfu"])
    if train13_obj is not None:
        summ.update(train_13m_tokens_per_s=train13_obj["value"], train_13m_ms=train13_obj["ms_per_step"])
    if prefill_obj is not None:
        summ.update(prefill_350m_tokens_per_s=prefill_obj["value"])
    if decode_obj is not None:
        summ.update(decode_117m_tokens_per_s=decode_obj["value"])
    line["summary"] = summ
    print(json.dumps(line))


if __name__ == "__main__":
    main()
