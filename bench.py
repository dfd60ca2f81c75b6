"""Benchmark of the hybrid AdamW + Newton-Schulz Muon optimizer step on B200.

python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]
               [--ns-mode reference|bf16|tf32|fp32]

Newton-Schulz modes: reference (the reference's bf16 rounding points, bf16 tensor
cores; default), bf16 (B rounded to bf16 too), tf32 (tf32 rounding points,
kind::tf32 tensor cores), fp32 (no rounding points, three-pass tf32 products).
The tf32 and fp32 modes report against the dense TF32 peak measured in the run
(divided by 3 for fp32).

Workloads (synthetic, seeded; shapes from the reference model family):
  hybrid_1b   (default) d_model 2048, 24 layers, FFN 8192, vocab 32000, untied lm_head;
              Muon on the block matrices, AdamW on embed / lm_head / LayerNorm; fp32.
  hybrid_8b   d_model 4096, 32 layers, GQA k/v [1024, 4096], FFN 14336, vocab 32000;
              bf16 grads with fp32 master params, loss scale 2^16, bf16 param copies.
  adamw_arena isolated fused AdamW over 2^28 fp32 params (t = 10, wd 0.1, divisor 4).
  ns_batch    isolated Newton-Schulz on 64 x [4096, 4096] + 32 x [4096, 14336].
  chatbot     the Chatbot(vocab 512, 2 layers, d_model 64) step (latency-bound).
  ns_probe, ns_probe_sq
              small profiling cases (8 x [2048, 8192], 32 x [2048, 2048]).

Rank 0 prints one JSON line. Multi-GPU runs use torchrun (one process per GPU):
Muon matrices are owned whole by one rank, the AdamW arena is split evenly, and
inside the timed region every rank's results reach every other rank: by default
the step itself pushes each finished chunk into the peers' arenas over NVLink
(--exchange fused), or NCCL all-gathers the arenas after the step (--exchange
nccl). The e2e number steps from pinned host buffers through mmn_optim_step_host.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# The benchmark's metric as the configurations name it; `value` is the params/s
# part (whole job), ms_per_step the step time, components the AdamW GB/s and NS
# TFLOP/s, and params_per_s_per_gpu the per-GPU rate.
METRIC = "hybrid AdamW+Muon step ms & params/s/GPU; AdamW HBM GB/s; NS TFLOPS"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM bytes (read + write) per algorithmic Newton-Schulz flop of the GEMM
# kernels of one reference-mode optimizer step (5 iterations, the last one fused
# with the parameter update), from the ncu capture of the 8 x [2048, 8192]
# profiling case (profiles/ns_gemm_probe_full.md): 5763.1 MB per 6.1848e12 flop.
# Traffic grows with the flops of a class, so the per-step traffic of a workload
# is this ratio times its Newton-Schulz flops.
NS_DRAM_BYTES_PER_FLOP = 5763.1e6 / 6.1848e12
# DRAM bytes per element of the isolated AdamW kernel measured by ncu on the
# 2^28 arena: read p, g, m, v and write p, m, v (profiles/adamw_arena.md).
ADAMW_DRAM_BYTES_PER_PARAM = 28.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return PEAKS_FALLBACK, "fallback"


def measure_tf32_peak(dev, sustained_s=3.0):
    """Dense TF32 tensor-core peak of this GPU, measured the way the bf16 peak
    is: cuBLAS fp32 GEMM with TF32 allowed, 8192^3 (2*N^3 flops), best of 10 on
    CUDA events (burst) and back to back for sustained_s seconds (sustained).
    Run before the timed region, only for the TF32 Newton-Schulz mode."""
    import torch

    n = 8192
    a = torch.randn(n, n, device=f"cuda:{dev}")
    b = torch.randn(n, n, device=f"cuda:{dev}")
    c = torch.empty(n, n, device=f"cuda:{dev}")
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        for _ in range(3):
            torch.mm(a, b, out=c)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.mm(a, b, out=c)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(1, int(sustained_s * 1e3 / best))
        e0.record()
        for _ in range(reps):
            torch.mm(a, b, out=c)
        e1.record()
        e1.synchronize()
        sus = e0.elapsed_time(e1) / reps
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b, c
    flops = 2.0 * n ** 3
    return flops / (best / 1e3) / 1e12, flops / (sus / 1e3) / 1e12


# ------------------------------------------------------------------ workloads
def hybrid_model(d, n_layer, ffn, vocab, kv_dim=None):
    """(name, shape, route) in optimizer call order (lm_head; blocks last..first:
    ffn2, ffn, out, q, k, v, ln2.gamma, ln2.beta, ln1.gamma, ln1.beta; embed),
    routed the tagged way: block matrices -> Muon, embed / lm_head / LN -> AdamW."""
    kv = kv_dim or d
    out = [("lm_head", (vocab, d), "adamw")]
    for layer in reversed(range(n_layer)):
        b = f"blocks.{layer}."
        out += [(b + "ffn2", (d, ffn), "muon"), (b + "ffn", (ffn, d), "muon"),
                (b + "out", (d, d), "muon"), (b + "q", (d, d), "muon"),
                (b + "k", (kv, d), "muon"), (b + "v", (kv, d), "muon"),
                (b + "ln2.gamma", (d,), "adamw"), (b + "ln2.beta", (d,), "adamw"),
                (b + "ln1.gamma", (d,), "adamw"), (b + "ln1.beta", (d,), "adamw")]
    out.append(("embed", (vocab, d), "adamw"))
    return out


WORKLOADS = {
    "hybrid_1b": dict(model=lambda: hybrid_model(2048, 24, 8192, 32000), grad="f32",
                      desc="hybrid step, d_model 2048, 24 layers, FFN 8192, vocab 32000"),
    "hybrid_8b": dict(model=lambda: hybrid_model(4096, 32, 14336, 32000, kv_dim=1024),
                      grad="bf16",
                      desc="hybrid step, d_model 4096, 32 layers, GQA kv 1024, FFN 14336, "
                           "vocab 32000, bf16 grads + fp32 master, loss scale 2^16"),
    "chatbot": dict(model=lambda: [(n, s, "auto") for n, s in
                                   __import__("magicmindnet_b200").chatbot_param_order(512, 2, 64)],
                    grad="f32", desc="Chatbot(vocab 512, n_layer 2, d_model 64) hybrid step"),
    "adamw_arena": dict(model=lambda: [("arena", (1 << 28,), "adamw")], grad="f32",
                        desc="fused AdamW over 2^28 fp32 params, t=10, wd 0.1, divisor 4"),
    "ns_batch": dict(model=lambda: [(f"sq{i}", (4096, 4096), "muon") for i in range(64)] +
                     [(f"ffn{i}", (4096, 14336), "muon") for i in range(32)], grad="f32",
                     desc="Newton-Schulz on 64 x [4096,4096] + 32 x [4096,14336]"),
    "ns_probe": dict(model=lambda: [(f"ffn{i}", (2048, 8192), "muon") for i in range(8)],
                     grad="f32", desc="Newton-Schulz on 8 x [2048,8192] (profiling case: "
                                      "X is 268 MB, larger than L2; about 1.5 GB on the device)"),
    "ns_probe_sq": dict(model=lambda: [(f"sq{i}", (2048, 2048), "muon") for i in range(32)],
                        grad="f32", desc="Newton-Schulz on 32 x [2048,2048] (profiling case: "
                                         "X is 268 MB, larger than L2; about 1.5 GB on the device)"),
}


def count_params(model):
    n = 0
    for _, s, _ in model:
        k = 1
        for d in s:
            k *= d
        n += k
    return n


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i - 5] for r in self.rows if len(r) > 8 for i in range(5, 9)
                          if r[i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


# ------------------------------------------------------------ CPU baseline
def cpu_baseline(workload: str, model, sample_s: float = 15.0):
    """The oracle (a C port of the reference's CPU step) timed on this host's
    cores on a bounded sample of the workload, extrapolated to one full step
    by the sample's share of the step's work. Returns a dict for the JSON line."""
    import numpy as np

    from oracle import reference_optim as R

    cores = R.lib().ref_max_threads()
    rng = np.random.default_rng(0)
    n_total = count_params(model)
    muon = [s for _, s, r in model if r == "muon" or (r == "auto" and R.classify_param(s) == R.MATRIX)]
    adamw_n = n_total - sum(s[0] * s[1] for s in muon)
    t_full = 0.0
    parts = []
    # AdamW: time a slice, scale by element count.
    if adamw_n:
        k = min(adamw_n, 1 << 24)
        p = rng.normal(0, 0.02, k).astype(np.float32)
        g = rng.normal(0, 1e-3, k).astype(np.float32)
        m = np.zeros(k, np.float32)
        v = np.zeros(k, np.float32)
        dt = min(R.lib().ref_adamw_step_timed(R._ptr(p), R._ptr(m), R._ptr(v), R._ptr(g), k, 3e-4,
                                               0.9, 0.95, 1e-8, 0.01, 10, 1.0, 0)
                 for _ in range(3))
        t_full += dt * adamw_n / k
        parts.append(f"AdamW {k} elems x{adamw_n / k:.1f}")
    # Newton-Schulz: one matrix per shape class, scaled down so the sample stays
    # bounded, extrapolated by flop count.
    classes = {}
    for s in muon:
        n, mm = min(s), max(s)
        classes[(n, mm)] = classes.get((n, mm), 0) + 1
    budget = sample_s / max(len(classes), 1)
    for (n, mm), cnt in classes.items():
        f_full = 5 * (4.0 * n * n * mm + 2.0 * n ** 3)
        sn, sm = n, mm
        while 5 * (4.0 * sn * sn * sm + 2.0 * sn ** 3) > 5e10 and sn > 64:
            sn //= 2
            sm //= 2
        g = rng.normal(0, 1e-2, (sn, sm)).astype(np.float32)
        t0 = time.perf_counter()
        R.newton_schulz5(g, 5, order=R.GEMM_F32_FMA)
        dt = time.perf_counter() - t0
        f_s = 5 * (4.0 * sn * sn * sm + 2.0 * sn ** 3)
        t_full += dt * (f_full / f_s) * cnt
        parts.append(f"NS [{sn},{sm}] for {cnt} x [{n},{mm}] (flop-scaled)")
        if dt > budget:
            break
    return {"value": n_total / t_full if t_full else None, "unit": "params/s", "cores": cores,
            "kind": "port", "sample": "; ".join(parts), "step_s_extrapolated": t_full}


# --------------------------------------------------------------------- ours
def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch

    import magicmindnet_b200 as mmn

    torch.cuda.set_device(local_rank)
    dev = local_rank
    spec = WORKLOADS[args.workload]
    model = spec["model"]()
    n_total = count_params(model)
    is_8b = args.workload == "hybrid_8b"
    if args.workload == "adamw_arena":
        adamw = mmn.AdamWConfig(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    elif args.workload == "chatbot":
        adamw = mmn.AdamWConfig(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    else:
        adamw = mmn.AdamWConfig()
    dp = world > 1 and args.grad_reduce != "none"
    # loss-scaled sharded steps: each rank scans only what it steps and tells
    # the others (mmn_optim_scan_grads), unless --scan full
    shard_scan = (is_8b and world > 1 and not dp and args.scan == "shard"
                  and args.exchange == "fused")
    cfg = mmn.StepConfig(adamw=adamw, muon=mmn.MuonConfig(), ns_mode=args.ns_mode,
                         grad_dtype=spec["grad"], bf16_param_shadow=is_8b, loss_scaling=is_8b,
                         rank=rank, world_size=world, use_graph=True,
                         reduce_grads=dp and args.grad_reduce == "fused", scan_shard=shard_scan)
    stream = torch.cuda.current_stream(dev)
    step = mmn.OptimizerStep([(k, s, r) for k, (_, s, r) in enumerate(model)], cfg, device=dev,
                             stream=stream.cuda_stream)
    # seeded synthetic values, generated on the device
    gen = torch.Generator(device=f"cuda:{dev}").manual_seed(0)
    for k, (_, s, _) in enumerate(model):
        step.param(k).normal_(0, 0.02, generator=gen)
        gv = step.grad(k)
        if gv.dtype == torch.bfloat16:
            gv.copy_((torch.randn(s, device=f"cuda:{dev}", generator=gen) * (1e-3 * 65536.0)))
        else:
            gv.normal_(0, 1e-2 if args.workload in ("adamw_arena", "ns_batch") else 1e-3,
                       generator=gen)
    if is_8b:
        for k in range(len(model)):
            b = step.param_bf16(k)
            b.copy_(step.param(k))
    if args.workload == "adamw_arena":
        step.set_state(0, "m", np.random.default_rng(0).normal(0, 1e-3, 1 << 28).astype(np.float32))
        step.set_state(0, "v", np.abs(np.random.default_rng(1).normal(0, 1e-4, 1 << 28)).astype(np.float32))
        step.adamw_step = 9  # the timed steps run at t = 10, 11, ...
    divisor = 4.0 if args.workload == "adamw_arena" else 1.0
    torch.cuda.synchronize()

    gl = step.gather_layout()
    gathers = []
    reduces = []
    fused = world > 1 and (args.exchange == "fused" or args.grad_reduce == "fused")
    if fused:
        # the step's own kernels store this rank's parameters into every peer
        step.connect_peers()
    elif world > 1:
        import torch.distributed as dist
        from magicmindnet_b200.step import _view

        use16 = is_8b
        for key, region in (("adamw_param", "adamw_region"), ("muon_param", "muon_region")):
            ptr = gl[key + ("_bf16" if use16 else "")]
            if ptr and gl[region]:
                full = _view(ptr, (gl[region] * world,), "bf16" if use16 else "f32", dev)
                gathers.append((full, full[rank * gl[region]:(rank + 1) * gl[region]]))
    if dp and args.grad_reduce == "nccl":
        # NCCL baseline of the grad reduction: an in-place reduce-scatter of each
        # grad arena into this rank's region (the arenas are rank-major)
        from magicmindnet_b200.step import _view

        plan = mmn.shard_plan([(k, s, r) for k, (_, s, r) in enumerate(model)], world)
        gdt, gsz = ("bf16", 2) if spec["grad"] == "bf16" else ("f32", 4)
        for route, region in (("adamw", "adamw_region"), ("muon", "muon_region")):
            ks = [k for k, (_, _, r) in enumerate(model) if r == route]
            if ks and gl[region]:
                base = step.grad(ks[0]).data_ptr() - plan["offset"][ks[0]] * gsz
                full = _view(base, (gl[region] * world,), gdt, dev)
                reduces.append((full, full[rank * gl[region]:(rank + 1) * gl[region]]))

    def one_step():
        if shard_scan:
            step.scan_grads()
        if dp and args.grad_reduce == "fused":
            step.reduce_grads()
        elif reduces:
            import torch.distributed as dist

            for full, mine in reduces:
                dist.reduce_scatter_tensor(mine, full)
        step.step(divisor)
        if fused:
            step.exchange_fence()
        if gathers:
            import torch.distributed as dist

            for full, mine in gathers:
                dist.all_gather_into_tensor(full, mine)

    # TF32 roofline denominator, measured before the warm-up so that the timed
    # region is untouched
    tf32_peak = measure_tf32_peak(dev) if args.ns_mode in ("tf32", "fp32") else None
    inj = []
    for i in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(dev)).split(",")[0])
                          if os.environ.get("CUDA_VISIBLE_DEVICES", "").isdigit() else dev)
    # the timed steps record per-phase CUDA events (launched without the graph;
    # the warm-up steps captured and replayed it, at the same speed)
    step.enable_timing(True)
    clocks.start()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.steps):
        if is_8b and i % 100 == 50:
            inj.append(i)  # one injected inf grad per 100 steps
            step.grad(0).view(-1)[0] = float("inf")
        one_step()
        if is_8b and i % 100 == 50:
            step.grad(0).view(-1)[0] = 1e-3 * 65536.0
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    # per-phase device times averaged over the timed steps (CUDA events the
    # library records on the streams its kernels run on)
    phase = {k2: [v] for k2, v in step.last_timing().items()}
    step.enable_timing(False)
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        import torch.distributed as dist

        tt = torch.tensor([ms], device=f"cuda:{dev}")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    value = n_total / (ms / 1e3)

    # --- e2e: host grads in, host params out through the public API
    # (mmn_optim_step_host: the copies are pipelined with the compute per chunk).
    # Each rank copies in the grads it steps and copies back the params it
    # stepped; with the peer exchange the device arenas are complete as well.
    e2e = None
    if args.e2e and not dp:
        plan = mmn.shard_plan([(k, s, r) for k, (_, s, r) in enumerate(model)], world)
        areg = plan["adamw_region"]
        stepped = []  # elements of every slot this rank steps
        for k, (_, s, r) in enumerate(model):
            n = int(np.prod(s))
            if plan["owner"][k] >= 0:
                stepped.append(n if plan["owner"][k] == rank else 0)
            else:
                off = plan["offset"][k]
                stepped.append(max(0, min(off + n, (rank + 1) * areg) - max(off, rank * areg)))
        gsz = 2 if spec["grad"] == "bf16" else 4
        full_in = is_8b and world > 1 and not shard_scan  # the scan reads every grad
        pin_g = [step.grad(k).cpu().pin_memory() if stepped[k] or full_in else None
                 for k in range(len(model))]
        pin_p = [torch.empty(s, dtype=torch.float32).pin_memory() if stepped[k] else None
                 for k, (_, s, _) in enumerate(model)]
        no_g = [None] * len(model)
        bi = sum((int(np.prod(s)) if full_in else stepped[k]) * gsz
                 for k, (_, s, _) in enumerate(model))
        bo = sum(stepped) * 4

        def host_step():
            if shard_scan:
                # this rank's grads in and scanned, every rank's verdict in, then the step
                step.scan_grads(pin_g)
                step.step_host(no_g, pin_p, divisor)
            else:
                step.step_host(pin_g, pin_p, divisor)
            if fused:
                step.exchange_fence()
            if gathers:
                import torch.distributed as dist

                for full, mine in gathers:
                    dist.all_gather_into_tensor(full, mine)
                torch.cuda.current_stream(dev).synchronize()

        for _ in range(2):
            host_step()
        e_steps = max(1, min(args.steps, 10))
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(e_steps):
            host_step()
        e_ms = (time.perf_counter() - t0) * 1e3 / e_steps
        if world > 1:
            import torch.distributed as dist

            tt = torch.tensor([e_ms, bi, bo], dtype=torch.float64, device=f"cuda:{dev}")
            mx = tt.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            dist.all_reduce(tt, op=dist.ReduceOp.SUM)
            e_ms, bi, bo = float(mx[0]), int(tt[1]), int(tt[2])
        e2e = {"value": n_total / (e_ms / 1e3), "unit": "params/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
               "api": "mmn_optim_step_host (pinned host buffers, synchronous)",
               "timing": "host wall clock per step, max over ranks"}

    pk, pk_kind = peaks()
    med = {k: (statistics.median(v) if v else 0.0) for k, v in phase.items()}
    ns_flops = step.ns_flops()
    total, n_adamw, n_muon = step.param_counts()
    # AdamW algorithmic bytes: read p, g, m, v and write p, m, v (28 B/param at fp32);
    # bf16 grads read 2 B instead of 4, and the bf16 copy adds 2 B written.
    a_bytes_per = (28 if spec["grad"] == "f32" else 26) + (2 if is_8b else 0)
    a_elems_rank = n_adamw / world
    comp = {
        "adamw": {"ms": med["adamw"], "bytes_per_param": a_bytes_per,
                  "GB/s": (a_bytes_per * a_elems_rank / (med["adamw"] / 1e3) / 1e9)
                  if med["adamw"] else None},
        "newton_schulz": {"ms": med["newton_schulz"], "flops": ns_flops,
                          "TFLOP/s": (ns_flops / (med["newton_schulz"] / 1e3) / 1e12)
                          if med["newton_schulz"] else None},
        "muon_momentum_ms": med["muon_momentum"], "muon_update_ms": med["muon_update"],
        "step_ms_events": med["step"],
        "note": "phase times are averaged over the timed steps. AdamW runs on a side stream "
                "concurrently with the Newton-Schulz GEMMs, so in hybrid workloads its event "
                "time includes waiting for SMs; its kernel rate is the adamw_arena workload's",
    }
    if n_muon and med["newton_schulz"] > 0:
        ach = ns_flops / (med["newton_schulz"] / 1e3) / 1e12
        sustained = args.workload.startswith("hybrid")
        if args.ns_mode in ("tf32", "fp32"):
            # the dense TF32 rate is half the bf16 one and not in the peaks file:
            # measured in this run, before the timed region. The fp32 mode forms
            # every product from three tf32 MMAs, so its ceiling is a third.
            split = 3.0 if args.ns_mode == "fp32" else 1.0
            peak = (tf32_peak[1] if sustained else tf32_peak[0]) / split
            peak_src = ("measured in this run: cuBLAS tf32 8192^3, "
                        + ("sustained" if sustained else "best of 10")
                        + (", / 3 (three tf32 MMAs per fp32 product)" if split > 1 else ""))
        else:
            peak = pk["bf16_tflops_sustained"] if sustained else pk["bf16_tflops"]
            peak_src = pk_kind
        roof = {"bound": "tensor", "kernel": "ns_gemm (tcgen05, Gram + Square + Poly per iteration)",
                "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                "peak_source": peak_src,
                "traffic": ns_flops * NS_DRAM_BYTES_PER_FLOP if args.ns_mode == "reference" else None,
                "traffic_unit": "DRAM bytes per step of the NS kernels (ncu ratio of the "
                                "8 x [2048,8192] capture, scaled by flops)",
                "flops_per_step": ns_flops}
    else:
        ach = a_bytes_per * a_elems_rank / (med["adamw"] / 1e3) / 1e9
        roof = {"bound": "hbm", "kernel": "adamw_kernel", "achieved": ach, "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": ach / pk["hbm_gbs"], "peak_source": pk_kind,
                "traffic": ADAMW_DRAM_BYTES_PER_PARAM * a_elems_rank,
                "traffic_unit": "DRAM bytes per launch (ncu: 28 B per param on the 2^28 arena)",
                "algorithmic_bytes": a_bytes_per * a_elems_rank}
    per_step, per_reduce = step.kernel_launches()
    launches_per_step = per_step + (per_reduce if (dp and args.grad_reduce == "fused") or shard_scan
                                    else 0)
    line = {
        "metric": METRIC, "value": value, "unit": "params/s", "n_gpus": world,
        "params_per_s_per_gpu": value / world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": ("f32 (NS GEMMs " + {"tf32": "tf32 x tf32", "fp32": "3 x tf32 split fp32"}.get(
                      args.ns_mode, "bf16 x bf16") + " -> f32)")
                 if not is_8b else "bf16 grads/params, f32 master",
        "data": "synthetic (seeded normal params/grads)",
        "config": {"workload": args.workload, "desc": spec["desc"], "params": n_total,
                   "adamw_params": n_adamw, "muon_params": n_muon, "ns_mode": args.ns_mode,
                   "parallelism": f"shard{world}" if world > 1 else "single",
                   "exchange": ("copy-engine pushes over NVLink per chunk + 1-element all-reduce fence"
                                if fused else
                                "NCCL all-gather of the parameter arenas") if world > 1 else None,
                   "grad_reduce": ({"fused": "mmn_optim_reduce_grads: rank-ordered sum over "
                                             "NVLink fused with the non-finite scan",
                                    "nccl": "NCCL reduce-scatter of the grad arenas"}
                                   [args.grad_reduce] if dp else
                                   "none (grads already reduced, as the configurations assume)"),
                   "nonfinite_scan": (("sharded: each rank scans what it steps and sets every "
                                       "rank's flag (mmn_optim_scan_grads)") if shard_scan else
                                      "every rank scans every grad") if is_8b else None,
                   "l2": "inputs larger than L2 (no flush needed)"},
        "roofline": roof, "components": comp, "clocks": clk, "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
    }
    if is_8b:
        line["loss_scale"] = dict(zip(("scale", "skipped_steps"), step.loss_scale()))
        line["injected_inf_steps"] = inj
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload, model)
    step.close()
    return line


def run_reference(args, rank, world):
    if rank != 0:
        return None
    spec = WORKLOADS[args.workload]
    model = spec["model"]()
    vals = []
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(args.workload, model, sample_s=2.0)
        if i >= args.warmup:
            vals.append(cb)
    v = statistics.median(c["value"] for c in vals)
    ms = statistics.median(c["step_s_extrapolated"] for c in vals) * 1e3
    cb = dict(vals[-1])
    cb["value"] = v
    return {"metric": METRIC, "value": v, "unit": "params/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic (seeded normal params/grads)",
            "config": {"workload": args.workload, "desc": spec["desc"],
                       "params": count_params(model)},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "params/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="hybrid_1b", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ns-mode", default="reference", choices=["reference", "bf16", "tf32", "fp32"])
    ap.add_argument("--no-e2e", dest="e2e", action="store_false")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="fused", choices=["fused", "nccl"],
                    help="multi-GPU parameter exchange: copy-engine pushes over NVLink inside "
                         "the step (CUDA IPC) or an NCCL all-gather after the step")
    ap.add_argument("--scan", default="shard", choices=["shard", "full"],
                    help="multi-GPU loss-scaled steps: each rank scans only the grads it "
                         "steps and sets every rank's skip flag (shard), or every rank scans "
                         "every grad (full)")
    ap.add_argument("--grad-reduce", default="none", choices=["none", "fused", "nccl"],
                    help="multi-GPU: also time the data-parallel grad reduction before each "
                         "step (fused: mmn_optim_reduce_grads over NVLink; nccl: "
                         "reduce-scatter). Default: grads are already reduced, as the "
                         "benchmark configurations assume")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local_rank}"))
    line = run_ours(args, rank, world, local_rank)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
