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
# with the parameter update): 5763.1 MB of dram__bytes_read.sum +
# dram__bytes_write.sum per 6.1848e12 flop, summed over the Gram, Square and
# Poly launches of one step of the 8 x [2048, 8192] case
# (ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none
#  -k regex:ns_gemm python bench.py --workload ns_probe --steps 1 --warmup 3
#  --no-e2e --no-cpu-baseline). Traffic grows with the flops of a class, so the
# per-step traffic of a workload is this ratio times its Newton-Schulz flops.
NS_DRAM_BYTES_PER_FLOP = 5763.1e6 / 6.1848e12
# DRAM bytes per element of the isolated AdamW kernel: read p, g, m, v and write
# p, m, v, as ncu's dram__bytes_read.sum + dram__bytes_write.sum of one
# adamw_kernel launch on the 2^28 arena gives (7.52 GB per launch).
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
def _ns_flops(n, m, steps=5):
    return steps * (4.0 * n * n * m + 2.0 * n ** 3)


class RefSampler:
    """The oracle (a C port of the reference's CPU step) timed on this host's
    cores on a bounded sample of one optimizer step of `model`, extrapolated to
    the whole step.

    A sample is AdamW over a slice of at most 2^24 elements (scaled by element
    count) and, for every Newton-Schulz shape class, one matrix shrunk until its
    flops are at most `sample_flops` (the reference runs every matrix of the
    class through the same code). Calibration times one full-size matrix of
    every class whose flops are at most `full_cap` once, so that the sample of
    that class is scaled by the measured full/sample time ratio; larger classes
    are scaled by their flop ratio. threads = 0 uses every host thread."""

    def __init__(self, model, threads=0, sample_flops=5e10, full_cap=1.2e12, calibrate=True):
        import numpy as np

        from oracle import reference_optim as R

        self.R, self.np = R, np
        self.threads = threads
        self.cores = R.lib().ref_max_threads() if threads <= 0 else threads
        self.rng = np.random.default_rng(0)
        self.n_total = count_params(model)
        muon = [s for _, s, r in model
                if r == "muon" or (r == "auto" and R.classify_param(s) == R.MATRIX)]
        self.adamw_n = self.n_total - sum(s[0] * s[1] for s in muon)
        self.k = min(self.adamw_n, 1 << 24)
        self.classes = {}
        for s in muon:
            key = (min(s), max(s))
            self.classes[key] = self.classes.get(key, 0) + 1
        self.sample = {}
        for (n, m) in self.classes:
            sn, sm = n, m
            while _ns_flops(sn, sm) > sample_flops and sn > 64:
                sn //= 2
                sm //= 2
            self.sample[(n, m)] = (sn, sm)
        self.ratio = {c: _ns_flops(*c) / _ns_flops(*self.sample[c]) for c in self.classes}
        self.calibration = {}
        if calibrate:
            for c in self.classes:
                if _ns_flops(*c) > full_cap or self.sample[c] == c:
                    continue
                t_full = self._time_ns(c)
                t_samp = min(self._time_ns(self.sample[c]) for _ in range(2))
                self.ratio[c] = t_full / t_samp
                self.calibration[f"{c[0]}x{c[1]}"] = {
                    "full_s": round(t_full, 3), "sample_s": round(t_samp, 3),
                    "flop_ratio": round(_ns_flops(*c) / _ns_flops(*self.sample[c]), 2),
                    "time_ratio": round(self.ratio[c], 2)}

    def _time_ns(self, shape):
        g = self.rng.normal(0, 1e-2, shape).astype(self.np.float32)
        t0 = time.perf_counter()
        self.R.newton_schulz5(g, 5, order=self.R.GEMM_F32_FMA, threads=self.threads)
        return time.perf_counter() - t0

    def step(self):
        """One sampled step: (extrapolated seconds of the whole step, seconds
        the sample took)."""
        np, R = self.np, self.R
        w0 = time.perf_counter()
        t_full = 0.0
        if self.adamw_n:
            k = self.k
            p = self.rng.normal(0, 0.02, k).astype(np.float32)
            g = self.rng.normal(0, 1e-3, k).astype(np.float32)
            m = np.zeros(k, np.float32)
            v = np.zeros(k, np.float32)
            dt = R.lib().ref_adamw_step_timed(R._ptr(p), R._ptr(m), R._ptr(v), R._ptr(g), k,
                                              3e-4, 0.9, 0.95, 1e-8, 0.01, 10, 1.0, self.threads)
            t_full += dt * self.adamw_n / k
        for c, cnt in self.classes.items():
            t_full += self._time_ns(self.sample[c]) * self.ratio[c] * cnt
        return t_full, time.perf_counter() - w0

    def describe(self):
        parts = []
        if self.adamw_n:
            parts.append(f"AdamW {self.k} of {self.adamw_n} elems")
        for c, cnt in self.classes.items():
            how = "time-scaled from a full-size run" if f"{c[0]}x{c[1]}" in self.calibration \
                else "flop-scaled"
            parts.append(f"NS [{self.sample[c][0]},{self.sample[c][1]}] for {cnt} x "
                         f"[{c[0]},{c[1]}] ({how})")
        return "; ".join(parts)

    def sampled_fraction(self):
        """Share of the step's work one sample runs (elements for AdamW, flops
        for Newton-Schulz, each weighted by its extrapolated time share)."""
        tot = sum(_ns_flops(*c) * cnt for c, cnt in self.classes.items())
        smp = sum(_ns_flops(*self.sample[c]) for c in self.classes)
        return {"adamw_elems": self.k / self.adamw_n if self.adamw_n else None,
                "ns_flops": smp / tot if tot else None}


def cpu_baseline(workload: str, model):
    """The oracle on this host's cores for the JSON line's cpu_baseline: every
    thread (calibrated on full-size matrices where that is bounded) and one
    thread (the reference is single-threaded), each one sampled step,
    extrapolated to the whole step and labelled as such."""
    allt = RefSampler(model)
    t_all, w_all = allt.step()
    one = RefSampler(model, threads=1, sample_flops=1e10, calibrate=False)
    t_one, w_one = one.step()
    return {"value": allt.n_total / t_all, "unit": "params/s", "cores": allt.cores,
            "kind": "port", "extrapolated": True, "sample": allt.describe(),
            "sample_s": round(w_all, 3), "step_s_extrapolated": t_all,
            "sampled_fraction": allt.sampled_fraction(), "calibration": allt.calibration,
            "single_thread": {"value": one.n_total / t_one, "unit": "params/s", "cores": 1,
                              "extrapolated": True, "sample": one.describe(),
                              "sample_s": round(w_one, 3), "step_s_extrapolated": t_one}}


# --------------------------------------------------------------------- ours
def fill_workload(step, workload, model, dev):
    """Seeded synthetic values of a workload, generated on the device in slot
    order (the same values on every GPU and every rank):
    params ~ N(0, 0.02); grads ~ N(0, 1e-3) (N(0, 1e-2) for the isolated AdamW
    and Newton-Schulz workloads; bf16 grads carry the 2^16 loss scale);
    the isolated AdamW arena also gets m ~ N(0, 1e-3), v ~ |N(0, 1e-4)| and the
    step count 9 (its first timed step runs at t = 10), the isolated
    Newton-Schulz batch a velocity ~ N(0, 1e-3)."""
    import torch

    gen = torch.Generator(device=f"cuda:{dev}").manual_seed(0)
    for k, (_, s, _) in enumerate(model):
        step.param(k).normal_(0, 0.02, generator=gen)
        gv = step.grad(k)
        if gv.dtype == torch.bfloat16:
            gv.copy_((torch.randn(s, device=f"cuda:{dev}", generator=gen) * (1e-3 * 65536.0)))
        else:
            gv.normal_(0, 1e-2 if workload in ("adamw_arena", "ns_batch") else 1e-3,
                       generator=gen)
    if step.config.bf16_param_shadow:
        for k in range(len(model)):
            step.param_bf16(k).copy_(step.param(k))
    if workload == "adamw_arena":
        n = model[0][1][0]
        m = torch.empty(n, device=f"cuda:{dev}").normal_(0, 1e-3, generator=gen)
        step.set_state(0, "m", m)
        m.normal_(0, 1e-4, generator=gen).abs_()
        step.set_state(0, "v", m)
        del m
        step.adamw_step = 9  # the timed steps run at t = 10, 11, ...
    if workload == "ns_batch":
        for k, (_, s, _) in enumerate(model):
            vel = torch.empty(s, device=f"cuda:{dev}").normal_(0, 1e-3, generator=gen)
            step.set_state(k, "velocity", vel)
        del vel
    torch.cuda.synchronize(dev)


def isolated_kernels(dev, pk, pk_kind, ns_modes=("reference", "tf32", "fp32")):
    """The configurations' isolated kernel workloads, timed with CUDA events in
    the same run after the main workload has freed its memory: the fused AdamW
    over the 2^28-element arena (t = 10, wd 0.1, divisor 4; 28 B per param) and
    Newton-Schulz on 64 x [4096, 4096] + 32 x [4096, 14336] (velocity ~ N(0,
    1e-3), 5 iterations) in the reference recipe, the TF32 mode and the fp32 mode
    (the one within 1e-4 of exact Newton-Schulz). 3 warm-up and 3 timed steps
    each; inputs larger than L2. Fractions are of the measured peaks (HBM copy
    bandwidth; cuBLAS bf16 burst; the dense TF32 peak measured here, before the
    timed steps, and a third of it for the fp32 mode's three tf32 products)."""
    import torch

    import magicmindnet_b200 as mmn

    out = {}
    stream = torch.cuda.current_stream(dev)

    def timed(workload, cfg, divisor, warmup=3, steps=3):
        model = WORKLOADS[workload]["model"]()
        step = mmn.OptimizerStep([(k, s, r) for k, (_, s, r) in enumerate(model)], cfg,
                                 device=dev, stream=stream.cuda_stream)
        fill_workload(step, workload, model, dev)
        for _ in range(warmup):
            step.step(divisor)
        if workload == "adamw_arena":
            step.adamw_step = 9  # the timed steps run at t = 10, 11, 12
        torch.cuda.synchronize(dev)
        step.enable_timing(True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step.step(divisor)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ph = step.last_timing()
        flops = step.ns_flops()
        step.close()
        torch.cuda.empty_cache()
        return e0.elapsed_time(e1) / steps, ph, flops

    adamw = mmn.AdamWConfig(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    ms, ph, _ = timed("adamw_arena", mmn.StepConfig(adamw=adamw, use_graph=False), 4.0)
    byts = ADAMW_DRAM_BYTES_PER_PARAM * (1 << 28)
    out["adamw_arena"] = {"kernel_ms": ph["adamw"], "step_ms": ms,
                          "GB/s": byts / (ph["adamw"] / 1e3) / 1e9,
                          "frac": byts / (ph["adamw"] / 1e3) / 1e9 / pk["hbm_gbs"],
                          "peak": pk["hbm_gbs"], "peak_source": pk_kind,
                          "bytes_per_launch": byts}
    tf32 = None
    for mode in ns_modes:
        if mode in ("tf32", "fp32"):
            tf32 = tf32 or measure_tf32_peak(dev)
            peak, src = tf32[0] / (3.0 if mode == "fp32" else 1.0), "measured in this run: " \
                "cuBLAS tf32 8192^3, best of 10"
        else:
            peak, src = pk["bf16_tflops"], pk_kind
        ms, ph, flops = timed("ns_batch", mmn.StepConfig(ns_mode=mode, use_graph=True), 1.0)
        tf = flops / (ph["newton_schulz"] / 1e3) / 1e12
        out[f"ns_batch_{mode}"] = {"ns_ms": ph["newton_schulz"], "step_ms": ms,
                                   "momentum_ms": ph["muon_momentum"],
                                   "norm_ms": ph["muon_norm"], "flops": flops,
                                   "TFLOP/s": tf, "peak": peak, "frac": tf / peak,
                                   "peak_source": src}
    return out


def _param_checksums(step, n_slots):
    """Per-slot exact checksums of the parameters every rank holds after the
    exchange (fp32, or the bf16 copies when the fp32 master stays with its
    owner): the integer sum of the bit patterns and a position-weighted one."""
    import torch

    rows = []
    for k in range(n_slots):
        t = step.param_bf16(k) if step.config.bf16_param_shadow else step.param(k)
        bits = t.view(torch.int16 if t.dtype == torch.bfloat16 else torch.int32).reshape(-1)
        b = bits.to(torch.int64)
        w = torch.arange(b.numel(), device=b.device, dtype=torch.int64) % 4093 + 1
        rows.append(torch.stack([b.sum(), (b * w).sum()]))
        del b, w
    return torch.stack(rows)


def parity_vs_single(step, model, cfg, workload, n_steps, inj, divisor, rank, world, dev):
    """After a sharded run: every rank's parameters against one GPU stepping the
    same seeded workload unsharded, bit for bit. Each rank checksums every
    slot; the handles are closed; rank 0 replays the n_steps steps (with the
    same injected non-finite grads) on its own GPU and compares. Returns the
    verdict every rank agrees on."""
    import torch
    import torch.distributed as dist

    import magicmindnet_b200 as mmn

    cs = _param_checksums(step, len(model))
    mx, mn = cs.clone(), cs.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    dist.all_reduce(mn, op=dist.ReduceOp.MIN)
    step.close()
    torch.cuda.synchronize(dev)
    dist.barrier()
    ok = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
    if rank == 0:
        one_cfg = mmn.StepConfig(**{**cfg.__dict__, "rank": 0, "world_size": 1,
                                    "reduce_grads": False, "scan_shard": False})
        single = mmn.OptimizerStep([(k, s, r) for k, (_, s, r) in enumerate(model)], one_cfg,
                                   device=dev, stream=torch.cuda.current_stream(dev).cuda_stream)
        fill_workload(single, workload, model, dev)
        g0 = single.grad(0).view(-1)
        for i in range(n_steps):  # the grad edits and the steps share one stream
            if i in inj:
                g0[0] = float("inf")
            single.step(divisor)
            if i in inj:
                g0[0] = 1e-3 * 65536.0
        single.sync()
        ref = _param_checksums(single, len(model))
        single.close()
        ok[0] = int(torch.equal(mx, mn) and torch.equal(mx, ref))
    dist.broadcast(ok, 0)
    return bool(ok.item())


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
    fill_workload(step, args.workload, model, dev)
    divisor = 4.0 if args.workload == "adamw_arena" else 1.0
    torch.cuda.synchronize()
    n_done = 0  # steps taken so far (the multi-GPU parity replay repeats them)

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
    inj_global = []
    for i in range(args.warmup):
        one_step()
        n_done += 1
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
            inj_global.append(n_done)
            step.grad(0).view(-1)[0] = float("inf")
        one_step()
        n_done += 1
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
            n_done += 1
        e_steps = max(1, min(args.steps, 10))
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(e_steps):
            host_step()
        e_ms = (time.perf_counter() - t0) * 1e3 / e_steps
        n_done += e_steps
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
        if world == 1:
            # The PCIe floor on this box: the same per-slot copies (grads in on
            # one stream, params out on another, pinned buffers), no compute.
            # The grads copied in are the values already there; params are only read.
            h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

            def copies():
                for k in range(len(model)):
                    if pin_g[k] is not None:
                        with torch.cuda.stream(h2d):
                            step.grad(k).copy_(pin_g[k], non_blocking=True)
                    if pin_p[k] is not None:
                        with torch.cuda.stream(d2h):
                            pin_p[k].copy_(step.param(k), non_blocking=True)
                h2d.synchronize()
                d2h.synchronize()

            torch.cuda.synchronize(dev)
            copies()
            t0 = time.perf_counter()
            for _ in range(3):
                copies()
            floor = (time.perf_counter() - t0) * 1e3 / 3
            e2e["copy_floor_ms"] = floor
            e2e["vs_copy_floor"] = e_ms / floor
            e2e["copy_floor"] = ("the same host<->device copies alone, both directions at once "
                                 "on two streams, host wall clock, mean of 3")

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
        "muon_momentum_ms": med["muon_momentum"],
        "muon_norm": {"ms": med["muon_norm"], "elems": n_muon / world,
                      "note": "the sequential fp32 sums of squares of the Newton-Schulz inputs "
                              "(bf16, 2 B read per element), one launch for every matrix"},
        "muon_update_ms": med["muon_update"],
        "step_ms_events": med["step"],
        "exchange_exposed_ms": (ms - med["step"]) if world > 1 else None,
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
    if world > 1 and not dp:
        # the sharded result against one GPU stepping the same workload, bit for bit
        line["parity_vs_1gpu"] = parity_vs_single(step, model, cfg, args.workload, n_done,
                                                  set(inj_global), divisor, rank, world, dev)
        line["parity_steps"] = n_done
    else:
        if world > 1:
            line["parity_vs_1gpu"] = None  # local grads differ per rank under --grad-reduce
        step.close()
    if world == 1 and args.kernels and args.workload.startswith("hybrid"):
        torch.cuda.empty_cache()
        comp["isolated"] = isolated_kernels(dev, pk, pk_kind)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload, model)
    return line


def run_reference(args, rank, world):
    """The reference arm: the oracle port of the reference's CPU step on this
    host's cores (no Rust toolchain exists to build the reference itself). Each
    of the warm-up and timed steps is one bounded sample of the workload's step
    (RefSampler), extrapolated to the whole step; ms_per_step is that
    extrapolated step time and sample_ms_per_step what the samples took."""
    if rank != 0:
        return None
    spec = WORKLOADS[args.workload]
    model = spec["model"]()
    smp = RefSampler(model)
    full, wall = [], []
    for i in range(args.warmup + args.steps):
        t, w = smp.step()
        if i >= args.warmup:
            full.append(t)
            wall.append(w)
    t_med = statistics.median(full)
    v = smp.n_total / t_med
    one = RefSampler(model, threads=1, sample_flops=1e10, calibrate=False)
    t_one, w_one = one.step()
    cb = {"value": v, "unit": "params/s", "cores": smp.cores, "kind": "port",
          "extrapolated": True, "sample": smp.describe(),
          "sampled_fraction": smp.sampled_fraction(), "calibration": smp.calibration,
          "single_thread": {"value": one.n_total / t_one, "unit": "params/s", "cores": 1,
                            "extrapolated": True, "sample": one.describe(),
                            "sample_s": round(w_one, 3), "step_s_extrapolated": t_one}}
    return {"metric": METRIC, "value": v, "unit": "params/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_med * 1e3,
            "sample_ms_per_step": statistics.median(wall) * 1e3, "extrapolated": True,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "impl": "reference", "data": "synthetic (seeded normal params/grads)",
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
    ap.add_argument("--no-kernels", dest="kernels", action="store_false",
                    help="skip the isolated AdamW-arena and Newton-Schulz-batch timings that "
                         "a one-GPU hybrid run adds to its components")
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
    if line.get("parity_vs_1gpu") is False:
        print("sharded parameters differ from the one-GPU step", file=sys.stderr, flush=True)
        sys.exit(3)


if __name__ == "__main__":
    main()
