"""CPU oracle for the MagicMindNet optimizer step — TEST INFRASTRUCTURE ONLY.

Python mirror of the Rust optimizer structs in crates/mmn-optim/src/lib.rs on top
of the C restatement in mmn_optim_ref.c. Only tests/, the smoke check and the
CPU-baseline leg of bench.py import this module; the product path never does.

State handling follows the reference exactly:
  * AdamW keeps ONE step counter per instance, advanced on every step_param
    call (lib.rs:41-43), so every tensor stepped in one model step sees a
    different bias-correction t.
  * m, v and Muon velocity are created lazily as zeros per caller id
    (lib.rs:45-46, 150-153) and never freed.
  * Routing is by shape only (lib.rs:196-202).

Parity status: partially pinned (see mmn_optim_ref.h). The reference cannot be
run here (Rust, no toolchain); its own tests pin only the accumulator average and
the routing table.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libmmn_optim_ref.so")

GEMM_F32_SEQ, GEMM_F32_FMA, GEMM_F64 = 0, 1, 2
# Newton-Schulz products formed by numpy's float64 matrix multiply (a BLAS
# dgemm): the GEMM_F64 recipe (fp64 sums rounded once to fp32) with another
# fp64 summation order, fast enough for the full-size matrices (4096 x 14336)
# on the host cores. Only newton_schulz5 / ns_iteration accept it.
GEMM_BLAS64 = 3
NS_REFERENCE, NS_BF16, NS_TF32, NS_FP32 = 0, 1, 2, 3

_f = ctypes.c_float
_i64 = ctypes.c_int64
_fp = ctypes.POINTER(ctypes.c_float)


def build() -> str:
    """Compile the oracle with its Makefile (gcc) and return the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.ref_bf16_round.restype = _f
        L.ref_bf16_round.argtypes = [_f]
        L.ref_tf32_round.restype = _f
        L.ref_tf32_round.argtypes = [_f]
        L.ref_adamw_step.argtypes = [_fp, _fp, _fp, _fp, _i64, _f, _f, _f, _f, _f, _i64, _f]
        L.ref_adamw_step_timed.restype = ctypes.c_double
        L.ref_adamw_step_timed.argtypes = [_fp, _fp, _fp, _fp, _i64, _f, _f, _f, _f, _f,
                                           _i64, _f, ctypes.c_int]
        L.ref_muon_momentum.argtypes = [_fp, _fp, _fp, _i64, _f, ctypes.c_int, _f]
        L.ref_newton_schulz5.argtypes = [_fp, _i64, _i64, ctypes.c_int, _fp, ctypes.c_int,
                                         ctypes.c_int, _fp, ctypes.c_int]
        L.ref_ns_iteration.argtypes = [_fp, _i64, _i64, _fp, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int]
        L.ref_gemm.argtypes = [_fp, _fp, _fp, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int]
        L.ref_muon_apply.argtypes = [_fp, _fp, _i64, _i64, _f]
        L.ref_muon_scale.restype = _f
        L.ref_muon_scale.argtypes = [_i64, _i64]
        L.ref_bias_correction.restype = _f
        L.ref_bias_correction.argtypes = [_f, _i64]
        L.ref_grad_average.argtypes = [_fp, _fp, _i64, _i64]
        L.ref_max_threads.restype = ctypes.c_int
        L.ref_ns_round_array.argtypes = [_fp, _fp, _i64, ctypes.c_int]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Vectorised bf16 round-to-nearest-even (same rule as ref_bf16_round)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    lo = u & 0xFFFF
    hi = u >> 16
    up = (lo > 0x8000) | ((lo == 0x8000) & ((hi & 1) == 1))
    r = ((hi + up.astype(np.uint64)) << 16)
    r = np.where(nan, (u | 0x00400000) & 0xFFFF0000, r)
    return r.astype(np.uint32).view(np.float32).reshape(x.shape)


def tf32_round(x: np.ndarray) -> np.ndarray:
    """Vectorised tf32 round-to-nearest-even of finite values (same rule as
    ref_tf32_round): 10 mantissa bits kept, rounding on the 13 dropped."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = (u + 0xFFF + ((u >> 13) & 1)) & 0xFFFFE000
    keep = (u & 0x7F800000) == 0x7F800000
    r = np.where(keep, u, r)
    return r.astype(np.uint32).view(np.float32).reshape(x.shape)


def bias_correction(beta: float, t: int) -> float:
    return float(lib().ref_bias_correction(beta, t))


def muon_scale(rows: int, cols: int) -> float:
    return float(lib().ref_muon_scale(rows, cols))


def adamw_update(p, m, v, g, *, lr, betas, eps, weight_decay, t, grad_divisor=1.0):
    """In-place AdamW update of one tensor at step count t (lib.rs:41-60)."""
    lib().ref_adamw_step(_ptr(p), _ptr(m), _ptr(v), _ptr(np.ascontiguousarray(g, np.float32)),
                         p.size, lr, betas[0], betas[1], eps, weight_decay, t, grad_divisor)


def muon_momentum(vel, g, *, momentum, nesterov, grad_divisor=1.0):
    u = np.empty_like(vel)
    lib().ref_muon_momentum(_ptr(vel), _ptr(np.ascontiguousarray(g, np.float32)), _ptr(u),
                            vel.size, momentum, int(nesterov), grad_divisor)
    return u


def gemm(a, b, order=GEMM_F64, threads=0):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    c = np.empty((a.shape[0], b.shape[1]), np.float32)
    lib().ref_gemm(_ptr(a), _ptr(b), _ptr(c), a.shape[0], b.shape[1], a.shape[1], order, threads)
    return c


def pad_to_square(g: np.ndarray) -> np.ndarray:
    """lib.rs:89-99: a non-2-D input is zero-padded row-major into side x side,
    side = ceil(sqrt(len)) computed in f32."""
    if g.ndim == 2:
        return np.ascontiguousarray(g, np.float32)
    n = g.size
    side = int(np.ceil(np.sqrt(np.float32(n), dtype=np.float32)))
    out = np.zeros(side * side, np.float32)
    out[:n] = g.reshape(-1)
    return out.reshape(side, side)


_NS_A, _NS_B, _NS_C = np.float32(3.4445), np.float32(-4.7750), np.float32(2.0315)  # lib.rs:84-86
_NS_EPS = np.float32(1e-7)  # lib.rs:87


def _ns_round(x, variant):
    """The rounding point of a Newton-Schulz variant (ns_round in mmn_optim_ref.c)."""
    x = np.ascontiguousarray(x, np.float32)
    if variant == NS_FP32:
        return x
    out = np.empty_like(x)
    lib().ref_ns_round_array(_ptr(x), _ptr(out), x.size, variant)
    return out


def _ns_iteration_blas64(x, variant):
    """ref_ns_iteration (lib.rs:112-120) with the three products formed in float64
    by numpy's matmul and rounded once to float32; the elementwise steps are the
    same float32 operations in the same order."""
    x64 = x.astype(np.float64)
    a = _ns_round((x64 @ x64.T).astype(np.float32), variant)               # :114-115
    a64 = a.astype(np.float64)
    sq = _ns_round((a64 @ a64).astype(np.float32), variant)                # :116
    b = a * _NS_B + sq * _NS_C                                              # :117
    if variant == NS_BF16:
        b = bf16_round(b)
    del a, a64, sq
    bx = (b.astype(np.float64) @ x64).astype(np.float32)
    return _ns_round(x * _NS_A + bx, variant)                              # :118-119


def _newton_schulz5_blas64(g2, steps, variant):
    """ref_newton_schulz5 (lib.rs:101-126) with GEMM_BLAS64 products: transpose
    when rows > cols, round, divide by the Frobenius norm (a sequential float32
    sum of squares, as lib.rs:109; fp64 sum rounded once in NS_TF32 and NS_FP32), iterate,
    transpose back."""
    rows, cols = g2.shape
    transposed = rows > cols
    x = _ns_round(np.ascontiguousarray(g2.T if transposed else g2), variant)
    if variant in (NS_FP32, NS_TF32):
        s = np.float32(np.sum(np.square(x, dtype=np.float64)))
    else:
        s = np.cumsum((x * x).reshape(-1), dtype=np.float32)[-1]  # sequential, in order
    norm = np.fmax(np.sqrt(np.float32(s)), _NS_EPS)  # f32::max: a NaN gives the other
    x = (x / norm).astype(np.float32)
    for _ in range(steps):
        x = _ns_iteration_blas64(x, variant)
    out = np.ascontiguousarray(x.T if transposed else x)
    return out, float(norm)


def newton_schulz5(g, steps=5, order=GEMM_F32_FMA, variant=NS_REFERENCE, threads=0,
                   return_norm=False):
    """newton_schulz5 (lib.rs:83-126). Output has the (padded) 2-D input shape."""
    g2 = pad_to_square(np.asarray(g, np.float32))
    if order == GEMM_BLAS64:
        out, nrm = _newton_schulz5_blas64(g2, steps, variant)
        return (out, nrm) if return_norm else out
    rows, cols = g2.shape
    out = np.empty((rows, cols), np.float32)
    norm = _f(0.0)
    lib().ref_newton_schulz5(_ptr(g2), rows, cols, steps, _ptr(out), order, variant,
                             ctypes.byref(norm), threads)
    return (out, float(norm.value)) if return_norm else out


def ns_iteration(x, order=GEMM_F64, variant=NS_REFERENCE, threads=0):
    x = np.ascontiguousarray(x, np.float32)
    if order == GEMM_BLAS64:
        return _ns_iteration_blas64(x, variant)
    y = np.empty_like(x)
    lib().ref_ns_iteration(_ptr(x), x.shape[0], x.shape[1], _ptr(y), order, variant, threads)
    return y


def muon_apply(p, o, lr):
    lib().ref_muon_apply(_ptr(p), _ptr(np.ascontiguousarray(o, np.float32)), p.shape[0],
                         p.shape[1] if p.ndim > 1 else 1, lr)


class AdamWConfig:
    """lib.rs:6-22; defaults lr 3e-4, betas (0.9, 0.95), eps 1e-8, wd 0.01."""

    def __init__(self, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01):
        self.lr, self.betas, self.eps, self.weight_decay = lr, tuple(betas), eps, weight_decay


class MuonConfig:
    """lib.rs:63-80; defaults lr 0.02, momentum 0.95, nesterov, 5 steps."""

    def __init__(self, lr=0.02, momentum=0.95, nesterov=True, ns_steps=5):
        self.lr, self.momentum, self.nesterov, self.ns_steps = lr, momentum, nesterov, ns_steps


class AdamW:
    """lib.rs:24-61."""

    def __init__(self, config: AdamWConfig):
        self.config = config
        self.step = 0
        self.m: dict[int, np.ndarray] = {}
        self.v: dict[int, np.ndarray] = {}

    def step_param(self, pid: int, param: np.ndarray, grad: np.ndarray, grad_divisor=1.0):
        self.step += 1
        m = self.m.setdefault(pid, np.zeros(param.shape, np.float32))
        v = self.v.setdefault(pid, np.zeros(param.shape, np.float32))
        c = self.config
        adamw_update(param, m, v, grad, lr=c.lr, betas=c.betas, eps=c.eps,
                     weight_decay=c.weight_decay, t=self.step, grad_divisor=grad_divisor)


class Muon:
    """lib.rs:128-176."""

    def __init__(self, config: MuonConfig, order=GEMM_F32_FMA, variant=NS_REFERENCE):
        self.config = config
        self.velocity: dict[int, np.ndarray] = {}
        self.order, self.variant = order, variant

    def step_matrix(self, pid: int, param: np.ndarray, grad: np.ndarray, grad_divisor=1.0):
        g2 = np.ascontiguousarray(grad, np.float32)
        if g2.ndim != 2:
            side = int(np.ceil(np.sqrt(np.float32(g2.size), dtype=np.float32)))
            g2 = g2.reshape(side, side)  # lib.rs:146-149 (panics unless len == side^2)
        vel = self.velocity.setdefault(pid, np.zeros(g2.shape, np.float32))
        c = self.config
        u = muon_momentum(vel, g2, momentum=c.momentum, nesterov=c.nesterov,
                          grad_divisor=grad_divisor)
        o = newton_schulz5(u, c.ns_steps, order=self.order, variant=self.variant)
        muon_apply(param, o, c.lr)


MATRIX, OTHER = "Matrix", "Other"


def classify_param(shape) -> str:
    """lib.rs:196-202."""
    return MATRIX if len(shape) == 2 and shape[0] > 1 and shape[1] > 1 else OTHER


class HybridOptimizer:
    """lib.rs:183-210."""

    def __init__(self, muon: MuonConfig, adamw: AdamWConfig, order=GEMM_F32_FMA,
                 variant=NS_REFERENCE):
        self.muon = Muon(muon, order, variant)
        self.adamw = AdamW(adamw)

    def step(self, pid, param, grad, route=None, grad_divisor=1.0):
        kind = route or classify_param(param.shape)
        if kind == MATRIX:
            self.muon.step_matrix(pid, param, grad, grad_divisor)
        else:
            self.adamw.step_param(pid, param, grad, grad_divisor)


class GradAccumulator:
    """lib.rs:212-262."""

    def __init__(self):
        self.grads: list[np.ndarray] = []
        self.micro_batches = 0
        self.param_index = 0

    def clear(self):
        self.grads.clear()
        self.micro_batches = 0
        self.param_index = 0

    def begin_micro_batch(self):
        self.param_index = 0

    def finish_micro_batch(self):
        self.micro_batches += 1
        self.param_index = 0

    def add_param_grad(self, grad):
        if self.param_index < len(self.grads):
            self.grads[self.param_index] += np.asarray(grad, np.float32)
        else:
            self.grads.append(np.array(grad, np.float32, copy=True))
        self.param_index += 1

    def averaged_grad(self, index):
        s = self.grads[index]
        out = np.empty_like(s)
        lib().ref_grad_average(_ptr(s), _ptr(out), s.size, self.micro_batches)
        return out

    def __len__(self):
        return len(self.grads)


class LossScaleState:
    """Dynamic loss scaling for bf16 grads. NEW BEHAVIOUR with no reference
    counterpart (the reference trains in fp32 without loss scaling), defined
    here so the GPU path has something to be checked against:
      * grads arrive multiplied by `scale` and rounded to bf16; the step uses
        g = float(g_bf16) / scale (exact for a power-of-two scale);
      * if any grad of any tensor is non-finite the whole step is skipped:
        params, m, v, velocity and the AdamW call counter stay as they are,
        the scale halves and the clean-step count resets;
      * after `growth_interval` consecutive clean steps the scale doubles."""

    def __init__(self, scale=65536.0, growth_interval=2000):
        self.scale = np.float32(scale)
        self.growth_interval = growth_interval
        self.good = 0
        self.skipped = 0

    def unscale(self, g_bf16_values):
        return (np.asarray(g_bf16_values, np.float32) / self.scale).astype(np.float32)

    def check(self, grads) -> bool:
        """True when the step may run (all grads finite)."""
        return all(np.isfinite(g).all() for g in grads)

    def update(self, stepped: bool) -> None:
        if not stepped:
            self.scale = np.float32(self.scale * np.float32(0.5))
            self.good = 0
            self.skipped += 1
            return
        self.good += 1
        if self.good >= self.growth_interval:
            self.scale = np.float32(self.scale * np.float32(2.0))
            self.good = 0


def grad_allreduce(local_grads, bf16=False) -> np.ndarray:
    """Data-parallel grad reduction before the step. NEW BEHAVIOUR with no
    reference counterpart (the reference trains in one process), defined here so
    the multi-GPU path has something to be checked against:
      * the ranks' local grads are summed in rank order in fp32: s = g_0, then
        s = s + g_r for r = 1 .. W-1, each add rounded to nearest even;
      * bf16 grads are widened to fp32 exactly, summed that way and rounded to
        bf16 once (round to nearest even).
    local_grads: one float32 array per rank (bf16 grads as their float32
    values). Returns the sum as float32 (bf16-rounded values when bf16)."""
    s = np.asarray(local_grads[0], np.float32).copy()
    for g in local_grads[1:]:
        np.add(s, np.asarray(g, np.float32), out=s)
    return bf16_round(s) if bf16 else s


def bf16_from_bits(bits) -> np.ndarray:
    """float32 values of bf16 bit patterns (uint16 or int16 arrays)."""
    return (np.asarray(bits).view(np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_bits(x) -> np.ndarray:
    """uint16 bit patterns of bf16(x) (round to nearest even)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)
