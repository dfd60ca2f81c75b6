"""The fp32 Newton-Schulz mode (MMN_NS_FP32) on the tensor cores against the
oracle's REF_NS_FP32 recipe and against exact (fp64) Newton-Schulz.

The mode runs the iteration of crates/mmn-optim/src/lib.rs:112-120 with no
rounding points: X, A = XX^T and A2 = A A stay fp32 values, each stored as a
hi + lo pair of tf32 planes, and every product is formed from three tf32 MMAs
(hi*hi + hi*lo + lo*hi) accumulated in fp32. It has no reference counterpart
(the reference rounds to bf16 four times per iteration); the oracle defines it.

Tolerance: 1e-4 relative Frobenius for newton_schulz5 and for Muon parameter
updates, the bar the task sets for an fp32 Newton-Schulz; one iteration and
its A, A2 within 5e-5 (the three-pass product drops the lo*lo term, 2^-22 of
each product, and the tensor cores accumulate each MMA's products before the
fp32 add). Without rounding points nothing is amplified, so five iterations
stay within the one-iteration error.
"""
import ctypes

import numpy as np
import pytest

from conftest import chatbot_params, rel_fro

pytestmark = pytest.mark.gpu

NS_A, NS_B, NS_C = 3.4445, -4.7750, 2.0315
ADAMW = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)


def exact_ns(g, steps=5):
    """Newton-Schulz in fp64 with no rounding points."""
    x = np.asarray(g, np.float64)
    tr = x.shape[0] > x.shape[1]
    if tr:
        x = x.T
    x = x / max(np.linalg.norm(x), 1e-7)
    for _ in range(steps):
        a = x @ x.T
        x = NS_A * x + (NS_B * a + NS_C * (a @ a)) @ x
    return x.T if tr else x


def gpu_iteration(x, norm):
    from magicmindnet_b200 import _native as N

    n, m = x.shape
    a = np.empty((n, n), np.float32)
    a2 = np.empty((n, n), np.float32)
    xn = np.empty((n, m), np.float32)
    x = np.ascontiguousarray(x, np.float32)
    N.check(N.lib().mmn_newton_schulz_iteration(
        x.ctypes.data, n, m, ctypes.c_float(norm), N.NS_FP32, a.ctypes.data, a2.ctypes.data,
        xn.ctypes.data, 0))
    return a, a2, xn


@pytest.mark.parametrize("shape", [(64, 64), (64, 256), (100, 300), (256, 256), (384, 640),
                                   (1, 8)])
def test_fp32_iteration_matches_oracle(mmn, oracle, shape):
    rng = np.random.default_rng(sum(shape))
    n, m = shape
    y = rng.normal(0, 1e-2, (n, m)).astype(np.float32)
    norm = max(np.float32(np.sqrt(np.sum(y * y, dtype=np.float32))), np.float32(1e-7))
    a, a2, xn = gpu_iteration(y, norm)
    x0 = (y / norm).astype(np.float32)
    a_ref = oracle.gemm(x0, x0.T.copy(), oracle.GEMM_F64)
    assert rel_fro(a, a_ref) <= 5e-5
    np.testing.assert_array_equal(a, a.T)
    assert rel_fro(a2, oracle.gemm(a_ref, a_ref, oracle.GEMM_F64)) <= 5e-5
    assert rel_fro(xn, oracle.ns_iteration(x0, oracle.GEMM_F64, oracle.NS_FP32)) <= 5e-5
    # a later iteration (norm divisor 1) from the oracle's own X
    x2 = oracle.ns_iteration(oracle.ns_iteration(x0, oracle.GEMM_F64, oracle.NS_FP32),
                             oracle.GEMM_F64, oracle.NS_FP32)
    _, _, xn2 = gpu_iteration(x2, 1.0)
    assert rel_fro(xn2, oracle.ns_iteration(x2, oracle.GEMM_F64, oracle.NS_FP32)) <= 5e-5


@pytest.mark.parametrize("shape", [(64, 64), (64, 256), (256, 64), (512, 64), (100, 37),
                                   (300, 300), (512, 1536), (4, 4), (1, 5)])
def test_fp32_newton_schulz5_within_1e4(mmn, oracle, shape):
    rng = np.random.default_rng(11)
    g = rng.normal(0, 1e-2, shape).astype(np.float32)
    out = mmn.newton_schulz5(g, 5, ns_mode="fp32")
    ref = oracle.newton_schulz5(g, 5, order=oracle.GEMM_F64, variant=oracle.NS_FP32)
    assert out.shape == ref.shape and np.isfinite(out).all()
    assert rel_fro(out, ref) <= 1e-4
    assert rel_fro(out, exact_ns(g)) <= 1e-4


def test_fp32_transpose_rule_and_determinism(mmn):
    rng = np.random.default_rng(3)
    g = rng.normal(0, 1e-2, (96, 320)).astype(np.float32)
    a = mmn.newton_schulz5(g, ns_mode="fp32")
    b = mmn.newton_schulz5(np.ascontiguousarray(g.T), ns_mode="fp32")
    np.testing.assert_array_equal(a.T, b)
    g2 = rng.normal(0, 1e-2, (320, 768)).astype(np.float32)
    np.testing.assert_array_equal(mmn.newton_schulz5(g2, ns_mode="fp32"),
                                  mmn.newton_schulz5(g2, ns_mode="fp32"))


def test_fp32_zero_steps_returns_normalised_input(mmn, oracle):
    rng = np.random.default_rng(6)
    g = rng.normal(0, 1e-2, (48, 80)).astype(np.float32)
    out = mmn.newton_schulz5(g, 0, ns_mode="fp32")
    ref = oracle.newton_schulz5(g, 0, variant=oracle.NS_FP32)
    # X = hi + lo carries u to 2^-22; the GPU norm is a tree sum
    np.testing.assert_allclose(out, ref, rtol=2e-6, atol=0)


def test_fp32_muon_and_batched_step_within_1e4(mmn, oracle):
    """Muon::step_matrix and the batched Chatbot step in the fp32 mode: AdamW
    tensors and the velocity bit-exact, Muon updates within 1e-4."""
    rng = np.random.default_rng(0)
    shapes = [(64, 64), (64, 256), (256, 64), (512, 64), (33, 17)]
    gpu = mmn.Muon(mmn.MuonConfig(), ns_mode="fp32")
    ref = oracle.Muon(oracle.MuonConfig(), order=oracle.GEMM_F64, variant=oracle.NS_FP32)
    for i, s in enumerate(shapes):
        p = rng.normal(0, 0.02, s).astype(np.float32)
        pr = p.copy()
        for _ in range(2):
            g = rng.normal(0, 1e-3, s).astype(np.float32)
            before = pr.copy()
            gpu.step_matrix(i, p, g)
            ref.step_matrix(i, pr, g)
            assert rel_fro(p - before, pr - before) <= 1e-4, s
            np.testing.assert_array_equal(gpu.export_velocity(i, s).view(np.uint32),
                                          ref.velocity[i].view(np.uint32))
            p[:] = pr

    named = chatbot_params(np.random.default_rng(1))
    order = [n for n, _ in named]
    p_ref = {n: v.copy() for n, v in named}
    step = mmn.OptimizerStep([(k, p_ref[n].shape, "auto") for k, n in enumerate(order)],
                             mmn.StepConfig(adamw=mmn.AdamWConfig(**ADAMW),
                                            muon=mmn.MuonConfig(), ns_mode="fp32"))
    for k, n in enumerate(order):
        step.set_param(k, p_ref[n])
    hyb = oracle.HybridOptimizer(oracle.MuonConfig(), oracle.AdamWConfig(**ADAMW),
                                 order=oracle.GEMM_F64, variant=oracle.NS_FP32)
    for s in range(2):
        grads = {n: rng.normal(0, 1e-3, p_ref[n].shape).astype(np.float32) for n in order}
        before = {n: p_ref[n].copy() for n in order}
        for k, n in enumerate(order):
            hyb.step(k, p_ref[n], grads[n])
            step.set_grad(k, grads[n])
        step.step()
        step.sync()
        for k, n in enumerate(order):
            out = step.get_param(k)
            if oracle.classify_param(p_ref[n].shape) == oracle.MATRIX:
                assert rel_fro(out - before[n], p_ref[n] - before[n]) <= 1e-4, (s, n)
                step.set_param(k, p_ref[n])
            else:
                np.testing.assert_array_equal(out.view(np.uint32), p_ref[n].view(np.uint32))
    step.close()


def _exact_ns_fp64_on_gpu(g, steps=5):
    """Exact Newton-Schulz in fp64 computed on the GPU with torch (the fp64
    form of exact_ns, for sizes the CPU would take minutes on)."""
    import torch

    x = torch.from_numpy(g).cuda().double()
    tr = x.shape[0] > x.shape[1]
    if tr:
        x = x.T
    x = x / max(torch.linalg.norm(x).item(), 1e-7)
    for _ in range(steps):
        a = x @ x.T
        x = NS_A * x + (NS_B * a + NS_C * (a @ a)) @ x
    return (x.T if tr else x).cpu().numpy()


@pytest.mark.parametrize("shape", [(4096, 14336), (14336, 4096), (4096, 4096)])
def test_fp32_and_tf32_full_size_against_fp64(mmn, shape):
    """The largest Newton-Schulz shapes of the benchmark configurations (the
    4096 x 14336 FFN matrices and 4096 x 4096 projections), one matrix each,
    against fp64 Newton-Schulz: fp32 mode within 1e-4, TF32 mode within 4e-3."""
    g = np.random.default_rng(5).normal(0, 1e-2, shape).astype(np.float32)
    exact = _exact_ns_fp64_on_gpu(g)
    assert rel_fro(mmn.newton_schulz5(g, 5, ns_mode="fp32"), exact) <= 1e-4
    assert rel_fro(mmn.newton_schulz5(g, 5, ns_mode="tf32"), exact) <= 4e-3
