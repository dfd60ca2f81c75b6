"""The TF32 Newton-Schulz mode (MMN_NS_TF32) on the tensor cores against the
oracle's REF_NS_TF32 recipe.

The mode keeps the reference recipe (crates/mmn-optim/src/lib.rs:104-119) and
moves its four rounding points from bf16 to tf32: X, A = XX^T and A2 = A A are
held as tf32 values in fp32 words and multiplied with kind::tf32 MMAs, fp32
accumulate, B = b*A + c*A2 kept exact by two accumulators. It has no reference
counterpart; the oracle defines it.

Tolerances (relative Frobenius unless stated):
  - one iteration from the same input: A and A2 within one tf32 ulp plus the
    fp32 accumulation bound per entry on at most 2% of entries, the next X
    within 3e-4 (a rounding flip moves an entry by one tf32 ulp, 2^-11
    relative, and a few percent of entries flip between two fp32 summation
    orders: about 1e-4);
  - newton_schulz5 end to end against the oracle's tf32 recipe: 3e-3. The
    quintic amplifies tf32 rounding flips the way it amplifies bf16 ones
    (slope 3.44 near zero, about 480x over five iterations), so two correct
    fp32 summation orders of the oracle itself end 6e-4 to 9e-4 apart;
  - against exact Newton-Schulz (fp64, no rounding): 4e-3, where the bf16
    reference recipe sits at 0.9e-2 to 1.6e-2;
  - Muon parameter updates: 3e-3; AdamW and the velocity stay bit-exact.
"""
import ctypes

import numpy as np
import pytest

from conftest import chatbot_params, rel_fro

pytestmark = pytest.mark.gpu

NS_A, NS_B, NS_C = 3.4445, -4.7750, 2.0315
ADAMW = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)


def exact_ns(g, steps=5):
    """Newton-Schulz in fp64 with no rounding points (lib.rs:101-124 without
    its bf16 casts)."""
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
        x.ctypes.data, n, m, ctypes.c_float(norm), N.NS_TF32, a.ctypes.data, a2.ctypes.data,
        xn.ctypes.data, 0))
    return a, a2, xn


def tf32_rounding_check(a, b, abs_terms):
    """Entries of two tf32-rounded GEMM outputs may differ by one tf32 ulp (a
    rounding flip) plus the fp32 accumulation error, bounded by 2^-16 of the
    sum of absolute products. Returns the fraction of differing entries and
    the worst ratio to that bound."""
    diff = np.abs(a - b)
    mag = np.maximum(np.abs(a), np.abs(b))
    ulp = np.exp2(np.floor(np.log2(np.maximum(mag, 1e-30))) - 10)
    bound = ulp + np.ldexp(abs_terms, -16)
    return float((a != b).mean()), float(np.max(diff / bound))


@pytest.mark.parametrize("shape", [(64, 64), (64, 256), (100, 300), (256, 256), (384, 640),
                                   (1, 8)])
def test_tf32_first_iteration_matches_oracle(mmn, oracle, shape):
    rng = np.random.default_rng(hash(shape) % 2**32)
    n, m = shape
    y = oracle.tf32_round(rng.normal(0, 1e-2, (n, m)).astype(np.float32))
    norm = max(np.float32(np.sqrt(np.sum(y * y, dtype=np.float32))), np.float32(1e-7))
    a, a2, xn = gpu_iteration(y, norm)
    x0 = (y / norm).astype(np.float32)
    a_ref = oracle.tf32_round(oracle.gemm(x0, x0.T.copy(), oracle.GEMM_F64))
    ax = np.abs(x0)
    frac, worst = tf32_rounding_check(a, a_ref, oracle.gemm(ax, ax.T.copy(), oracle.GEMM_F64))
    assert frac <= 0.02 and worst <= 1.0, (frac, worst)
    np.testing.assert_array_equal(a, a.T)  # symmetric by construction
    np.testing.assert_array_equal(a, oracle.tf32_round(a))  # stored as tf32 values
    a2_own = oracle.tf32_round(oracle.gemm(a, a, oracle.GEMM_F64))
    aa = np.abs(a)
    frac, worst = tf32_rounding_check(a2, a2_own, oracle.gemm(aa, aa, oracle.GEMM_F64))
    assert frac <= 0.02 and worst <= 1.0, (frac, worst)
    xn_ref = oracle.ns_iteration(x0, oracle.GEMM_F64, oracle.NS_TF32)
    assert rel_fro(xn, xn_ref) <= 3e-4
    np.testing.assert_array_equal(xn, oracle.tf32_round(xn))


@pytest.mark.parametrize("shape", [(64, 256), (256, 256), (128, 640)])
def test_tf32_later_iteration_matches_oracle(mmn, oracle, shape):
    rng = np.random.default_rng(7)
    n, m = shape
    y = oracle.tf32_round(rng.normal(0, 1e-2, (n, m)).astype(np.float32))
    norm = np.float32(np.sqrt(np.sum(y * y, dtype=np.float32)))
    x1 = oracle.ns_iteration((y / norm).astype(np.float32), oracle.GEMM_F64, oracle.NS_TF32)
    x2 = oracle.ns_iteration(x1, oracle.GEMM_F64, oracle.NS_TF32)
    _, _, xn = gpu_iteration(x2, 1.0)
    assert rel_fro(xn, oracle.ns_iteration(x2, oracle.GEMM_F64, oracle.NS_TF32)) <= 3e-4


@pytest.mark.parametrize("shape", [(64, 64), (64, 256), (256, 64), (512, 64), (100, 37),
                                   (300, 300), (512, 1536), (4, 4), (1, 5)])
def test_tf32_newton_schulz5_end_to_end(mmn, oracle, shape):
    rng = np.random.default_rng(11)
    g = rng.normal(0, 1e-2, shape).astype(np.float32)
    out = mmn.newton_schulz5(g, 5, ns_mode="tf32")
    ref = oracle.newton_schulz5(g, 5, order=oracle.GEMM_F64, variant=oracle.NS_TF32)
    assert out.shape == ref.shape and np.isfinite(out).all()
    assert rel_fro(out, ref) <= 3e-3
    assert rel_fro(out, exact_ns(g)) <= 4e-3
    if min(shape) >= 64:
        # the point of the mode: several times closer to exact Newton-Schulz
        # than the bf16 reference recipe on the same input
        bf = mmn.newton_schulz5(g, 5, ns_mode="reference")
        assert rel_fro(out, exact_ns(g)) * 3 < rel_fro(bf, exact_ns(g))


def test_tf32_transpose_rule_and_determinism(mmn):
    rng = np.random.default_rng(3)
    g = rng.normal(0, 1e-2, (96, 320)).astype(np.float32)
    a = mmn.newton_schulz5(g, ns_mode="tf32")
    b = mmn.newton_schulz5(np.ascontiguousarray(g.T), ns_mode="tf32")
    np.testing.assert_array_equal(a.T, b)
    g2 = rng.normal(0, 1e-2, (320, 768)).astype(np.float32)
    np.testing.assert_array_equal(mmn.newton_schulz5(g2, ns_mode="tf32"),
                                  mmn.newton_schulz5(g2, ns_mode="tf32"))


def test_tf32_scaled_identity_stays_diagonal(mmn, oracle):
    """NS of s*I stays diagonal with one value on the diagonal, the scalar
    recurrence x -> tf32(a*x + (b*A + c*A2)*x), A = tf32(x*x), A2 = tf32(A*A)
    from x0 = 1/sqrt(n) (the oracle test pins the recurrence exactly; the
    GPU's tree-summed norm may move x0 by an ulp, so 2e-3 here)."""
    n = 48
    out = mmn.newton_schulz5(np.eye(n, dtype=np.float32) * np.float32(0.37), 5, ns_mode="tf32")
    assert np.count_nonzero(out - np.diag(np.diag(out))) == 0
    d = np.diag(out)
    assert np.all(d == d[0])
    ref = oracle.newton_schulz5(np.eye(n, dtype=np.float32) * np.float32(0.37), 5,
                                order=oracle.GEMM_F64, variant=oracle.NS_TF32)
    np.testing.assert_allclose(d, np.diag(ref), rtol=2e-3)


def test_tf32_muon_and_batched_step_vs_oracle(mmn, oracle):
    """Muon::step_matrix and the batched Chatbot step in the TF32 mode: AdamW
    tensors and the velocity bit-exact, Muon updates within 3e-3."""
    rng = np.random.default_rng(0)
    shapes = [(64, 64), (64, 256), (256, 64), (512, 64), (33, 17)]
    gpu = mmn.Muon(mmn.MuonConfig(), ns_mode="tf32")
    ref = oracle.Muon(oracle.MuonConfig(), order=oracle.GEMM_F64, variant=oracle.NS_TF32)
    for i, s in enumerate(shapes):
        p = rng.normal(0, 0.02, s).astype(np.float32)
        pr = p.copy()
        for _ in range(2):
            g = rng.normal(0, 1e-3, s).astype(np.float32)
            before = pr.copy()
            gpu.step_matrix(i, p, g)
            ref.step_matrix(i, pr, g)
            assert rel_fro(p - before, pr - before) <= 3e-3, s
            np.testing.assert_array_equal(gpu.export_velocity(i, s).view(np.uint32),
                                          ref.velocity[i].view(np.uint32))
            p[:] = pr

    named = chatbot_params(np.random.default_rng(1))
    order = [n for n, _ in named]
    p_ref = {n: v.copy() for n, v in named}
    step = mmn.OptimizerStep([(k, p_ref[n].shape, "auto") for k, n in enumerate(order)],
                             mmn.StepConfig(adamw=mmn.AdamWConfig(**ADAMW),
                                            muon=mmn.MuonConfig(), ns_mode="tf32"))
    for k, n in enumerate(order):
        step.set_param(k, p_ref[n])
    hyb = oracle.HybridOptimizer(oracle.MuonConfig(), oracle.AdamWConfig(**ADAMW),
                                 order=oracle.GEMM_F64, variant=oracle.NS_TF32)
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
                assert rel_fro(out - before[n], p_ref[n] - before[n]) <= 3e-3, (s, n)
                step.set_param(k, p_ref[n])
            else:
                np.testing.assert_array_equal(out.view(np.uint32), p_ref[n].view(np.uint32))
    step.close()
