"""Newton-Schulz on the tensor cores against the oracle.

The reference recipe (crates/mmn-optim/src/lib.rs:112-120) rounds to bf16 at
four points per iteration, and the quintic's slope of 3.44 near zero amplifies
every rounding flip, so two correct fp32 GEMM summation orders drift apart over
five iterations (the oracle alone shows ~6e-3 between its fp32 and fp64
orders; tests/test_oracle.py pins that). Parity is therefore checked in layers:

  1. one iteration from the same input: the bf16 GEMM outputs A, A2 agree
     elementwise up to 1 bf16 ulp on a small fraction of entries, and the next
     X within 1e-3 relative Frobenius;
  2. the full five iterations: within 2e-2 relative Frobenius (the stated
     bf16-mode tolerance; the reference-order spread itself is ~6e-3);
  3. exact properties: transpose rule and run-to-run determinism.
"""
import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu

ITER_SHAPES = [(64, 64), (64, 256), (128, 512), (256, 256), (100, 300), (1, 8), (200, 1000),
               (384, 640)]


def first_iter_input(oracle, rng, n, m):
    g = rng.normal(0, 1e-2, (n, m)).astype(np.float32)
    y = oracle.bf16_round(g)
    norm = np.float32(np.sqrt(np.sum(y * y, dtype=np.float32)))
    norm = max(norm, np.float32(1e-7))
    return y, norm


def gpu_iteration(mmn, x, norm, mode="reference"):
    import ctypes

    from magicmindnet_b200 import _native as N

    n, m = x.shape
    a = np.empty((n, n), np.float32)
    a2 = np.empty((n, n), np.float32)
    xn = np.empty((n, m), np.float32)
    x = np.ascontiguousarray(x, np.float32)
    N.check(N.lib().mmn_newton_schulz_iteration(
        x.ctypes.data, n, m, ctypes.c_float(norm), {"reference": 0, "bf16": 1}[mode],
        a.ctypes.data, a2.ctypes.data, xn.ctypes.data, 0))
    return a, a2, xn


def bf16_rounding_check(a, b, abs_terms):
    """Compares two bf16-rounded GEMM outputs. Each entry may differ by one bf16
    ulp (a rounding flip) plus the fp32 accumulation error, bounded here by
    2^-16 of the sum of the absolute products (abs_terms). Returns the
    fraction of differing entries and the worst ratio to that bound."""
    diff = np.abs(a - b)
    mag = np.maximum(np.abs(a), np.abs(b))
    ulp = np.exp2(np.floor(np.log2(np.maximum(mag, 1e-30))) - 7)
    bound = ulp + np.ldexp(abs_terms, -16)
    return float((a != b).mean()), float(np.max(diff / bound))


@pytest.mark.parametrize("shape", ITER_SHAPES)
def test_first_iteration_matches_oracle(mmn, oracle, shape):
    rng = np.random.default_rng(hash(shape) % 2**32)
    n, m = shape
    y, norm = first_iter_input(oracle, rng, n, m)
    a, a2, xn = gpu_iteration(mmn, y, norm)
    x0 = (y / norm).astype(np.float32)
    # oracle pieces with fp64 accumulation (closest to exact)
    a_ref = oracle.bf16_round(oracle.gemm(x0, x0.T.copy(), oracle.GEMM_F64))
    a2_ref = oracle.bf16_round(oracle.gemm(a_ref, a_ref, oracle.GEMM_F64))
    xn_ref = oracle.ns_iteration(x0, oracle.GEMM_F64)
    ax = np.abs(x0)
    frac, worst = bf16_rounding_check(a, a_ref, oracle.gemm(ax, ax.T.copy(), oracle.GEMM_F64))
    assert frac <= 0.02 and worst <= 1.0, (frac, worst)
    np.testing.assert_array_equal(a, a.T)  # symmetric by construction
    # A2 from the GPU's own A isolates the second product from flips in A
    a2_ref_own = oracle.bf16_round(oracle.gemm(a, a, oracle.GEMM_F64))
    aa = np.abs(a)
    frac, worst = bf16_rounding_check(a2, a2_ref_own, oracle.gemm(aa, aa, oracle.GEMM_F64))
    assert frac <= 0.02 and worst <= 1.0, (frac, worst)
    assert rel_fro(a2, a2_ref) <= 1e-3
    assert rel_fro(xn, xn_ref) <= 1e-3


@pytest.mark.parametrize("shape", [(64, 256), (256, 256), (128, 640)])
def test_later_iteration_matches_oracle(mmn, oracle, shape):
    """An iteration on a bf16-valued X (norm divisor 1), as in iterations 2-5."""
    rng = np.random.default_rng(7)
    n, m = shape
    y, norm = first_iter_input(oracle, rng, n, m)
    x1 = oracle.ns_iteration((y / norm).astype(np.float32), oracle.GEMM_F64)
    x2 = oracle.ns_iteration(x1, oracle.GEMM_F64)
    _, _, xn = gpu_iteration(mmn, x2, 1.0)
    xn_ref = oracle.ns_iteration(x2, oracle.GEMM_F64)
    assert rel_fro(xn, xn_ref) <= 1e-3


@pytest.mark.parametrize("shape", [(64, 64), (64, 256), (256, 64), (512, 64), (100, 37), (300, 300),
                                   (4, 4), (1, 5)])
@pytest.mark.parametrize("mode", ["reference", "bf16"])
def test_newton_schulz5_end_to_end(mmn, oracle, shape, mode):
    """Each mode against the oracle running the same recipe: 2e-2 relative
    Frobenius. The bf16 mode is also held to 2e-2 against the reference
    recipe itself for matrices with min(shape) >= 64; on smaller ones the bf16
    rounding of B alone moves the result by up to ~3e-2 (a property of the
    recipe, visible between the oracle's own two variants)."""
    rng = np.random.default_rng(11)
    g = rng.normal(0, 1e-2, shape).astype(np.float32)
    out = mmn.newton_schulz5(g, 5, ns_mode=mode)
    variant = oracle.NS_BF16 if mode == "bf16" else oracle.NS_REFERENCE
    ref = oracle.newton_schulz5(g, 5, order=oracle.GEMM_F64, variant=variant)
    assert out.shape == ref.shape
    assert np.isfinite(out).all()
    assert rel_fro(out, ref) <= 2e-2
    if mode == "bf16" and min(shape) >= 64:
        ref_r = oracle.newton_schulz5(g, 5, order=oracle.GEMM_F64)
        assert rel_fro(out, ref_r) <= 2e-2


def test_newton_schulz5_transpose_rule_is_exact(mmn):
    rng = np.random.default_rng(3)
    g = rng.normal(0, 1e-2, (96, 320)).astype(np.float32)
    a = mmn.newton_schulz5(g)
    b = mmn.newton_schulz5(np.ascontiguousarray(g.T))
    np.testing.assert_array_equal(a.T, b)


def test_newton_schulz5_is_deterministic(mmn):
    rng = np.random.default_rng(4)
    g = rng.normal(0, 1e-2, (256, 768)).astype(np.float32)
    np.testing.assert_array_equal(mmn.newton_schulz5(g), mmn.newton_schulz5(g))


def test_reference_unit_tests(mmn):
    """lib.rs:295-300 (identity -> finite) and lib.rs:322-328 (nonzero)."""
    o = mmn.newton_schulz5(np.eye(2, dtype=np.float32))
    assert np.isfinite(o).all()
    g = np.fromfunction(lambda i, j: (i + j) * 0.1, (4, 4)).astype(np.float32)
    assert np.abs(mmn.newton_schulz5(g)).sum() > 1e-6


def test_non_2d_input_is_zero_padded(mmn, oracle):
    rng = np.random.default_rng(5)
    g = rng.normal(0, 1e-2, (10,)).astype(np.float32)  # side = 4, padded with 6 zeros
    out = mmn.newton_schulz5(g)
    ref = oracle.newton_schulz5(g, order=oracle.GEMM_F64)
    assert out.shape == (4, 4)
    assert rel_fro(out, ref) <= 2e-2


def test_zero_steps_returns_normalised_input(mmn, oracle):
    rng = np.random.default_rng(6)
    g = rng.normal(0, 1e-2, (48, 80)).astype(np.float32)
    out = mmn.newton_schulz5(g, 0)
    ref = oracle.newton_schulz5(g, 0)
    # the GPU reproduces the reference's sequential fp32 norm exactly
    np.testing.assert_array_equal(out, ref)
