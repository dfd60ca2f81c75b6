"""The momentum pass and the sequential norm inside the batched step, bit for
bit. With zero Newton-Schulz iterations the Muon update is
p -= lr * sqrt(rows/cols) * bf16(u) / norm (crates/mmn-optim/src/lib.rs:
154-175, the norm of :109), so a batched step's parameters and velocities must
equal the oracle's bit for bit: a wrong element order in the norm, a momentum
step run twice or skipped, or an inexact norm all show. Covered: shapes of both
orientations side by side (transposed, rows not a multiple of 8, small and
stagnating sizes), three steps (the velocity carried over), fp32 grads and bf16
loss-scaled grads, and a non-finite grad early in a large matrix (its sum
settles at inf or NaN while the momentum still runs over the rest)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(2048, 8192), (8192, 2048), (1000, 1024), (1024, 1000), (200, 300), (64, 256),
          (2048, 8192)]


def _finite_bits_equal(a, b, msg):
    np.testing.assert_array_equal(a, b, err_msg=msg)  # NaN positions equal
    fin = np.isfinite(a)
    np.testing.assert_array_equal(a[fin].view(np.uint32), b[fin].view(np.uint32), err_msg=msg)


def _run(mmn, oracle, grads_for, *, bf16=False, steps=3):
    cfg = mmn.MuonConfig(ns_steps=0)
    kw = dict(grad_dtype="bf16", loss_scaling=True, loss_scale_init=1024.0) if bf16 else {}
    step = mmn.OptimizerStep([(k, s, "muon") for k, s in enumerate(SHAPES)],
                             mmn.StepConfig(muon=cfg, use_graph=False, **kw), device=0)
    rng = np.random.default_rng(5)
    p_ref = [rng.normal(0, 0.02, s).astype(np.float32) for s in SHAPES]
    for k in range(len(SHAPES)):
        step.set_param(k, p_ref[k])
    ref = oracle.Muon(oracle.MuonConfig(cfg.lr, cfg.momentum, cfg.nesterov, 0),
                      order=oracle.GEMM_F64)
    for it in range(steps):
        gs = grads_for(it)
        for k, g in enumerate(gs):
            if bf16:
                step.set_grad(k, oracle.bf16_bits(oracle.bf16_round(g * np.float32(1024.0))))
            else:
                step.set_grad(k, g)
        step.step()
        step.sync()
        for k, g in enumerate(gs):
            if bf16:
                g = (oracle.bf16_round(g * np.float32(1024.0)) / np.float32(1024.0)).astype(
                    np.float32)
            ref.step_matrix(k, p_ref[k], g)
        for k, s in enumerate(SHAPES):
            _finite_bits_equal(step.get_state(k, "velocity"), ref.velocity[k],
                               f"velocity, step {it}, {s}")
            _finite_bits_equal(step.get_param(k), p_ref[k], f"param, step {it}, {s}")
    step.close()


def _normal_grads(seed):
    def grads_for(it):
        rng = np.random.default_rng(seed + it)
        return [rng.normal(0, 1e-3, s).astype(np.float32) for s in SHAPES]
    return grads_for


def test_fused_momentum_and_norm_fp32_grads(mmn, oracle):
    _run(mmn, oracle, _normal_grads(10))


def test_fused_momentum_and_norm_bf16_loss_scaled_grads(mmn, oracle):
    _run(mmn, oracle, _normal_grads(20), bf16=True, steps=2)


@pytest.mark.parametrize("bad", [np.inf, np.nan])
def test_non_finite_grad_in_a_fused_matrix(mmn, oracle, bad):
    """A non-finite grad at element 7 of a 2048 x 8192 matrix: its sum settles
    at once, the momentum still runs over the other 16.8M elements of that
    matrix, and every other matrix is untouched by it."""
    base = _normal_grads(30)

    def grads_for(it):
        gs = base(it)
        if it == 1:
            gs[0].reshape(-1)[7] = bad
        return gs

    _run(mmn, oracle, grads_for, steps=2)
