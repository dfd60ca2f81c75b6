"""Reference-mode Muon parity at full size, one matrix of every shape class the
two large benchmark configurations step.

  - the 1.34e9-parameter configuration (d_model 2048, FFN 8192): q/k/v/out
    [2048, 2048], ffn [8192, 2048] (stepped transposed: the fused last
    iteration writes the transposed fp32 parameters) and ffn2 [2048, 8192]
    (the CTA-pair transposed Poly with K = 2048), inside the real whole-model
    step;
  - the 5.36e9-parameter configuration (d_model 4096, GQA k/v [1024, 4096], FFN
    14336): q/out [4096, 4096], k/v [1024, 4096], ffn [14336, 4096] and ffn2
    [4096, 14336], two layers of them stepped together in fp32.

Each checked matrix carries a non-zero velocity, so the comparison covers the
whole Muon step of crates/mmn-optim/src/lib.rs:141-175: momentum, Nesterov
input, newton_schulz5 (:83-126) and p -= lr * sqrt(rows/cols) * O. The oracle
runs the same recipe with float64 products (GEMM_BLAS64, equal bit for bit to
its fp64 order on smaller shapes). Bars: the update within 2e-2 relative
Frobenius (the reference-mode tolerance), velocity bit-exact, and one
iteration from the same input within 1e-3."""
import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu


def _oracle_muon(oracle, p0, g, vel0, cfg):
    ref = oracle.Muon(oracle.MuonConfig(cfg.lr, cfg.momentum, cfg.nesterov, cfg.ns_steps),
                      order=oracle.GEMM_BLAS64)
    ref.velocity[0] = vel0.copy()
    p = p0.copy()
    ref.step_matrix(0, p, g)
    return p, ref.velocity[0]


def _check_slots(mmn, oracle, step, names, slots, vel0):
    cfg = mmn.MuonConfig()
    before = {k: (step.param(k).cpu().numpy(), step.grad(k).cpu().numpy()) for k in slots}
    step.step()
    step.sync()
    for k in slots:
        p0, g = before[k]
        p_ref, vel_ref = _oracle_muon(oracle, p0, g, vel0[k], cfg)
        p_gpu = step.param(k).cpu().numpy()
        vel_gpu = step.get_state(k, "velocity")
        np.testing.assert_array_equal(vel_gpu.view(np.uint32), vel_ref.view(np.uint32),
                                      err_msg=names[k])
        rel = rel_fro(p_gpu - p0, p_ref - p0)
        assert rel <= 2e-2, f"{names[k]} {p0.shape}: update differs by {rel:.3e}"


def _seed_velocity(step, slots, shapes, seed):
    rng = np.random.default_rng(seed)
    vel0 = {}
    for k in slots:
        v = rng.normal(0, 1e-3, shapes[k]).astype(np.float32)
        step.set_state(k, "velocity", v)
        vel0[k] = v
    return vel0


def test_hybrid_1b_every_muon_shape_class(mmn, oracle):
    import torch

    import bench

    model = bench.WORKLOADS["hybrid_1b"]["model"]()
    names = [n for n, _, _ in model]
    shapes = [s for _, s, _ in model]
    step = mmn.OptimizerStep([(k, s, r) for k, (_, s, r) in enumerate(model)],
                             mmn.StepConfig(use_graph=False), device=0)
    gen = torch.Generator(device="cuda").manual_seed(0)
    for k, (_, s, _) in enumerate(model):
        step.param(k).normal_(0, 0.02, generator=gen)
        step.grad(k).normal_(0, 1e-3, generator=gen)
    slots = [names.index(n) for n in ("blocks.0.ffn", "blocks.0.ffn2", "blocks.0.q",
                                      "blocks.23.k")]
    vel0 = _seed_velocity(step, slots, shapes, 1)
    _check_slots(mmn, oracle, step, names, slots, vel0)
    step.close()


def _layers_8b(n_layer=2):
    d, kv, ffn = 4096, 1024, 14336
    out = []
    for layer in reversed(range(n_layer)):
        b = f"blocks.{layer}."
        out += [(b + "ffn2", (d, ffn)), (b + "ffn", (ffn, d)), (b + "out", (d, d)),
                (b + "q", (d, d)), (b + "k", (kv, d)), (b + "v", (kv, d))]
    return out


def test_hybrid_8b_every_muon_shape_class(mmn, oracle):
    import torch

    layers = _layers_8b()
    names = [n for n, _ in layers]
    shapes = [s for _, s in layers]
    step = mmn.OptimizerStep([(k, s, "muon") for k, s in enumerate(shapes)],
                             mmn.StepConfig(use_graph=False), device=0)
    gen = torch.Generator(device="cuda").manual_seed(2)
    for k in range(len(layers)):
        step.param(k).normal_(0, 0.02, generator=gen)
        step.grad(k).normal_(0, 1e-3, generator=gen)
    slots = [names.index(n) for n in ("blocks.1.ffn2", "blocks.1.ffn", "blocks.0.q",
                                      "blocks.0.v")]
    vel0 = _seed_velocity(step, slots, shapes, 3)
    _check_slots(mmn, oracle, step, names, slots, vel0)
    step.close()


@pytest.mark.parametrize("shape", [(2048, 2048), (2048, 8192), (1024, 4096), (4096, 4096),
                                   (4096, 14336)])
def test_one_iteration_full_size(mmn, oracle, shape):
    """The first iteration (division by the norm, A = bf16(XX^T), A2, the
    polynomial) from the same bf16 input: next X within 1e-3 of the oracle."""
    from test_gpu_newton_schulz import first_iter_input, gpu_iteration

    rng = np.random.default_rng(sum(shape))
    n, m = shape
    y, norm = first_iter_input(oracle, rng, n, m)
    _, _, xn = gpu_iteration(mmn, y, norm)
    x0 = (y / norm).astype(np.float32)
    xn_ref = oracle.ns_iteration(x0, oracle.GEMM_BLAS64)
    assert rel_fro(xn, xn_ref) <= 1e-3
