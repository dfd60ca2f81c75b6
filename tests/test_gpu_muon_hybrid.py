"""Muon::step_matrix, HybridOptimizer::step and the batched whole-model step on
the GPU against the oracle, on the Chatbot (vocab 512, 2 layers,
d_model 64) with grads ~ N(0, 1e-3) for three consecutive steps.

Tolerances: AdamW tensors bit-exact; Muon velocity bit-exact; Muon parameter
updates within 2e-2 relative Frobenius (see test_gpu_newton_schulz.py for why
the bf16 rounding points of the reference recipe set that floor)."""
import numpy as np
import pytest

from conftest import chatbot_params, rel_fro

pytestmark = pytest.mark.gpu

ADAMW = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_muon_step_matrix_vs_oracle(mmn, oracle):
    rng = np.random.default_rng(0)
    shapes = [(64, 64), (64, 256), (256, 64), (512, 64), (33, 17)]
    gpu = mmn.Muon(mmn.MuonConfig())
    ref = oracle.Muon(oracle.MuonConfig(), order=oracle.GEMM_F64)
    ps = [rng.normal(0, 0.02, s).astype(np.float32) for s in shapes]
    pr = [p.copy() for p in ps]
    for step in range(3):
        for i, s in enumerate(shapes):
            g = rng.normal(0, 1e-3, s).astype(np.float32)
            before = pr[i].copy()
            gpu.step_matrix(i, ps[i], g)
            ref.step_matrix(i, pr[i], g)
            assert rel_fro(ps[i] - before, pr[i] - before) <= 2e-2, (step, s)
            # velocity arithmetic is elementwise: bit-exact
            np.testing.assert_array_equal(bits(gpu.export_velocity(i, s)), bits(ref.velocity[i]))
            ps[i][:] = pr[i]  # re-align so the next step starts from the same params


def test_muon_reference_unit_test(mmn):
    """lib.rs:330-342 muon_step_matrix_changes_weights."""
    p = np.fromfunction(lambda i, j: 1.0 + (i + j) * 0.01, (4, 4)).astype(np.float32)
    g = np.fromfunction(lambda i, j: 0.1 + i * 0.02 + j * 0.03, (4, 4)).astype(np.float32)
    before = p.copy()
    mmn.Muon(mmn.MuonConfig(lr=0.1)).step_matrix(0, p, g)
    assert not np.array_equal(p, before)


def test_hybrid_routes_like_reference(mmn):
    """lib.rs:344-369: a 4x4 matrix goes to Muon, a [3,1] column to AdamW."""
    opt = mmn.HybridOptimizer(mmn.MuonConfig(lr=0.1), mmn.AdamWConfig())
    p = np.fromfunction(lambda i, j: 1.0 + (i + j) * 0.01, (4, 4)).astype(np.float32)
    g = np.fromfunction(lambda i, j: 0.1 + i * 0.02 + j * 0.03, (4, 4)).astype(np.float32)
    before = p.copy()
    opt.step(0, p, g)
    assert not np.array_equal(p, before)
    assert opt.adamw.step == 0
    v = np.array([[1.0], [2.0], [3.0]], np.float32)
    opt.step(1, v, np.full((3, 1), 0.5, np.float32))
    assert v[0, 0] != 1.0 and opt.adamw.step == 1


def _run_chatbot(mmn, oracle, routing, id_scheme, batched, use_graph=True):
    rng = np.random.default_rng(0)
    named = chatbot_params(rng)
    order = [n for n, _ in named]
    p_gpu = {n: v.copy() for n, v in named}
    p_ref = {n: v.copy() for n, v in named}
    tagged = routing == "tagged"

    def route(name, shape):
        if tagged and (name in ("embed", "lm_head") or len(shape) == 1):
            return "adamw"
        return "auto"

    ref = oracle.HybridOptimizer(oracle.MuonConfig(), oracle.AdamWConfig(**ADAMW),
                                 order=oracle.GEMM_F64)
    if batched:
        step = mmn.OptimizerStep(
            [(k, p_gpu[n].shape, route(n, p_gpu[n].shape)) for k, n in enumerate(order)],
            mmn.StepConfig(adamw=mmn.AdamWConfig(**ADAMW), muon=mmn.MuonConfig(),
                           fresh_state=id_scheme == "train", use_graph=use_graph))
        for k, n in enumerate(order):
            step.set_param(k, p_gpu[n])
    else:
        hyb = mmn.HybridOptimizer(mmn.MuonConfig(), mmn.AdamWConfig(**ADAMW))
    worst = 0.0
    for s in range(3):
        grads = {n: rng.normal(0, 1e-3, p_ref[n].shape).astype(np.float32) for n in order}
        before = {n: p_ref[n].copy() for n in order}
        for k, n in enumerate(order):
            pid = k if id_scheme == "stable" else 22 * s + k
            r = route(n, p_ref[n].shape)
            ref.step(pid, p_ref[n], grads[n],
                     route=None if r == "auto" else ("Other" if r == "adamw" else "Matrix"))
            if batched:
                step.set_grad(k, grads[n])
            else:
                hyb.step(pid, p_gpu[n], grads[n],
                         route=None if r == "auto" else ("Other" if r == "adamw" else "Matrix"))
        if batched:
            step.step()
            step.sync()
            for k, n in enumerate(order):
                p_gpu[n] = step.get_param(k)
        for n in order:
            kind = route(n, p_ref[n].shape)
            is_muon = kind == "muon" or (kind == "auto" and oracle.classify_param(p_ref[n].shape)
                                          == oracle.MATRIX)
            if is_muon:
                err = rel_fro(p_gpu[n] - before[n], p_ref[n] - before[n])
                worst = max(worst, err)
                assert err <= 2e-2, (s, n, err)
                p_gpu[n][:] = p_ref[n]  # next step starts from the same params
                if batched:
                    step.set_param(order.index(n), p_gpu[n])
            else:
                np.testing.assert_array_equal(bits(p_gpu[n]), bits(p_ref[n]), err_msg=n)
    return worst


@pytest.mark.parametrize("routing", ["reference", "tagged"])
@pytest.mark.parametrize("id_scheme", ["stable", "train"])
def test_chatbot_hybrid_per_call(mmn, oracle, routing, id_scheme):
    _run_chatbot(mmn, oracle, routing, id_scheme, batched=False)


@pytest.mark.parametrize("routing", ["reference", "tagged"])
@pytest.mark.parametrize("id_scheme", ["stable", "train"])
@pytest.mark.parametrize("use_graph", [True, False])
def test_chatbot_hybrid_batched(mmn, oracle, routing, id_scheme, use_graph):
    _run_chatbot(mmn, oracle, routing, id_scheme, batched=True, use_graph=use_graph)
