"""bf16 grads with fp32 master params, dynamic loss scaling, non-finite skip
and bf16 parameter copies (the step of the 5.36e9-parameter GQA model) against the oracle's
definition of that behaviour (oracle.LossScaleState)."""
import numpy as np
import pytest

from conftest import chatbot_params, rel_fro

pytestmark = pytest.mark.gpu

ADAMW = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("use_graph", [True, False])
def test_loss_scaled_bf16_step_with_skip_and_growth(mmn, oracle, use_graph):
    rng = np.random.default_rng(0)
    named = chatbot_params(rng)
    order = [n for n, _ in named]
    p_ref = {n: v.copy() for n, v in named}
    step = mmn.OptimizerStep(
        [(k, p_ref[n].shape) for k, n in enumerate(order)],
        mmn.StepConfig(adamw=mmn.AdamWConfig(**ADAMW), muon=mmn.MuonConfig(), grad_dtype="bf16",
                       bf16_param_shadow=True, loss_scaling=True, loss_scale_init=65536.0,
                       growth_interval=2, use_graph=use_graph))
    for k, n in enumerate(order):
        step.set_param(k, p_ref[n])
    ref = oracle.HybridOptimizer(oracle.MuonConfig(), oracle.AdamWConfig(**ADAMW),
                                 order=oracle.GEMM_F64)
    ls = oracle.LossScaleState(65536.0, growth_interval=2)
    muon_k = [k for k, n in enumerate(order) if oracle.classify_param(p_ref[n].shape) == oracle.MATRIX]
    for s in range(5):
        raw = {n: rng.normal(0, 1e-3, p_ref[n].shape).astype(np.float32) for n in order}
        scaled = {n: oracle.bf16_round(raw[n] * ls.scale) for n in order}
        if s == 1:  # one injected non-finite grad
            scaled[order[muon_k[0]]].reshape(-1)[7] = np.inf
        for k, n in enumerate(order):
            step.set_grad(k, oracle.bf16_bits(scaled[n]))
        before = {k: step.get_param(k) for k in range(len(order))}
        state_before = {k: step.get_state(k, "velocity" if k in muon_k else "m")
                        for k in range(len(order))}
        t_before = step.adamw_step
        step.step()
        step.sync()
        ok = ls.check(scaled.values())
        if ok:
            for k, n in enumerate(order):
                ref.step(k, p_ref[n], ls.unscale(scaled[n]))
        ls.update(ok)
        scale, skipped = step.loss_scale()
        assert scale == ls.scale and skipped == ls.skipped, (s, scale, ls.scale)
        if not ok:
            assert step.adamw_step == t_before
            for k in range(len(order)):
                np.testing.assert_array_equal(bits(step.get_param(k)), bits(before[k]))
                st = step.get_state(k, "velocity" if k in muon_k else "m")
                np.testing.assert_array_equal(bits(st), bits(state_before[k]))
            continue
        for k, n in enumerate(order):
            got = step.get_param(k)
            if k in muon_k:
                assert rel_fro(got - before[k], p_ref[n] - before[k]) <= 2e-2, (s, n)
                step.set_param(k, p_ref[n])  # realign
                got = p_ref[n]
            else:
                np.testing.assert_array_equal(bits(got), bits(p_ref[n]), err_msg=n)
            shadow = step.param_bf16(k).float().cpu().numpy()
            np.testing.assert_array_equal(bits(shadow), bits(oracle.bf16_round(step.get_param(k))))
    # growth: 3 clean steps after the skip with interval 2 -> one doubling
    assert ls.scale == np.float32(65536.0)
