"""The AdamW-only callers of the reference reuse the same batched step: the
Classifier's train_step (head, then backbone; crates/mmn-models/src/chatbot.rs:
1483-1548) and the diffusion UNet's train_step_denoise (down, mid, up conv
weights; :2277-2320). Both pass a fresh param_id on every call, so AdamW state
starts at zero each call while the instance step count keeps advancing. The
batched step with use_hybrid = False and fresh_state must equal the oracle's
per-call AdamW sequence bit for bit."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("which", ["classifier", "diffusion"])
def test_adamw_only_callers_batched_equals_per_call(mmn, oracle, which):
    order = (mmn.classifier_param_order(5, 48) if which == "classifier"
             else mmn.diffusion_param_order())
    rng = np.random.default_rng(21)
    cfg = mmn.StepConfig(adamw=mmn.AdamWConfig(lr=1e-3), use_hybrid=False, fresh_state=True,
                         use_graph=False)
    step = mmn.OptimizerStep([(k, s) for k, (_, s) in enumerate(order)], cfg, device=0)
    assert step.routes == ["adamw"] * len(order)
    ref = oracle.AdamW(oracle.AdamWConfig(1e-3, (0.9, 0.95), 1e-8, 0.01))
    params = [rng.normal(0, 0.05, s).astype(np.float32) for _, s in order]
    for k, p in enumerate(params):
        step.set_param(k, p)
    param_id = 0
    for _ in range(3):
        grads = [rng.normal(0, 1e-2, s).astype(np.float32) for _, s in order]
        for k, g in enumerate(grads):
            step.set_grad(k, g)
            ref.step_param(param_id, params[k], g)  # a new id every call
            param_id += 1
        step.step()
        step.sync()
    for k, (name, _) in enumerate(order):
        np.testing.assert_array_equal(_bits(step.get_param(k)), _bits(params[k]), err_msg=name)
    assert step.adamw_step == ref.step == 3 * len(order)
    step.close()
