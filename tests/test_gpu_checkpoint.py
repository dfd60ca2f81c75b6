"""Optimizer-state checkpoints on the GPU: stepping, saving, loading into a
fresh handle and stepping both again must give identical parameters and state
bit for bit (resume equivalence), including the AdamW call counter and the
loss-scaling state after a skipped step."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MODEL = ([(f"m{i}", (96, 160), "auto") for i in range(18)] +
         [(f"t{i}", (160, 96), "auto") for i in range(3)] +
         [("ln.gamma", (160,), "auto"), ("emb", (300, 64), "adamw"), ("odd", (7, 5), "auto")])


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _grads(rng, bf16, scale=1.0):
    import torch

    out = []
    for _, s, _ in MODEL:
        g = rng.normal(0, 1e-3, s).astype(np.float32) * np.float32(scale)
        out.append(torch.from_numpy(g).bfloat16().view(torch.int16).numpy().view(np.uint16)
                   if bf16 else g)
    return out


def _handle(mmn, cfg, params):
    step = mmn.OptimizerStep([(k, s, r) for k, (_, s, r) in enumerate(MODEL)], cfg, device=0)
    for k, p in enumerate(params):
        step.set_param(k, p)
    return step


def _run(step, grads):
    for k, g in enumerate(grads):
        step.set_grad(k, g)
    step.step()
    step.sync()


@pytest.mark.parametrize("bf16", [False, True])
def test_resume_from_checkpoint_is_bit_exact(mmn, tmp_path, bf16):
    rng = np.random.default_rng(5)
    cfg = (mmn.StepConfig(grad_dtype="bf16", bf16_param_shadow=True, loss_scaling=True,
                          loss_scale_init=1024.0, growth_interval=3, use_graph=False)
           if bf16 else mmn.StepConfig(use_graph=False))
    params = [rng.normal(0, 0.02, s).astype(np.float32) for _, s, _ in MODEL]
    names = [n for n, _, _ in MODEL]
    a = _handle(mmn, cfg, params)
    for it in range(3):
        g = _grads(rng, bf16, 1024.0 if bf16 else 1.0)
        if bf16 and it == 1:
            g[2].reshape(-1)[3] = 0x7F80  # +inf: skipped, scale halves
        _run(a, g)
    path = str(tmp_path / "optim.safetensors")
    mmn.save_state(a, path, names)
    b = _handle(mmn, cfg, [a.get_param(k) for k in range(len(MODEL))])
    mmn.load_state(b, path, names)
    assert b.adamw_step == a.adamw_step
    assert b.loss_state() == a.loss_state()
    for it in range(2):
        g = _grads(rng, bf16, 1024.0 if bf16 else 1.0)
        _run(a, g)
        _run(b, g)
    for k, (name, s, _) in enumerate(MODEL):
        np.testing.assert_array_equal(_bits(a.get_param(k)), _bits(b.get_param(k)), err_msg=name)
        which = ("m", "v") if a.routes[k] == "adamw" else ("velocity",)
        for w in which:
            np.testing.assert_array_equal(_bits(a.get_state(k, w)), _bits(b.get_state(k, w)),
                                          err_msg=f"{name}.{w}")
    assert b.loss_state() == a.loss_state()
    if bf16:
        assert a.loss_state()[1] == 1
    a.close()
    b.close()


def test_load_rejects_a_different_handle(mmn, tmp_path):
    rng = np.random.default_rng(6)
    params = [rng.normal(0, 0.02, s).astype(np.float32) for _, s, _ in MODEL]
    a = _handle(mmn, mmn.StepConfig(use_graph=False), params)
    _run(a, _grads(rng, False))
    path = str(tmp_path / "optim.safetensors")
    mmn.save_state(a, path)
    other = _handle(mmn, mmn.StepConfig(adamw=mmn.AdamWConfig(lr=1e-3), use_graph=False), params)
    with pytest.raises(ValueError):
        mmn.load_state(other, path)
    with pytest.raises(ValueError):
        mmn.load_state(a, path, [f"x{k}" for k in range(len(MODEL))])
    a.close()
    other.close()
