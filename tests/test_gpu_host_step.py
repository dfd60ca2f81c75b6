"""mmn_optim_step_host: the step from host buffers (grads in, params out, copies
pipelined per chunk) must give bit for bit what the device-resident step gives
for the same grads: the copies move bytes and change no arithmetic. The model
has more than 16 matrices of one shape (and their transposes) so that a shape
class is split into several Newton-Schulz chunks."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _model():
    shapes = [(256, 512)] * 20 + [(512, 256)] * 5 + [(128, 128)] * 17
    shapes += [(1000, 64), (64,), (300,), (7, 5), (3, 3, 4)]
    routes = ["auto"] * len(shapes)
    routes[shapes.index((1000, 64))] = "adamw"
    return [(k, s, r) for k, (s, r) in enumerate(zip(shapes, routes))]


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    import torch

    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).bfloat16().view(
        torch.int16).numpy().view(np.uint16).copy()


def _grads(rng, model, bf16: bool, scale: float = 1.0):
    out = []
    for _, s, _ in model:
        g = rng.normal(0, 1e-3, s).astype(np.float32) * np.float32(scale)
        out.append(_bf16_bits(g) if bf16 else g)
    return out


def _pair(mmn, model, **cfg):
    rng = np.random.default_rng(7)
    a = mmn.OptimizerStep(model, mmn.StepConfig(**cfg), device=0)
    b = mmn.OptimizerStep(model, mmn.StepConfig(**cfg), device=0)
    for k, (_, s, _) in enumerate(model):
        p = rng.normal(0, 0.02, s).astype(np.float32)
        a.set_param(k, p)
        b.set_param(k, p)
    return a, b


def _device_step(step, grads, divisor=1.0):
    for k, g in enumerate(grads):
        step.set_grad(k, g)
    step.step(divisor)
    step.sync()
    return [step.get_param(k) for k in range(len(grads))]


def _same(x, y, what):
    np.testing.assert_array_equal(np.asarray(x).view(np.uint32), np.asarray(y).view(np.uint32),
                                  err_msg=what)


@pytest.mark.parametrize("variant", ["f32", "ns0", "bf16_loss_scale"])
def test_host_step_equals_device_step(mmn, variant):
    model = _model()
    bf = variant == "bf16_loss_scale"
    cfg = dict(use_graph=False)
    if variant == "ns0":
        cfg["muon"] = mmn.MuonConfig(ns_steps=0)
    if bf:
        cfg.update(grad_dtype="bf16", bf16_param_shadow=True, loss_scaling=True,
                   loss_scale_init=1024.0, growth_interval=2)
    a, b = _pair(mmn, model, **cfg)
    rng = np.random.default_rng(11)
    for it in range(3):
        grads = _grads(rng, model, bf, 1024.0 if bf else 1.0)
        if bf and it == 1:
            grads[3].reshape(-1)[5] = 0x7F80  # +inf: the step is skipped everywhere
        divisor = 2.0 if it == 2 else 1.0
        want = _device_step(a, grads, divisor)
        out = [np.full(s, np.nan, np.float32) for _, s, _ in model]
        b.step_host(grads, out, divisor)
        for k in range(len(model)):
            _same(out[k], want[k], f"{variant} step {it} slot {k} (host output)")
            _same(b.get_param(k), want[k], f"{variant} step {it} slot {k} (device master)")
        if bf:
            assert b.loss_scale() == a.loss_scale()
    if bf:
        assert a.loss_scale()[1] == 1
    assert b.adamw_step == a.adamw_step
    a.close()
    b.close()


def test_host_step_pinned_tensors_and_skipped_slots(mmn):
    import torch

    model = _model()
    a, b = _pair(mmn, model, use_graph=False)
    rng = np.random.default_rng(3)
    grads = _grads(rng, model, False)
    want = _device_step(a, grads)

    # pinned torch buffers; slot 0's grad is placed on the device beforehand
    # (None = no copy in), odd slots' params are not read back (None)
    pin_g = [None if k == 0 else torch.from_numpy(g).pin_memory() for k, g in enumerate(grads)]
    b.set_grad(0, grads[0])
    pin_p = [None if k % 2 else torch.full(s, float("nan")).pin_memory()
             for k, (_, s, _) in enumerate(model)]
    b.step_host(pin_g, pin_p)
    for k in range(len(model)):
        if pin_p[k] is not None:
            _same(pin_p[k].numpy(), want[k], f"slot {k} (pinned output)")
        _same(b.get_param(k), want[k], f"slot {k} (device master)")

    # a second step from pinned buffers matches a second device step
    grads2 = _grads(rng, model, False)
    want2 = _device_step(a, grads2)
    pin_p2 = [torch.empty(s).pin_memory() for _, s, _ in model]
    b.step_host([torch.from_numpy(g).pin_memory() for g in grads2], pin_p2)
    for k in range(len(model)):
        _same(pin_p2[k].numpy(), want2[k], f"slot {k} (second step)")
    a.close()
    b.close()


def test_host_step_rejects_bad_buffers(mmn):
    model = _model()
    step = mmn.OptimizerStep(model, mmn.StepConfig(use_graph=False), device=0)
    grads = [np.zeros(s, np.float32) for _, s, _ in model]
    params = [np.zeros(s, np.float32) for _, s, _ in model]
    with pytest.raises(ValueError):
        step.step_host(grads[:-1], params)
    bad = list(grads)
    bad[2] = np.zeros(7, np.float32)
    with pytest.raises(ValueError):
        step.step_host(bad, params)
    bad = list(params)
    bad[1] = np.zeros(model[1][1], np.float64)
    with pytest.raises(ValueError):
        step.step_host(grads, bad)
    step.close()
