"""The benchmark configurations at full size, checked through properties that do
not need the oracle to run the whole workload:

  - AdamW on the 2^28-element arena (t = 10, wd 0.1, divisor 4): elementwise, so
    2^20 sampled elements (plus both ends) must match the oracle bit for bit;
  - Newton-Schulz on 64 x [4096, 4096] + 32 x [4096, 14336]: run-to-run
    determinism of the whole batch, independence from the batch a matrix runs
    in, and the transpose rule NS(G^T) = NS(G)^T at the largest shape;
  - the 1.34e9-parameter hybrid step: sampled AdamW elements bit-exact against the
    oracle, one [2048, 2048] Muon matrix against the oracle's Muon step within the
    Newton-Schulz tolerance (2e-2 relative Frobenius of the update);
  - the 5.36e9-parameter step with bf16 grads and loss scaling: a non-finite grad
    anywhere leaves every parameter and the AdamW counter unchanged and halves
    the scale; the next clean step moves the parameters.

Everything is generated on the device from fixed seeds."""
import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _sample_idx(n, k, seed):
    rng = np.random.default_rng(seed)
    idx = np.unique(np.concatenate([rng.integers(0, n, k), np.arange(8), n - 1 - np.arange(8)]))
    return idx


def test_adamw_arena_2p28_sampled_bitexact(mmn, oracle):
    import torch

    n = 1 << 28
    cfg = mmn.StepConfig(adamw=mmn.AdamWConfig(lr=3e-4, betas=(0.9, 0.95), eps=1e-8,
                                               weight_decay=0.1), use_graph=False)
    step = mmn.OptimizerStep([(0, (n,), "adamw")], cfg, device=0)
    gen = torch.Generator(device="cuda").manual_seed(0)
    step.param(0).normal_(0, 0.02, generator=gen)
    step.grad(0).normal_(0, 1e-2, generator=gen)
    m = torch.empty(n, device="cuda").normal_(0, 1e-3, generator=gen)
    v = torch.empty(n, device="cuda").normal_(0, 1e-4, generator=gen).abs_()
    step.set_state(0, "m", m.cpu().numpy())
    step.set_state(0, "v", v.cpu().numpy())
    step.adamw_step = 9  # this step runs at t = 10
    idx_t = torch.from_numpy(_sample_idx(n, 1 << 20, 1)).cuda()
    p0 = step.param(0)[idx_t].cpu().numpy()
    g0 = step.grad(0)[idx_t].cpu().numpy()
    m0, v0 = m[idx_t].cpu().numpy(), v[idx_t].cpu().numpy()
    del m, v
    step.step(4.0)
    step.sync()
    p1 = step.param(0)[idx_t].cpu().numpy()
    m1 = step.get_state(0, "m")[idx_t.cpu().numpy()]
    oracle.adamw_update(p0, m0, v0, g0, lr=3e-4, betas=(0.9, 0.95), eps=1e-8,
                        weight_decay=0.1, t=10, grad_divisor=4.0)
    np.testing.assert_array_equal(_bits(p1), _bits(p0))
    np.testing.assert_array_equal(_bits(m1), _bits(m0))
    assert step.adamw_step == 10
    step.close()


NS_BATCH_SHAPES = [(4096, 4096)] * 64 + [(4096, 14336)] * 32


def _ns_handle(mmn, shapes, seed_of):
    """Muon-only step over `shapes`; matrix k gets grads from seed seed_of(k),
    params zero, so p_new = -(lr * scale) * O exactly."""
    import torch

    step = mmn.OptimizerStep([(k, s, "muon") for k, s in enumerate(shapes)],
                             mmn.StepConfig(use_graph=False), device=0)
    for k, s in enumerate(shapes):
        gen = torch.Generator(device="cuda").manual_seed(seed_of(k))
        step.param(k).zero_()
        step.grad(k).normal_(0, 1e-2, generator=gen)
    return step


def test_newton_schulz_4096_batch_deterministic_and_batch_independent(mmn):
    import torch

    a = _ns_handle(mmn, NS_BATCH_SHAPES, lambda k: 1000 + k)
    a.step()
    a.sync()
    b = _ns_handle(mmn, NS_BATCH_SHAPES, lambda k: 1000 + k)
    b.step()
    b.sync()
    for k in range(len(NS_BATCH_SHAPES)):
        assert torch.equal(a.param(k), b.param(k)), k
    b.close()
    # the same matrices in other batches (a chunk of their own, other neighbours)
    pick = [0, 37, 63, 64, 80, 95]
    c = _ns_handle(mmn, [NS_BATCH_SHAPES[k] for k in pick], lambda j: 1000 + pick[j])
    c.step()
    c.sync()
    for j, k in enumerate(pick):
        assert torch.equal(c.param(j), a.param(k)), k
        assert torch.isfinite(a.param(k)).all()
    a.close()
    c.close()


def test_newton_schulz_transpose_rule_full_size(mmn):
    import torch

    gen = torch.Generator(device="cuda").manual_seed(7)
    g = torch.empty((4096, 14336), device="cuda").normal_(0, 1e-2, generator=gen)
    o = mmn.newton_schulz5(g)
    ot = mmn.newton_schulz5(g.t().contiguous())
    torch.cuda.synchronize()
    assert torch.equal(ot, o.t())
    assert torch.isfinite(o).all()


def _hybrid_step(mmn, model, cfg):
    import torch

    step = mmn.OptimizerStep([(k, s, r) for k, (_, s, r) in enumerate(model)], cfg, device=0)
    gen = torch.Generator(device="cuda").manual_seed(0)
    for k, (_, s, _) in enumerate(model):
        step.param(k).normal_(0, 0.02, generator=gen)
        gv = step.grad(k)
        if gv.dtype == torch.bfloat16:
            gv.copy_(torch.randn(s, device="cuda", generator=gen) * (1e-3 * 65536.0))
        else:
            gv.normal_(0, 1e-3, generator=gen)
    return step


def test_hybrid_1b_full_step_sampled_parity(mmn, oracle):
    import torch

    import bench

    model = bench.WORKLOADS["hybrid_1b"]["model"]()
    step = _hybrid_step(mmn, model, mmn.StepConfig(use_graph=False))
    names = [n for n, _, _ in model]
    # AdamW: lm_head (first call, t = 1), a LayerNorm vector, embed (last call)
    a_slots = [names.index("lm_head"), names.index("blocks.11.ln2.gamma"), names.index("embed")]
    t_of = {}
    t = 0
    for k, (_, _, r) in enumerate(model):
        if r == "adamw":
            t += 1
            t_of[k] = t
    before = {}
    for k in a_slots:
        n = step.param(k).numel()
        idx = torch.from_numpy(_sample_idx(n, 1 << 16, k)).cuda()
        before[k] = (idx, step.param(k).view(-1)[idx].cpu().numpy(),
                     step.grad(k).view(-1)[idx].cpu().numpy())
    q = names.index("blocks.0.q")
    q_p0 = step.param(q).cpu().numpy()
    q_g = step.grad(q).cpu().numpy()
    step.step()
    step.sync()
    cfg = mmn.AdamWConfig()
    for k, (idx, p0, g0) in before.items():
        m0 = np.zeros_like(p0)
        v0 = np.zeros_like(p0)
        oracle.adamw_update(p0, m0, v0, g0, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                            weight_decay=cfg.weight_decay, t=t_of[k])
        np.testing.assert_array_equal(_bits(step.param(k).view(-1)[idx].cpu().numpy()),
                                      _bits(p0), err_msg=names[k])
    ref = oracle.Muon(oracle.MuonConfig())
    q_ref = q_p0.copy()
    ref.step_matrix(0, q_ref, q_g)
    q_gpu = step.param(q).cpu().numpy()
    assert rel_fro(q_gpu - q_p0, q_ref - q_p0) <= 2e-2
    step.close()


def test_hybrid_8b_full_nonfinite_skip_then_step(mmn):
    import torch

    import bench

    model = bench.WORKLOADS["hybrid_8b"]["model"]()
    cfg = mmn.StepConfig(grad_dtype="bf16", bf16_param_shadow=True, loss_scaling=True,
                         loss_scale_init=65536.0, use_graph=False)
    step = _hybrid_step(mmn, model, cfg)
    gl = step.gather_layout()
    from magicmindnet_b200.step import _view

    arenas = [_view(gl["adamw_param"], (gl["adamw_region"],), "f32", 0),
              _view(gl["muon_param"], (gl["muon_region"],), "f32", 0)]

    def checksum(a):  # exact: integer sum of the bit patterns, in pieces
        return sum(int(c.view(torch.int32).sum(dtype=torch.int64)) for c in a.split(1 << 27))

    sums0 = [checksum(a) for a in arenas]
    snap = [a[: 1 << 24].clone() for a in arenas]
    scale0, skipped0 = step.loss_scale()
    t0 = step.adamw_step
    # one +inf in the last Muon matrix's grads: the whole step is skipped
    last = max(k for k, (_, _, r) in enumerate(model) if r == "muon")
    step.grad(last).view(-1)[12345] = float("inf")
    step.step()
    step.sync()
    assert step.loss_scale() == (scale0 / 2, skipped0 + 1)
    assert step.adamw_step == t0
    for a, s0, sn in zip(arenas, sums0, snap):
        assert checksum(a) == s0
        assert torch.equal(a[: 1 << 24], sn)
    # clean grads again: the next step moves every arena
    step.grad(last).view(-1)[12345] = 0.0
    step.step()
    step.sync()
    assert step.loss_scale()[1] == skipped0 + 1
    assert step.adamw_step == t0 + sum(1 for _, _, r in model if r == "adamw")
    for a, sn in zip(arenas, snap):
        assert not torch.equal(a[: 1 << 24], sn)
        assert torch.isfinite(a[: 1 << 24]).all()
    step.close()
