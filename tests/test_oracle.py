"""The CPU oracle against the reference's own known answers and against
closed forms derived from the arithmetic of crates/mmn-optim/src/lib.rs.
No GPU needed."""
import os

import numpy as np
import pytest

from conftest import rel_fro


def test_reference_grad_accumulator_average(oracle):
    """lib.rs:283-293: the average of 1 and 3 is 2 within 1e-6."""
    acc = oracle.GradAccumulator()
    acc.begin_micro_batch()
    acc.add_param_grad(np.array([[1.0]], np.float32))
    acc.finish_micro_batch()
    acc.begin_micro_batch()
    acc.add_param_grad(np.array([[3.0]], np.float32))
    acc.finish_micro_batch()
    assert abs(acc.averaged_grad(0)[0, 0] - 2.0) < 1e-6


def test_reference_grad_accumulator_clear(oracle):
    """lib.rs:371-381."""
    acc = oracle.GradAccumulator()
    acc.begin_micro_batch()
    acc.add_param_grad(np.array([[1.0]], np.float32))
    acc.finish_micro_batch()
    assert acc.micro_batches == 1
    acc.clear()
    assert acc.micro_batches == 0 and len(acc) == 0


def test_reference_routing_table(oracle):
    """lib.rs:302-320."""
    assert oracle.classify_param((64, 32)) == oracle.MATRIX
    assert oracle.classify_param((16,)) == oracle.OTHER
    assert oracle.classify_param((16, 1)) == oracle.OTHER
    assert oracle.classify_param((1, 3, 3, 3)) == oracle.OTHER


def test_reference_ns_finite_and_nonzero(oracle):
    """lib.rs:295-300 and lib.rs:322-328."""
    assert np.isfinite(oracle.newton_schulz5(np.eye(2, dtype=np.float32))).all()
    g = np.fromfunction(lambda i, j: (i + j) * 0.1, (4, 4)).astype(np.float32)
    assert np.abs(oracle.newton_schulz5(g)).sum() > 1e-6


def test_reference_changes_weights(oracle):
    """lib.rs:269-280, 330-369."""
    p = np.array([[1.0]], np.float32)
    oracle.AdamW(oracle.AdamWConfig(lr=0.1)).step_param(0, p, np.array([[0.5]], np.float32))
    assert p[0, 0] != 1.0
    p = np.fromfunction(lambda i, j: 1.0 + (i + j) * 0.01, (4, 4)).astype(np.float32)
    g = np.fromfunction(lambda i, j: 0.1 + i * 0.02 + j * 0.03, (4, 4)).astype(np.float32)
    before = p.copy()
    oracle.Muon(oracle.MuonConfig(lr=0.1)).step_matrix(0, p, g)
    assert not np.array_equal(p, before)


def test_bf16_rounding_is_nearest_even(oracle):
    f = oracle.lib().ref_bf16_round
    one = np.float32(1.0)
    ulp = np.float32(2.0 ** -7)
    assert f(float(one + ulp / 2)) == 1.0  # tie -> even (1.0)
    assert f(float(one + ulp + ulp / 2)) == float(one + 2 * ulp)  # tie -> even (up)
    assert f(float(one + ulp / 2 + np.float32(2.0 ** -20))) == float(one + ulp)
    assert f(3.0e38) == float("inf") or f(3.0e38) > 3e38  # overflow rounds to inf
    assert np.isnan(f(float("nan")))


def test_adamw_first_call_closed_form(oracle):
    """First call, m = v = 0: m_hat ~ g and v_hat ~ g^2, so
    p' = (p - lr * g / (|g| + eps)) * (1 - lr * wd)."""
    rng = np.random.default_rng(0)
    p = rng.normal(0, 1, 1000).astype(np.float32)
    g = rng.normal(0, 1e-3, 1000).astype(np.float32)
    q = p.copy()
    oracle.AdamW(oracle.AdamWConfig(1e-3, (0.9, 0.999), 1e-8, 0.01)).step_param(0, q, g)
    want = (p.astype(np.float64) - 1e-3 * g / (np.abs(g) + 1e-8)) * (1 - 1e-3 * 0.01)
    np.testing.assert_allclose(q, want, rtol=1e-6, atol=1e-9)


def test_adamw_step_counter_is_per_instance(oracle):
    """The second tensor of a step uses t = 2 on its very first update."""
    rng = np.random.default_rng(1)
    opt = oracle.AdamW(oracle.AdamWConfig(1e-3, (0.9, 0.999), 1e-8, 0.0))
    a = rng.normal(0, 1, 8).astype(np.float32)
    b = rng.normal(0, 1, 8).astype(np.float32)
    g = rng.normal(0, 1e-3, 8).astype(np.float32)
    opt.step_param(0, a, g)
    b2 = b.copy()
    opt.step_param(1, b, g)
    m = (1 - np.float32(0.9)) * g
    v = (1 - np.float32(0.999)) * g * g
    mh = m / (1 - np.float32(0.9) ** 2)
    vh = v / (1 - np.float32(0.999) ** 2)
    np.testing.assert_allclose(b, b2 - 1e-3 * mh / (np.sqrt(vh) + 1e-8), rtol=1e-6)


def test_ns_scaled_identity_follows_scalar_recurrence(oracle):
    """NS of s*I_n stays diagonal; every diagonal entry follows
    x <- bf16(a*x + (b*bf16(x^2) + c*bf16(bf16(x^2)^2)) * x) from x0 = 1/sqrt(n)."""
    n = 8
    out = oracle.newton_schulz5(np.eye(n, dtype=np.float32) * 0.37)
    assert np.count_nonzero(out - np.diag(np.diag(out))) == 0
    x = np.float32(oracle.bf16_round(np.float32(0.37))) / np.float32(
        np.sqrt(np.float32(n) * oracle.bf16_round(np.float32(0.37)) ** 2))
    a, b, c = np.float32(3.4445), np.float32(-4.7750), np.float32(2.0315)
    for _ in range(5):
        x2 = oracle.bf16_round(np.float32(x * x))
        x4 = oracle.bf16_round(np.float32(x2 * x2))
        x = oracle.bf16_round(np.float32(x * a + np.float32(np.float32(x2 * b) + np.float32(x4 * c)) * x))
    np.testing.assert_allclose(np.diag(out), np.full(n, x), rtol=0, atol=0)


def test_tf32_round_known_answers(oracle):
    """Nearest-even on the 13 dropped mantissa bits; exact values unchanged."""
    f = np.float32
    cases = {
        0x3F800000: 0x3F800000,  # 1.0 exact
        0x3F801000: 0x3F800000,  # tie, kept value even -> down
        0x3F803000: 0x3F804000,  # tie, kept value odd -> up
        0x3F800FFF: 0x3F800000,  # below half -> down
        0x3F801001: 0x3F802000,  # above half -> up
        0xBF803000: 0xBF804000,  # sign kept
        0x7F800000: 0x7F800000,  # inf
    }
    for src, want in cases.items():
        x = np.array([src], np.uint32).view(f)
        assert oracle.tf32_round(x).view(np.uint32)[0] == want, hex(src)
        assert np.array([oracle.lib().ref_tf32_round(float(x[0]))], f).view(np.uint32)[0] == want


def test_ns_tf32_scaled_identity_follows_scalar_recurrence(oracle):
    """The TF32 recipe on s*I_n: every diagonal entry follows
    x <- tf32(a*x + (b*tf32(x^2) + c*tf32(tf32(x^2)^2)) * x) from x0 = 1/sqrt(n)."""
    n = 8
    out = oracle.newton_schulz5(np.eye(n, dtype=np.float32) * 0.37, variant=oracle.NS_TF32)
    assert np.count_nonzero(out - np.diag(np.diag(out))) == 0
    t = lambda v: oracle.tf32_round(np.array([v], np.float32))[0]
    y = t(np.float32(0.37))
    s = np.float32(0)
    for _ in range(n):
        s = np.float32(s + np.float32(y * y))
    x = np.float32(y / np.float32(np.sqrt(s)))
    a, b, c = np.float32(3.4445), np.float32(-4.7750), np.float32(2.0315)
    for _ in range(5):
        x2 = t(np.float32(x * x))
        x4 = t(np.float32(x2 * x2))
        x = t(np.float32(x * a + np.float32(np.float32(x2 * b) + np.float32(x4 * c)) * x))
    np.testing.assert_allclose(np.diag(out), np.full(n, x), rtol=0, atol=0)


def test_ns_tf32_recipe_is_closer_to_exact_than_bf16(oracle):
    """The TF32 mode's reason to exist: on a 128 x 384 input it ends several
    times closer to Newton-Schulz without rounding than the bf16 recipe."""
    g = np.random.default_rng(8).normal(0, 1e-2, (128, 384)).astype(np.float32)
    x = g.astype(np.float64) / np.linalg.norm(g.astype(np.float64))
    for _ in range(5):
        a = x @ x.T
        x = 3.4445 * x + (-4.7750 * a + 2.0315 * (a @ a)) @ x
    t = oracle.newton_schulz5(g, order=oracle.GEMM_F64, variant=oracle.NS_TF32)
    b = oracle.newton_schulz5(g, order=oracle.GEMM_F64)
    err = lambda o: np.linalg.norm(o - x) / np.linalg.norm(x)
    assert err(t) < 4e-3 and err(t) * 4 < err(b)


def test_ns_fp32_recipe_matches_exact_newton_schulz(oracle):
    """The fp32 mode's recipe (no rounding points, norm summed once in fp64)
    is Newton-Schulz in fp32 arithmetic: within 1e-5 of the fp64 iteration."""
    g = np.random.default_rng(9).normal(0, 1e-2, (96, 256)).astype(np.float32)
    x = g.astype(np.float64) / np.linalg.norm(g.astype(np.float64))
    for _ in range(5):
        a = x @ x.T
        x = 3.4445 * x + (-4.7750 * a + 2.0315 * (a @ a)) @ x
    o = oracle.newton_schulz5(g, order=oracle.GEMM_F32_SEQ, variant=oracle.NS_FP32)
    assert np.linalg.norm(o - x) / np.linalg.norm(x) < 1e-5


def test_ns_transpose_rule_exact(oracle):
    rng = np.random.default_rng(2)
    g = rng.normal(0, 1e-2, (24, 40)).astype(np.float32)
    np.testing.assert_array_equal(oracle.newton_schulz5(g).T, oracle.newton_schulz5(g.T.copy()))


def test_muon_zero_velocity_nesterov_input(oracle):
    """With zero velocity: u = (1-mu)*g + mu*(1-mu)*g."""
    g = np.random.default_rng(3).normal(0, 1, 100).astype(np.float32)
    vel = np.zeros(100, np.float32)
    u = oracle.muon_momentum(vel, g, momentum=0.95, nesterov=True)
    om = np.float32(1) - np.float32(0.95)
    np.testing.assert_array_equal(vel, om * g)
    np.testing.assert_array_equal(u, g * om + (om * g) * np.float32(0.95))


def test_muon_scale_factor(oracle):
    assert oracle.muon_scale(256, 64) == np.float32(2.0)
    assert oracle.muon_scale(64, 256) == np.float32(0.5)
    assert oracle.muon_scale(512, 64) == np.sqrt(np.float32(8.0))


def test_ns_pad_non_2d(oracle):
    g = np.arange(10, dtype=np.float32)
    pad = oracle.pad_to_square(g)
    assert pad.shape == (4, 4) and pad.reshape(-1)[:10].tolist() == list(range(10))
    assert not pad.reshape(-1)[10:].any()


def test_ns_summation_order_sensitivity(oracle):
    """Why the Newton-Schulz tolerance is 2e-2 and not 1e-4: the reference recipe
    rounds to bf16 four times per iteration and amplifies rounding flips, so the
    oracle's own fp32 and fp64 summation orders already drift apart by more than
    1e-4 after five iterations, while one iteration from the same input agrees
    to well under 1e-3."""
    rng = np.random.default_rng(4)
    g = rng.normal(0, 1e-2, (128, 256)).astype(np.float32)
    o32 = oracle.newton_schulz5(g, order=oracle.GEMM_F32_SEQ)
    o64 = oracle.newton_schulz5(g, order=oracle.GEMM_F64)
    spread = rel_fro(o32, o64)
    assert 1e-4 < spread < 2e-2
    y = oracle.bf16_round(g)
    x0 = (y / np.float32(np.sqrt(np.sum(y * y, dtype=np.float32)))).astype(np.float32)
    one = rel_fro(oracle.ns_iteration(x0, oracle.GEMM_F32_SEQ), oracle.ns_iteration(x0, oracle.GEMM_F64))
    assert one < 1e-3


@pytest.mark.parametrize("order", [0, 1, 2])
def test_gemm_orders_agree(oracle, order):
    rng = np.random.default_rng(5)
    a = rng.normal(0, 1, (37, 53)).astype(np.float32)
    b = rng.normal(0, 1, (53, 71)).astype(np.float32)
    np.testing.assert_allclose(oracle.gemm(a, b, order), a.astype(np.float64) @ b, rtol=1e-4,
                               atol=1e-4)


# ------------------------------------------------------------------ golden vectors
def _golden():
    import json

    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                           "known_answers.json")) as f:
        return json.load(f)


def _f32(hexes):
    return np.array([int(h, 16) for h in hexes], np.uint32).view(np.float32)


def test_oracle_matches_golden_known_answers(oracle):
    """tests/golden/known_answers.json restates the reference's arithmetic in
    numpy (tests/golden/make_golden.py); the C oracle must reproduce it bit
    for bit."""
    G = _golden()
    a = G["adamw"]
    for t in a["tensors"]:
        p = _f32(t["p"]).copy()
        m = np.zeros_like(p)
        v = np.zeros_like(p)
        oracle.adamw_update(p, m, v, _f32(t["g"]), lr=_f32([a["lr"]])[0],
                            betas=(_f32([a["beta1"]])[0], _f32([a["beta2"]])[0]),
                            eps=_f32([a["eps"]])[0], weight_decay=_f32([a["weight_decay"]])[0],
                            t=t["t"])
        for name, got in (("p_out", p), ("m_out", m), ("v_out", v)):
            np.testing.assert_array_equal(got.view(np.uint32), _f32(t[name]).view(np.uint32),
                                          err_msg=name)
    mm = G["muon_momentum"]
    vel = np.zeros(len(mm["g"]), np.float32)
    u = oracle.muon_momentum(vel, _f32(mm["g"]), momentum=_f32([mm["momentum"]])[0], nesterov=True)
    np.testing.assert_array_equal(vel.view(np.uint32), _f32(mm["vel_out"]).view(np.uint32))
    np.testing.assert_array_equal(u.view(np.uint32), _f32(mm["u"]).view(np.uint32))
    for e in G["muon_scale"]:
        assert oracle.muon_scale(e["rows"], e["cols"]) == _f32([e["scale"]])[0], e
    ident = G["ns_scaled_identity"]
    n, s = ident["n"], _f32([ident["s"]])[0]
    for name, variant in (("bf16", oracle.NS_REFERENCE), ("tf32", oracle.NS_TF32)):
        out = oracle.newton_schulz5(np.eye(n, dtype=np.float32) * s, variant=variant)
        np.testing.assert_array_equal(np.diag(out), np.full(n, _f32([ident["diag"][name]])[0]))
    acc = G["grad_accumulator"]
    avg = np.empty(1, np.float32)
    total = np.array([sum(x[0] for x in acc["micro_batches"])], np.float32)
    oracle.lib().ref_grad_average(oracle._ptr(total), oracle._ptr(avg), 1,
                                  len(acc["micro_batches"]))
    assert avg[0] == _f32(acc["average"])[0]
    for kind, shapes in G["routing"].items():
        for shp in shapes:
            assert oracle.classify_param(tuple(shp)) == kind, shp


def _np_round(x, variant, oracle):
    if variant == oracle.NS_TF32:
        return oracle.tf32_round(x)
    if variant == oracle.NS_FP32:
        return np.asarray(x, np.float32)
    return oracle.bf16_round(x)


def _np_newton_schulz5(g, steps, variant, oracle):
    """An independent numpy restatement of newton_schulz5 (lib.rs:83-126) with
    fp64 products rounded once to fp32, the rounding points of each variant,
    and the reference's sequential fp32 norm (fp64 once for the TF32 and fp32
    modes)."""
    f = np.float32
    tr = g.shape[0] > g.shape[1]
    x = _np_round(g.T if tr else g, variant, oracle).astype(f)
    if variant in (oracle.NS_FP32, oracle.NS_TF32):
        s = f(np.sum(x.astype(np.float64) ** 2))
    else:
        s = f(0)
        for v in x.ravel():
            s = f(s + f(v * v))
    x = (x / max(f(np.sqrt(s)), f(1e-7))).astype(f)
    a, b, c = f(3.4445), f(-4.7750), f(2.0315)
    for _ in range(steps):
        A = _np_round((x.astype(np.float64) @ x.T.astype(np.float64)).astype(f), variant, oracle)
        A2 = _np_round((A.astype(np.float64) @ A.astype(np.float64)).astype(f), variant, oracle)
        B = (A * b + A2 * c).astype(f)
        if variant == oracle.NS_BF16:
            B = oracle.bf16_round(B)
        BX = (B.astype(np.float64) @ x.astype(np.float64)).astype(f)
        x = _np_round((x * a + BX).astype(f), variant, oracle)
    return (x.T if tr else x).astype(f)


@pytest.mark.parametrize("variant", [0, 1, 2, 3])
def test_oracle_ns_matches_independent_numpy_restatement(oracle, variant):
    """The oracle's C recipe (fp64 GEMM order) against the numpy restatement,
    five iterations, both orientations: bit for bit. With K <= 20 the fp64 sums
    of fp32 products are exact in both, so every rounding point sees the same
    value."""
    rng = np.random.default_rng(40 + variant)
    for shape in ((12, 20), (20, 12), (16, 16)):
        g = rng.normal(0, 1e-2, shape).astype(np.float32)
        got = oracle.newton_schulz5(g, 5, order=oracle.GEMM_F64, variant=variant)
        want = _np_newton_schulz5(g, 5, variant, oracle)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=str(shape))


@pytest.mark.parametrize("variant", [0, 1, 2, 3])
def test_blas64_products_equal_the_fp64_order(oracle, variant):
    """GEMM_BLAS64 (numpy float64 matmul, used for the full-size Newton-Schulz
    checks) against the oracle's own fp64 GEMM order: five iterations and one
    iteration bit for bit, both orientations, K up to 1024. Two fp64 sums of
    bf16 products differ by far less than an fp32 rounding step, so every
    rounding point sees the same fp32 value."""
    rng = np.random.default_rng(60 + variant)
    for shape in ((64, 256), (300, 200), (256, 1024)):
        g = rng.normal(0, 1e-2, shape).astype(np.float32)
        a, na = oracle.newton_schulz5(g, 5, order=oracle.GEMM_F64, variant=variant,
                                      return_norm=True)
        b, nb = oracle.newton_schulz5(g, 5, order=oracle.GEMM_BLAS64, variant=variant,
                                      return_norm=True)
        assert na == nb
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32), err_msg=str(shape))
        x = g if shape[0] <= shape[1] else np.ascontiguousarray(g.T)
        x = (oracle._ns_round(x, variant) / np.float32(na)).astype(np.float32)
        np.testing.assert_array_equal(oracle.ns_iteration(x, oracle.GEMM_F64, variant),
                                      oracle.ns_iteration(x, oracle.GEMM_BLAS64, variant))


def test_grad_allreduce_is_the_rank_ordered_fp32_sum(oracle):
    """The data-parallel reduction the multi-GPU path is checked against: per
    element, a float32 running sum in rank order (a scalar restatement here),
    bf16 grads rounded once at the end, non-finite values propagated. The order
    matters: three ranks with a cancelling pair give another result reversed."""
    rng = np.random.default_rng(70)
    world = 3
    locs = [rng.normal(0, 1e-3, 97).astype(np.float32) for _ in range(world)]
    locs[0][5], locs[1][5], locs[2][5] = np.float32(1e8), np.float32(-1e8), np.float32(3.0)
    locs[1][9] = np.inf
    locs[2][11] = np.nan
    got = oracle.grad_allreduce(locs)
    for i in range(97):
        s = np.float32(locs[0][i])
        for r in range(1, world):
            s = np.float32(s + locs[r][i])
        assert got[i].view(np.uint32) == s.view(np.uint32) or (np.isnan(got[i]) and np.isnan(s)), i
    assert got[5] == 3.0 and oracle.grad_allreduce(locs[::-1])[5] == 0.0
    assert np.isposinf(got[9]) and np.isnan(got[11])
    # bf16: widen, sum in fp32, round once (not after every add)
    b = [oracle.bf16_round(x * np.float32(1024.0)) for x in locs]
    got16 = oracle.grad_allreduce(b, bf16=True)
    np.testing.assert_array_equal(got16.view(np.uint32),
                                  oracle.bf16_round(oracle.grad_allreduce(b)).view(np.uint32))
    step = b[0]
    for x in b[1:]:
        step = oracle.bf16_round(step + x)
    assert (oracle.bf16_round(oracle.grad_allreduce(b)) != step)[np.isfinite(step)].any()
    # bf16 bit patterns read back as float32 values
    bits = oracle.bf16_bits(b[0])
    np.testing.assert_array_equal(oracle.bf16_from_bits(bits).view(np.uint32),
                                  b[0].view(np.uint32))
