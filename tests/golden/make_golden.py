"""Generates tests/golden/known_answers.json: known answers of the reference's
optimizer arithmetic (crates/mmn-optim/src/lib.rs), restated here in numpy
float32 with the reference's operation order and NOT through the oracle, so
that the oracle (tests/test_oracle.py) and the GPU (tests/test_gpu_golden.py)
are pinned against an independent statement of the same arithmetic. numpy
float32 scalar and array operations round each operation to float32, like
Rust's f32 arithmetic (no fused multiply-add). Values are stored as the hex of
their float32 bit patterns.

Run: python tests/golden/make_golden.py   (writes known_answers.json beside it)
"""
import json
import os

import numpy as np

F = np.float32
HERE = os.path.dirname(os.path.abspath(__file__))


def bits(a):
    return [f"{int(u):08x}" for u in np.ascontiguousarray(a, np.float32).view(np.uint32).ravel()]


def bf16(x):
    """half 2.7.1 bf16::from_f32 on finite values: round to nearest, ties to even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def tf32(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0xFFF + ((u >> 13) & 1)) & 0xFFFFE000
    return r.astype(np.uint32).view(np.float32)


def adamw(p, m, v, g, lr, b1, b2, eps, wd, t):
    """AdamW::step_param (lib.rs:41-60) for step count t in {1, 2}, where
    b.powf(t) is exactly b (t = 1) or the correctly rounded b*b (t = 2)."""
    m = b1 * m + (F(1) - b1) * g                     # :47-49
    v = b2 * v + (F(1) - b2) * g * g                 # :50-52
    bc1 = F(1) - (b1 if t == 1 else F(b1 * b1))      # :53
    bc2 = F(1) - (b2 if t == 1 else F(b2 * b2))      # :54
    m_hat = m / bc1
    v_hat = v / bc2
    p = p - lr * (m_hat / (np.sqrt(v_hat) + eps))    # :55-57
    p = p * (F(1) - lr * wd)                         # :58-59
    return p.astype(F), m.astype(F), v.astype(F)


def main():
    rng = np.random.default_rng(2026)
    out = {}
    # AdamW: two tensors stepped by one instance, so the second sees t = 2 on
    # its first update (the per-instance counter, lib.rs:41-43), then the first
    # tensor again at t = 3 is not included (powf of a non-trivial exponent).
    lr, b1, b2, eps, wd = F(1e-3), F(0.9), F(0.999), F(1e-8), F(0.01)
    p1 = rng.normal(0, 0.02, 257).astype(F)
    g1 = rng.normal(0, 1e-3, 257).astype(F)
    g1[:4] = [0.0, 1e-30, -3.5, 7.0]  # zero, tiny, large grads
    p2 = rng.normal(0, 0.02, (5, 7)).astype(F)
    g2 = rng.normal(0, 1e-3, (5, 7)).astype(F)
    z1, z2 = np.zeros_like(p1), np.zeros_like(p2)
    q1, m1, v1 = adamw(p1, z1, z1, g1, lr, b1, b2, eps, wd, 1)
    q2, m2, v2 = adamw(p2, z2, z2, g2, lr, b1, b2, eps, wd, 2)
    out["adamw"] = {"lr": bits([lr])[0], "beta1": bits([b1])[0], "beta2": bits([b2])[0],
                    "eps": bits([eps])[0], "weight_decay": bits([wd])[0],
                    "tensors": [{"shape": list(p.shape), "p": bits(p), "g": bits(g),
                                 "p_out": bits(q), "m_out": bits(m), "v_out": bits(v), "t": t}
                                for p, g, q, m, v, t in ((p1, g1, q1, m1, v1, 1),
                                                         (p2, g2, q2, m2, v2, 2))]}
    # Muon momentum with zero velocity and Nesterov (lib.rs:154-165)
    mu = F(0.95)
    g = rng.normal(0, 1e-3, 64).astype(F)
    vel = mu * np.zeros_like(g) + (F(1) - mu) * g
    u = g * (F(1) - mu) + vel * mu
    out["muon_momentum"] = {"momentum": bits([mu])[0], "g": bits(g), "vel_out": bits(vel),
                            "u": bits(u)}
    # sqrt(rows / cols) of lib.rs:169-171
    out["muon_scale"] = [{"rows": r, "cols": c, "scale": bits([np.sqrt(F(r) / F(c))])[0]}
                         for r, c in ((64, 256), (256, 64), (512, 64), (33, 17), (4096, 14336))]
    # newton_schulz5 of s * I_n (lib.rs:83-126): the diagonal follows a scalar
    # recurrence; the norm is the sequential f32 sum of n equal squares (:109)
    n, s0 = 8, F(0.37)
    a, b, c = F(3.4445), F(-4.7750), F(2.0315)
    rec = {}
    for name, rnd in (("bf16", bf16), ("tf32", tf32)):
        y = rnd(np.array([s0], F))[0]
        acc = F(0)
        for _ in range(n):
            acc = F(acc + F(y * y))
        x = F(y / np.sqrt(acc))
        for _ in range(5):
            x2 = rnd(np.array([F(x * x)], F))[0]
            x4 = rnd(np.array([F(x2 * x2)], F))[0]
            x = rnd(np.array([F(x * a + F(F(x2 * b) + F(x4 * c)) * x)], F))[0]
        rec[name] = bits([x])[0]
    out["ns_scaled_identity"] = {"n": n, "s": bits([s0])[0], "diag": rec}
    # GradAccumulator (lib.rs:283-293) and the routing table (lib.rs:303-320)
    out["grad_accumulator"] = {"micro_batches": [[1.0], [3.0]], "average": bits([F(4.0) / F(2)])}
    out["routing"] = {"Matrix": [[64, 32], [2, 2]], "Other": [[16], [16, 1], [1, 3, 3, 3]]}
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", os.path.join(HERE, "known_answers.json"))


if __name__ == "__main__":
    main()
