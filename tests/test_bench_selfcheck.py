"""The benchmark's own multi-GPU check, on CPU: after a sharded run every rank
checksums every slot's parameters exactly (bench._param_checksums: the integer
sum of the bit patterns and a position-weighted one), and the ranks compare
them by all-reduce MAX and MIN. Here: the checksums tell a one-ulp change and a
swap of two elements apart, cover the bf16 parameter copies, and two gloo ranks
disagree exactly when one rank's parameters differ."""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class _Cfg:
    def __init__(self, bf16):
        self.bf16_param_shadow = bf16


class _FakeStep:
    """The two accessors _param_checksums uses, over host tensors."""

    def __init__(self, params, bf16=False):
        self.params = params
        self.config = _Cfg(bf16)

    def param(self, k):
        return self.params[k]

    def param_bf16(self, k):
        return self.params[k]


def _params(seed, bf16=False):
    import torch

    g = torch.Generator().manual_seed(seed)
    ps = [torch.randn(s, generator=g) * 0.02 for s in ((64, 48), (300,), (17, 5, 3))]
    return [p.bfloat16() for p in ps] if bf16 else ps


@pytest.mark.parametrize("bf16", [False, True])
def test_checksums_see_one_ulp_and_a_swap(bf16):
    import torch

    import bench

    base = _params(0, bf16)
    cs0 = bench._param_checksums(_FakeStep(base, bf16), len(base))
    assert torch.equal(cs0, bench._param_checksums(_FakeStep([p.clone() for p in base], bf16), 3))

    ulp = [p.clone() for p in base]
    flat = ulp[1].view(torch.int16 if bf16 else torch.int32).reshape(-1)
    flat[123] += 1  # the next representable value
    cs1 = bench._param_checksums(_FakeStep(ulp, bf16), 3)
    assert not torch.equal(cs1[1], cs0[1]) and torch.equal(cs1[0], cs0[0])

    swap = [p.clone() for p in base]
    f = swap[0].reshape(-1)
    f[[3, 900]] = f[[900, 3]]
    cs2 = bench._param_checksums(_FakeStep(swap, bf16), 3)
    assert cs2[0, 0] == cs0[0, 0]  # the plain sum cannot see a swap...
    assert cs2[0, 1] != cs0[0, 1]  # ...the position-weighted one does


def _rank(rank, world, port, perturb, q):
    import sys

    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    import bench

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        ps = _params(7)
        if perturb and rank == 1:
            ps[2].reshape(-1)[40] = torch.nextafter(ps[2].reshape(-1)[40], torch.tensor(1.0))
        cs = bench._param_checksums(_FakeStep(ps), len(ps))
        mx, mn = cs.clone(), cs.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(mn, op=dist.ReduceOp.MIN)
        q.put((rank, bool(torch.equal(mx, mn))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("perturb", [False, True])
def test_two_ranks_agree_only_on_equal_parameters(perturb):
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, perturb, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == {0: not perturb, 1: not perturb}
