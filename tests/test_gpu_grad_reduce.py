"""mmn_grad_reduce and mmn_grad_nonfinite_scan: the data-parallel grad
reduction and the sharded non-finite scan (the steps before the optimizer on
each rank) on caller-owned buffers, through the C ABI.

The sources stand in for the ranks' local grads. On one GPU they are buffers of
that GPU, which runs the same kernels that mmn_optim_reduce_grads runs over
NVLink mappings; the sum must equal the oracle's rank-ordered sum
(oracle.grad_allreduce) bit for bit, fp32 and bf16, ragged lengths included.
The non-finite flag is checked both ways, and bad arguments are refused before
any kernel runs. The scan raises every rank's flag (here: words of one GPU)
on one Inf or NaN and none on finite grads. With two GPUs one source, and one
flag, also live on the peer GPU.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _reduce(srcs, dst, numel, bf16, flag=None, device=0):
    import torch

    from magicmindnet_b200 import _native as N

    arr = (ctypes.c_void_p * len(srcs))(*[ctypes.c_void_p(p) for p in srcs])
    return N.lib().mmn_grad_reduce(arr, len(srcs), ctypes.c_void_p(dst), numel,
                                   N.DTYPE_BF16 if bf16 else N.DTYPE_F32,
                                   ctypes.c_void_p(flag) if flag is not None else None, device,
                                   ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))


def _local(n, world, bf16, seed, device="cuda"):
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    out = []
    for _ in range(world):
        g = torch.empty(n, device=device).normal_(0, 1e-3, generator=gen)
        out.append((g * 1024.0).bfloat16() if bf16 else g)
    return out


def _host(t, oracle):
    import torch

    if t.dtype == torch.bfloat16:
        return oracle.bf16_from_bits(t.view(torch.int16).cpu().numpy())
    return t.cpu().numpy()


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
@pytest.mark.parametrize("world,n", [(2, 1), (2, 7), (3, 1000), (8, 4099), (4, 1 << 20),
                                     (8, (1 << 22) + 5)])
def test_sum_equals_oracle_rank_order(mmn, oracle, bf16, world, n):
    import torch

    from magicmindnet_b200 import _native as N

    srcs = _local(n, world, bf16, seed=1000 + world + n)
    want = oracle.grad_allreduce([_host(g, oracle) for g in srcs], bf16)
    dst = torch.full((n,), float("nan"), device="cuda",
                     dtype=torch.bfloat16 if bf16 else torch.float32)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.check(_reduce([g.data_ptr() for g in srcs], dst.data_ptr(), n, bf16, flag.data_ptr()))
    torch.cuda.synchronize()
    got = _host(dst, oracle)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    assert int(flag.item()) == 0
    # in place: the destination is the first rank's own buffer
    N.check(_reduce([g.data_ptr() for g in srcs], srcs[0].data_ptr(), n, bf16))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_host(srcs[0], oracle).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
def test_nonfinite_sum_sets_the_flag(mmn, bf16):
    import torch

    from magicmindnet_b200 import _native as N

    dt = torch.bfloat16 if bf16 else torch.float32
    n = 10007
    for where, how in [(0, "inf"), (n - 1, "nan"), (5000, "overflow")]:
        srcs = [torch.full((n,), 1e-3, device="cuda", dtype=dt) for _ in range(3)]
        if how == "overflow":  # every input finite, their sum is not
            srcs[0][where] = 3e38
            srcs[2][where] = 3e38
        else:
            srcs[1][where] = float(how)
        dst = torch.empty(n, device="cuda", dtype=dt)
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        N.check(_reduce([g.data_ptr() for g in srcs], dst.data_ptr(), n, bf16, flag.data_ptr()))
        torch.cuda.synchronize()
        assert int(flag.item()) == 1, (where, how)
        assert not torch.isfinite(dst[where].float()).item()
    # a flag already raised stays raised over a finite sum (it is never cleared here)
    srcs = [torch.full((n,), 1e-3, device="cuda", dtype=dt) for _ in range(2)]
    flag = torch.ones(1, dtype=torch.int32, device="cuda")
    N.check(_reduce([g.data_ptr() for g in srcs], dst.data_ptr(), n, bf16, flag.data_ptr()))
    torch.cuda.synchronize()
    assert int(flag.item()) == 1


def test_bad_arguments_are_refused_before_any_kernel(mmn):
    import torch

    from magicmindnet_b200 import _native as N

    n = 1024
    srcs = [torch.ones(n + 8, device="cuda") for _ in range(2)]
    dst = torch.zeros(n + 8, device="cuda")
    ptrs = [g.data_ptr() for g in srcs]
    assert _reduce(ptrs[:1], dst.data_ptr(), n, False) == N.MMN_E_INVALID  # one source
    assert _reduce(ptrs * 5, dst.data_ptr(), n, False) == N.MMN_E_INVALID  # ten sources
    assert _reduce([ptrs[0] + 4, ptrs[1]], dst.data_ptr(), n, False) == N.MMN_E_INVALID
    assert _reduce(ptrs, dst.data_ptr() + 4, n, False) == N.MMN_E_INVALID
    assert _reduce(ptrs, ptrs[0] + 16, n, False) == N.MMN_E_INVALID  # partial overlap
    host = np.zeros(n + 4, np.float32)
    haddr = host.ctypes.data + (-host.ctypes.data) % 16  # aligned: refused as host memory
    assert _reduce([haddr, ptrs[1]], dst.data_ptr(), n, False) == N.MMN_E_INVALID
    assert b"host memory" in N.lib().mmn_last_error()
    assert _reduce(ptrs, dst.data_ptr(), -1, False) == N.MMN_E_INVALID
    torch.cuda.synchronize()
    assert bool((dst == 0).all().item())  # nothing was written
    N.check(_reduce(ptrs, dst.data_ptr(), 0, False))  # empty: nothing to do


def test_peer_source_on_a_second_gpu(mmn, oracle):
    import torch

    from magicmindnet_b200 import _native as N

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    n = (1 << 20) + 3
    local = _local(n, 2, False, seed=77)
    peer = _local(n, 1, False, seed=78, device="cuda:1")[0]
    torch.cuda.synchronize(1)
    want = oracle.grad_allreduce([_host(local[0], oracle), _host(peer, oracle),
                                  _host(local[1], oracle)])
    dst = torch.empty(n, device="cuda:0")
    N.check(_reduce([local[0].data_ptr(), peer.data_ptr(), local[1].data_ptr()],
                    dst.data_ptr(), n, False))
    torch.cuda.synchronize(0)
    np.testing.assert_array_equal(_host(dst, oracle).view(np.uint32), want.view(np.uint32))


def _scan(grads, numel, bf16, flags, device=0):
    import torch

    from magicmindnet_b200 import _native as N

    arr = (ctypes.c_void_p * len(flags))(*[ctypes.c_void_p(p) for p in flags])
    return N.lib().mmn_grad_nonfinite_scan(
        ctypes.c_void_p(grads), numel, N.DTYPE_BF16 if bf16 else N.DTYPE_F32, arr, len(flags),
        device, ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
@pytest.mark.parametrize("n", [1, 13, 4096, (1 << 22) + 7])
def test_sharded_scan_raises_every_rank_flag(mmn, bf16, n):
    """The sharded scan's kernel (each rank scans its part and raises all ranks'
    flags), with the ranks' flags as words of one GPU: a clean part raises
    none, one Inf or NaN anywhere (vector body or scalar tail) raises all."""
    import torch

    from magicmindnet_b200 import _native as N

    dt = torch.bfloat16 if bf16 else torch.float32
    g = torch.empty(n, device="cuda", dtype=dt).normal_(0, 1e-3)
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    ptrs = [flags.data_ptr() + 4 * k for k in range(8)]
    N.check(_scan(g.data_ptr(), n, bf16, ptrs))
    torch.cuda.synchronize()
    assert int(flags.sum().item()) == 0
    for pos, bad in [(n - 1, float("inf")), (n // 2, float("nan")), (0, float("-inf"))]:
        g2 = g.clone()
        g2[pos] = bad
        flags.zero_()
        N.check(_scan(g2.data_ptr(), n, bf16, ptrs[:5]))
        torch.cuda.synchronize()
        assert flags.cpu().tolist() == [1] * 5 + [0] * 3, (pos, bad)
    # the largest finite values are not flagged
    g.fill_(torch.finfo(dt).max)
    flags.zero_()
    N.check(_scan(g.data_ptr(), n, bf16, ptrs))
    torch.cuda.synchronize()
    assert int(flags.sum().item()) == 0


def test_sharded_scan_refuses_bad_arguments(mmn):
    import torch

    from magicmindnet_b200 import _native as N

    g = torch.zeros(64, device="cuda")
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    f = [flags.data_ptr(), flags.data_ptr() + 4]
    assert _scan(g.data_ptr() + 4, 32, False, f) == N.MMN_E_INVALID  # misaligned grads
    assert _scan(g.data_ptr(), 32, False, []) == N.MMN_E_INVALID
    assert _scan(g.data_ptr(), 32, False, f * 5) == N.MMN_E_INVALID  # ten flags
    assert _scan(g.data_ptr(), 32, False, [flags.data_ptr() + 2]) == N.MMN_E_INVALID
    host = np.zeros(8, np.int32)
    assert _scan(g.data_ptr(), 32, False, [host.ctypes.data]) == N.MMN_E_INVALID
    assert _scan(g.data_ptr(), -1, False, f) == N.MMN_E_INVALID
    N.check(_scan(g.data_ptr(), 0, False, f))
    torch.cuda.synchronize()
    assert int(flags.sum().item()) == 0


def test_sharded_scan_raises_a_peer_flag(mmn):
    import torch

    from magicmindnet_b200 import _native as N

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    g = torch.zeros(1000, device="cuda:0")
    g[999] = float("nan")
    mine = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    peer = torch.zeros(1, dtype=torch.int32, device="cuda:1")
    N.check(_scan(g.data_ptr(), 1000, False, [mine.data_ptr(), peer.data_ptr()]))
    torch.cuda.synchronize(0)
    assert int(mine.item()) == 1 and int(peer.item()) == 1
