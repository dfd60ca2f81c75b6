"""mmn_newton_schulz5_noalloc: the entry point for callers that cannot call
cudaMalloc (device memory owned by another allocator or a fixed arena, hosts
that forbid allocation after start-up, paths that cannot afford cudaMalloc's
implicit synchronisation). Its scratch is a fixed array inside the library.

Called through the C ABI on device buffers, twice in a row per case, and
compared with the allocating entry point mmn_newton_schulz5. Both run the same
kernels on the same input, so the results must agree bit for bit; a scratch
layout fault (a wrong X ping-pong buffer, overlapping partial sums or
descriptors, a region left uncleared) would break that. Each case is also held
to the oracle within the Newton-Schulz tolerance of the suite (2e-2 relative
Frobenius). The cases cover zero and even step counts (the result then sits in
the other X buffer, or comes straight from the normalised input), both
orientations, both arithmetic modes and shapes at the ends of the fixed
scratch. This file is named to be collected last."""
import ctypes

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu


def _run(fn_name, g, out, steps, mode):
    from magicmindnet_b200 import _native as N

    L = N.lib()
    if fn_name == "noalloc":
        rc = L.mmn_newton_schulz5_noalloc(ctypes.c_void_p(g.data_ptr()), g.shape[0], g.shape[1],
                                          steps, mode, ctypes.c_void_p(out.data_ptr()), 0, None)
    else:
        shape = N.shape_array(g.shape)
        rc = L.mmn_newton_schulz5(ctypes.c_void_p(g.data_ptr()), shape, 2, steps, mode,
                                  ctypes.c_void_p(out.data_ptr()), 0, None, N.MEM_DEVICE)
    N.check(rc)


CASES = [
    ((256, 1024), 0, 5),
    ((1024, 256), 0, 5),
    ((300, 200), 1, 5),
    ((200, 300), 0, 0),
    ((512, 128), 0, 4),
    ((128, 512), 1, 4),
    ((1024, 1024), 0, 5),   # largest square: min side at the limit
    ((1023, 1025), 0, 5),   # padded strides, scratch nearly full
    ((1, 1048576), 0, 5),   # rows * cols at the limit
]


@pytest.mark.parametrize("shape,mode,steps", CASES)
def test_noalloc_matches_allocating_entry_point(mmn, oracle, shape, mode, steps):
    import torch

    rng = np.random.default_rng(123 + steps)
    for call in range(2):  # two calls in a row share the fixed scratch
        g_host = rng.normal(0, 1e-2, shape).astype(np.float32)
        g = torch.from_numpy(g_host).cuda()
        out_fixed = torch.full(shape, float("nan"), device="cuda")
        out_alloc = torch.empty(shape, device="cuda")
        _run("noalloc", g, out_fixed, steps, mode)
        _run("alloc", g, out_alloc, steps, mode)
        torch.cuda.synchronize()
        a = out_fixed.cpu().numpy()
        b = out_alloc.cpu().numpy()
        assert np.isfinite(a).all(), call
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32), err_msg=str(call))
        if call == 0:
            variant = oracle.NS_BF16 if mode == 1 else oracle.NS_REFERENCE
            ref = oracle.newton_schulz5(g_host, steps, order=oracle.GEMM_F64, variant=variant)
            assert rel_fro(a, ref) <= 2e-2


def test_noalloc_rejects_sizes_beyond_its_scratch(mmn):
    from magicmindnet_b200 import _native as N

    L = N.lib()
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    rc = L.mmn_newton_schulz5_noalloc(dummy, 2048, 2048, 5, 0, dummy, 0, None)
    assert rc == N.MMN_E_UNSUPPORTED
    assert b"1048576" in L.mmn_last_error()
    rc = L.mmn_newton_schulz5_noalloc(dummy, 1025, 1025, 5, 0, dummy, 0, None)
    assert rc == N.MMN_E_UNSUPPORTED
    rc = L.mmn_newton_schulz5_noalloc(dummy, 2, 1048577, 5, 0, dummy, 0, None)
    assert rc == N.MMN_E_UNSUPPORTED
