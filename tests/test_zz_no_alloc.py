"""mmn_newton_schulz5_noalloc: the entry point for callers that cannot call
cudaMalloc (device memory owned by another allocator or a fixed arena, hosts
that forbid allocation after start-up, paths that cannot afford cudaMalloc's
implicit synchronisation). Its scratch is a fixed array inside the library.

Called through the C ABI on device buffers, twice in a row, and compared with
the allocating entry point mmn_newton_schulz5 within the Newton-Schulz
tolerance used elsewhere in the suite (2e-2 relative Frobenius; the two paths
run the same kernels, so they normally agree exactly). This file is named to
be collected last."""
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


@pytest.mark.parametrize("shape,mode", [((256, 1024), 0), ((1024, 256), 0), ((300, 200), 1),
                                        ((1024, 1024), 0)])
def test_noalloc_matches_allocating_entry_point(mmn, shape, mode):
    import torch

    rng = np.random.default_rng(123)
    for call in range(2):  # two calls in a row share the fixed scratch
        g = torch.from_numpy(rng.normal(0, 1e-2, shape).astype(np.float32)).cuda()
        out_fixed = torch.full(shape, float("nan"), device="cuda")
        out_alloc = torch.empty(shape, device="cuda")
        _run("noalloc", g, out_fixed, 5, mode)
        _run("alloc", g, out_alloc, 5, mode)
        torch.cuda.synchronize()
        a = out_fixed.cpu().numpy()
        b = out_alloc.cpu().numpy()
        assert np.isfinite(a).all(), call
        assert rel_fro(a, b) <= 2e-2, call


def test_noalloc_rejects_sizes_beyond_its_scratch(mmn):
    from magicmindnet_b200 import _native as N

    L = N.lib()
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    rc = L.mmn_newton_schulz5_noalloc(dummy, 2048, 2048, 5, 0, dummy, 0, None)
    assert rc == N.MMN_E_UNSUPPORTED
    assert b"1048576" in L.mmn_last_error()
    rc = L.mmn_newton_schulz5_noalloc(dummy, 1025, 1025, 5, 0, dummy, 0, None)
    assert rc == N.MMN_E_UNSUPPORTED
