"""Failure detection on the device without a fault: the bounded wait that every
pipelined kernel uses gives up after its limit, reports MMN_E_TIMEOUT through
the status word, and leaves the context usable."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports(mmn):
    from magicmindnet_b200 import _native as N

    t0 = time.monotonic()
    rc = N.lib().mmn_selftest_bounded_wait(0, 200_000_000)  # 200 ms
    dt = time.monotonic() - t0
    assert rc == N.MMN_E_TIMEOUT, N.lib().mmn_last_error()
    assert 0.2 <= dt < 5.0
    assert b"gave up" in N.lib().mmn_last_error()
    # the device is still usable afterwards
    g = np.random.default_rng(0).normal(0, 1e-2, (64, 96)).astype(np.float32)
    out = mmn.newton_schulz5(g)
    assert np.isfinite(out).all()
    assert N.lib().mmn_selftest_bounded_wait(0, 0) == N.MMN_E_INVALID
