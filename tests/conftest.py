import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle import reference_optim as R

    R.lib()
    return R


@pytest.fixture(scope="session")
def mmn():
    """The product package; GPU tests fail (not skip) without a usable B200."""
    import magicmindnet_b200 as m

    assert m.is_available(), "GPU tests need a B200 (sm_100a) device"
    return m


def rel_fro(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))


def init_linear(rng, out_dim, in_dim):
    """crates/mmn-nn/src/lib.rs:300-304: U(-s/2, s/2), s = sqrt(2/(in+out))."""
    s = np.sqrt(2.0 / (in_dim + out_dim))
    return rng.uniform(-s / 2, s / 2, (out_dim, in_dim)).astype(np.float32)


def chatbot_params(rng, vocab=512, n_layer=2, d=64):
    """Chatbot(vocab 512, 2 layers, d_model 64) parameter values in optimizer
    call order, with the reference's init distributions (Linear U(-s/2,s/2),
    Embedding U(-1,1), LN gamma=1/beta=0)."""
    from magicmindnet_b200.step import chatbot_param_order

    out = []
    for name, shape in chatbot_param_order(vocab, n_layer, d):
        if name == "embed":
            v = rng.uniform(-1, 1, shape).astype(np.float32)
        elif name.endswith("gamma"):
            v = np.ones(shape, np.float32)
        elif name.endswith("beta"):
            v = np.zeros(shape, np.float32)
        else:
            v = init_linear(rng, shape[0], shape[1])
        out.append((name, v))
    return out
