"""The GPU against tests/golden/known_answers.json, the numpy restatement of
the reference's arithmetic (tests/golden/make_golden.py): AdamW with the
per-instance step counter and Muon's momentum, bit for bit."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _f32(hexes):
    return np.array([int(h, 16) for h in hexes], np.uint32).view(np.float32)


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "known_answers.json")) as f:
        return json.load(f)


def test_adamw_matches_golden(mmn, golden):
    a = golden["adamw"]
    cfg = mmn.AdamWConfig(lr=float(_f32([a["lr"]])[0]),
                          betas=(float(_f32([a["beta1"]])[0]), float(_f32([a["beta2"]])[0])),
                          eps=float(_f32([a["eps"]])[0]),
                          weight_decay=float(_f32([a["weight_decay"]])[0]))
    opt = mmn.AdamW(cfg)
    for k, t in enumerate(a["tensors"]):  # one instance: the second tensor runs at t = 2
        p = _f32(t["p"]).reshape(t["shape"]).copy()
        opt.step_param(k, p, _f32(t["g"]).reshape(t["shape"]))
        assert opt.step == t["t"]
        np.testing.assert_array_equal(p.view(np.uint32).ravel(), _f32(t["p_out"]).view(np.uint32))
        n = p.size
        for which in ("m", "v"):
            np.testing.assert_array_equal(opt.export_state(k, which, n).view(np.uint32),
                                          _f32(t[which + "_out"]).view(np.uint32), err_msg=which)
    opt.close()


def test_muon_momentum_matches_golden(mmn, golden):
    mm = golden["muon_momentum"]
    g = _f32(mm["g"]).reshape(8, 8)
    opt = mmn.Muon(mmn.MuonConfig(momentum=float(_f32([mm["momentum"]])[0])))
    p = np.zeros((8, 8), np.float32)
    opt.step_matrix(0, p, g)
    np.testing.assert_array_equal(opt.export_velocity(0, (8, 8)).view(np.uint32).ravel(),
                                  _f32(mm["vel_out"]).view(np.uint32))
    opt.close()
