"""The C++ mirrors of the reference's Rust optimizer API (include/mmn_optim.hpp)
and of its trainer's optimizer loop (include/mmn_train.hpp), compiled with g++
against the C-ABI library: the reference's own unit tests of
crates/mmn-optim/src/lib.rs:264-382 restated in C++ (tests/cpp/), parity of
the same calls with the CPU oracle, and the training loop against an oracle
replay. The CPU parts need no GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _compile(tmp_path_factory, name):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ is not installed")
    from magicmindnet_b200 import _native as N
    from magicmindnet_b200 import build as B
    from oracle import reference_optim as R

    B.build()
    R.build()
    lib_dir = os.path.dirname(N.LIB_PATH)
    ref_dir = os.path.dirname(R._LIB_PATH)
    out = str(tmp_path_factory.mktemp("cpp") / name)
    cmd = [gxx, "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "oracle"),
           "-I", os.path.join(ROOT, "tests", "cpp"),
           os.path.join(ROOT, "tests", "cpp", name + ".cpp"), "-o", out,
           "-L", lib_dir, "-lmmn_optim_cuda", "-L", ref_dir, "-lmmn_optim_ref",
           f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{ref_dir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return out


@pytest.fixture(scope="module")
def cpp_test_binary(tmp_path_factory):
    return _compile(tmp_path_factory, "test_optim_api")


@pytest.fixture(scope="module")
def train_loop_binary(tmp_path_factory):
    """The trainer's optimizer loop (include/mmn_train.hpp) and its oracle replay."""
    return _compile(tmp_path_factory, "test_train_loop")


def test_train_loop_cpu_part(train_loop_binary):
    """The loop against a literal restatement of train_with_encoder on the
    oracle: flushes (the ragged last batch too), averaging, ids, counters."""
    r = subprocess.run([train_loop_binary, "--cpu-only"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout


@pytest.mark.gpu
def test_train_loop_on_gpu(train_loop_binary):
    """The GPU trainer against the oracle replay: AdamW bit for bit, Muon within
    2e-2 of its update, over two epochs of ragged batches."""
    r = subprocess.run([train_loop_binary], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout


def test_cpp_mirror_cpu_part(cpp_test_binary):
    r = subprocess.run([cpp_test_binary, "--cpu-only"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout


@pytest.mark.gpu
def test_cpp_mirror_on_gpu(cpp_test_binary):
    r = subprocess.run([cpp_test_binary], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout
