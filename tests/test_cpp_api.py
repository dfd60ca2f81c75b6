"""The C++ mirror of the reference's Rust optimizer API (include/mmn_optim.hpp)
compiled with g++ against the C-ABI library: the reference's own unit tests of
crates/mmn-optim/src/lib.rs:264-382 restated in C++ (tests/cpp/), plus parity
of the same calls with the CPU oracle. The CPU part needs no GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def cpp_test_binary(tmp_path_factory):
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
    out = str(tmp_path_factory.mktemp("cpp") / "test_optim_api")
    cmd = [gxx, "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "oracle"),
           os.path.join(ROOT, "tests", "cpp", "test_optim_api.cpp"), "-o", out,
           "-L", lib_dir, "-lmmn_optim_cuda", "-L", ref_dir, "-lmmn_optim_ref",
           f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{ref_dir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return out


def test_cpp_mirror_cpu_part(cpp_test_binary):
    r = subprocess.run([cpp_test_binary, "--cpu-only"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout


@pytest.mark.gpu
def test_cpp_mirror_on_gpu(cpp_test_binary):
    r = subprocess.run([cpp_test_binary], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout
