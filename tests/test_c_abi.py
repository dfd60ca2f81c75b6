"""The C ABI from plain C99 (the language of the header and of any FFI that
binds it): tests/c/test_c_abi.c is compiled with -std=c99 -pedantic -Werror,
linked against the built library and run. No GPU is needed."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_c99_program_links_and_calls_the_library(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    from magicmindnet_b200 import _native as N

    lib_dir = os.path.dirname(N.LIB_PATH)
    assert os.path.exists(N.LIB_PATH), "build the library first"
    exe = str(tmp_path / "test_c_abi")
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                    "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "test_c_abi.c"),
                    "-L", lib_dir, "-lmmn_optim_cuda", "-Wl,-rpath," + lib_dir, "-o", exe],
                   check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "c abi ok" in r.stdout
