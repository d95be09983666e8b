"""Build and run the C++ shim test (tests/cpp/test_shim.cpp) against
libtpmd.so: failure paths on CPU, a full decode on the GPU."""
from __future__ import annotations

import os
import subprocess

import pytest

from conftest import PKG, ROOT

SRC = os.path.join(ROOT, "tests", "cpp", "test_shim.cpp")


@pytest.fixture(scope="module")
def shim_bin(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("shim") / "test_shim")
    subprocess.run(["g++", "-O1", "-std=c++17", "-I", os.path.join(ROOT, "include"), SRC, "-o", out,
                    "-L", PKG, "-ltpmd", f"-Wl,-rpath,{PKG}"], check=True)
    return out


def test_shim_failure_paths(shim_bin):
    r = subprocess.run([shim_bin], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "OK" in r.stdout


@pytest.mark.gpu
def test_shim_decode_on_gpu(shim_bin):
    r = subprocess.run([shim_bin, "gpu"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    print(r.stdout)
