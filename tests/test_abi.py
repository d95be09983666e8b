"""The C ABI (include/tpmd.h) without compute: the library loads, exports
every declared symbol, validates arguments, and agrees with the oracle on the
load-time scale folding."""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np
import pytest

import oracle as O
import tpmd
from conftest import ROOT, gpu_available
from tpmd import synth


def declared_symbols():
    src = "".join(open(os.path.join(ROOT, "include", h)).read()
                  for h in ("tpmd.h", "tpme.h", "tpfm.h", "tpae.h", "tppl.h"))
    return sorted(set(re.findall(r"\b((?:tpmd|tpme|tpfm|tpae|tppl|tpk)_[a-z0-9_]+)\s*\(", src)))


def test_exports_every_declared_symbol():
    L = tpmd.load_library()
    names = declared_symbols()
    assert len(names) >= 18
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert set(names) == set(tpmd.EXPORTS)


def test_library_links_no_vendor_math_library():
    """every contraction on the path is the library's own tcgen05 code: the
    shared object depends on the C/C++ runtime only (CUDA runtime linked
    statically, NCCL opened at run time by the multi-GPU group), not on
    cuBLAS, cuBLASLt, cuDNN or a CUDA runtime of the host process"""
    import subprocess
    so = tpmd.LIB_PATH
    deps = subprocess.run(["ldd", so], capture_output=True, text=True, check=True).stdout
    for lib in ("cublas", "cudnn", "cudart", "nccl", "torch"):
        assert lib not in deps, (lib, deps)


def test_abi_version():
    assert tpmd.load_library().tpmd_abi_version() == 1


def test_scale_for_matches_oracle():
    for name, shape in synth.tensor_shapes().items():
        ne = synth.ggml_ne(shape)
        assert tpmd.scale_for(name, ne) == O.scale_for(name, ne), name
    for name, ne in [("enc.fc.0.weight", (512, 512)), ("enc.net_app.convs.0.0.weight", (1, 1, 3, 64)),
                     ("enc.x.conv2.1.weight", (3, 3, 64, 128)), ("enc.x.skip.1.weight", (1, 1, 64, 128)),
                     ("enc.y.conv1.1.bias", (64,)), ("dec.direction.Q", (20, 512))]:
        assert tpmd.scale_for(name, ne) == O.scale_for(name, ne), name


def test_null_arguments_fail_cleanly():
    L = tpmd.load_library()
    assert L.tpk_bilinear_gather(None, 0, 4, 2, 2, None, 1, 0, 0, None, None) == -1
    assert b"null" in L.tpk_last_error()
    assert L.tpk_im2col_cf(None, 4, 4, 4, 1, 3, 3, 1, 1, 1, 1, 1, 1, None, 0, None) == -1
    buf = (C.c_float * 16)()
    assert L.tpk_im2col_cf(buf, 0, 4, 4, 1, 3, 3, 1, 1, 1, 1, 1, 1, buf, 0, None) == -1
    assert b"bad shape" in L.tpk_last_error()
    # NULL handle: -1, never a crash
    assert L.tpmd_prepare(None) == -1
    assert L.tpmd_decode(None, None, 1, None) == -1
    assert L.tpmd_last_error(None) == b"no context"
    L.tpmd_destroy(None)


def test_create_rejects_bad_arguments():
    with pytest.raises(tpmd.TpmdError):
        tpmd.MotionDecoder(dtype=7)
    with pytest.raises(tpmd.TpmdError):
        tpmd.MotionDecoder(max_batch=0)


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU path")
def test_create_without_gpu_fails_loudly():
    with pytest.raises(tpmd.TpmdError):
        tpmd.MotionDecoder(device=0)
