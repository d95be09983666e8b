"""The allocation-free decode entry point (tpmd_decode_noalloc).

It serves callers that cannot call cudaMalloc while they decode: real-time
frame loops that must not risk an allocator stall or an out-of-memory error
mid-stream, and hosts whose memory manager owns the GPU's memory. Its scratch
is a static device array inside libtpmd.so. Checked through the C ABI
against the regular device entry point, on two calls in a row (the second
runs over the scratch the first left behind), at the same tolerance as the
batch-composition tests: bit-identical frames, each call's device status
read through tpmd_device_status. This file is named to be collected last."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import tpmd
from metrics import cosine, max_abs

pytestmark = pytest.mark.gpu


def test_noalloc_matches_decode_device(model):
    import torch
    L = tpmd.load_library()
    dec = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, max_batch=2)
    dec.set_tensors(model["w"])
    dec.prepare()
    dec.set_feats(model["feats"])
    st = torch.from_numpy(model["styles"][:2]).cuda()
    ref = torch.empty((2, 3, 512, 512), device="cuda")
    dec.decode_device(st.data_ptr(), 2, ref.data_ptr(), 0)
    torch.cuda.synchronize()
    ref = ref.cpu().numpy()
    for i in range(2):  # two calls in a row through the shared static scratch
        out = torch.full((1, 3, 512, 512), float("nan"), device="cuda")
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rc = L.tpmd_decode_noalloc(C.c_void_p(dec._h), C.c_void_p(st[i:i + 1].data_ptr()), 1,
                                   C.c_void_p(out.data_ptr()), None)
        assert rc == 0, L.tpmd_last_error(C.c_void_p(dec._h)).decode()
        torch.cuda.synchronize()
        if i == 1:  # past the first call's one-time set-up, the device's free memory is untouched
            assert torch.cuda.mem_get_info()[0] == free0
        # the frames count only once the device status is clean
        rc = L.tpmd_device_status(C.c_void_p(dec._h), None)
        assert rc == 0, L.tpmd_last_error(C.c_void_p(dec._h)).decode()
        got = out.cpu().numpy()[0]
        print(f"noalloc call {i}: cos {cosine(got, ref[i]):.9f} max-abs {max_abs(got, ref[i]):.3e}")
        assert np.array_equal(got, ref[i])


def test_noalloc_rejects_what_does_not_fit(model):
    import torch
    L = tpmd.load_library()
    dec = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, max_batch=2)
    dec.set_tensors(model["w"])
    dec.prepare()
    dec.set_feats(model["feats"])
    st = torch.zeros((2, 512), device="cuda")
    out = torch.empty((2, 3, 512, 512), device="cuda")
    rc = L.tpmd_decode_noalloc(C.c_void_p(dec._h), C.c_void_p(st.data_ptr()), 2,
                               C.c_void_p(out.data_ptr()), None)
    assert rc == -1
    assert b"exceeds its static scratch" in L.tpmd_last_error(C.c_void_p(dec._h))
    d32 = tpmd.MotionDecoder(0, tpmd.DTYPE_F32, max_batch=1)
    d32.set_tensors(model["w"])
    d32.prepare()
    d32.set_feats(model["feats"])
    rc = L.tpmd_decode_noalloc(C.c_void_p(d32._h), C.c_void_p(st.data_ptr()), 1,
                               C.c_void_p(out.data_ptr()), None)
    assert rc == -1
    assert b"f16" in L.tpmd_last_error(C.c_void_p(d32._h))
