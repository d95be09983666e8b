"""Device-side failure detection without a GPU fault.

Every pipeline wait in the tcgen05 kernels is bounded; on expiry a kernel
sets the handle's device error flag, issues no further work, frees its
tensor memory and returns, so the CUDA context stays usable. The test hook
tpmd_debug_expire_wait makes the next decode's first tcgen05 conv wait on an
mbarrier that nothing completes, with a 1 ms limit. The tests check that the
expiry reaches the caller the way the reference reports errors
(src/tp.cpp:70-83: an int status and the last-error string): as -1 from the
synchronous host entry point, and through tpmd_device_status after the
asynchronous device entry point; and that the next decode is bit-identical
to one on a fresh handle."""
from __future__ import annotations

import numpy as np
import pytest

import tpmd

pytestmark = pytest.mark.gpu

WAIT_NS = 1_000_000  # 1 ms


def _dec(model):
    d = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, 2)
    d.set_tensors(model["w"])
    d.prepare()
    d.set_feats(model["feats"])
    return d


@pytest.fixture(scope="module")
def clean_frames(model):
    return _dec(model).decode(model["styles"][:2])


def test_expired_wait_fails_host_decode(model, clean_frames):
    d = _dec(model)
    d.debug_expire_wait(WAIT_NS)
    with pytest.raises(tpmd.TpmdError, match="timed out"):
        d.decode(model["styles"][:2])
    # the hook fires once; the flag was read and cleared by the failing call
    assert np.array_equal(d.decode(model["styles"][:2]), clean_frames)


def test_expired_wait_reported_by_device_status(model, clean_frames):
    import torch
    d = _dec(model)
    st = torch.from_numpy(model["styles"][:2]).cuda()
    out = torch.empty((2, 3, 512, 512), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    d.device_status(stream)  # nothing pending
    d.debug_expire_wait(WAIT_NS)
    d.decode_device(st.data_ptr(), 2, out.data_ptr(), stream)  # enqueues: rc 0
    with pytest.raises(tpmd.TpmdError, match="timed out"):
        d.device_status(stream)
    d.device_status(stream)  # read and cleared
    d.decode_device(st.data_ptr(), 2, out.data_ptr(), stream)
    d.device_status(stream)
    assert np.array_equal(out.cpu().numpy(), clean_frames)


def test_hook_rejects_bad_arguments(model):
    d = _dec(model)
    with pytest.raises(tpmd.TpmdError, match="wait_ns"):
        d.debug_expire_wait(0)
    d32 = tpmd.MotionDecoder(0, tpmd.DTYPE_F32, 1)
    with pytest.raises(tpmd.TpmdError, match="tcgen05"):
        d32.debug_expire_wait(WAIT_NS)
