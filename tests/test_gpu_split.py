"""The host decode's split schedule (tpmd_decode / tpmd_decode_rgb24 on a
tcgen05 handle): the levels up to r128 run once per group of frames, the r256
and r512 levels in parts whose frames are copied to the host while the next
part computes. Each frame still sums the same terms in the same order as in a
whole-chunk decode, so the frames must be bit-identical to
tpmd_decode_device's, whatever the grouping: one group of parts (fewer than
16 frames in a chunk), two groups (16 or more), several chunks of max_batch
frames, and the plain sub-batch schedule it replaces (TPMD_NO_SPLIT)."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as O
import tpmd

pytestmark = pytest.mark.gpu


def _dec(model, max_batch):
    d = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, max_batch)
    d.set_tensors(model["w"])
    d.prepare()
    d.set_feats(model["feats"])
    return d


def _styles(model, n):
    st = np.concatenate([model["styles"]] * (n // len(model["styles"]) + 1))[:n]
    return np.ascontiguousarray(st + 0.01 * np.arange(n, dtype=np.float32)[:, None])  # distinct frames


def _device_frames(d, st):
    import torch
    s_d = torch.from_numpy(st).cuda()
    f_d = torch.empty((len(st), 3, 512, 512), device="cuda")
    d.decode_device(s_d.data_ptr(), len(st), f_d.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return f_d.cpu().numpy()


# (frames, max_batch): one group of parts; two groups; chunks of max_batch
# then a short last chunk; two groups with parts of several sizes
@pytest.mark.parametrize("n,max_batch", [(4, 8), (7, 8), (16, 16), (20, 8), (23, 24)])
def test_split_host_decode_matches_device(model, n, max_batch):
    d = _dec(model, max_batch)
    st = _styles(model, n)
    ref = _device_frames(d, st)
    host = d.decode(st)
    assert np.array_equal(host, ref)
    host2 = d.decode(st)  # again, through the cached graphs of every part
    assert np.array_equal(host2, ref)


def test_split_rgb24_and_plain_schedule_agree(model):
    d = _dec(model, 24)
    st = _styles(model, 23)
    ref = _device_frames(d, st)
    rgb = d.decode_rgb24(st)
    assert np.array_equal(rgb, O.chw_to_rgb24(ref))
    os.environ["TPMD_NO_SPLIT"] = "1"
    try:
        plain = d.decode(st)
    finally:
        del os.environ["TPMD_NO_SPLIT"]
    assert np.array_equal(plain, ref)
