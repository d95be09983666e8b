"""Allocation proof of the decode loop, the device-side counterpart of the
reference's bench/tp-allocproof.cpp (zero allocations per frame once the
graphs exist): after a first call, which captures and instantiates the
chunk's CUDA graphs, further decodes leave the device's free memory
unchanged, through the device entry point and through the host entry point
with its split schedule."""
from __future__ import annotations

import numpy as np
import pytest

import tpmd

pytestmark = pytest.mark.gpu


def test_decodes_allocate_nothing_after_the_first(model):
    import torch
    d = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, max_batch=16)
    d.set_tensors(model["w"])
    d.prepare()
    d.set_feats(model["feats"])
    st = np.ascontiguousarray(np.concatenate([model["styles"]] * 4)[:16])
    s_d = torch.from_numpy(st).cuda()
    f_d = torch.empty((16, 3, 512, 512), device="cuda")
    f_h = np.empty((16, 3, 512, 512), np.float32)
    stream = torch.cuda.current_stream().cuda_stream
    d.decode_device(s_d.data_ptr(), 16, f_d.data_ptr(), stream)  # graphs captured here
    d.decode(st, out=f_h)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        d.decode_device(s_d.data_ptr(), 16, f_d.data_ptr(), stream)
        d.decode(st, out=f_h)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert np.array_equal(f_h, f_d.cpu().numpy())
