"""The GPU output conversion to RGB24 through the C ABI, bit-exact against
the oracle's restatement of tools/tp-cli.cpp:43-53: the op on edge values and
random frames, and tpmd_decode_rgb24 against the oracle's conversion of the
same frames from tpmd_decode (both sides deterministic)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import tpmd
from test_rgb24 import edge_values

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,h,w", [(1, 64, 64), (3, 512, 512), (2, 6, 10)])
def test_op_bit_exact(n, h, w):
    import torch
    rng = np.random.default_rng(n * h)
    v = rng.standard_normal(n * 3 * h * w).astype(np.float32) * 1.5
    ev = edge_values()
    k = min(ev.size, v.size)
    v[:k] = ev[:k]
    frames = v.reshape(n, 3, h, w)
    out = torch.zeros((n, h, w, 3), dtype=torch.uint8, device="cuda")
    tpmd.chw_to_rgb24(torch.from_numpy(frames).cuda(), out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.chw_to_rgb24(frames))


def test_op_rejects_bad_shapes():
    import torch
    f = torch.zeros((1, 3, 3, 3), device="cuda")
    o = torch.zeros((1, 3, 3, 3), dtype=torch.uint8, device="cuda")
    with pytest.raises(tpmd.TpmdError, match="multiple of 4"):
        tpmd.chw_to_rgb24(f, o)


def test_decode_rgb24_matches_f32_decode(model):
    d = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, 2)
    d.set_tensors(model["w"])
    d.prepare()
    d.set_feats(model["feats"])
    st = np.concatenate([model["styles"], model["styles"][:1] + 0.01])  # 5 frames, 3 sub-batches
    f32 = d.decode(st)
    rgb = d.decode_rgb24(st)
    assert rgb.shape == (5, 512, 512, 3)
    assert np.array_equal(rgb, O.chw_to_rgb24(f32))
