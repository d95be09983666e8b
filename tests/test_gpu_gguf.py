"""The decoder loaded from a motion_ae GGUF file (tpmd_load_gguf, the
decoder half of tp_ctx::load, src/tp.cpp:32-38) equals the decoder loaded
tensor by tensor from the same scale-folded host copies: identical prepared
weight arena and identical frames."""
import numpy as np
import pytest
import torch

import gguf_writer as gw
import tpmd
from tpmd.multi import arena_tensor

pytestmark = pytest.mark.gpu


def _from_file(path, dtype):
    d = tpmd.MotionDecoder(0, dtype, 4)
    d.load_gguf(path)
    d.prepare()
    return d


def _from_tensors(w, dtype):
    d = tpmd.MotionDecoder(0, dtype, 4)
    d.set_tensors(w)
    d.prepare()
    return d


@pytest.mark.parametrize("dtype", [tpmd.DTYPE_F32, tpmd.DTYPE_F16])
def test_gguf_load_equals_tensor_load(model, tmp_path, dtype):
    p = str(tmp_path / "motion_ae_f32.gguf")
    rng = np.random.default_rng(3)
    extra = [("enc.net_app.convs.0.0.weight", rng.standard_normal((8, 3, 3, 3)).astype(np.float32), "f32"),
             ("dec.direction.weight", rng.standard_normal((512, 20)).astype(np.float32), "f32")]
    gw.write(p, extra + [(n, a.reshape(gw.torch_shape(n, a.shape)), "f32") for n, a in model["raw"].items()])
    a, b = _from_file(p, dtype), _from_tensors(model["w"], dtype)
    dev = torch.device("cuda", 0)
    wa, wb = arena_tensor(a, 0, dev), arena_tensor(b, 0, dev)
    assert wa.numel() == wb.numel() and torch.equal(wa, wb)
    for d in (a, b):
        d.set_feats(model["feats"])
    st = model["styles"][:2]
    fa, fb = a.decode(st), b.decode(st)
    assert np.array_equal(fa, fb)
    a.close()
    b.close()


def test_gguf_load_reports_missing_tensor(model, tmp_path):
    p = str(tmp_path / "partial.gguf")
    items = [(n, a.reshape(gw.torch_shape(n, a.shape)), "f32") for n, a in model["raw"].items()
             if n != "dec.to_rgbs.3.bias"]
    gw.write(p, items)
    d = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, 4)
    d.load_gguf(p)
    with pytest.raises(tpmd.TpmdError, match="dec.to_rgbs.3.bias"):
        d.prepare()
    d.close()


def test_gguf_load_rejects_wrong_architecture(model, tmp_path):
    p = str(tmp_path / "arch.gguf")
    gw.write(p, [("dec.input.input", model["raw"]["dec.input.input"], "f32")], arch="lia")
    d = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, 4)
    with pytest.raises(tpmd.TpmdError, match="unexpected architecture 'lia'"):
        d.load_gguf(p)
    d.close()
