"""The B200 motion encoder (tpme_*) against the oracle's restatement of
motion_enc::run (src/motion_enc.cpp:46-184), float32 both sides; its GGUF
path; and the device hand-off of the pyramid to the decoder
(tpmd_set_feats_device), which must equal the host set_feats path."""
import numpy as np
import pytest

import gguf_writer as gw
import oracle as O
import tpmd
from metrics import cosine
from tpmd import synth

pytestmark = pytest.mark.gpu

# float32 on both sides, different summation orders: per-output cosine and
# max-abs relative to the output's scale
COS_MIN = 1 - 1e-6
REL_MAX = 1e-4


@pytest.fixture(scope="module")
def enc_model():
    raw = synth.make_encoder_weights(0)
    w = synth.fold(raw, O.scale_for)
    img = synth.make_image(0)
    ref = O.Encoder(w).run(img)
    return dict(raw=raw, w=w, img=img, ref=ref)


@pytest.fixture(scope="module")
def encoder(enc_model):
    e = tpmd.MotionEncoder(0)
    e.set_tensors(enc_model["w"])
    e.prepare()
    yield e
    e.close()


def _close(got, ref, what):
    c = cosine(got, ref)
    err = float(np.abs(got - ref).max())
    scale = max(1.0, float(np.abs(ref).max()))
    assert c >= COS_MIN and err <= REL_MAX * scale, f"{what}: cos {c:.9f} max-abs {err:.3e}"


def test_encoder_matches_oracle(encoder, enc_model):
    got = encoder.run(enc_model["img"])
    ref = enc_model["ref"]
    for k in ("appearance", "lam", "motion"):
        _close(got[k], ref[k], k)
    for j in range(7):
        assert got["feats"][j].shape == ref["feats"][j].shape
        _close(got["feats"][j], ref["feats"][j], f"feat{j}")


def test_encoder_is_deterministic(encoder, enc_model):
    a = encoder.run(enc_model["img"])
    b = encoder.run(enc_model["img"])
    for k in ("appearance", "lam", "motion"):
        assert np.array_equal(a[k], b[k])
    for j in range(7):
        assert np.array_equal(a["feats"][j], b["feats"][j])


def test_encoder_gguf_equals_tensor_load(encoder, enc_model, tmp_path, model):
    p = str(tmp_path / "motion_ae_f32.gguf")
    items = [(n, a.reshape(gw.torch_shape(n, a.shape)), "f32") for n, a in model["raw"].items()]
    items += [(n, a, "f32") for n, a in enc_model["raw"].items()]
    gw.write(p, items)
    e = tpmd.MotionEncoder(0)
    e.load_gguf(p)
    e.prepare()
    a, b = e.run(enc_model["img"]), encoder.run(enc_model["img"])
    for k in ("appearance", "lam", "motion"):
        assert np.array_equal(a[k], b[k]), k
    for j in range(7):
        assert np.array_equal(a["feats"][j], b["feats"][j]), j
    e.close()


@pytest.mark.parametrize("dtype", [tpmd.DTYPE_F32, tpmd.DTYPE_F16])
def test_feats_device_handoff_equals_host_path(encoder, enc_model, model, dtype):
    out = encoder.run(enc_model["img"])
    d_dev = tpmd.MotionDecoder(0, dtype, 4)
    d_host = tpmd.MotionDecoder(0, dtype, 4)
    for d in (d_dev, d_host):
        d.set_tensors(model["w"])
        d.prepare()
    d_dev.set_feats_device(encoder.feat_ptrs())
    d_host.set_feats(out["feats"])
    st = model["styles"][:2]
    assert np.array_equal(d_dev.decode(st), d_host.decode(st))
    d_dev.close()
    d_host.close()


def test_encoder_errors(enc_model):
    e = tpmd.MotionEncoder(0)
    with pytest.raises(tpmd.TpmdError, match="weights not prepared"):
        e.run(enc_model["img"])
    with pytest.raises(tpmd.TpmdError, match="unknown tensor"):
        e.set_tensors({"enc.nope": np.zeros(3, np.float32)})
    with pytest.raises(tpmd.TpmdError, match="size mismatch"):
        e.set_tensors({"enc.fc.0.bias": np.zeros(3, np.float32)})
    part = {k: v for k, v in enc_model["w"].items() if k != "enc.fc.2.weight"}
    e.set_tensors(part)
    with pytest.raises(tpmd.TpmdError, match="missing tensor enc.fc.2.weight"):
        e.prepare()
    with pytest.raises(tpmd.TpmdError, match="no encoder run"):
        e.feat_ptrs()
    e.close()
