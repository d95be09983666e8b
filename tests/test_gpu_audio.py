"""The B200 audio encoder (tpae_*) against the oracle's restatement of
audio_model::encode (src/audio_enc.cpp:55-236), float32 both sides (the GPU's
tcgen05 GEMMs by the three-pass TF32 split); exact, padded and cropped
inputs; the GGUF path."""
import numpy as np
import pytest

import gguf_writer as gw
import oracle as O
import tpmd
from metrics import cosine
from tpmd import synth

pytestmark = pytest.mark.gpu


def _enc(cfg, w):
    e = tpmd.AudioEncoder(cfg, 0)
    e.set_tensors(w)
    e.prepare()
    return e


@pytest.mark.parametrize("cfg", [synth.AUDIO_SMALL, synth.AUDIO_CONFIG], ids=["small", "base"])
def test_encode_matches_oracle(cfg):
    w = synth.make_audio_weights(cfg, 0)
    au = synth.make_audio(2.0, 0)
    e = _enc(cfg, w)
    o = O.Aud(cfg, w)
    for n, S in ((au.size, 50), (au.size - 123, 50), (au.size, 37)):  # exact, padded, cropped
        got, ref = e.encode(au[:n], S), o.encode(au[:n], S)
        assert cosine(got, ref) > 1 - 1e-6
        assert np.abs(got - ref).max() < 1e-3 * np.abs(ref).max()
    e.close()


def test_encode_30s_clip_deterministic():
    cfg = synth.AUDIO_CONFIG
    w = synth.make_audio_weights(cfg, 0)
    au = synth.make_audio(30.0, 1)
    e = _enc(cfg, w)
    a = e.encode(au, 750)
    b = e.encode(au, 750)
    assert a.shape == (750, 512) and np.isfinite(a).all() and np.array_equal(a, b)
    e.close()


def test_gguf_load_and_config_check(tmp_path):
    cfg = synth.AUDIO_SMALL
    w = synth.make_audio_weights(cfg, 0)
    kv = [("float.audio.n_layers", gw.T_U32, cfg["n_layers"]), ("float.audio.hidden_size", gw.T_U32, cfg["hidden"]),
          ("float.audio.conv_kernel.0", gw.T_U32, cfg["conv_kernel"][0]), ("float.audio.ln_eps", gw.T_F32, cfg["ln_eps"])]
    p = str(tmp_path / "audio_f32.gguf")
    gw.write(p, [(n, a, "f32") for n, a in w.items()], arch="float-audio", extra_kv=kv)
    a = tpmd.AudioEncoder(cfg, 0)
    a.load_gguf(p)
    a.prepare()
    b = _enc(cfg, w)
    au = synth.make_audio(1.0, 2)
    assert np.array_equal(a.encode(au, 25), b.encode(au, 25))
    wrong = tpmd.AudioEncoder(dict(cfg, n_layers=3), 0)
    with pytest.raises(tpmd.TpmdError, match="float.audio.n_layers"):
        wrong.load_gguf(p)
    for s in (a, b, wrong):
        s.close()


def test_errors():
    cfg = synth.AUDIO_SMALL
    with pytest.raises(tpmd.TpmdError, match="invalid config"):
        tpmd.AudioEncoder(dict(cfg, n_heads=3), 0)
    e = tpmd.AudioEncoder(cfg, 0)
    with pytest.raises(tpmd.TpmdError, match="not prepared"):
        e.encode(np.zeros(16000, np.float32), 25)
    e.set_tensors(synth.make_audio_weights(cfg, 0))
    e.prepare()
    with pytest.raises(tpmd.TpmdError, match="too short"):
        e.encode(np.zeros(100, np.float32), 1)
    e.close()
