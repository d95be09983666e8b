"""The end-to-end generator (tppl_*, generate_impl of src/pipeline.cpp:99-186)
against the oracle stages chained the same way in Python: motion encoder,
audio encoder, two sampler chunks with the autoregressive context, decoder
styles = appearance + motion, and decoded frames. float32 throughout."""
import numpy as np
import pytest

import oracle as O
import tpmd
from metrics import cosine
from tpmd import synth

pytestmark = pytest.mark.gpu

FMT = synth.FMT_SMALL
AUD = synth.AUDIO_SMALL512


@pytest.fixture(scope="module")
def case(model):
    w_enc = synth.fold(synth.make_encoder_weights(0), O.scale_for)
    w_aud = synth.make_audio_weights(AUD, 0)
    w_fmt = synth.make_fmt_weights(FMT, 0)
    img = synth.make_image(0)
    audio = synth.make_audio(3.0, 0)  # 75 frames: two chunks, the second padded
    n = tpmd.Pipeline(0, "f32", FMT, AUD).n_frames(audio.size)
    noise = np.random.default_rng(5).standard_normal((2, 50, 512)).astype(np.float32)
    return dict(w_enc=w_enc, w_aud=w_aud, w_fmt=w_fmt, w_dec=model["w"], img=img, audio=audio, n=n, noise=noise)


def _oracle_styles(c, emotion=3):
    e = O.Encoder(c["w_enc"]).run(c["img"])
    wa = O.Aud(AUD, c["w_aud"]).encode(c["audio"], c["n"])
    f = O.Fmt(FMT, c["w_fmt"])
    P, CF, D = 10, 50, 512
    prev_x, prev_wa = np.zeros((P, D), np.float32), np.zeros((P, D), np.float32)
    r_d = []
    for ck in range(2):
        idx = np.minimum(np.arange(ck * CF, ck * CF + CF), c["n"] - 1)
        wa_t = wa[idx]
        out = f.sample(e["motion"], prev_wa, wa_t, prev_x, c["noise"][ck], emotion)
        r_d.append(out)
        prev_x, prev_wa = out[CF - P:], wa_t[CF - P:]
    r_d = np.concatenate(r_d)[:c["n"]]
    return e, e["appearance"][None] + r_d


@pytest.fixture(scope="module")
def pipe(case):
    p = tpmd.Pipeline(0, "f32", FMT, AUD, max_batch=16)
    p.set_weights(case["w_enc"], case["w_aud"], case["w_fmt"], case["w_dec"])
    yield p
    p.close()


def test_styles_match_oracle_chain(pipe, case):
    got = pipe.styles(case["img"], case["audio"], 3, noise=case["noise"])
    _, ref = _oracle_styles(case)
    assert got.shape == (75, 512)
    assert cosine(got, ref) > 1 - 1e-6
    for t in (0, 49, 50, 74):  # both chunks, the chunk boundary, the padded tail
        assert cosine(got[t], ref[t]) > 1 - 1e-5, t


def test_frames_match_oracle_decoder(pipe, case):
    frames = pipe.generate(case["img"], case["audio"], 3, noise=case["noise"])
    e, styles = _oracle_styles(case)
    dec = O.Decoder(case["w_dec"], e["feats"])
    for t in (0, 60):
        ref = dec.decode(styles[t], mode=0)
        c = cosine(frames[t], ref)
        assert c > 0.999, (t, c, float(np.abs(frames[t] - ref).max()))


def test_seeded_noise_and_callback(pipe, case):
    a = pipe.styles(case["img"], case["audio"], 3, seed=7)
    b = pipe.styles(case["img"], case["audio"], 3, seed=7)
    c = pipe.styles(case["img"], case["audio"], 3, seed=8)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    seen = []
    frames = pipe.generate(case["img"], case["audio"], 3, seed=7)

    def cb(i, f):
        seen.append(i)
        assert np.array_equal(f, frames[i])
        return 1 if i == 20 else 0  # stop early

    n = pipe.generate_cb(case["img"], case["audio"], 3, cb, seed=7)
    assert n == 75 and seen == list(range(21))


def test_pipeline_rejects_mismatched_stages():
    with pytest.raises(tpmd.TpmdError, match="dim_a"):
        tpmd.Pipeline(0, "f32", FMT, synth.AUDIO_SMALL)


def test_styles_cb_chunks_match_styles(pipe, case):
    ref = pipe.styles(case["img"], case["audio"], 3, noise=case["noise"])
    seen = []

    def cb(f0, st):
        seen.append((f0, st.copy()))
        return 0

    assert pipe.styles_cb(case["img"], case["audio"], 3, cb, noise=case["noise"]) == 75
    assert [f for f, _ in seen] == [0, 50] and seen[1][1].shape == (25, 512)  # the padded tail is not passed
    assert np.array_equal(np.concatenate([s for _, s in seen]), ref)
    calls = []
    pipe.styles_cb(case["img"], case["audio"], 3, lambda f0, st: calls.append(f0) or 1, noise=case["noise"])
    assert calls == [0]  # a nonzero return stops the sampler
