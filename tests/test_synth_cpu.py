"""The seeded synthetic inputs that stand in for the benchmark configs
(no public dataset is involved) follow the configs' stated shapes and
distributions: config 0's 20-direction QR-orthonormal motion basis,
w_src ~ N(0, 1)^512 and alpha ~ N(0, 0.5)^20; config 2's per-frame random
walk (start N(0, 0.5), steps N(0, 0.05), clipped to [-3, 3]); the feature
pyramid's shapes (r = 8..512, channels 512/512/512/256/128/64/32) with N(0, 1)
channels; random-init weights with modulation biases 1 and the normalised
[1,3,3,1] x [1,3,3,1] blur kernel (times 4, the up-sampling gain); config
4's band-limited (80-4000 Hz) audio and the portrait image in [-1, 1].
Seeded: equal seeds give equal arrays."""
from __future__ import annotations

import numpy as np

from tpmd import synth

ST_OC = (512, 512, 512, 256, 128, 64, 32)


def test_motion_basis_and_config0_styles():
    w_src, q = synth.make_basis(0)
    assert w_src.shape == (512,) and q.shape == (512, 20)
    np.testing.assert_allclose(q.T @ q, np.eye(20), atol=1e-5)
    assert abs(float(w_src.mean())) < 0.15 and abs(float(w_src.std()) - 1.0) < 0.1
    st = synth.styles_config0(0, n=400)
    alpha = (st - w_src[None, :]) @ q  # recover alpha through the orthonormal basis
    assert abs(float(alpha.std()) - 0.5) < 0.02 and abs(float(alpha.mean())) < 0.02
    np.testing.assert_array_equal(st, synth.styles_config0(0, n=400))


def test_config2_random_walk():
    w_src, q = synth.make_basis(0)
    st = synth.styles_walk(0, n=2000)
    alpha = (st - w_src[None, :]) @ q
    steps = np.diff(alpha, axis=0)
    inner = np.abs(alpha[1:]) < 2.9  # steps away from the clip bound
    assert abs(float(steps[inner].std()) - 0.05) < 0.003
    assert float(np.abs(alpha).max()) <= 3.0 + 1e-4
    assert abs(float(alpha[0].std()) - 0.5) < 0.25  # the start, one 20-vector drawn N(0, 0.5)
    # per-clip seeds: a clip index gives another walk, the same index the same one
    assert not np.array_equal(synth.styles_walk(0, 50, clip=1), synth.styles_walk(0, 50, clip=0))
    np.testing.assert_array_equal(synth.styles_walk(0, 50, clip=3), synth.styles_walk(0, 50, clip=3))


def test_feats_pyramid(model):
    for feats in (model["feats"], synth.make_feats(0, smooth=False)):  # smooth (seed 0), white
        assert len(feats) == 7
        for j, f in enumerate(feats):
            r = 8 << j
            assert f.shape == (r * r, ST_OC[j]) and f.dtype == np.float32
            if r >= 64:
                assert abs(float(f.mean())) < 0.05 and abs(float(f.std()) - 1.0) < 0.05
    sm = model["feats"][6]
    # the smooth maps are spatially correlated, the white ones are not
    img = sm[:, 0].reshape(512, 512)
    assert float(np.corrcoef(img[:, :-1].ravel(), img[:, 1:].ravel())[0, 1]) > 0.9


def test_random_init_weights():
    w = synth.make_weights(0)
    bk = synth.blur_kernel4()
    k1 = np.array([1, 3, 3, 1], np.float64)
    # normalised, times 4: the checkpoint's blur kernels include the gain of
    # the 2x up-sampling (src/motion_dec.cpp:158)
    np.testing.assert_allclose(bk, 4.0 * np.outer(k1, k1) / np.outer(k1, k1).sum(), rtol=1e-6)
    mods = [n for n in w if n.endswith("modulation.bias")]
    assert mods and all(np.all(w[n] == 1.0) for n in mods)
    others = [n for n in w if n.endswith("bias") and not n.endswith("modulation.bias")]
    assert others and all(np.all(w[n] == 0.0) for n in others)
    shapes = synth.tensor_shapes()
    assert set(w) == set(shapes) and all(w[n].shape == tuple(shapes[n]) for n in w)
    np.testing.assert_array_equal(w["dec.convs.0.conv.weight"], synth.make_weights(0)["dec.convs.0.conv.weight"])


def test_config4_audio_and_image():
    sr = 16000
    x = synth.make_audio(2.0, seed=0, sr=sr)
    assert x.shape == (2 * sr,) and abs(float(x.mean())) < 1e-4 and abs(float(x.std()) - 1.0) < 1e-3
    spec = np.abs(np.fft.rfft(x.astype(np.float64))) ** 2
    f = np.fft.rfftfreq(x.size, 1.0 / sr)
    outside = spec[(f < 60) | (f > 4100)].sum() / spec.sum()
    assert outside < 0.01  # band-limited to 80-4000 Hz (the envelope spreads a few Hz)
    img = synth.make_image(0)
    assert img.shape == (3, 512, 512) and img.dtype == np.float32
    assert float(img.min()) >= -1.0 and float(img.max()) <= 1.0
