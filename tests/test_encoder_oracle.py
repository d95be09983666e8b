"""The oracle's motion-encoder restatement (folded weights, f32, the graph of
src/motion_enc.cpp:46-184) against an independent float64 torch formulation
of the unfolded LIA encoder (tests/torch_lia.py): pins the restatement's
composition, folding and layouts. CPU only."""
import numpy as np
import pytest

import oracle as O
import torch_lia
from metrics import cosine
from tpmd import synth


@pytest.fixture(scope="module")
def enc_case():
    raw = synth.make_encoder_weights(0)
    img = synth.make_image(0)
    return raw, img


def test_oracle_encoder_matches_torch_float64(enc_case):
    raw, img = enc_case
    got = O.Encoder(synth.fold(raw, O.scale_for)).run(img)
    ref = torch_lia.TorchEncoder(raw).run(img)
    for k in ("appearance", "lam", "motion"):
        assert cosine(got[k], ref[k]) > 1 - 1e-9, k
        assert np.abs(got[k] - ref[k]).max() < 1e-4 * max(1.0, np.abs(ref[k]).max()), k
    for j in range(7):
        g, r = got["feats"][j], ref["feats"][j]
        assert g.shape == ((8 << j) ** 2, O.ST_OC[j])
        assert cosine(g, r) > 1 - 1e-9, j
        assert np.abs(g - r).max() < 1e-4 * max(1.0, np.abs(r).max()), j


def test_oracle_encoder_rejects_bad_tensors(enc_case):
    raw, _ = enc_case
    w = synth.fold(raw, O.scale_for)
    bad = dict(w)
    bad["enc.fc.4.bias"] = np.zeros(21, np.float32)
    with pytest.raises(RuntimeError, match="enc.fc.4.bias"):
        O.Encoder(bad)
    part = {k: v for k, v in w.items() if k != "dec.direction.Q"}
    with pytest.raises(RuntimeError, match="missing tensor dec.direction.Q"):
        O.Encoder(part).run(np.zeros((3, 512, 512), np.float32))
