"""The oracle's audio encoder (src/audio_enc.cpp:55-236) against an
independent float64 torch wav2vec2 formulation (tests/torch_lia.py). CPU."""
import numpy as np
import pytest

import oracle as O
import torch_lia
import tpmd
from metrics import cosine
from tpmd import synth


@pytest.mark.parametrize("cfg", [synth.AUDIO_SMALL, synth.AUDIO_CONFIG], ids=["small", "base"])
def test_oracle_audio_matches_torch_float64(cfg):
    w = synth.make_audio_weights(cfg, 0)
    au = synth.make_audio(2.0, 0)
    for n, S in ((au.size, 50), (au.size - 123, 50), (au.size, 37)):  # exact, padded, cropped
        got = O.Aud(cfg, w).encode(au[:n], S)
        ref = torch_lia.TorchAudio(cfg, w).encode(au[:n], S)
        assert got.shape == (S, cfg["dim_w"])
        assert cosine(got, ref) > 1 - 1e-9
        assert np.abs(got - ref).max() < 1e-4 * np.abs(ref).max()


def test_default_config_is_the_references():
    c = tpmd.default_audio_config()
    assert (c["n_layers"], c["n_heads"], c["hidden"], c["ffn"], c["dim_w"]) == (12, 12, 768, 3072, 512)
    assert c["conv_kernel"] == (10, 3, 3, 3, 3, 2, 2) and c["conv_stride"] == (5, 2, 2, 2, 2, 2, 2)
    assert c["conv_dim"] == (512,) * 7 and (c["pos_kernel"], c["pos_groups"]) == (128, 16)
    assert (c["sample_rate"], c["fps"]) == (16000, 25) and abs(c["ln_eps"] - 1e-5) < 1e-10
