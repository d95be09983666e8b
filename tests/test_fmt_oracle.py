"""The oracle's flow-matching transformer and chunk sampler (src/fmt.cpp:
9-211, src/pipeline.cpp:15-91) against an independent float64 torch DiT
(tests/torch_lia.py) and a direct restatement of the Euler/CFG loop. CPU."""
import numpy as np
import pytest

import oracle as O
import torch_lia
import tpmd
from metrics import cosine
from tpmd import synth


def _inputs(cfg, seed=1):
    rng = np.random.default_rng(seed)
    T = cfg["chunk_frames"] + cfg["prev_frames"]
    CD = cfg["dim_w"] + cfg["dim_a"] + cfg["dim_e"]
    return (rng.standard_normal((T, cfg["dim_w"])).astype(np.float32),
            rng.standard_normal((3, T, CD)).astype(np.float32))


@pytest.mark.parametrize("cfg", [synth.FMT_SMALL, synth.FMT_CONFIG], ids=["small", "config4"])
def test_oracle_forward_matches_torch_float64(cfg):
    w = synth.make_fmt_weights(cfg, 0)
    x60, cond = _inputs(cfg)
    for t in (0.0, 0.5555556, 1.0):
        v = O.Fmt(cfg, w).forward(x60, cond, t)
        r = torch_lia.TorchFmt(cfg, w).forward(x60, cond, t)
        assert cosine(v, r) > 1 - 1e-9
        assert np.abs(v - r).max() < 1e-4 * np.abs(r).max()


def test_oracle_sampler_matches_its_definition():
    cfg = synth.FMT_SMALL
    w = synth.make_fmt_weights(cfg, 0)
    io = synth.make_fmt_chunk(cfg, 0)
    f = O.Fmt(cfg, w)
    got = f.sample(io["wr"], io["prev_wa"], io["cond_audio"], io["prev_x"], io["x0"], io["emotion"])
    # the loop of src/pipeline.cpp:19-91 written out with the torch forward
    D, P, CF, nfe = cfg["dim_w"], cfg["prev_frames"], cfg["chunk_frames"], cfg["nfe"]
    T, CD = P + CF, D + cfg["dim_a"] + cfg["dim_e"]
    cond = np.zeros((3, T, CD), np.float32)
    for b in range(3):
        for fr in range(T):
            cond[b, fr, :D] = io["wr"]
            wa = io["prev_wa"][fr] if fr < P else io["cond_audio"][fr - P]
            if not (b == 0 and fr >= P):
                cond[b, fr, D:2 * D] = wa
            if b == 1:
                cond[b, fr, D + cfg["dim_a"] + io["emotion"]] = 1.0
    tf = torch_lia.TorchFmt(cfg, w)
    x = io["x0"].astype(np.float64)
    for s in range(nfe - 1):
        x60 = np.concatenate([io["prev_x"], x]).astype(np.float32)
        v = tf.forward(x60, cond, np.float32(s / (nfe - 1)))
        u, fu, a = v[0], v[1], v[2]
        vc = (u + cfg["a_cfg"] * (a - u)) + cfg["e_cfg"] * (fu - a)
        x = x + (np.float32((s + 1) / (nfe - 1)) - np.float32(s / (nfe - 1))) * vc[P:]
    assert cosine(got, x) > 1 - 1e-7
    assert np.abs(got - x).max() < 1e-3 * np.abs(x).max()


def test_default_config_is_the_references():
    c = tpmd.default_fmt_config()
    want = dict(dim_h=1024, depth=8, n_heads=8, dim_w=512, dim_a=512, dim_e=7, chunk_frames=50,
                prev_frames=10, attn_window=2, t_freq_dim=256, nfe=10, mlp_ratio=4.0, a_cfg=2.0, e_cfg=1.0)
    for k, v in want.items():
        assert c[k] == v, k
    assert abs(c["ln_eps"] - 1e-6) < 1e-12
