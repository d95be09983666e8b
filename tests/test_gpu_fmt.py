"""The B200 flow-matching sampler (tpfm_*) against the oracle's restatement
(src/fmt.cpp:9-211, src/pipeline.cpp:15-91): one CFG-batched forward and a
whole 9-step chunk, float32 (tcgen05 GEMMs by the three-pass TF32 split) and
f16-weight modes; the GGUF path with its hyper-parameter check."""
import numpy as np
import pytest

import gguf_writer as gw
import oracle as O
import tpmd
from metrics import cosine
from tpmd import synth

pytestmark = pytest.mark.gpu

CONFIGS = [synth.FMT_SMALL, synth.FMT_CONFIG]
IDS = ["small", "config4"]


def _inputs(cfg, seed=1):
    rng = np.random.default_rng(seed)
    T = cfg["chunk_frames"] + cfg["prev_frames"]
    CD = cfg["dim_w"] + cfg["dim_a"] + cfg["dim_e"]
    return (rng.standard_normal((T, cfg["dim_w"])).astype(np.float32),
            rng.standard_normal((3, T, CD)).astype(np.float32))


def _sampler(cfg, w, dtype):
    s = tpmd.FmtSampler(cfg, 0, dtype)
    s.set_tensors(w)
    s.prepare()
    return s


@pytest.mark.parametrize("cfg", CONFIGS, ids=IDS)
def test_forward_f32_matches_oracle(cfg):
    w = synth.make_fmt_weights(cfg, 0)
    x60, cond = _inputs(cfg)
    s = _sampler(cfg, w, tpmd.DTYPE_F32)
    o = O.Fmt(cfg, w)
    for t in (0.0, 0.4444444, 1.0):
        v, r = s.forward(x60, cond, t), o.forward(x60, cond, t)
        assert cosine(v, r) > 1 - 1e-6
        assert np.abs(v - r).max() < 1e-3 * np.abs(r).max()
    s.close()


@pytest.mark.parametrize("cfg", CONFIGS, ids=IDS)
def test_chunk_f32_matches_oracle(cfg):
    w = synth.make_fmt_weights(cfg, 0)
    io = synth.make_fmt_chunk(cfg, 0)
    args = (io["wr"], io["prev_wa"], io["cond_audio"], io["prev_x"], io["x0"], io["emotion"])
    s = _sampler(cfg, w, tpmd.DTYPE_F32)
    got = s.sample(*args)
    again = s.sample(*args)  # graph replay
    ref = O.Fmt(cfg, w).sample(*args)
    assert np.array_equal(got, again)
    assert cosine(got, ref) > 1 - 1e-6
    assert np.abs(got - ref).max() < 1e-3 * np.abs(ref).max()
    s.close()


def test_chunk_f16_close_to_f32_oracle():
    cfg = synth.FMT_CONFIG
    w = synth.make_fmt_weights(cfg, 0)
    io = synth.make_fmt_chunk(cfg, 0)
    args = (io["wr"], io["prev_wa"], io["cond_audio"], io["prev_x"], io["x0"], io["emotion"])
    s = _sampler(cfg, w, tpmd.DTYPE_F16)
    got = s.sample(*args)
    ref = O.Fmt(cfg, w).sample(*args)
    # f16 weights and GEMM inputs, f32 accumulation: the reference's fast mode
    assert cosine(got, ref) > 0.999
    s.close()


def test_gguf_load_and_config_check(tmp_path):
    cfg = synth.FMT_SMALL
    w = synth.make_fmt_weights(cfg, 0)
    kv = [("float.fmt." + k, gw.T_U32, v) for k, v in (("dim_h", cfg["dim_h"]), ("depth", cfg["depth"]),
                                                         ("n_heads", cfg["n_heads"]), ("nfe", cfg["nfe"]))]
    kv += [("float.fmt.a_cfg_scale", gw.T_F32, cfg["a_cfg"]), ("float.fmt.ln_eps", gw.T_F32, cfg["ln_eps"])]
    p = str(tmp_path / "fmt_f32.gguf")
    gw.write(p, [(n, a, "f32") for n, a in w.items()], arch="float-fmt", extra_kv=kv)
    keys = tpmd.gguf_kv(p, "float-fmt")
    assert keys["float.fmt.dim_h"] == cfg["dim_h"] and keys["general.architecture"] == "float-fmt"
    a = tpmd.FmtSampler(cfg, 0, tpmd.DTYPE_F32)
    a.load_gguf(p)
    a.prepare()
    b = _sampler(cfg, w, tpmd.DTYPE_F32)
    x60, cond = _inputs(cfg)
    assert np.array_equal(a.forward(x60, cond, 0.25), b.forward(x60, cond, 0.25))
    wrong = tpmd.FmtSampler(dict(cfg, depth=3), 0, tpmd.DTYPE_F32)
    with pytest.raises(tpmd.TpmdError, match="float.fmt.depth"):
        wrong.load_gguf(p)
    for s in (a, b, wrong):
        s.close()


def test_errors():
    cfg = synth.FMT_SMALL
    with pytest.raises(tpmd.TpmdError, match="invalid config"):
        tpmd.FmtSampler(dict(cfg, n_heads=3), 0)
    s = tpmd.FmtSampler(cfg, 0)
    x60, cond = _inputs(cfg)
    with pytest.raises(tpmd.TpmdError, match="not prepared"):
        s.forward(x60, cond, 0.0)
    with pytest.raises(tpmd.TpmdError, match="unknown tensor"):
        s.set_tensors({"blocks.9.attn.qkv.weight": np.zeros(4, np.float32)})
    w = synth.make_fmt_weights(cfg, 0)
    del w["decoder.linear.bias"]
    s.set_tensors(w)
    with pytest.raises(tpmd.TpmdError, match="missing tensor decoder.linear.bias"):
        s.prepare()
    s.close()
