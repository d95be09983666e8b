"""Graph-level pin of the oracle against the reference's own code.

oracle/ref_build.py compiles the reference's src/motion_dec.cpp,
src/motion_enc.cpp and src/gguf_load.cpp where they lie, over the ggml
stand-in in oracle/refgraph/ (stock ggml ops restated from their
definitions; the patched ops are the reference's own constructors and CPU
forward functions from patches/ggml-tp-ops.patch). These tests load a
motion_ae GGUF file through the reference's loader (with its
motion_ae_scale folding), run its prepare(), its exact parity graph, its
fast batched graph in f32 and in its f16 mode, and its motion encoder, and
compare each with the oracle on the same seeded inputs.

Tolerances: derived weights bit-exact; f32 graphs 1 - cosine <= 1e-8 (the
two sides sum in different orders); the f16 fast graph 1 - cosine <= 3e-5 on
frames (f16 rounding of GEMM operands turns order-level differences into
occasional one-ulp flips that the warp amplifies level by level) and the same
SSIM against the fp32 frames within 0.001.

Skipped when oracle/_ref/libtpgraph.so is absent (no reference tree)."""
from __future__ import annotations

import numpy as np
import pytest

import gguf_writer as gw
import oracle as O
from metrics import cosine, max_abs, ssim

pytestmark = pytest.mark.skipif(O.graph_lib() is None, reason="oracle/_ref/libtpgraph.so not built")


def _write(path, raw, dt):
    gw.write(path, [(n, a.reshape(gw.torch_shape(n, a.shape)), dt) for n, a in raw.items()])


@pytest.fixture(scope="module")
def parity_inputs():
    from tpmd import synth
    raw = synth.make_weights(seed=0, bias_std=0.1, flow_gain=synth.PARITY_FLOW_GAIN)
    return dict(raw=raw, feats=synth.make_feats(seed=0), styles=synth.styles_config0(seed=0, n=2))


@pytest.fixture(scope="module")
def f32_file(parity_inputs, tmp_path_factory):
    p = str(tmp_path_factory.mktemp("refgraph") / "motion_ae_f32.gguf")
    _write(p, parity_inputs["raw"], "f32")
    return p


@pytest.fixture(scope="module")
def ref32(f32_file):
    return O.RefGraph(f32_file)


@pytest.fixture(scope="module")
def oracle32(parity_inputs):
    from tpmd import synth
    return O.Decoder(synth.fold(parity_inputs["raw"], O.scale_for), parity_inputs["feats"])


def test_loader_folds_like_the_oracle(parity_inputs, ref32):
    """weights_t::load + motion_ae_scale (src/gguf_load.cpp:50-197,
    src/motion_enc.cpp:14-45) against the oracle's scale table"""
    from tpmd import synth
    want = synth.fold(parity_inputs["raw"], O.scale_for)
    for name, a in want.items():
        got = ref32.tensor(name)
        assert np.array_equal(got, a.reshape(-1)), name


def test_prepare_matches_oracle_derivation(parity_inputs, ref32):
    """motion_dec::prepare (src/motion_dec.cpp:31-226): S_aug for all 15
    demodulated convs, the sub-pixel up-conv matrices and the cf GEMM
    matrices, bit for bit"""
    from tpmd import synth
    w = synth.fold(parity_inputs["raw"], O.scale_for)
    shapes = synth.tensor_shapes()
    names = ["dec.conv1.conv.weight"] + [f"dec.convs.{i}.conv.weight" for i in range(14)]
    for nm in names:
        oc, ic = shapes[nm][-4], shapes[nm][-3]
        W = w[nm].reshape(oc, ic, 3, 3)
        assert np.array_equal(ref32.tensor("saug." + nm).reshape(oc, ic + 1), O.saug(W, ic, oc)), nm
        if ".convs." in nm and int(nm.split(".")[2]) % 2 == 0:
            K = w[nm.replace("conv.weight", "conv.blur.kernel")]
            assert np.array_equal(ref32.tensor("tsubcf." + nm).reshape(4 * oc, 9 * ic),
                                  O.tsubcf(W, K, ic, oc)), nm
        elif ".convs." in nm:
            # cf rows r = ic + IC*(kw + 3 kh)
            acf = W.transpose(0, 2, 3, 1).reshape(oc, 9 * ic)
            assert np.array_equal(ref32.tensor("acf." + nm).reshape(oc, 9 * ic), acf), nm


def test_exact_graph_taps_and_frame(parity_inputs, ref32, oracle32):
    """the reference's parity graph (src/motion_dec.cpp:794-888) against the
    oracle's mode 0, every tap of every level and the frame"""
    st = parity_inputs["styles"][0]
    ref32.build(taps=True)
    ref32.set_feats(parity_inputs["feats"])
    img = ref32.decode(st, taps=True)
    ref = oracle32.decode(st, mode=0, keep_taps=True)
    worst = 0.0
    names = ["conv1_4"] + [f"r{8 << j}.{k}" for j in range(7)
                           for k in ("conv1", "conv2", "flowmap", "grid", "warp", "out", "rgb")]
    for name in names:
        a, b = ref32.tap(name), oracle32.tap(name)
        assert a.shape == b.shape, name
        d = 1.0 - cosine(a, b)
        worst = max(worst, d)
        assert d <= 1e-8, (name, d, max_abs(a, b))
    d = 1.0 - cosine(img, ref)
    print(f"exact graph: worst tap 1-cos {worst:.2e}; frame 1-cos {d:.2e} max-abs {max_abs(img, ref):.2e}")
    assert d <= 1e-8


def test_fast_graph_f32(parity_inputs, ref32, oracle32):
    """the reference's fast batched graph (src/motion_dec.cpp:889-1123, two
    frames per dispatch, CPU flavour) against the oracle's sub-pixel mode"""
    assert ref32.build(batch=2) == 2
    ref32.set_feats(parity_inputs["feats"])
    imgs = ref32.decode_batch(parity_inputs["styles"])
    for i, st in enumerate(parity_inputs["styles"]):
        ref = oracle32.decode(st, mode=1)
        d = 1.0 - cosine(imgs[i], ref)
        print(f"fast graph f32 frame {i}: 1-cos {d:.2e} max-abs {max_abs(imgs[i], ref):.2e}")
        assert d <= 1e-8


def test_fast_graph_f16(parity_inputs, oracle32, tmp_path):
    """the reference's f16 mode (an f16 motion_ae file loaded with keep_f16,
    src/tp.cpp:24-27) against the oracle's emulation of that arithmetic
    (mode 1 | REF_F16_GRAPH) on the same f16-rounded file values"""
    from tpmd import synth
    raw = parity_inputs["raw"]
    p = str(tmp_path / "motion_ae_f16.gguf")
    _write(p, raw, "f16")
    rg = O.RefGraph(p, keep_f16=True)
    rg.build(batch=2)
    rg.set_feats(parity_inputs["feats"])
    imgs = rg.decode_batch(parity_inputs["styles"])
    raw16 = {k: v.astype(np.float16).astype(np.float32) for k, v in raw.items()}
    od16 = O.Decoder(synth.fold(raw16, O.scale_for), parity_inputs["feats"])
    for i, st in enumerate(parity_inputs["styles"]):
        emu = od16.decode(st, mode=1 | O.REF_F16_GRAPH)
        fp32 = oracle32.decode(st, mode=0)
        d = 1.0 - cosine(imgs[i], emu)
        s_ref, s_emu = ssim(imgs[i], fp32), ssim(emu, fp32)
        print(f"fast graph f16 frame {i}: 1-cos {d:.2e}; SSIM vs fp32: reference {s_ref:.5f}, "
              f"emulation {s_emu:.5f}")
        assert d <= 3e-5
        assert abs(s_ref - s_emu) <= 1e-3


def test_encoder_graph(tmp_path):
    """motion_enc::run (src/motion_enc.cpp:46-184) against the oracle's
    encoder: appearance, lambda, motion and the seven decoder feats"""
    from tpmd import synth
    renc = synth.make_encoder_weights(0)
    rdec = synth.make_weights(seed=0)
    p = str(tmp_path / "motion_ae_f32.gguf")
    _write(p, {**renc, **rdec}, "f32")
    rg = O.RefGraph(p)
    img = synth.make_image(0)
    r = rg.encode(img)
    o = O.Encoder(synth.fold(renc, O.scale_for)).run(img)
    for k in ("appearance", "lam", "motion"):
        assert 1.0 - cosine(r[k], o[k]) <= 1e-9, k
    for j in range(7):
        assert 1.0 - cosine(r["feats"][j], o["feats"][j]) <= 1e-9, j
