"""CPU tests of the oracle: pinned to the reference's own op code (golden
vectors, and live when oracle/_ref is built), to the reference's test_ops.cpp
known-answer checks, and to independent torch formulations."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from metrics import cosine, max_abs
from tpmd import synth


def _gather_case(d, name, m):
    feat, grid = d[name + ".feat"], d[name + ".grid"]
    return O.bilinear_gather(feat, m["W"], m["H"], grid, m["planar"], m["sp"])


def test_golden_gather(golden):
    d, meta = golden
    names = [n for n, m in meta.items() if m["op"] == "gather"]
    assert len(names) >= 6
    for n in names:
        got = _gather_case(d, n, meta[n])
        np.testing.assert_allclose(got, d[n + ".out"], rtol=1e-6, atol=1e-7, err_msg=n)


def test_golden_im2col_bit_exact(golden):
    d, meta = golden
    for n, m in meta.items():
        if m["op"] != "im2col_cf":
            continue
        got = O.im2col_cf(d[n + ".src"], m["IC"], m["IW"], m["IH"], m["N"], m["KW"], m["KH"],
                          m["s0"], m["s1"], m["p0"], m["p1"], m["d0"], m["d1"], m["f16"])
        ref = d[n + ".out"]
        assert got.shape == ref.shape, n
        assert np.array_equal(got.view(np.uint16 if m["f16"] else np.uint32),
                              ref.view(np.uint16 if m["f16"] else np.uint32)), n


def test_golden_fused_ops(golden):
    d, meta = golden
    for axis in (0, 2):
        n = f"bias_lrelu_axis{axis}"
        got = O.bias_lrelu((d[n + ".x"], meta[n]["ne"]), d[n + ".b"], axis)
        np.testing.assert_array_equal(got, d[n + ".out"])
    m = meta["subpix"]
    np.testing.assert_array_equal(
        O.subpix_lrelu(d["subpix.g0"], d["subpix.g1"], d["subpix.b"], m["W"], m["H"], m["OC"]),
        d["subpix.out"])
    m = meta["subpix_cl"]
    np.testing.assert_array_equal(
        O.subpix_lrelu_cl(d["subpix_cl.y4"], d["subpix_cl.b"], m["OC"], m["W"] * m["H"], m["B"], m["W"]),
        d["subpix_cl.out"])
    m = meta["upfirdn"]
    np.testing.assert_allclose(O.upfirdn2x(d["upfirdn.x"], d["upfirdn.k"], m["W"], m["H"], m["CB"]),
                               d["upfirdn.out"], rtol=1e-6, atol=1e-7)
    np.testing.assert_array_equal(O.clsp(d["clsp.cl"], d["clsp.m"], 7, 30), d["clsp.mul"])
    np.testing.assert_allclose(O.clsp(d["clsp.cl"], d["clsp.m"], 7, 30, d["clsp.o"]),
                               d["clsp.lerp"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(O.flow_grid(d["flow_grid.fl"], d["flow_grid.xs"], 30),
                               d["flow_grid.out"], rtol=1e-6, atol=1e-7)


@pytest.mark.skipif(O.ref_lib() is None, reason="reference op code not built here")
def test_live_reference_ops():
    """oracle vs the reference's CPU functions and CUDA kernels (run on the host)"""
    rng = np.random.default_rng(7)
    for c, w, h, f16, planar, sp in [(40, 9, 11, False, False, False), (16, 33, 7, True, True, True),
                                     (512, 4, 4, True, False, False)]:
        feat = rng.standard_normal((w * h, c)).astype(np.float16 if f16 else np.float32)
        g = rng.uniform(-1.2, 1.2, (w * h * 2, 2)).astype(np.float32)
        grid = np.ascontiguousarray(g.T) if planar else g
        a = O.bilinear_gather(feat, w, h, grid, planar, sp)
        for impl in ("ref_cpu", "ref_cu"):
            np.testing.assert_allclose(a, O.bilinear_gather(feat, w, h, grid, planar, sp, impl=impl),
                                       rtol=1e-6, atol=1e-7)
    src = rng.standard_normal((3, 9, 10, 48)).astype(np.float32)
    for f16 in (False, True):
        a = O.im2col_cf(src, 48, 10, 9, 3, dst_f16=f16)
        b = O.im2col_cf(src, 48, 10, 9, 3, dst_f16=f16, impl="ref_cu")
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


def _naive_upfirdn(x, W, C, k, up, pad0, pad1):
    """the reference test's double-precision upfirdn2d (tests/test_ops.cpp:16-40)"""
    UW = W * up
    PW = UW + pad0 + pad1
    OW = PW - 4 + 1
    pad = np.zeros((C, PW, PW))
    pad[:, pad0:pad0 + UW:up, pad0:pad0 + UW:up] = x.reshape(C, W, W)
    out = np.zeros((C, OW, OW))
    kk = k.reshape(4, 4)
    for a in range(4):
        for b in range(4):
            out += kk[a, b] * pad[:, a:a + OW, b:b + OW]
    return out


def test_reference_upfirdn_kats():
    """tests/test_ops.cpp:63-106: blur pad (2,2) and upsample2x against naive
    upfirdn at 1e-5 on mt19937-seeded-style N(0,1) inputs, W = 6, C = 3,
    normalised [1,3,3,1] kernel"""
    rng = np.random.default_rng(42)
    W, C = 6, 3
    x = rng.standard_normal(C * W * W).astype(np.float32)
    k1 = np.array([1, 3, 3, 1], np.float64)
    k = np.outer(k1, k1)
    k = (k / k.sum()).astype(np.float32)
    got = O.blur(x.reshape(C, W, W), k.ravel(), W, W, C, 2, 2)
    ref = _naive_upfirdn(x, W, C, k, 1, 2, 2)
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() < 1e-5
    got = O.upfirdn2x(x, k.ravel(), W, W, C).reshape(C, 2 * W, 2 * W)
    ref = _naive_upfirdn(x, W, C, k, 2, 2, 1)
    assert np.abs(got - ref).max() < 1e-5


def test_gather_vs_torch_grid_sample():
    rng = np.random.default_rng(3)
    for c, w, h in [(8, 16, 16), (5, 7, 12)]:
        feat = rng.standard_normal((w * h, c)).astype(np.float32)
        grid = rng.uniform(-1.1, 1.1, (w * h, 2)).astype(np.float32)
        got = O.bilinear_gather(feat, w, h, grid)
        ft = torch.tensor(feat, dtype=torch.float64).T.reshape(1, c, h, w)
        gt = torch.tensor(grid, dtype=torch.float64).reshape(1, 1, -1, 2)
        ref = torch.nn.functional.grid_sample(ft, gt, mode="bilinear", padding_mode="zeros",
                                              align_corners=False)[0, :, 0].T.numpy()
        assert np.abs(got - ref).max() < 1e-5


def test_tsubcf_equals_conv_transpose_then_blur():
    """the fast graph's composed sub-pixel up-conv kernel (motion_dec.cpp
    :144-191) equals torch conv_transpose2d(stride 2) followed by the blur"""
    rng = np.random.default_rng(1)
    IC, OC, H = 8, 4, 5
    Wt = rng.standard_normal((OC, IC, 3, 3)).astype(np.float32)
    K = synth.blur_kernel4()
    x = torch.tensor(rng.standard_normal((1, IC, H, H)))
    y = torch.nn.functional.conv_transpose2d(x, torch.tensor(Wt, dtype=torch.float64).transpose(0, 1),
                                             stride=2)
    kb = torch.tensor(K, dtype=torch.float64)[None, None].repeat(OC, 1, 1, 1)
    ref = torch.nn.functional.conv2d(torch.nn.functional.pad(y, (1, 1, 1, 1)), kb, groups=OC)[0].numpy()
    T = O.tsubcf(Wt, K, IC, OC)
    w4 = torch.tensor(T.reshape(4 * OC, 3, 3, IC).transpose(0, 3, 1, 2), dtype=torch.float64)
    y4 = torch.nn.functional.conv2d(x, w4, padding=1)[0].numpy()
    out = np.zeros_like(ref)
    for k in range(4):
        out[:, k >> 1::2, k & 1::2] = y4[k * OC:(k + 1) * OC]
    assert np.abs(out - ref).max() < 1e-5


def test_saug():
    rng = np.random.default_rng(2)
    Wt = rng.standard_normal((6, 5, 3, 3)).astype(np.float32)
    s = O.saug(Wt, 5, 6)
    ref = 0.5 * (Wt.astype(np.float64) ** 2).sum((2, 3))
    np.testing.assert_allclose(s[:, :5], ref, rtol=1e-6)
    assert np.all(s[:, 5] == np.float32(0.5e-8))


def test_scale_for_table():
    """motion_ae_scale (src/motion_enc.cpp:14-45) on the decoder's names"""
    r2 = np.sqrt(2.0)
    assert O.scale_for("dec.convs.0.conv.weight", (3, 3, 512, 512)) == pytest.approx(1 / np.sqrt(9 * 512))
    assert O.scale_for("dec.convs.3.conv.modulation.weight", (512, 512)) == pytest.approx(1 / np.sqrt(512))
    assert O.scale_for("dec.convs.3.activate.bias", (512,)) == pytest.approx(r2)
    assert O.scale_for("dec.to_rgbs.2.conv.1.bias", (1, 1, 3, 1)) == pytest.approx(r2)
    assert O.scale_for("dec.to_rgbs.2.conv.0.weight", (1, 1, 512, 3)) == pytest.approx(r2 / np.sqrt(512))
    assert O.scale_for("dec.to_flows.6.conv.weight", (1, 1, 32, 3)) == pytest.approx(1 / np.sqrt(32))
    assert O.scale_for("dec.to_flows.6.bias", (1, 1, 3, 1)) == 1.0
    assert O.scale_for("dec.convs.0.conv.blur.kernel", (4, 4)) == 1.0
    assert O.scale_for("dec.direction.Q", (20, 512)) == 1.0


def test_decoder_modes_agree(model, oracle_dec, oracle_frames):
    """exact graph (zero-stuff up-conv) vs sub-pixel graph: the identity the
    reference's fast graph relies on, end to end"""
    sub = oracle_dec.decode(model["styles"][0], mode=1)
    assert cosine(sub, oracle_frames[0]) >= 0.9999, max_abs(sub, oracle_frames[0])


def test_decoder_vs_independent_torch(model, oracle_frames):
    """oracle (folded, S_aug, f32) vs an unfolded float64 torch formulation"""
    from torch_lia import TorchLIA
    ref = TorchLIA(model["raw"], model["feats"]).decode(model["styles"][0])
    c = cosine(oracle_frames[0], ref)
    print(f"oracle vs torch fp64: cos {c:.8f} max-abs {max_abs(oracle_frames[0], ref):.3e}")
    assert c >= 0.9999


def test_decoder_taps_shapes(model, oracle_dec):
    oracle_dec.decode(model["styles"][1], mode=0, keep_taps=True)
    assert oracle_dec.tap("conv1_4").size == 512 * 16
    for j in range(7):
        r, oc = 8 << j, O.ST_OC[j]
        assert oracle_dec.tap(f"r{r}.conv1").size == oc * r * r
        assert oracle_dec.tap(f"r{r}.grid").size == 2 * r * r
        assert oracle_dec.tap(f"r{r}.rgb").size == 3 * r * r
    with pytest.raises(KeyError):
        oracle_dec.tap("nope")


def test_decoder_rejects_bad_tensors(model):
    w = dict(model["w"])
    w["dec.convs.0.conv.weight"] = w["dec.convs.0.conv.weight"][:10]
    with pytest.raises(ValueError):
        O.Decoder(w, model["feats"])
    w = dict(model["w"])
    del w["dec.to_rgbs.3.bias"]
    with pytest.raises(ValueError):
        O.Decoder(w, model["feats"])


def test_reference_f16_arithmetic_meets_gate(model, oracle_dec, oracle_frames):
    """the reference's f16 mode (its f16 fast graph, emulated and pinned in
    test_refgraph.py) meets SSIM >= 0.99 against fp32 on the parity
    configuration, so the gate is one the reference itself passes"""
    from metrics import ssim
    f16 = oracle_dec.decode(model["styles"][0], mode=1 | O.REF_F16_GRAPH)
    s = ssim(f16, oracle_frames[0])
    print(f"reference-f16 emulation: ssim {s:.5f} cos {cosine(f16, oracle_frames[0]):.6f}")
    assert s >= 0.99
