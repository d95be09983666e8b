"""GPU parity of the whole decoder through the C ABI against the fp32
oracle (the reference's exact graph restated).

Gates (from the task's north star): fp32 mode per-frame cosine >= 0.9999
with max-abs reported; f16 mode SSIM >= 0.99 against the fp32 oracle frames.
Inputs: random-init weights, smooth N(0,1) feature fields (see
tpmd.synth.make_feats for why white-noise maps are not a parity input)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import tpmd
from metrics import cosine, max_abs, ssim

pytestmark = pytest.mark.gpu


def make_dec(model, dtype, max_batch=8):
    d = tpmd.MotionDecoder(0, dtype, max_batch)
    d.set_tensors(model["w"])
    d.prepare()
    d.set_feats(model["feats"])
    return d


@pytest.fixture(scope="module")
def dec32(model):
    return make_dec(model, tpmd.DTYPE_F32)


@pytest.fixture(scope="module")
def dec16(model):
    return make_dec(model, tpmd.DTYPE_F16)


def _style_vec(model, base, lat):
    w = model["w"]
    return (w[base + ".modulation.weight"].astype(np.float64) @ lat.astype(np.float64)
            + w[base + ".modulation.bias"])


@pytest.mark.parametrize("level", range(7))
def test_taps_f32(model, dec32, oracle_dec, level):
    lat = model["styles"][0]
    oracle_dec.decode(lat, mode=0, keep_taps=True)
    r = 8 << level
    t = dec32.taps(lat, level)
    s2 = _style_vec(model, f"dec.convs.{2 * level + 1}.conv", lat)[:, None, None]
    pairs = [("conv1", O_tap(oracle_dec, f"r{r}.conv1", t["conv1"].shape) * s2),
             ("conv2", O_tap(oracle_dec, f"r{r}.conv2", t["conv2"].shape)),
             ("rgb", O_tap(oracle_dec, f"r{r}.rgb", t["rgb"].shape))]
    if level < 6:
        s_next = _style_vec(model, f"dec.convs.{2 * level + 2}.conv", lat)[:, None, None]
        pairs += [("flowmap", O_tap(oracle_dec, f"r{r}.flowmap", t["flowmap"].shape)),
                  ("trunk", O_tap(oracle_dec, f"r{r}.out", t["trunk"].shape) * s_next)]
    for name, ref in pairs:
        c = cosine(t[name], ref)
        print(f"level {level} {name}: cos {c:.9f} max-abs {max_abs(t[name], ref):.3e}")
        assert c >= 0.9999, (level, name, c)


def O_tap(d, name, shape):
    return d.tap(name).reshape(shape)


def test_frames_f32(model, dec32, oracle_frames):
    frames = dec32.decode(model["styles"])
    for i in range(len(frames)):
        c = cosine(frames[i], oracle_frames[i])
        print(f"f32 frame {i}: cos {c:.9f} max-abs {max_abs(frames[i], oracle_frames[i]):.3e}")
        assert c >= 0.9999


def test_frames_f16(model, dec16, oracle_frames):
    frames = dec16.decode(model["styles"])
    for i in range(len(frames)):
        c, s = cosine(frames[i], oracle_frames[i]), ssim(frames[i], oracle_frames[i])
        print(f"f16 frame {i}: cos {c:.7f} ssim {s:.5f} max-abs {max_abs(frames[i], oracle_frames[i]):.3e}")
        assert s >= 0.99
        assert c >= 0.999


@pytest.mark.parametrize("which", ["f32", "f16"])
def test_batch_invariance(model, dec32, dec16, which):
    """a frame decodes to the same bits alone or inside a batch"""
    d = dec32 if which == "f32" else dec16
    st = model["styles"]
    together = d.decode(st)
    for i in range(len(st)):
        alone = d.decode(st[i:i + 1])
        assert np.array_equal(alone[0], together[i]), i


def test_more_frames_than_batch(model):
    d = make_dec(model, tpmd.DTYPE_F16, max_batch=2)
    st = np.concatenate([model["styles"], model["styles"][:1]])
    out = d.decode(st)
    ref = make_dec(model, tpmd.DTYPE_F16, max_batch=8).decode(st)
    assert np.array_equal(out, ref)


def test_device_decode_matches_host(model, dec16):
    import torch
    st = model["styles"]
    host = dec16.decode(st)
    s_d = torch.from_numpy(st).cuda()
    f_d = torch.empty((len(st), 3, 512, 512), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    dec16.decode_device(s_d.data_ptr(), len(st), f_d.data_ptr(), stream)
    torch.cuda.synchronize()
    assert np.array_equal(f_d.cpu().numpy(), host)


def test_errors_are_reported(model):
    d = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, 2)
    with pytest.raises(tpmd.TpmdError, match="not prepared"):
        d.decode(model["styles"][:1])
    with pytest.raises(tpmd.TpmdError, match="unknown tensor"):
        d.set_tensors({"dec.nope": np.zeros(3, np.float32)})
    with pytest.raises(tpmd.TpmdError, match="expected"):
        d.set_tensors({"dec.convs.0.activate.bias": np.zeros(3, np.float32)})
    with pytest.raises(tpmd.TpmdError, match="missing"):
        d.prepare()
    d.set_tensors(model["w"])
    d.prepare()
    with pytest.raises(tpmd.TpmdError, match="feats not set"):
        d.decode(model["styles"][:1])


def test_kernel_launch_count(dec16, dec32):
    # style, den, conv1 input, conv1, then per level up-conv, conv2, tail;
    # with tcgen05 the four levels with OC <= 256 fuse conv2 and tail
    assert dec32.kernel_launches(8) == 25
    assert dec16.kernel_launches(8) == 21
    assert dec16.kernel_launches(9) == 42


def test_stress_random_init(stress_model):
    """plain random init (ToFlow gain 1, chaotic): fp32 still meets cosine
    0.9999; f16 must be within 0.01 SSIM of the reference's own f16
    arithmetic (emulated by the oracle), which itself ends near 0.95 here"""
    import oracle as O
    m = stress_model
    od = O.Decoder(m["w"], m["feats"])
    st = m["styles"][:2]
    d32, d16 = make_dec(m, tpmd.DTYPE_F32), make_dec(m, tpmd.DTYPE_F16)
    g32, g16 = d32.decode(st), d16.decode(st)
    for i in range(len(st)):
        ref = od.decode(st[i], mode=0)
        ref16 = od.decode(st[i], mode=1 | O.REF_F16_GRAPH)
        c32 = cosine(g32[i], ref)
        s16, sref = ssim(g16[i], ref), ssim(ref16, ref)
        print(f"stress frame {i}: f32 cos {c32:.7f}; f16 ssim {s16:.4f} vs reference-f16 {sref:.4f}")
        assert c32 >= 0.9999
        assert s16 >= sref - 0.01


def _dec_with_conv(model, kind):
    import os
    old = os.environ.get("TPMD_CONV")
    os.environ["TPMD_CONV"] = kind
    try:
        return make_dec(model, tpmd.DTYPE_F16)
    finally:
        if old is None:
            del os.environ["TPMD_CONV"]
        else:
            os.environ["TPMD_CONV"] = old


@pytest.mark.parametrize("level", range(7))
def test_tcgen05_matches_simt_f16(model, level):
    """the tcgen05 convs against the FFMA convs on identical f16 storage:
    only the accumulation order differs"""
    tc, simt = _dec_with_conv(model, "tc"), _dec_with_conv(model, "simt")
    lat = model["styles"][0]
    a, b = tc.taps(lat, level), simt.taps(lat, level)
    for k in a:
        c = cosine(a[k], b[k])
        print(f"level {level} {k}: tc vs simt cos {c:.9f} max-abs {max_abs(a[k], b[k]):.3e}")
        assert c >= 0.9999, (level, k, c)


def test_strip_heights_agree(model):
    """the r512 conv2 work units are strips of 8, 16 or 32 output rows,
    chosen from the batch size; every output row sums the same kernel rows in
    the same order, so the frames are bit-identical"""
    st = np.concatenate([model["styles"]] * 24)[:24]
    st = st + 0.01 * np.arange(24, dtype=np.float32)[:, None]  # 24 distinct frames
    outs = [make_dec(model, tpmd.DTYPE_F16, max_batch=mb).decode(st) for mb in (24, 12, 8)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
