"""GPU parity of the op-level kernels (tpk_bilinear_gather, tpk_im2col_cf)
through the C ABI: against the golden vectors produced by the reference's own
op code and against the oracle at the config-1 sweep shapes."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import tpmd

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_gather(feat, W, H, grid, planar, sp):
    C = feat.shape[-1]
    N = grid.size // 2
    out = torch.empty((C, N) if sp else (N, C), dtype=torch.float32, device="cuda")
    tpmd.bilinear_gather(dev(feat), W, H, dev(grid), out, planar=planar, out_sp=sp)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_gather_golden(golden):
    d, meta = golden
    for n, m in meta.items():
        if m["op"] != "gather":
            continue
        got = run_gather(d[n + ".feat"], m["W"], m["H"], d[n + ".grid"], m["planar"], m["sp"])
        np.testing.assert_allclose(got, d[n + ".out"], rtol=1e-6, atol=1e-7, err_msg=n)


def test_im2col_golden_bit_exact(golden):
    d, meta = golden
    for n, m in meta.items():
        if m["op"] != "im2col_cf":
            continue
        ref = d[n + ".out"]
        out = torch.empty(ref.shape, dtype=torch.float16 if m["f16"] else torch.float32, device="cuda")
        tpmd.im2col_cf(dev(d[n + ".src"]), m["IC"], m["IW"], m["IH"], m["N"], out, m["KW"], m["KH"],
                       m["s0"], m["s1"], m["p0"], m["p1"], m["d0"], m["d1"])
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint8), ref.view(np.uint8)), n


@pytest.mark.parametrize("C,R", [(32, 512), (64, 256), (128, 128), (256, 64), (512, 32), (512, 8)])
@pytest.mark.parametrize("f16", [False, True])
def test_gather_sweep_vs_oracle(C, R, f16):
    """config 1(b): grid uniform in [-1.1, 1.1] (zero padding exercised)"""
    rng = np.random.default_rng(C * 1000 + R)
    feat = rng.standard_normal((R * R, C)).astype(np.float16 if f16 else np.float32)
    grid = rng.uniform(-1.1, 1.1, (R * R, 2)).astype(np.float32)
    got = run_gather(feat, R, R, grid, False, False)
    ref = O.bilinear_gather(feat, R, R, grid)
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)


def test_gather_max_size_checksum():
    """C = 512 at 512 x 512, f16: full-size run checked on a strided sample
    of points against the oracle"""
    R, C = 512, 512
    rng = np.random.default_rng(5)
    feat = rng.standard_normal((R * R, C)).astype(np.float16)
    grid = rng.uniform(-1.1, 1.1, (R * R, 2)).astype(np.float32)
    got = run_gather(feat, R, R, grid, False, False)
    idx = np.arange(0, R * R, 97)
    ref = O.bilinear_gather(feat, R, R, grid[idx])
    np.testing.assert_allclose(got[idx], ref, rtol=1e-6, atol=1e-6)


def test_gather_layouts_agree():
    rng = np.random.default_rng(9)
    C, R = 64, 32
    feat = rng.standard_normal((R * R, C)).astype(np.float32)
    grid = rng.uniform(-1.1, 1.1, (R * R, 2)).astype(np.float32)
    a = run_gather(feat, R, R, grid, False, False)
    b = run_gather(feat, R, R, np.ascontiguousarray(grid.T), True, False)
    c = run_gather(feat, R, R, grid, False, True)
    assert np.array_equal(a, b)
    assert np.array_equal(a, c.T)


def test_gather_empty_and_ragged():
    import ctypes as C
    feat = dev(np.ones((4, 3), np.float32))
    # N = 0: succeeds without touching dst (which may be NULL)
    assert tpmd.load_library().tpk_bilinear_gather(C.c_void_p(feat.data_ptr()), 0, 3, 2, 2, None, 0,
                                                   0, 0, None, None) == 0
    rng = np.random.default_rng(11)
    for C in (1, 3, 7, 13):
        feat = rng.standard_normal((25, C)).astype(np.float16)
        g = rng.uniform(-1.2, 1.2, (40, 2)).astype(np.float32)
        np.testing.assert_allclose(run_gather(feat, 5, 5, g, False, False),
                                   O.bilinear_gather(feat, 5, 5, g), rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("IC,R,N", [(32, 64, 2), (64, 128, 1), (512, 16, 3), (24, 20, 2), (3, 9, 1)])
@pytest.mark.parametrize("f16", [False, True])
def test_im2col_sweep_bit_exact(IC, R, N, f16):
    """config 1(c): 3x3 pad 1 stride 1, bit-exact against the oracle"""
    rng = np.random.default_rng(IC + R)
    src = rng.standard_normal((N, R, R, IC)).astype(np.float32)
    ref = O.im2col_cf(src, IC, R, R, N, dst_f16=f16)
    out = torch.empty(ref.shape, dtype=torch.float16 if f16 else torch.float32, device="cuda")
    tpmd.im2col_cf(dev(src), IC, R, R, N, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint8), ref.view(np.uint8))
