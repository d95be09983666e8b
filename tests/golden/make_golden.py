"""Generate tests/golden/ops_golden.npz from the reference's own op code.

Runs only where the reference tree is present (it builds oracle/_ref/ via
oracle/ref_build.py, which compiles the patched ggml CPU ops and CUDA kernels
of patches/ggml-tp-ops.patch as host code). Each case stores its seeded
inputs, its parameters and the reference outputs; tests compare the oracle
(CPU) and the CUDA kernels (GPU) against them. Cases cover the shapes the
decoder uses, ragged channel counts, non-square maps, both grid layouts,
both output layouts, f32/f16 features, grid points on and beyond the border
(zero padding), and strided / dilated / asymmetric-padding im2col.

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "ops_golden.npz")

GATHER_CASES = [
    # name, C, W, H, f16, planar, sp, npts
    ("g_c32_w16_f32", 32, 16, 16, False, False, False, 512),
    ("g_c64_w8_f16_planar", 64, 8, 8, True, True, False, 192),
    ("g_c48_w12x10_f32_sp", 48, 12, 10, False, False, True, 300),
    ("g_c21_w7x9_f16_ragged", 21, 7, 9, True, False, False, 150),
    ("g_c512_w8_f16", 512, 8, 8, True, False, False, 100),
    ("g_c3_w5_f32_planar_sp", 3, 5, 5, False, True, True, 77),
    ("g_c256_w16_f32", 256, 16, 16, False, False, False, 200),
]
IM2COL_CASES = [
    # name, IC, IW, IH, N, KW, KH, s0, s1, p0, p1, d0, d1, f16
    ("i_ic32_8x8_n2_f32", 32, 8, 8, 2, 3, 3, 1, 1, 1, 1, 1, 1, False),
    ("i_ic32_8x8_n2_f16", 32, 8, 8, 2, 3, 3, 1, 1, 1, 1, 1, 1, True),
    ("i_ic24_7x5_s2_f16", 24, 7, 5, 1, 3, 3, 2, 2, 1, 1, 1, 1, True),
    ("i_ic5_6x6_mixed_f32", 5, 6, 6, 2, 3, 2, 1, 2, 2, 0, 2, 1, False),
    ("i_ic64_4x4_n3_f16", 64, 4, 4, 3, 3, 3, 1, 1, 1, 1, 1, 1, True),
    ("i_ic512_4x4_n1_f16", 512, 4, 4, 1, 3, 3, 1, 1, 1, 1, 1, 1, True),
]


def special_grid(rng, n):
    """uniform [-1.1, 1.1] plus border / exact-pixel / far-away points"""
    g = rng.uniform(-1.1, 1.1, (n, 2)).astype(np.float32)
    specials = np.array([[-1, -1], [1, 1], [-1, 1], [0, 0], [1.0001, 0], [-1.0001, 0.5],
                         [5, 5], [-7, 0.1], [0.999, -0.999]], np.float32)
    k = min(len(specials), n)
    g[:k] = specials[:k]
    return g


def main() -> int:
    subprocess.run([sys.executable, os.path.join(ROOT, "oracle", "ref_build.py")], check=True)
    if O.ref_lib() is None:
        print("make_golden: reference op code unavailable (reference tree absent)")
        return 1
    rng = np.random.default_rng(20261201)
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}
    for name, c, w, h, f16, planar, sp, n in GATHER_CASES:
        feat = rng.standard_normal((w * h, c)).astype(np.float16 if f16 else np.float32)
        g = special_grid(rng, n)
        grid = np.ascontiguousarray(g.T) if planar else g
        out = O.bilinear_gather(feat, w, h, grid, planar, sp, impl="ref_cpu")
        out_cu = O.bilinear_gather(feat, w, h, grid, planar, sp, impl="ref_cu")
        assert np.array_equal(out, out_cu), name
        arrays[name + ".feat"] = feat
        arrays[name + ".grid"] = grid
        arrays[name + ".out"] = out
        meta[name] = dict(op="gather", C=c, W=w, H=h, f16=f16, planar=planar, sp=sp, N=n)
    for name, ic, iw, ih, n, kw, kh, s0, s1, p0, p1, d0, d1, f16 in IM2COL_CASES:
        src = rng.standard_normal((n, ih, iw, ic)).astype(np.float32)
        out = O.im2col_cf(src, ic, iw, ih, n, kw, kh, s0, s1, p0, p1, d0, d1, f16, impl="ref_cu")
        arrays[name + ".src"] = src
        arrays[name + ".out"] = out
        meta[name] = dict(op="im2col_cf", IC=ic, IW=iw, IH=ih, N=n, KW=kw, KH=kh, s0=s0, s1=s1,
                          p0=p0, p1=p1, d0=d0, d1=d1, f16=f16)
    # fused pointwise ops (reference CPU forward functions)
    ne = (6, 5, 4, 2)
    x = rng.standard_normal(int(np.prod(ne))).astype(np.float32)
    for axis in (0, 2):
        b = rng.standard_normal(ne[axis]).astype(np.float32)
        nm = f"bias_lrelu_axis{axis}"
        arrays[nm + ".x"], arrays[nm + ".b"] = x, b
        arrays[nm + ".out"] = O.bias_lrelu((x, ne), b, axis, impl="ref_cpu")
        meta[nm] = dict(op="bias_lrelu", ne=list(ne), axis=axis)
    W, H, OC = 5, 4, 3
    g0 = rng.standard_normal(W * H * 2 * OC).astype(np.float32)
    g1 = rng.standard_normal(W * H * 2 * OC).astype(np.float32)
    bb = rng.standard_normal(OC).astype(np.float32)
    arrays["subpix.g0"], arrays["subpix.g1"], arrays["subpix.b"] = g0, g1, bb
    arrays["subpix.out"] = O.subpix_lrelu(g0, g1, bb, W, H, OC, impl="ref_cpu")
    meta["subpix"] = dict(op="subpix_lrelu", W=W, H=H, OC=OC)
    y4 = rng.standard_normal(4 * OC * W * H * 2).astype(np.float32)
    arrays["subpix_cl.y4"], arrays["subpix_cl.b"] = y4, bb
    arrays["subpix_cl.out"] = O.subpix_lrelu_cl(y4, bb, OC, W * H, 2, W, impl="ref_cpu")
    meta["subpix_cl"] = dict(op="subpix_lrelu_cl", W=W, H=H, OC=OC, B=2)
    k4 = (np.outer([1, 3, 3, 1], [1, 3, 3, 1]) / 16.0).astype(np.float32).ravel()
    xu = rng.standard_normal(W * H * 6).astype(np.float32)
    arrays["upfirdn.x"], arrays["upfirdn.k"] = xu, k4
    arrays["upfirdn.out"] = O.upfirdn2x(xu, k4, W, H, 6, impl="ref_cpu")
    meta["upfirdn"] = dict(op="upfirdn2x", W=W, H=H, CB=6)
    cl = rng.standard_normal(7 * 30).astype(np.float32)
    m = rng.uniform(0, 1, 30).astype(np.float32)
    o = rng.standard_normal(7 * 30).astype(np.float32)
    arrays["clsp.cl"], arrays["clsp.m"], arrays["clsp.o"] = cl, m, o
    arrays["clsp.mul"] = O.clsp(cl, m, 7, 30, impl="ref_cpu")
    arrays["clsp.lerp"] = O.clsp(cl, m, 7, 30, o, impl="ref_cpu")
    meta["clsp"] = dict(op="clsp", C=7, N=30)
    fl = rng.standard_normal(3 * 30).astype(np.float32) * np.float32(3)
    xs = rng.standard_normal(2 * 30).astype(np.float32)
    arrays["flow_grid.fl"], arrays["flow_grid.xs"] = fl, xs
    arrays["flow_grid.out"] = O.flow_grid(fl, xs, 30, impl="ref_cpu")
    meta["flow_grid"] = dict(op="flow_grid", N=30)

    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(meta)} cases)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
