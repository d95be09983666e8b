"""bench.py's algorithmic counts, which set roofline.achieved: the conv GEMM
flops of one frame in the executed sub-pixel form, per stage (up-conv 0.302,
1.208, 4.832, then 9.664 four times; conv2 0.302, 1.208, then 4.832 five
times; conv1 0.0755 GFLOP), 70.74 GFLOP in all, which with the 1x1 ToFlow /
ToRGB convs (0.197) and the modulation GEMVs (0.007) is the decoder's 70.95;
and the fused conv2+tail's bytes, which drop the conv2 output's HBM round
trip."""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402

UP = (0.302, 1.208, 4.832, 9.664, 9.664, 9.664, 9.664)
C2 = (0.302, 1.208, 4.832, 4.832, 4.832, 4.832, 4.832)


@pytest.mark.parametrize("j", range(7))
def test_gemm_flops_per_stage(j):
    r = 8 << j
    up, _ = bench.kernel_work(f"upconv_r{r}", 1, 2)
    c2, _ = bench.kernel_work(f"conv2_r{r}", 1, 2)
    assert up / 1e9 == pytest.approx(UP[j], abs=5e-4)
    assert c2 / 1e9 == pytest.approx(C2[j], abs=5e-4)
    # a launch of nb frames is nb times one frame's work
    assert bench.kernel_work(f"upconv_r{r}", 50, 2)[0] == pytest.approx(50 * up)


def test_whole_decoder_flops():
    names = ["conv1"] + [f"{k}_r{8 << j}" for j in range(7) for k in ("upconv", "conv2")]
    total = sum(bench.kernel_work(n, 1, 2)[0] for n in names)
    assert bench.kernel_work("conv1", 1, 2)[0] / 1e9 == pytest.approx(0.0755, abs=1e-4)
    assert (total + 0.197e9 + 0.007e9) / 1e9 == pytest.approx(70.95, abs=0.01)


def test_fused_tail_bytes():
    """conv2+tail at r512: the conv input (64 B a pixel, f16), the frame
    (12 B a pixel, f32), the r256 skip planes and the weights; no conv2
    output write and read"""
    f, b = bench.kernel_work("conv2tail_r512", 50, 2)
    f2, b2 = bench.kernel_work("conv2_r512", 50, 2)
    _, bt = bench.kernel_work("tail_r512", 50, 2)
    assert f == f2
    assert b == b2 + bt - 2 * 50 * 512 * 512 * 32 * 2
    assert b / 50 == pytest.approx(21.8e6, rel=0.01)
