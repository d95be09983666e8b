"""The output conversion CHW f32 -> RGB24 (tools/tp-cli.cpp:43-53: clamp to
[-1, 1], then (unsigned char) ((v + 1) / 2 * 255) in f32) in the oracle,
against the same formula in numpy float32 on the edge values: +-1, values
one ulp inside and outside the clamp, values one ulp either side of every
byte boundary, infinities, and random values; byte work, so bit-exact."""
from __future__ import annotations

import numpy as np

import oracle as O


def formula(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, np.float32)
    v = np.where(v < np.float32(-1), np.float32(-1), np.where(v > np.float32(1), np.float32(1), v))
    s = (v + np.float32(1)) / np.float32(2) * np.float32(255)
    return np.trunc(s.astype(np.float32)).astype(np.uint8)


def edge_values() -> np.ndarray:
    one = np.float32(1)
    vals = [-np.inf, -2.0, np.nextafter(-one, -2 * one), -1.0, np.nextafter(-one, 0 * one), -0.5, 0.0,
            1e-30, np.nextafter(one, 0 * one), 1.0, np.nextafter(one, 2 * one), 2.0, np.inf]
    for k in range(256):  # either side of each byte boundary
        b = np.float32(2.0 * k / 255.0 - 1.0)
        vals += [np.nextafter(b, -2 * one), b, np.nextafter(b, 2 * one)]
    return np.asarray(vals, np.float32)


def test_oracle_matches_formula():
    ev = edge_values()
    rng = np.random.default_rng(0)
    v = np.concatenate([ev, rng.standard_normal(3 * 4096 - ev.size).astype(np.float32) * 1.5])
    frames = v[: 3 * 4096].reshape(1, 3, 64, 64)
    got = O.chw_to_rgb24(frames)
    want = formula(frames).transpose(0, 2, 3, 1)
    assert np.array_equal(got, want)
    assert got.dtype == np.uint8 and got.shape == (1, 64, 64, 3)


def test_clamp_endpoints():
    f = np.array([-5.0, -1.0, 1.0, 5.0], np.float32).reshape(1, 1, 1, 4).repeat(3, 1)
    assert O.chw_to_rgb24(f)[0, 0, :, 0].tolist() == [0, 0, 255, 255]
