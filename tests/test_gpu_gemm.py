"""The library's tcgen05 GEMM (tpk_gemm; the sampler's and the audio
encoder's contractions) against float64 numpy on the same inputs.

Bounds, per output element, relative to S = sum_k |x_k w_k|:
* f32 operands (three-pass TF32 split): |err| <= 2e-6 S (about 2^-20 per
  product plus f32 accumulation);
* f16 operands, f32 accumulation: |err| <= 2e-6 S against the product of
  the f16-rounded operands.
Shapes cover split-K over a thread-block cluster (few tiles, long K),
ragged M/N/K, the sampler's M = 180 and 60 row counts, the audio encoder's
750-frame rows, heads as column blocks and groups as row blocks, the fused
epilogue (bias, scale, GELU) and repeat determinism."""
from __future__ import annotations

import numpy as np
import pytest

import tpmd

pytestmark = pytest.mark.gpu


def _t(a, dt=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dt is None else t.to(dt)


def _check(y, ref, bound, tol=2e-6):
    err = np.abs(y.astype(np.float64) - ref)
    worst = float(np.max(err / (bound + 1e-30)))
    assert worst <= tol, worst
    return worst


def _gelu_erf(v):
    from scipy.special import erf
    return 0.5 * v * (1.0 + erf(v / np.sqrt(2.0)))


def _gelu_tanh(v):
    return 0.5 * v * (1.0 + np.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3)))


SHAPES = [(180, 1024, 1024), (180, 3072, 1024), (60, 1024, 512), (180, 512, 4096), (750, 768, 768),
          (750, 3072, 768), (37, 77, 40), (1, 128, 64), (300, 130, 1536), (257, 64, 8)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_f32(M, N, K):
    import torch
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    X = rng.standard_normal((M, K)).astype(np.float32)
    W = rng.standard_normal((N, K)).astype(np.float32)
    Y = torch.empty((M, N), device="cuda")
    tpmd.gemm(_t(X), _t(W), Y, M, N, K)
    ref = X.astype(np.float64) @ W.astype(np.float64).T
    w = _check(Y.cpu().numpy(), ref, np.abs(X).astype(np.float64) @ np.abs(W).astype(np.float64).T)
    print(f"f32 {M}x{N}x{K}: worst |err| / sum|xw| = {w:.2e}")


@pytest.mark.parametrize("M,N,K", SHAPES[:6])
def test_gemm_f16(M, N, K):
    import torch
    rng = np.random.default_rng(M + N + K)
    X = rng.standard_normal((M, K)).astype(np.float16)
    W = rng.standard_normal((N, K)).astype(np.float16)
    Y = torch.empty((M, N), device="cuda")
    tpmd.gemm(_t(X), _t(W), Y, M, N, K)
    x, wt = X.astype(np.float64), W.astype(np.float64)
    w = _check(Y.cpu().numpy(), x @ wt.T, np.abs(x) @ np.abs(wt).T)
    print(f"f16 {M}x{N}x{K}: worst |err| / sum|xw| = {w:.2e}")


@pytest.mark.parametrize("act", [0, 1, 2])
def test_epilogue(act):
    import torch
    rng = np.random.default_rng(act)
    M, N, K = 180, 4096, 1024
    X = rng.standard_normal((M, K)).astype(np.float32) * 0.05
    W = rng.standard_normal((N, K)).astype(np.float32) * 0.05
    b = rng.standard_normal(N).astype(np.float32)
    Y = torch.empty((M, N), device="cuda")
    tpmd.gemm(_t(X), _t(W), Y, M, N, K, bias=_t(b), scale=0.125, act=act)
    v = (X.astype(np.float64) @ W.astype(np.float64).T + b) * 0.125
    ref = v if act == 0 else _gelu_erf(v) if act == 1 else _gelu_tanh(v)
    bound = (np.abs(X).astype(np.float64) @ np.abs(W).astype(np.float64).T + np.abs(b)) * 0.125 + 1e-3
    _check(Y.cpu().numpy(), ref, bound, tol=4e-6)


def test_heads_as_column_blocks():
    """attention scores: q [S][H] and k [S][H], head h = columns h*hd..;
    y[h][i][j] = q_i . k_j over the head's columns, rows padded to ld"""
    import torch
    rng = np.random.default_rng(5)
    S, nh, hd = 750, 12, 64
    H, ld = nh * hd, 752
    q = rng.standard_normal((S, H)).astype(np.float32)
    k = rng.standard_normal((S, H)).astype(np.float32)
    Y = torch.zeros((nh, S, ld), device="cuda")
    tpmd.gemm(_t(q), _t(k), Y, S, S, hd, ldx=H, ldw=H, ldy=ld, batch=nh, x_col_b=hd, w_col_b=hd, y_batch=S * ld)
    y = Y.cpu().numpy()
    for h in (0, 5, 11):
        qs = q[:, h * hd:(h + 1) * hd].astype(np.float64)
        ks = k[:, h * hd:(h + 1) * hd].astype(np.float64)
        _check(y[h, :, :S], qs @ ks.T, np.abs(qs) @ np.abs(ks).T)
    assert not y[:, :, S:].any()  # the padding columns are not written


def test_groups_as_row_blocks_and_padded_k():
    """grouped conv / attention-times-values form: X rows of group g start at
    g*M, W rows at g*N, K = 750 columns of 752-float rows (the last k-block
    reads past K: zero fill)"""
    import torch
    rng = np.random.default_rng(6)
    G, M, N, K, ld = 12, 750, 64, 750, 752
    X = np.zeros((G * M, ld), np.float32)
    X[:, :K] = rng.random((G * M, K), dtype=np.float32)
    X[:, K:] = np.nan  # never read
    W = np.zeros((G * N, ld), np.float32)
    W[:, :K] = rng.standard_normal((G * N, K)).astype(np.float32)
    W[:, K:] = np.nan
    Y = torch.zeros((M, G * N), device="cuda")
    tpmd.gemm(_t(X), _t(W), Y, M, N, K, ldx=ld, ldw=ld, ldy=G * N, batch=G, x_row_b=M, w_row_b=N, y_batch=N)
    y = Y.cpu().numpy()
    for g in (0, 7, 11):
        x = X[g * M:(g + 1) * M, :K].astype(np.float64)
        w = W[g * N:(g + 1) * N, :K].astype(np.float64)
        _check(y[:, g * N:(g + 1) * N], x @ w.T, np.abs(x) @ np.abs(w).T)


def test_split_k_deterministic():
    import torch
    rng = np.random.default_rng(9)
    M, N, K = 180, 1024, 4096
    X, W = _t(rng.standard_normal((M, K)).astype(np.float32)), _t(rng.standard_normal((N, K)).astype(np.float32))
    a, b = torch.empty((M, N), device="cuda"), torch.empty((M, N), device="cuda")
    tpmd.gemm(X, W, a, M, N, K)
    for _ in range(3):
        tpmd.gemm(X, W, b, M, N, K)
        assert torch.equal(a, b)


def test_bad_arguments():
    import torch
    X = torch.zeros((8, 10), device="cuda")
    Y = torch.zeros((8, 8), device="cuda")
    with pytest.raises(tpmd.TpmdError, match="stride"):
        tpmd.gemm(X, X, Y, 8, 8, 10)  # 40-byte rows: not a 16-byte multiple
    with pytest.raises(tpmd.TpmdError, match="act"):
        tpmd.gemm(Y, Y, Y, 8, 8, 8, act=7)
