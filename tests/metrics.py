"""Frame comparison metrics used by the parity gates (test helpers)."""
from __future__ import annotations

import numpy as np
from scipy.ndimage import gaussian_filter


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def ssim(x: np.ndarray, y: np.ndarray) -> float:
    """Mean SSIM over channels of CHW frames (Wang et al. 2004: Gaussian
    window sigma 1.5, K1 0.01, K2 0.03), data range taken from the reference
    frame y."""
    x = np.asarray(x, np.float64)
    y = np.asarray(y, np.float64)
    L = float(y.max() - y.min())
    c1, c2 = (0.01 * L) ** 2, (0.03 * L) ** 2
    vals = []
    for ch in range(x.shape[0]):
        a, b = x[ch], y[ch]
        f = lambda z: gaussian_filter(z, 1.5, truncate=3.5)  # noqa: E731
        mu_a, mu_b = f(a), f(b)
        saa = f(a * a) - mu_a ** 2
        sbb = f(b * b) - mu_b ** 2
        sab = f(a * b) - mu_a * mu_b
        m = ((2 * mu_a * mu_b + c1) * (2 * sab + c2)) / ((mu_a ** 2 + mu_b ** 2 + c1) * (saa + sbb + c2))
        vals.append(m.mean())
    return float(np.mean(vals))
