"""Seeded synthetic inputs shared by the golden-vector generator and the tests.

Every generator uses ``numpy.random.default_rng(seed)`` so the same arrays are
rebuilt bit-for-bit on any machine; fixtures therefore store only outputs plus
a checksum of the inputs they were made from.

The distributions follow the benchmark configurations: N(0, 0.02^2) weights
with a few x20 outlier input columns (config 1), Student-t heavy tails on 1%
of entries (config 2), Hessians H = X^T X / n with X rows N(0, diag(s^2)) and
per-channel s ~ LogNormal(0, 1) (config 3).
"""

from __future__ import annotations

import hashlib

import numpy as np

f32 = np.float32


def checksum(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:16]


def weight_outlier_cols(seed: int, M: int, N: int, frac: float = 0.001, mult: float = 20.0,
                        std: float = 0.02) -> np.ndarray:
    """fp32 weights N(0, std^2) (fp16-representable); max(1, frac*N) columns scaled by ``mult``."""
    rng = np.random.default_rng(seed)
    W = rng.standard_normal((M, N), dtype=np.float64) * std
    k = max(1, int(round(frac * N)))
    cols = rng.choice(N, size=k, replace=False)
    W[:, cols] *= mult
    return W.astype(np.float16).astype(f32)


def weight_heavy_tail(seed: int, M: int, N: int, frac: float = 0.01, std: float = 0.02) -> np.ndarray:
    rng = np.random.default_rng(seed)
    W = rng.standard_normal((M, N), dtype=np.float64) * std
    mask = rng.random((M, N)) < frac
    W[mask] += std * rng.standard_t(3, size=int(mask.sum()))
    return W.astype(np.float16).astype(f32)


def hessian_lognormal(seed: int, N: int, n_samples: int) -> np.ndarray:
    """H = X^T X / n, X [n, N] rows N(0, diag(s^2)), s_c ~ LogNormal(0, 1)."""
    rng = np.random.default_rng(seed)
    s = rng.lognormal(0.0, 1.0, size=N)
    X = rng.standard_normal((n_samples, N)) * s[None, :]
    H = X.T @ X / n_samples
    H = 0.5 * (H + H.T)
    return H.astype(f32)


def codes(seed: int, M: int, K: int, lo: int = -8, hi: int = 7) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=(M, K)).astype(np.int8)
