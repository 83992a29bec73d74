"""PiSO data-aware per-row scale search on the GPU (mirrors converter/piso.py).

The candidate factor tables come from ``torch.linspace`` exactly as the
reference builds them (piso.py:62-63, 135-136); the search runs in
``piso_kernel`` (libintcrush_b200).  Semantics follow the reference's
PyTorch implementation (coarse range [0.5, 2.0] for INT4 asymmetric).
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as nat
from ._dev import back, device_of, f32


def _table(lo, hi, n):
    v = torch.linspace(lo, hi, n, dtype=torch.float32).tolist()
    return (ctypes.c_float * n)(*v)


def _run(W, hessian_diag, num_coarse, num_fine, qmin, qmax, divisor, asym, lo, hi):
    if W.dim() != 2:
        raise ValueError(f"Expected 2D tensor, got {W.dim()}D")
    dev = device_of(W)
    Wd = f32(W, dev)
    M, N = Wd.shape
    h = f32(hessian_diag.reshape(-1)[:N], dev)
    if h.shape[0] != N:
        raise ValueError(f"hessian_diag length {h.shape[0]} != in_features {N}")
    scales = torch.empty(M, 1, dtype=torch.float32, device=dev)
    zp = torch.empty(M, 1, dtype=torch.int8, device=dev) if asym else None
    if M:
        nat.check(nat.load().ic_piso(Wd.data_ptr(), M, N, N, h.data_ptr(), int(asym), qmin, qmax, float(divisor),
                                     _table(lo, hi, num_coarse), num_coarse, _table(0.95, 1.05, num_fine), num_fine,
                                     scales.data_ptr(), nat.ptr(zp), nat.stream_ptr(dev)), "piso")
    if asym:
        return back(scales, W), back(zp, W)
    return back(scales, W)


def compute_piso_scales_int8(W, hessian_diag, num_coarse: int = 128, num_fine: int = 16):
    """Symmetric INT8 (piso.py:190-240)."""
    return _run(W, hessian_diag, num_coarse, num_fine, -128, 127, 127.0, False, 0.5, 2.0)


def compute_piso_scales_int8_asymmetric(W, hessian_diag, num_coarse: int = 128, num_fine: int = 16):
    """Asymmetric INT8, coarse [0.8, 1.2] (piso.py:243-295)."""
    return _run(W, hessian_diag, num_coarse, num_fine, -128, 127, 255.0, True, 0.8, 1.2)


def compute_piso_scales_int4(W, hessian_diag, num_coarse: int = 128, num_fine: int = 16):
    """Symmetric INT4 (piso.py:303-352)."""
    return _run(W, hessian_diag, num_coarse, num_fine, -8, 7, 7.0, False, 0.5, 2.0)


def compute_piso_scales_int4_asymmetric(W, hessian_diag, num_coarse: int = 128, num_fine: int = 16):
    """Asymmetric INT4, coarse [0.5, 2.0] (piso.py:355-408)."""
    return _run(W, hessian_diag, num_coarse, num_fine, -8, 7, 15.0, True, 0.5, 2.0)
