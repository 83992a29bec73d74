"""Per-row / per-group scales and RTN codes on the GPU (mirrors converter/scales.py).

Every public function keeps the reference's signature, padding rules and
return dtypes/shapes; the arithmetic runs in ``rtn_row_kernel``
(libintcrush_b200) with the reference's fp32 operation order.
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _native as nat
from ._dev import back, device_of, f32
from .config import SCALE_MAX, SCALE_MIN
from .rounding import _round_half_away_from_zero


def _pad_to_group_size(W: torch.Tensor, group_size: int) -> torch.Tensor:  # scales.py:16-22
    n = W.shape[1]
    if n % group_size != 0:
        W = F.pad(W, (0, group_size - n % group_size))
    return W


def _ratios(clipping_ratios):
    if clipping_ratios is not None and len(clipping_ratios) == 0:
        clipping_ratios = None
    if clipping_ratios is None:
        return None, 0
    return (ctypes.c_float * len(clipping_ratios))(*[float(r) for r in clipping_ratios]), len(clipping_ratios)


def _scales(W, group_size, clipping_ratios, bits, asym):
    if W.dim() != 2:
        raise ValueError(f"Expected 2D tensor, got {W.dim()}D")
    dev = device_of(W)
    Wp = _pad_to_group_size(f32(W, dev), group_size).contiguous()
    M, N = Wp.shape
    G = N // group_size
    s = torch.empty(M, G, dtype=torch.float16, device=dev)
    zp = torch.empty(M, G, dtype=torch.int8, device=dev) if asym else None
    arr, nr = _ratios(clipping_ratios)
    if M:
        nat.check(nat.load().ic_rtn_scales(Wp.data_ptr(), M, N, N, bits, int(asym), group_size, arr, nr,
                                           s.data_ptr(), nat.ptr(zp), nat.stream_ptr(dev)), "rtn_scales")
    return back(s, W), back(zp, W)


def _codes(W, scales, zero_points, group_size, bits):
    dev = device_of(W)
    Wp = _pad_to_group_size(f32(W, dev), group_size).contiguous()
    M, N = Wp.shape
    G = N // group_size
    s = scales.to(dev)
    if s.dtype != torch.float16:
        raise ValueError("scales must be float16 (the stored scale dtype)")
    s = s.reshape(M, G).contiguous()
    zp = None if zero_points is None else zero_points.to(dev).to(torch.int8).reshape(M, G).contiguous()
    q = torch.empty(M, N, dtype=torch.int8, device=dev)
    if M:
        nat.check(nat.load().ic_rtn_codes(Wp.data_ptr(), M, N, N, bits, int(zp is not None), group_size,
                                          s.data_ptr(), nat.ptr(zp), q.data_ptr(), N, nat.stream_ptr(dev)),
                  "rtn_codes")
    return back(q, W)


def calculate_scales(W: torch.Tensor, group_size: int = 128,
                     clipping_ratios: list[float] | None = None) -> torch.Tensor:
    """INT4 symmetric per-group scales max|W|/7 (scales.py:62-99) -> fp16 [out, groups]."""
    return _scales(W, group_size, clipping_ratios, 4, False)[0]


def quantize_weights(W: torch.Tensor, scales: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """INT4 codes round-half-away(W/s) clamped to [-8,7] (scales.py:102-123)."""
    return _codes(W, scales, None, group_size, 4)


def calculate_scales_int8(W: torch.Tensor, clipping_ratios: list[float] | None = None) -> torch.Tensor:
    """INT8 symmetric per-row scales max|W|/127 (scales.py:126-160) -> fp16 [out, 1]."""
    if W.dim() != 2:
        raise ValueError(f"Expected 2D tensor, got {W.dim()}D")
    return _scales(W, W.shape[1], clipping_ratios, 8, False)[0]


def quantize_weights_int8(W: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """INT8 codes (scales.py:163-178)."""
    if W.dim() != 2:
        raise ValueError(f"Expected 2D tensor, got {W.dim()}D")
    return _codes(W, scales, None, W.shape[1], 8)


def _fix_asymmetric_scale(scales, w_min, w_max, qmin: int, qmax: int):
    """Raise scales whose zero-point would clamp (scales.py:184-229); elementwise helper."""
    spread = float(qmax - qmin)
    zp_raw = qmin - _round_half_away_from_zero(w_min / scales)
    lo = zp_raw < qmin
    hi = zp_raw > qmax
    if lo.any():
        fix = (w_max.float() / spread).clamp(min=SCALE_MIN, max=SCALE_MAX)
        scales = torch.maximum(scales, torch.where(lo, fix, scales))
    if hi.any():
        fix = (-w_min.float() / spread).clamp(min=SCALE_MIN, max=SCALE_MAX)
        scales = torch.maximum(scales, torch.where(hi, fix, scales))
    return scales


def calculate_scales_asymmetric(W: torch.Tensor, group_size: int = 128,
                                clipping_ratios: list[float] | None = None):
    """INT4 asymmetric scales + zero-points (scales.py:232-282)."""
    return _scales(W, group_size, clipping_ratios, 4, True)


def quantize_weights_asymmetric(W, scales, zero_points, group_size: int = 128):
    """INT4 asymmetric codes (scales.py:285-313)."""
    return _codes(W, scales, zero_points, group_size, 4)


def calculate_scales_int8_asymmetric(W: torch.Tensor, clipping_ratios: list[float] | None = None):
    """INT8 asymmetric per-row scales + zero-points (scales.py:316-361)."""
    if W.dim() != 2:
        raise ValueError(f"Expected 2D tensor, got {W.dim()}D")
    return _scales(W, W.shape[1], clipping_ratios, 8, True)


def quantize_weights_int8_asymmetric(W, scales, zero_points):
    """INT8 asymmetric codes (scales.py:364-384)."""
    if W.dim() != 2:
        raise ValueError(f"Expected 2D tensor, got {W.dim()}D")
    return _codes(W, scales, zero_points, W.shape[1], 8)


def rtn_quantize_fused(W: torch.Tensor, rot_size: int, int_bits: int = 4, asymmetric: bool = False,
                       clipping_ratios: list[float] | None = None, want_codes: bool = True,
                       want_packed: bool = True) -> dict:
    """One pass: sanitize + rotate + per-row scale search + RTN + pack + verify statistics.

    The device-resident form of pipeline.py:527-559 + 890-931 + 1010-1013 for
    one RTN layer (weights with |w| > 1000 are zeroed first, as the pipeline
    does before rotating).  W fp16/bf16/fp32 [out, in] -> dict with ``codes`` int8
    [out, in_pad] (optional), ``packed`` uint8 [out, ceil(in_pad/2)] (INT4),
    ``scales`` fp16 [out, 1], ``zero_points`` int8 [out, 1] (asymmetric) and
    ``stats`` fp64 [mse, max_err] of the verify step, all on the GPU.
    """
    dev = device_of(W)
    Wd = W.to(dev)
    if Wd.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        Wd = Wd.float()
    Wd = Wd.contiguous()
    M, N = Wd.shape
    r = rot_size if rot_size else 1
    npad = -(-N // r) * r
    dt = {torch.float32: nat.IC_F32, torch.float16: nat.IC_F16, torch.bfloat16: nat.IC_BF16}[Wd.dtype]
    codes = torch.empty(M, npad, dtype=torch.int8, device=dev) if want_codes else None
    packed = (torch.empty(M, (npad + 1) // 2, dtype=torch.uint8, device=dev)
              if (want_packed and int_bits == 4) else None)
    s = torch.empty(M, 1, dtype=torch.float16, device=dev)
    zp = torch.empty(M, 1, dtype=torch.int8, device=dev) if asymmetric else None
    sq = torch.empty(M, dtype=torch.float64, device=dev)
    mx = torch.empty(M, dtype=torch.float32, device=dev)
    stats = torch.zeros(2, dtype=torch.float64, device=dev)
    arr, nr = _ratios(clipping_ratios)
    st = nat.stream_ptr(dev)
    lib = nat.load()
    if M:
        nat.check(lib.ic_rtn_fused(Wd.data_ptr(), dt, M, N, N, rot_size, int_bits, int(asymmetric), arr, nr,
                                   nat.ptr(codes), nat.ptr(packed), s.data_ptr(), nat.ptr(zp), sq.data_ptr(),
                                   mx.data_ptr(), st), "rtn_fused")
        nat.check(lib.ic_finalize_stats(sq.data_ptr(), mx.data_ptr(), M, float(M * npad), stats.data_ptr(), st),
                  "finalize_stats")
    return dict(codes=codes, packed=packed, scales=s, zero_points=zp, stats=stats)
