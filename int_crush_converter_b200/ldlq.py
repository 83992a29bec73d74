"""LDLQ on the GPU (mirrors converter/ldlq.py).

``ldlq_quantize_layer`` keeps the reference's signature and semantics:
calibration Hessian (2-D / 3-D / DLR) or weight-only H = W^T W / M (damped,
and the damped H is what greedy uses), per-element scales with sign-flip
rounding, iterative scale refinement with momentum / divergence / convergence
checks, greedy local search, final least-squares per-row scales.  The column
loop, the lazy update, the inverse, the W^T W product, the scale update and
the greedy search run in libintcrush_b200.
"""

from __future__ import annotations

import math
import os
import warnings

import torch

from . import _native as nat
from ._dev import back, device_of, f32, round4, split, workspace
from .config import (
    ABS_SCALE_FLOOR, CONVERGENCE_EPS, CONVERGENCE_IMPROVEMENT_THRESHOLD, DENOMINATOR_FLOOR, DIAG_MEAN_FLOOR,
    GEMM_PASSES, INT4_SCALE_DIVISOR, INT8_SCALE_DIVISOR, MSE_DIVERGENCE_THRESHOLD, SANITIZE_CEIL, SANITIZE_FLOOR,
    SCALE_CEIL_MULTIPLIER, SCALE_DTYPE, SCALE_FLOOR_MULTIPLIER, SCALE_MAX, SCALE_MIN, SCALE_MOMENTUM, SUPERBLOCK,
    W_NONZERO_THRESHOLD,
)
from .greedy import greedy_local_search
from .greedy import greedy_lowrank as greedy_lowrank_search
from .hessian import dlr_to_dense, hessian_pair, inverse_pair, woodbury_inverse
from .types import QuantizationResult


def weight_only_hessian(Wd: torch.Tensor) -> torch.Tensor:
    """H = W^T W / M (ldlq.py:186) with the product on the tensor cores (3xTF32)."""
    dev = Wd.device
    M, N = Wd.shape
    lib = nat.load()
    st = nat.stream_ptr(dev)
    ldt = round4(M)
    th = torch.zeros(N, ldt, device=dev)
    tl = torch.zeros(N, ldt, device=dev)
    nat.check(lib.ic_transpose(Wd.data_ptr(), None, M, N, N, 1.0, th.data_ptr(), None, ldt, st), "transpose")
    nat.check(lib.ic_split_tf32(th.data_ptr(), N, M, ldt, th.data_ptr(), tl.data_ptr(), ldt, st), "split")
    ldh = round4(N)
    H = torch.empty(N, ldh, device=dev)
    nat.check(lib.ic_gemm_tn(N, N, M, 1.0, th.data_ptr(), tl.data_ptr(), ldt, th.data_ptr(), tl.data_ptr(), ldt,
                             0.0, None, None, ldh, H.data_ptr(), None, ldh, 3, st), "gemm")
    return H[:, :N] / M


def _sanitize(s: torch.Tensor) -> torch.Tensor:  # ldlq.py:326-330
    if not torch.isfinite(s).all():
        s = torch.nan_to_num(s, nan=SANITIZE_FLOOR, posinf=SANITIZE_CEIL, neginf=SANITIZE_FLOOR).clamp(min=SANITIZE_FLOOR)
    return s


def _single_pass(Wd, hi, lo, ld, scale_2d, block_size, qmin, qmax):  # ldlq.py:282-366
    dev = Wd.device
    M, N = Wd.shape
    s2 = _sanitize(scale_2d.reshape(M, N)).contiguous()
    Q = torch.zeros(M, N, dtype=torch.int8, device=dev)
    W_work = Wd.clone()
    sb = max(1, SUPERBLOCK // block_size) * block_size
    lib = nat.load()
    ws = workspace(lib.ic_gptq_workspace_size(M, N, block_size, sb), dev)
    nat.check(lib.ic_ldlq_run(W_work.data_ptr(), N, M, N, hi.data_ptr(), lo.data_ptr(), ld, block_size, sb,
                              s2.data_ptr(), N, qmin, qmax, Q.data_ptr(), N, GEMM_PASSES, ws.data_ptr(), ws.numel(),
                              nat.stream_ptr(dev)), "ldlq_run")
    return Q


def _update_scales(Wd, Q, cur, flat):  # ldlq.py:553-599
    smin, smax = flat.aminmax()
    lo = max(smin.item() * SCALE_FLOOR_MULTIPLIER, ABS_SCALE_FLOOR)
    hi = smax.item() * SCALE_CEIL_MULTIPLIER
    new = cur.clone()
    nat.check(nat.load().ic_ldlq_update_scales(Wd.data_ptr(), Q.data_ptr(), new.data_ptr(), flat.data_ptr(),
                                               new.numel(), SCALE_MOMENTUM, 1 - SCALE_MOMENTUM, lo, hi,
                                               W_NONZERO_THRESHOLD, nat.stream_ptr(Wd.device)), "ldlq_update")
    return new


def _iterative(Wd, hi, lo, ld, flat, iterations, block_size, qmin, qmax):  # ldlq.py:479-550
    M, N = Wd.shape
    cur = _sanitize(flat.clone())
    prev_mse = float("inf")
    prev_scales = None
    Q_res = None
    for it in range(iterations):
        Qi = _single_pass(Wd, hi, lo, ld, cur, block_size, qmin, qmax)
        Q_res = Qi
        mse = (Wd - Qi.float() * cur.reshape(M, N)).double().abs().pow(2).mean().item()
        if not math.isfinite(mse):
            if prev_scales is not None:
                cur = prev_scales
            break
        if it > 0 and mse > prev_mse * MSE_DIVERGENCE_THRESHOLD:
            if prev_scales is not None:
                cur = prev_scales
            break
        impr = (prev_mse - mse) / (prev_mse + CONVERGENCE_EPS)
        if it > 0 and impr < CONVERGENCE_IMPROVEMENT_THRESHOLD:
            break
        prev_mse = mse
        if it < iterations - 1:
            prev_scales = cur.clone()
            cur = _update_scales(Wd, Qi, cur, flat)
    return Q_res


def _ls_scales(Q, Wd):  # ldlq.py:227-231, 262-265
    Qf = Q.float()
    num = (Qf * Wd).sum(dim=1, keepdim=True)
    den = (Qf * Qf).sum(dim=1, keepdim=True).clamp(min=DENOMINATOR_FLOOR)
    return (num / den).clamp(min=SCALE_MIN)


def ldlq_quantize_layer(W: torch.Tensor, hessian=None, block_size: int = 128, damping: float = 0.01,
                        int_bits: int = 4, iterations: int = 1, greedy_passes: int = 0,
                        rank_threshold: float = 0.01, greedy_lowrank: bool | None = None) -> QuantizationResult:
    """Quantize one weight matrix with LDLQ (ldlq.py:95-279).

    The greedy search uses the full-rank Hessian (the reference's CPU path,
    the parity oracle) unless ``greedy_lowrank`` (default: the environment
    variable IC_GREEDY_LOWRANK=1) selects the reference's GPU low-rank variant
    with ``rank_threshold`` (greedy.py:384-479, dispatched by
    ldlq._greedy_local_search, ldlq.py:602-647).
    """
    if int_bits not in (4, 8):
        raise ValueError(f"int_bits must be 4 or 8, got {int_bits}")
    if W.dim() != 2:
        raise ValueError(f"Expected 2D weight tensor, got {W.dim()}D")
    Hsrc = hessian["D"] if isinstance(hessian, dict) else hessian
    dev = device_of(W, Hsrc)
    Wd = f32(W, dev)
    M, N = Wd.shape
    div = INT8_SCALE_DIVISOR if int_bits == 8 else INT4_SCALE_DIVISOR
    qmin, qmax = (-128, 127) if int_bits == 8 else (-8, 7)
    fallbacks: list[str] = []

    if hessian is not None:
        if isinstance(hessian, dict):
            if hessian["D"].shape[0] != N:
                raise ValueError(f"DLR Hessian dim {hessian['D'].shape[0]} != in_features {N}")
            Hinv = woodbury_inverse(hessian["D"], hessian["U"], damping=damping)
            hi, lo = split(Hinv.contiguous())
            H = dlr_to_dense(hessian["D"], hessian["U"])
        else:
            Hd = f32(hessian, dev)
            if Hd.dim() == 3:  # ldlq.py:64-92: per-block damped inverse in a dense [N, N]
                nb, bs, _ = Hd.shape
                hi = torch.zeros(N, round4(N), device=dev)
                lo = torch.zeros_like(hi)
                H = torch.zeros(N, N, device=dev)
                for bi in range(nb):
                    c0, c1 = bi * bs, min(bi * bs + bs, N)
                    if c1 <= c0:
                        break
                    blk = Hd[bi, :c1 - c0, :c1 - c0].contiguous()
                    bh, bl, n = hessian_pair(blk, 0, dev, rotate=False)
                    inverse_pair(bh, bl, n, damping, H_fallback=blk)
                    hi[c0:c1, c0:c1] = bh[:n, :n]
                    lo[c0:c1, c0:c1] = bl[:n, :n]
                    H[c0:c1, c0:c1] = blk
            elif Hd.dim() == 2:
                if tuple(Hd.shape) != (N, N):
                    raise ValueError(f"Hessian shape {tuple(Hd.shape)} != ({N}, {N})")
                H = Hd
                hi, lo, n = hessian_pair(Hd, 0, dev, rotate=False)
                inverse_pair(hi, lo, n, damping, H_fallback=Hd)
            else:
                raise ValueError(f"Expected 2D tensor, 3D tensor, or DLR dict Hessian, got {Hd.dim()}D")
    else:
        warnings.warn("LDLQ: no calibration Hessian provided; using H = W^T W / M. This can perform worse than RTN. "
                      "Pass a calibration Hessian from GPTQ calibration data for best results.", stacklevel=2)
        H = weight_only_hessian(Wd)
        if not torch.isfinite(H).all():  # ldlq.py:189-205
            s = (Wd.abs().amax(dim=1, keepdim=True) / div).clamp(min=SCALE_MIN, max=SCALE_MAX)
            q = (Wd / s).round().clamp(qmin, qmax).to(torch.int8)
            d = Wd - q.float() * s
            return QuantizationResult(quantized_W=back(q, W), scales=back(s.to(SCALE_DTYPE), W), zero_points=None,
                                      mse=d.double().pow(2).mean().item(), max_err=d.abs().max().item(),
                                      method_used="rtn", fallbacks=["hessian_nan_rtn"])
        dm = H.diagonal().mean().clamp(min=DIAG_MEAN_FLOOR)
        H = H + damping * dm * torch.eye(N, device=dev)
        hi, lo, n = hessian_pair(H, 0, dev, rotate=False)
        inverse_pair(hi, lo, n, None, H_fallback=H)

    ld = hi.shape[1]
    rs = (Wd.abs().amax(dim=1, keepdim=True) / div).clamp(min=SCALE_MIN)
    flat = rs.expand(M, N).contiguous()
    if iterations > 1:
        Q = _iterative(Wd, hi, lo, ld, flat, iterations, block_size, qmin, qmax)
    else:
        Q = _single_pass(Wd, hi, lo, ld, flat, block_size, qmin, qmax)
    if greedy_passes > 0:
        gs = _ls_scales(Q, Wd)
        if greedy_lowrank is None:
            greedy_lowrank = os.environ.get("IC_GREEDY_LOWRANK", "") == "1"
        if greedy_lowrank:
            Q, _, _ = greedy_lowrank_search(Wd, Q, gs.expand(M, N).contiguous(), H, greedy_passes, qmin, qmax,
                                            rank_threshold=rank_threshold)
        else:
            Q = greedy_local_search(Wd, Q, gs.expand(M, N).contiguous(), H, greedy_passes, qmin, qmax)
    fs = _ls_scales(Q, Wd)
    d = Wd - Q.float() * fs
    return QuantizationResult(quantized_W=back(Q, W), scales=back(fs.to(SCALE_DTYPE), W), zero_points=None,
                              mse=d.double().pow(2).mean().item(), max_err=(d.abs().max().item() if d.numel() else 0.0),
                              method_used="ldlq_b200", fallbacks=fallbacks)
