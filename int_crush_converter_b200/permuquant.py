"""PermuQuant channel reordering (mirrors converter/permuquant.py) on the GPU.

The candidate order (second moments, optionally joined with activation
moments) and the quantization errors of the acceptance rule run in
libintcrush_b200 (ic_permuquant_order, ic_group_quant_error); the rule and the
alpha sweep keep the reference's logic.  The errors are exact per term and
summed in the original column order, so where the groups span whole rows (the
pipeline's INT4 setting, pipeline.py:604) a permutation leaves them unchanged
and is never accepted with tau >= 0, as in exact arithmetic; the reference's
own decision there rests on the rounding of two fp32 sums.
"""

from __future__ import annotations

import torch

from . import _native as nat
from ._dev import back, device_of

_DT = {torch.float32: nat.IC_F32, torch.float16: nat.IC_F16, torch.bfloat16: nat.IC_BF16}


def _dev_w(W: torch.Tensor, dev) -> torch.Tensor:
    Wd = W.to(dev)
    if Wd.dtype not in _DT:
        Wd = Wd.float()
    return Wd.contiguous()


def _order(W: torch.Tensor, act_mu2, alpha: float):
    dev = device_of(W, act_mu2)
    Wd = _dev_w(W, dev)
    M, N = Wd.shape
    key = torch.empty(N, dtype=torch.float32, device=dev)
    perm = torch.empty(N, dtype=torch.int32, device=dev)
    act = None if act_mu2 is None else act_mu2.to(dev, torch.float32).contiguous()
    nat.check(nat.load().ic_permuquant_order(Wd.data_ptr(), _DT[Wd.dtype], M, N, N, nat.ptr(act), float(alpha),
                                             key.data_ptr(), perm.data_ptr(), nat.stream_ptr(dev)),
              "permuquant_order")
    return key, perm


def channel_second_moments(W: torch.Tensor) -> torch.Tensor:
    """mean_i W[i, j]^2 per input channel (permuquant.py:13-22)."""
    key, _ = _order(W, None, 0.0)
    return back(key, W)


def find_permutation_weight(W: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """Channels by descending second moment (permuquant.py:25-40), int64 like argsort."""
    _, perm = _order(W, None, 0.0)
    return back(perm.long(), W)


def find_permutation_joint(W: torch.Tensor, act_mu2: torch.Tensor, alpha: float = 0.5,
                           group_size: int = 128) -> torch.Tensor:
    """Channels by descending act^alpha * w^(1-alpha) (permuquant.py:43-67)."""
    _, perm = _order(W, act_mu2, alpha)
    return back(perm.long(), W)


def _errors(Wd: torch.Tensor, perm, group_size: int, int_bits: int) -> float:
    M, N = Wd.shape
    dev = Wd.device
    row = torch.empty(M, dtype=torch.float64, device=dev)
    inv = torch.empty(N, dtype=torch.int32, device=dev) if perm is not None else None
    p32 = None if perm is None else perm.to(dev, torch.int32).contiguous()
    nat.check(nat.load().ic_group_quant_error(Wd.data_ptr(), _DT[Wd.dtype], M, N, N, nat.ptr(p32), int(group_size),
                                              int(int_bits), nat.ptr(inv), row.data_ptr(), nat.stream_ptr(dev)),
              "group_quant_error")
    return float(row.sum().item())


def compute_group_quant_error(W: torch.Tensor, group_size: int = 128, int_bits: int = 4) -> float:
    """Total squared RTN error of W (permuquant.py:70-105)."""
    dev = device_of(W)
    return _errors(_dev_w(W, dev), None, group_size, int_bits)


def find_permutation_with_acceptance(W: torch.Tensor, act_mu2: torch.Tensor | None = None, alpha: float = 0.5,
                                     group_size: int = 128, tau: float = 0.0,
                                     int_bits: int = 4) -> tuple[torch.Tensor, bool]:
    """Candidate order plus the acceptance rule: relative error improvement > tau
    (permuquant.py:108-150).  The permuted error is computed without forming
    W[:, perm]."""
    dev = device_of(W, act_mu2)
    Wd = _dev_w(W, dev)
    _, perm = _order(Wd, act_mu2, alpha)
    e0 = _errors(Wd, None, group_size, int_bits)
    e1 = _errors(Wd, perm, group_size, int_bits)
    rel = (e0 - e1) / e0 if e0 > 0 else 0.0
    return back(perm.long(), W), bool(rel > tau)


def sweep_alpha(W: torch.Tensor, act_mu2: torch.Tensor | None = None, group_size: int = 128, tau: float = 0.0,
                num_alpha: int = 11, int_bits: int = 4) -> tuple[torch.Tensor, float, bool]:
    """Best accepted permutation over alpha in [0, 1] (permuquant.py:153-211)."""
    if num_alpha < 1:
        raise ValueError(f"num_alpha must be >= 1, got {num_alpha}")
    if act_mu2 is None or num_alpha == 1:
        perm, accepted = find_permutation_with_acceptance(W, act_mu2, 0.0, group_size, tau, int_bits)
        return perm, 0.0, accepted
    dev = device_of(W, act_mu2)
    Wd = _dev_w(W, dev)
    best_perm, best_alpha, best_err, best_ok = None, 0.0, float("inf"), False
    for i in range(num_alpha):
        alpha = i / (num_alpha - 1)
        perm, accepted = find_permutation_with_acceptance(Wd, act_mu2, alpha, group_size, tau, int_bits)
        if accepted:
            err = _errors(Wd, perm, group_size, int_bits)
            if err < best_err:
                best_err, best_perm, best_alpha, best_ok = err, perm, alpha, True
    if best_perm is None:
        best_perm = torch.arange(W.shape[1], device=dev)
    return back(best_perm, W), best_alpha, best_ok


def apply_permutation_to_weight(W: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    """W[:, perm] (permuquant.py:214-225)."""
    return W[:, perm.to(W.device)]
