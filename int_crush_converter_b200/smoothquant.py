"""SmoothRot pre-step of the per-layer path (configs with SmoothQuant + rotation).

The pipeline smooths FFN down layers before rotating them
(pipeline.py:547-553 for W, 766-774 for H).  The hot form is fused into the
layer call: ``quantize_gptq_layer(..., smoothing=s)`` applies both inside the
rotation kernels' loads.  These two functions are the standalone mirrors of
the reference's, on the GPU, for callers that compose the steps themselves.
"""

from __future__ import annotations

import torch

from . import _native as nat
from ._dev import device_of

SMOOTHQUANT_AMAX_FLOOR = 1e-8  # config.py:148
SMOOTHQUANT_HESSIAN_FLOOR = 1e-8 ** 2  # config.py:148-152
SANITIZE_CEIL = 1e30  # config.py:78


def apply_smoothing_to_weight(weight: torch.Tensor, smoothing: torch.Tensor) -> torch.Tensor:
    """W_smooth[:, j] = W[:, j] * s_j, same dtype as W (smoothquant.py:54-69)."""
    dev = device_of(weight, smoothing)
    nat.require_device(dev)
    W = weight.to(dev)
    out = W * smoothing.to(dev).unsqueeze(0).to(W.dtype)
    return out if weight.is_cuda else out.cpu()


def _transform_hessian_for_smoothquant(hessian: torch.Tensor, smoothing_factors: torch.Tensor) -> torch.Tensor:
    """H / max(s_i s_j, 1e-16), capped at 1e30, for a 2-D Hessian (pipeline.py:99-137)."""
    if hessian.dim() != 2:
        raise ValueError("the device mirror handles the 2-D Hessian; 3-D and DLR keep the reference's path")
    dev = device_of(hessian, smoothing_factors)
    nat.require_device(dev)
    s = smoothing_factors.to(dev).float()
    outer = (s.unsqueeze(0) * s.unsqueeze(1)).clamp(min=SMOOTHQUANT_HESSIAN_FLOOR)
    out = (hessian.to(dev).float() / outer).clamp(max=SANITIZE_CEIL).to(hessian.dtype)
    return out if hessian.is_cuda else out.cpu()


def _factors(act: torch.Tensor, act_stride: int, weight: torch.Tensor, mode: int, alpha: float,
             nsamp: float, dev: torch.device) -> torch.Tensor:
    from .gptq import _DT
    W = weight.to(dev)
    if W.dtype not in _DT:
        W = W.float()
    W = W.contiguous()
    out = torch.empty(W.shape[1], dtype=torch.float32, device=dev)
    nat.check(nat.load().ic_smooth_factors(W.data_ptr(), _DT[W.dtype], W.shape[0], W.shape[1], W.shape[1],
                                           act.data_ptr(), act_stride, mode, float(alpha), float(nsamp),
                                           out.data_ptr(), nat.stream_ptr(dev)), "smooth_factors")
    return out


def compute_smoothing_factors(act_amax: torch.Tensor, weight: torch.Tensor, alpha: float = 0.5) -> torch.Tensor:
    """s_j = max(amax_j, 1e-8)^alpha / max(max_i |W_ij|, 1e-8)^(1-alpha) (smoothquant.py:11-52), on the GPU."""
    if act_amax.dim() != 1:
        raise ValueError(f"act_amax must be 1D [in_features], got {act_amax.dim()}D")
    if weight.dim() != 2:
        raise ValueError(f"weight must be 2D [out, in], got {weight.dim()}D")
    if act_amax.shape[0] != weight.shape[1]:
        raise ValueError(f"act_amax length {act_amax.shape[0]} != weight in_features {weight.shape[1]}")
    dev = device_of(weight, act_amax)
    a = act_amax.to(dev, torch.float32).contiguous()
    out = _factors(a, 1, weight, 0, alpha, 1.0, dev)
    return out if weight.is_cuda else out.cpu()


def compute_smoothing_from_hessian_diag(hessian_diag: torch.Tensor, weight: torch.Tensor, alpha: float = 0.5,
                                        num_calibration_samples: int = 128) -> torch.Tensor:
    """s_j = sqrt(max(H_jj / n, 1e-8))^alpha / max(max_i |W_ij|, 1e-8)^(1-alpha)
    (smoothquant.py:72-102), on the GPU.  ``hessian_diag`` may be the diagonal
    [in] or the full Hessian [in, in] (its diagonal is read in place)."""
    dev = device_of(weight, hessian_diag)
    n = max(1, int(num_calibration_samples))
    h = hessian_diag.to(dev, torch.float32).contiguous()
    stride = 1 if h.dim() == 1 else h.shape[1] + 1
    if h.shape[0] != weight.shape[1]:
        raise ValueError(f"hessian_diag length {h.shape[0]} != weight in_features {weight.shape[1]}")
    out = _factors(h, stride, weight, 1, alpha, float(n), dev)
    return out if weight.is_cuda else out.cpu()
