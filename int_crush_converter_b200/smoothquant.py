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
