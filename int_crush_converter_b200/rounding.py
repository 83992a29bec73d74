"""Rounding helper and the Hessian inverse (mirrors converter/rounding.py).

The column loops of rounding._gptq_block / _ldlq_round_column live in the
CUDA block kernels (csrc/gptq.cu); this module keeps the small elementwise
helper and the inverse with the reference's fallback chain.
"""

from __future__ import annotations

import torch


def _round_half_away_from_zero(x: torch.Tensor) -> torch.Tensor:
    """where(x >= 0, floor(x + 0.5), ceil(x - 0.5)) (rounding.py:106-112)."""
    return torch.where(x >= 0, torch.floor(x + 0.5), torch.ceil(x - 0.5))


def _invert_hessian(H: torch.Tensor) -> torch.Tensor:
    """Inverse with the reference's chain (rounding.py:19-34) on the GPU."""
    from .hessian import invert_dense
    return invert_dense(H, damping=None)[0]
