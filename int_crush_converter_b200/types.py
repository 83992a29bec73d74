"""Result record of the layer quantizers (mirrors converter/types.py:163-199)."""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class QuantizationResult:
    """Result of quantizing one weight layer.

    Same fields and meaning as the reference's ``QuantizationResult``:
    ``quantized_W`` int8 codes [out, in], ``scales`` fp16 [out, 1],
    ``zero_points`` int8 [out, 1] or None, ``mse`` / ``max_err`` of the
    dequantized weights against the input, ``method_used`` naming the path
    (``"gptq_b200"``, ``"ldlq_b200"``, ``"rtn_b200"``, ...) and ``fallbacks``
    listing numeric fallbacks taken.
    """

    quantized_W: torch.Tensor
    scales: torch.Tensor
    zero_points: torch.Tensor | None = None
    mse: float = 0.0
    max_err: float = 0.0
    method_used: str = ""
    fallbacks: list[str] = field(default_factory=list)
