"""INT4 packing on the GPU (mirrors converter/packing.py).

Two's-complement nibbles, low nibble = even column, odd widths padded with a
zero nibble (the ``packing_order="little"`` layout the pipeline records).
"""

from __future__ import annotations

import torch

from . import _native as nat
from ._dev import back, device_of

INT4_MIN = -8
INT4_MAX = 7
INT4_PACK_FACTOR = 2


class INT4PackingError(ValueError):
    """Raised when values are out of INT4 range during packing (packing.py:13-14)."""


def validate_int4_range(tensor: torch.Tensor) -> None:
    """Finiteness and range check (packing.py:17-27); raises INT4PackingError."""
    if tensor.numel() == 0:
        return
    if tensor.is_floating_point() and not torch.isfinite(tensor).all():
        raise INT4PackingError("Tensor contains NaN or Inf values")
    lo, hi = tensor.min(), tensor.max()
    if lo < INT4_MIN or hi > INT4_MAX:
        raise INT4PackingError(f"Values must be in [{INT4_MIN}, {INT4_MAX}], got [{lo.item()}, {hi.item()}]")


def pack_int4(values: torch.Tensor) -> torch.Tensor:
    """[..., K] INT4 values -> [..., ceil(K/2)] uint8 (packing.py:30-46)."""
    dev = device_of(values)
    v = values.to(dev)
    if v.is_floating_point():
        validate_int4_range(v)
    v = v.to(torch.int8)
    K = v.shape[-1]
    lead = v.shape[:-1]
    v2 = v.reshape(-1, K).contiguous()
    M = v2.shape[0]
    out = torch.empty(M, (K + 1) // 2, dtype=torch.uint8, device=dev)
    if v2.numel():
        nat.check(nat.load().ic_pack_int4(v2.data_ptr(), M, K, K, out.data_ptr(), (K + 1) // 2,
                                          nat.stream_ptr(dev)), "pack_int4")
    return back(out.reshape(*lead, (K + 1) // 2), values)


def unpack_int4(packed: torch.Tensor, K: int) -> torch.Tensor:
    """[..., ceil(K/2)] uint8 -> [..., K] int8 (packing.py:49-66)."""
    dev = device_of(packed)
    p = packed.to(dev).to(torch.uint8)
    lead = p.shape[:-1]
    p2 = p.reshape(-1, p.shape[-1]).contiguous()
    M = p2.shape[0]
    out = torch.empty(M, K, dtype=torch.int8, device=dev)
    if M and K:
        nat.check(nat.load().ic_unpack_int4(p2.data_ptr(), M, K, p2.shape[1], out.data_ptr(), K,
                                            nat.stream_ptr(dev)), "unpack_int4")
    return back(out.reshape(*lead, K), packed)
