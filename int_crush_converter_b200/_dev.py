"""Device-placement helpers shared by the API modules."""

from __future__ import annotations

import torch

from . import _native as nat


def device_of(*tensors) -> torch.device:
    """The CUDA device to run on: the first CUDA input's, else the current one."""
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            return nat.require_device(t.device)
    return nat.require_device(None)


def f32(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    return t.to(device=dev, dtype=torch.float32).contiguous()


def back(t, like: torch.Tensor):
    """Return ``t`` on the device of the caller's tensor ``like``."""
    if t is None:
        return None
    return t if t.device == like.device else t.to(like.device)


def round4(n: int) -> int:
    return (n + 3) & ~3


def split(t32: torch.Tensor, ld: int | None = None):
    """fp32 [r, c] -> TF32 (hi, lo) pair with leading dimension ``ld`` (>= c), zero padded."""
    r, c = t32.shape
    ld = ld or round4(c)
    hi = torch.zeros(r, ld, device=t32.device, dtype=torch.float32)
    lo = torch.zeros(r, ld, device=t32.device, dtype=torch.float32)
    if r and c:
        nat.check(nat.load().ic_split_tf32(t32.data_ptr(), r, c, t32.stride(0), hi.data_ptr(), lo.data_ptr(),
                                           ld, nat.stream_ptr(t32.device)), "split_tf32")
    return hi, lo


def workspace(nbytes: int, dev: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
