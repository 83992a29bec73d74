"""Greedy local search on the GPU (mirrors converter/greedy.py).

``greedy_local_search`` computes what greedy_local_search_pytorch
(greedy.py:487-541) computes -- coordinate descent over the whole integer
grid, full-rank Hessian -- with exact blocked cross terms on the tensor
cores.  (The reference's GPU dispatcher may instead take a low-rank
approximation, greedy.py:384-479; this path always keeps the full H, which is
what its CPU path and the parity oracle do.)
"""

from __future__ import annotations

import torch

from . import _native as nat
from ._dev import device_of, f32, split, workspace
from .config import GEMM_PASSES


def greedy_local_search(W: torch.Tensor, Q: torch.Tensor, scale_2d: torch.Tensor, H: torch.Tensor,
                        num_passes: int, clamp_min: int, clamp_max: int) -> torch.Tensor:
    """Returns int8 codes [M, N] minimising tr((Q*s - W) H (Q*s - W)^T) coordinate-wise."""
    dev = device_of(W, Q, H)
    Wd = f32(W, dev)
    M, N = Wd.shape
    Qd = Q.to(dev).float().round().clamp(-128, 127).to(torch.int8).contiguous()
    Sd = f32(scale_2d.expand(M, N) if scale_2d.shape != (M, N) else scale_2d, dev)
    hi, lo = split(f32(H, dev))
    lib = nat.load()
    ws = workspace(lib.ic_greedy_workspace_size(M, N), dev)
    if M and N and num_passes > 0:
        nat.check(lib.ic_greedy_run(Wd.data_ptr(), N, Qd.data_ptr(), N, Sd.data_ptr(), N, hi.data_ptr(),
                                    lo.data_ptr(), hi.shape[1], M, N, int(num_passes), int(clamp_min),
                                    int(clamp_max), GEMM_PASSES, ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)),
                  "greedy_run")
    out = Qd.clamp(clamp_min, clamp_max)
    return out if W.is_cuda else out.to(W.device)


greedy_local_search_pytorch = greedy_local_search  # name used by converter/ldlq.py:647
