"""Greedy local search on the GPU (mirrors converter/greedy.py).

``greedy_local_search`` computes what greedy_local_search_pytorch
(greedy.py:487-541) computes -- coordinate descent over the whole integer
grid, full-rank Hessian -- with exact blocked cross terms on the tensor
cores.  ``greedy_lowrank`` is the reference's GPU low-rank variant
(greedy_lowrank_triton, greedy.py:384-479): H approximated by its leading
eigenpairs plus the exact diagonal, one device pass per sweep over all
columns, the pass loop stopping when the proxy loss stops improving by 1%;
when the decomposition does not qualify it falls back to the full-rank search,
as the reference falls back to its v2 kernel.
"""

from __future__ import annotations

import os

import torch

from . import _native as nat
from ._dev import device_of, f32, split, workspace
from .config import (EIGENVALUE_FLOOR, GREEDY_GEMM_PASSES, LOWRANK_MAX_K, LOWRANK_MAX_RANK_FRAC, LOWRANK_SKETCH,
                     STALL_THRESHOLD)


def greedy_local_search(W: torch.Tensor, Q: torch.Tensor, scale_2d: torch.Tensor, H: torch.Tensor,
                        num_passes: int, clamp_min: int, clamp_max: int, *,
                        gemm_passes: int | None = None) -> torch.Tensor:
    """Returns int8 codes [M, N] minimising tr((Q*s - W) H (Q*s - W)^T) coordinate-wise.
    ``gemm_passes`` (1 or 3) sets the precision of the cross-term products;
    default: the environment variable IC_GREEDY_GEMM_PASSES, else
    ``config.GREEDY_GEMM_PASSES`` (3)."""
    if gemm_passes is None:
        gemm_passes = os.environ.get("IC_GREEDY_GEMM_PASSES") or GREEDY_GEMM_PASSES
    gp = int(gemm_passes)
    if gp not in (1, 3):
        raise ValueError(f"gemm_passes must be 1 or 3, got {gemm_passes}")
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
                                    int(clamp_max), gp, ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)),
                  "greedy_run")
    out = Qd.clamp(clamp_min, clamp_max)
    return out if W.is_cuda else out.to(W.device)


greedy_local_search_pytorch = greedy_local_search  # name used by converter/ldlq.py:647


def lowrank_decompose(H: torch.Tensor, rank_threshold: float = 0.01,
                      max_rank_frac: float = LOWRANK_MAX_RANK_FRAC):
    """(s_k, U_k, k, ok) as _lowrank_decompose_svd (greedy.py:322-349): the
    randomized SVD of the symmetric H (svd.svd_lowrank, two power iterations),
    eigenpairs above rank_threshold * s_max kept.  The sketch is
    LOWRANK_SKETCH = 64 columns (the reference sketches max(N/2, 64)); when all
    64 qualify the rank is not resolved and ok is False (full-rank fallback)."""
    from .svd import svd_lowrank
    N = H.shape[0]
    q = min(LOWRANK_SKETCH, N)
    U, s, _ = svd_lowrank(H, q=q, niter=2)
    smax = s[0].item()
    if not smax >= EIGENVALUE_FLOOR:
        return None, None, 0, False
    mask = s > smax * rank_threshold
    k = int(mask.sum().item())
    if k > max_rank_frac * N or k > LOWRANK_MAX_K or k >= q:
        return None, None, k, False
    return s[mask].contiguous(), U[:, mask].contiguous(), k, True


def greedy_lowrank(W: torch.Tensor, Q: torch.Tensor, scale_2d: torch.Tensor, H: torch.Tensor, num_passes: int,
                   clamp_min: int, clamp_max: int, rank_threshold: float = 0.01,
                   max_rank_frac: float = LOWRANK_MAX_RANK_FRAC, decomposition=None):
    """Low-rank greedy search (greedy.py:384-479).  Returns (int8 codes, k,
    used_lowrank); with used_lowrank False the codes come from the full-rank
    search (the reference's fallback).  ``decomposition`` = (s_k, U_k) skips
    the randomized decomposition (tests give both sides the same one)."""
    from .hessian import _abt
    dev = device_of(W, Q, H)
    Wd = f32(W, dev)
    M, N = Wd.shape
    Hd = f32(H, dev)
    if decomposition is not None:
        s_k, U_k = (f32(torch.as_tensor(t), dev).contiguous() for t in decomposition)
        k, ok = int(s_k.numel()), 1 <= s_k.numel() <= 64
    else:
        s_k, U_k, k, ok = lowrank_decompose(Hd, rank_threshold, max_rank_frac)
    if not ok:
        return greedy_local_search(W, Q, scale_2d, H, num_passes, clamp_min, clamp_max), k, False
    Qd = Q.to(dev).float().round().clamp(-128, 127).to(torch.int8).contiguous()
    Sd = f32(scale_2d.expand(M, N) if scale_2d.shape != (M, N) else scale_2d, dev).contiguous()
    err = (Qd.float() * Sd - Wd).contiguous()                      # greedy.py:437
    hdiag = Hd.diagonal().contiguous()
    U = U_k.contiguous()
    SU = (U * s_k.unsqueeze(0)).contiguous()                        # s_val * u_val
    elr = _abt(err, U.T.contiguous()).contiguous()                  # err @ U_k (greedy.py:443)
    lib = nat.load()
    st = nat.stream_ptr(dev)
    prev = float("inf")
    runs = 0
    for p in range(num_passes):
        runs += 1
        nat.check(lib.ic_greedy_lowrank_pass(err.data_ptr(), N, Qd.data_ptr(), N, Sd.data_ptr(), N,
                                             hdiag.data_ptr(), U.data_ptr(), SU.data_ptr(), k, elr.data_ptr(),
                                             M, N, int(clamp_min), int(clamp_max), st), "greedy_lowrank")
        proxy = (_abt(err, Hd) * err).sum().item()                  # greedy.py:464-467
        if p > 0 and proxy >= prev * STALL_THRESHOLD:               # greedy.py:473-476
            break
        prev = proxy
    out = Qd.clamp(clamp_min, clamp_max)
    greedy_lowrank.passes_run = runs
    return (out if W.is_cuda else out.to(W.device)), k, True
