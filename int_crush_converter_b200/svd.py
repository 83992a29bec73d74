"""SVD-absorbed low-rank split (mirrors converter/svd.py) on the GPU.

``decompose_weight(W, rank)`` returns the reference's :class:`SVDResult`
(L1 [out, r] fp16 = U S, L2 [r, in] fp16 = V^T, residual fp32 = W - L1 L2)
computed with the algorithm the reference calls, torch.svd_lowrank(W, q=r,
niter=2) (a randomized range finder with two power iterations, then the SVD of
the projected r x in matrix): every product on the library's 3xTF32 tensor-core
GEMM, the orthonormalisations by ic_orthonormalize (classical Gram-Schmidt
applied twice), the small SVD through the eigenpairs of B B^T by ic_sym_eig (cyclic
Jacobi).  The range finder draws its Gaussian test matrix from torch's CUDA
generator (the pipeline seeds it, pipeline.py:258-263), so, as with the
reference on different hardware, the factors are one valid randomized
approximation: parity is judged on the residual's energy.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as nat
from ._dev import back, device_of, f32
from .hessian import _abt


@dataclass
class SVDResult:
    """W ~= L1 @ L2 + residual (svd.py:20-33)."""

    L1: torch.Tensor
    L2: torch.Tensor
    residual: torch.Tensor


def _orth(X: torch.Tensor) -> torch.Tensor:
    X = X.contiguous()
    nat.check(nat.load().ic_orthonormalize(X.data_ptr(), X.shape[0], X.shape[1], X.shape[1],
                                           nat.stream_ptr(X.device)), "orthonormalize")
    return X


def svd_lowrank(A: torch.Tensor, q: int, niter: int = 2):
    """U [m, q], S [q], V [n, q] with A ~= U diag(S) V^T (torch.svd_lowrank's algorithm)."""
    m, n = A.shape
    if m < n:
        V, S, U = svd_lowrank(A.T.contiguous(), q, niter)
        return U, S, V
    dev = A.device
    At = A.T.contiguous()
    Rt = torch.randn(q, n, device=dev, dtype=torch.float32)
    Q = _orth(_abt(A, Rt))                        # A R
    for _ in range(niter):
        Q = _orth(_abt(At, Q.T.contiguous()))      # A^T Q
        Q = _orth(_abt(A, Q.T.contiguous()))       # A (A^T Q)
    B = _abt(Q.T.contiguous(), At).contiguous()   # Q^T A [q, n]
    C = _abt(B, B).contiguous()                   # B B^T [q, q]
    evals = torch.empty(q, device=dev, dtype=torch.float32)
    Ub = torch.empty(q, q, device=dev, dtype=torch.float32)
    nat.check(nat.load().ic_sym_eig(C.data_ptr(), q, C.shape[1], evals.data_ptr(), Ub.data_ptr(), q,
                                    nat.stream_ptr(dev)), "sym_eig")
    S = evals.clamp(min=0).sqrt()
    U = _abt(Q, Ub.T.contiguous())                                  # Q Ub [m, q]
    Vt = _abt(Ub.T.contiguous(), B.T.contiguous())                  # Ub^T B [q, n]
    Vt = Vt / torch.where(S > 0, S, torch.ones_like(S)).unsqueeze(1)
    return U.contiguous(), S, Vt.T.contiguous()


def decompose_weight(W: torch.Tensor, rank: int = 32) -> SVDResult:
    """L1 = U S (fp16), L2 = V^T (fp16), residual = W - L1 L2 in fp32 (svd.py:35-75)."""
    if W.dim() != 2:
        raise ValueError(f"decompose_weight requires a 2D tensor, got {W.dim()}D")
    out_features, in_features = W.shape
    r = min(rank, min(out_features, in_features))
    if r <= 0:
        raise ValueError(f"rank must be > 0, got {rank} (clamped to {r})")
    dev = device_of(W)
    Wd = f32(W, dev)
    U, S, V = svd_lowrank(Wd, r, niter=2)
    L1 = (U[:, :r] * S[:r].unsqueeze(0)).to(torch.float16)
    L2 = V[:, :r].T.contiguous().to(torch.float16)
    residual = Wd - _abt(L1.float().contiguous(), L2.float().T.contiguous())
    return SVDResult(L1=back(L1, W), L2=back(L2, W), residual=back(residual.contiguous(), W))
