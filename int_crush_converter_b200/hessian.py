"""Hessian preparation on the GPU: rotation into the TF32 pair layout, damping,
the tensor-core SPD inverse with the reference's fallback chain, DLR helpers.

Replaces gptq._prepare_hinv / _prepare_hessian (converter/gptq.py:91-121),
rounding._invert_hessian (rounding.py:19-34) and dlr.woodbury_inverse /
dlr_to_dense (dlr.py:75-132).
"""

from __future__ import annotations

import warnings

import torch

from . import _native as nat
from ._dev import device_of, f32, round4, workspace
from ._native import NotPositiveDefinite
from .config import DIAG_MEAN_FLOOR

__all__ = ["hessian_pair", "inverse_pair", "invert_dense", "dlr_to_dense", "woodbury_inverse",
           "NotPositiveDefinite"]


def hessian_pair(H: torch.Tensor, rot_size: int, dev: torch.device, rotate: bool = True):
    """2-D Hessian -> rotated (R^T H R) TF32 pair [npad, ld], ld = round4(npad), zero padded."""
    Hd = f32(H, dev)
    n = Hd.shape[0]
    r = rot_size if (rotate and rot_size and rot_size > 1) else 1
    npad = -(-n // r) * r
    ld = round4(npad)
    hi = torch.zeros(npad, ld, device=dev, dtype=torch.float32)
    lo = torch.zeros(npad, ld, device=dev, dtype=torch.float32)
    lib = nat.load()
    st = nat.stream_ptr(dev)
    if r > 1:
        if ld == npad:
            nat.check(lib.ic_rotate_hessian(Hd.data_ptr(), 1, n, n, r, hi.data_ptr(), lo.data_ptr(), npad, st),
                      "rotate_hessian")
        else:
            th = torch.empty(npad, npad, device=dev)
            tl = torch.empty(npad, npad, device=dev)
            nat.check(lib.ic_rotate_hessian(Hd.data_ptr(), 1, n, n, r, th.data_ptr(), tl.data_ptr(), npad, st),
                      "rotate_hessian")
            hi[:, :npad] = th
            lo[:, :npad] = tl
    else:
        nat.check(lib.ic_split_tf32(Hd.data_ptr(), n, n, n, hi.data_ptr(), lo.data_ptr(), ld, st), "split_tf32")
    return hi, lo, npad


def inverse_pair(hi: torch.Tensor, lo: torch.Tensor, n: int, damping: float | None,
                 H_fallback: torch.Tensor | None = None) -> str:
    """In-place (H + damping*mean(diag)*I)^-1 on a TF32 pair; returns the path taken.

    SPD -> the library's tensor-core Cholesky inverse (the reference's
    "cholesky" branch).
    Not positive definite -> torch.linalg.inv on the GPU ("inv"), then pinv
    with the reference's warning ("pinv").  ``H_fallback`` is the undamped fp32
    matrix in the same (rotated) space, needed only for those branches; when
    None the pair is re-read before the attempt.
    """
    dev = hi.device
    ld = hi.shape[1]
    if H_fallback is None:
        H_fallback = (hi[:n, :n] + lo[:n, :n]).clone()
    ws = workspace(nat.load().ic_spd_inverse_workspace_size(n), dev)
    st = nat.load().ic_spd_inverse(hi.data_ptr(), lo.data_ptr(), n, ld, -1.0 if damping is None else float(damping),
                                   ws.data_ptr(), ws.numel(), nat.stream_ptr(dev))
    if st == nat.IC_OK:
        return "cholesky"
    if st != nat.IC_ERR_NOT_PD:
        nat.check(st, "spd_inverse")
    Hd = H_fallback.to(dev, torch.float32)
    Hd = torch.tril(Hd) + torch.tril(Hd, -1).T
    if damping is not None:
        dm = Hd.diagonal().mean().clamp(min=DIAG_MEAN_FLOOR)
        Hd = Hd + damping * dm * torch.eye(n, device=dev, dtype=torch.float32)
    inv, info = torch.linalg.inv_ex(Hd)
    path = "inv"
    if int(info.item()) != 0 or not torch.isfinite(inv).all():
        warnings.warn("Hessian is singular/ill-conditioned; falling back to pseudoinverse. "
                      "This may produce inaccurate quantization scales.", stacklevel=3)
        inv = torch.linalg.pinv(Hd)
        path = "pinv"
    nat.check(nat.load().ic_split_tf32(inv.contiguous().data_ptr(), n, n, n, hi.data_ptr(), lo.data_ptr(), ld,
                                       nat.stream_ptr(dev)), "split_tf32")
    return path


def invert_dense(H: torch.Tensor, damping: float | None = None):
    """fp32 inverse of a dense matrix with the reference's chain; returns (Hinv, path)."""
    dev = device_of(H)
    hi, lo, n = hessian_pair(H, 0, dev, rotate=False)
    path = inverse_pair(hi, lo, n, damping, H_fallback=f32(H, dev))
    out = (hi[:n, :n] + lo[:n, :n])
    return (out if H.is_cuda else out.to(H.device)), path


def dlr_to_dense(D: torch.Tensor, U: torch.Tensor) -> torch.Tensor:
    """diag(D) + U U^T (dlr.py:127-132), the product on the tensor cores (3xTF32)."""
    dev = device_of(D, U)
    Ud = f32(U, dev)
    n, r = Ud.shape
    from ._dev import split
    uh, ul = split(Ud)
    out = torch.empty(n, round4(n), device=dev, dtype=torch.float32)
    nat.check(nat.load().ic_gemm_tn(n, n, r, 1.0, uh.data_ptr(), ul.data_ptr(), uh.shape[1], uh.data_ptr(),
                                    ul.data_ptr(), uh.shape[1], 0.0, None, None, out.shape[1], out.data_ptr(), None,
                                    out.shape[1], 3, nat.stream_ptr(dev)), "gemm")
    out = out[:, :n].contiguous()
    out.diagonal().add_(f32(D, dev))
    return out if D.is_cuda else out.to(D.device)


def _abt(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """A @ B^T in 3xTF32 on the tensor cores (ic_gemm_tn), fp32 [rows(A), rows(B)]."""
    from ._dev import split
    ah, al = split(A)
    bh, bl = split(B)
    m, n, k = A.shape[0], B.shape[0], A.shape[1]
    ld = round4(n)
    out = torch.empty(m, ld, device=A.device, dtype=torch.float32)
    if m and n:
        nat.check(nat.load().ic_gemm_tn(m, n, k, 1.0, ah.data_ptr(), al.data_ptr(), ah.shape[1], bh.data_ptr(),
                                        bl.data_ptr(), bh.shape[1], 0.0, None, None, ld, out.data_ptr(), None, ld, 3,
                                        nat.stream_ptr(A.device)), "gemm")
    return out[:, :n]


def woodbury_inverse(D, U, damping: float = 0.0, device=None) -> torch.Tensor:
    """(diag(D) + U U^T + lambda*I)^-1 by the Woodbury identity (dlr.py:75-124), on the GPU:
    Dinv - Z (I + U^T Z)^-1 Z^T with Z = Dinv U; the three products on the tensor
    cores (3xTF32), the r x r inverse with the library's SPD inverse."""
    dev = device_of(D, U)
    D = f32(D, dev)
    U = f32(U, dev)
    r = U.shape[1]
    if damping > 0.0:
        dm = (D + (U * U).sum(dim=1)).mean().clamp(min=DIAG_MEAN_FLOOR)
        D = D + damping * dm
    Dinv = 1.0 / D.clamp(min=1e-12)
    Z = (Dinv.unsqueeze(1) * U).contiguous()
    Mm = _abt(U.T.contiguous(), Z.T.contiguous())
    Mm.diagonal().add_(1.0)
    Minv, _ = invert_dense(Mm.contiguous(), None)
    Y = _abt(Z, Minv.contiguous())          # Z Minv (Minv symmetric)
    out = _abt(Y.contiguous(), Z).neg_()    # -(Z Minv) Z^T
    out.diagonal().add_(Dinv)
    out = out.contiguous()
    return out if device is None else out.to(device)
