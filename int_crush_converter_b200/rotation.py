"""ConvRot group Hadamard rotation on the GPU (mirrors converter/rotation.py).

``rotate_weights`` / ``rotate_activations`` / ``rotate_hessian`` keep the
reference's signatures, padding and return shapes, but run the butterfly
kernels of ``libintcrush_b200`` instead of dense ``x @ H.T`` products.  The
explicit Hadamard matrices remain available for inspection and tests.
"""

from __future__ import annotations

import math

import torch

from . import _native as nat
from ._dev import back, device_of, f32

_hadamard_cache: dict[tuple[int, str, str], torch.Tensor] = {}


def _is_power_of_four(n: int) -> bool:  # rotation.py:16-19
    return n >= 4 and (n & (n - 1)) == 0 and (n & 0x55555555) == n


def _is_power_of_two(n: int) -> bool:  # rotation.py:22-23
    return n > 0 and (n & (n - 1)) == 0


def make_hadamard_sylvester(n: int, dtype: torch.dtype = torch.float16, device: str = "cpu") -> torch.Tensor:
    """Normalised Sylvester Hadamard of size n (rotation.py:26-36)."""
    if not _is_power_of_two(n):
        raise ValueError(f"n must be a power of 2, got {n}")
    H = torch.tensor([[1.0]], dtype=dtype, device=device)
    base = torch.tensor([[1.0, 1.0], [1.0, -1.0]], dtype=dtype, device=device)
    while H.shape[0] < n:
        H = torch.kron(base, H)
    return H * (1.0 / math.sqrt(n))


def make_hadamard_regular(n: int, dtype: torch.dtype = torch.float16, device: str = "cpu") -> torch.Tensor:
    """Regular Hadamard H4^{kron k} / 2^k of size n = 4^k (rotation.py:39-62)."""
    if not _is_power_of_four(n):
        raise ValueError(f"Regular Hadamard requires power of 4, got {n}. Use rot_size=16/64/256.")
    H4 = torch.tensor([[1.0, 1.0, 1.0, -1.0], [1.0, 1.0, -1.0, 1.0], [1.0, -1.0, 1.0, 1.0],
                       [-1.0, 1.0, 1.0, 1.0]], dtype=dtype, device=device) / 2.0
    H = H4
    while H.shape[0] < n:
        H = torch.kron(H, H4)
    return H


def get_hadamard(size: int, dtype: torch.dtype = torch.float16, device: str = "cpu") -> torch.Tensor:
    key = (size, str(dtype), str(device))
    if key not in _hadamard_cache:
        _hadamard_cache[key] = make_hadamard_regular(size, dtype=dtype, device=device)
    return _hadamard_cache[key]


def clear_hadamard_cache() -> None:
    _hadamard_cache.clear()


_DT = {torch.float32: nat.IC_F32, torch.float16: nat.IC_F16, torch.bfloat16: nat.IC_BF16}


def _rotate_rows(x2d: torch.Tensor, rot_size: int, dev: torch.device) -> torch.Tensor:
    if x2d.dtype not in _DT:
        x2d = x2d.float()
    x2d = x2d.to(dev)
    if x2d.stride(-1) != 1 or x2d.stride(0) < x2d.shape[1]:
        x2d = x2d.contiguous()
    M, N = x2d.shape
    npad = -(-N // rot_size) * rot_size
    out = torch.empty(M, npad, device=dev, dtype=torch.float32)
    nat.check(nat.load().ic_rotate_weights(x2d.data_ptr(), _DT[x2d.dtype], M, N, max(x2d.stride(0), N), rot_size,
                                           out.data_ptr(), npad, nat.stream_ptr(dev)), "rotate_weights")
    return out


def rotate_weights(W: torch.Tensor, rot_size: int) -> torch.Tensor:
    """Group-wise Hadamard along in_features (rotation.py:95-125).

    Returns [out, in_padded] (zero padding up to a multiple of ``rot_size``) on
    W's device, computed in fp32; fp16/bf16 inputs come back in their dtype.
    """
    if W.dim() != 2:
        raise ValueError(f"Expected 2D tensor, got {W.dim()}D")
    if not _is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be a power of 2, got {rot_size}")
    dev = device_of(W)
    out = _rotate_rows(W, rot_size, dev)
    if W.dtype in (torch.float16, torch.bfloat16):
        out = out.to(W.dtype)
    return back(out, W)


def rotate_activations(x: torch.Tensor, rot_size: int) -> torch.Tensor:
    """Group-wise Hadamard of [..., in] activations (rotation.py:128-153)."""
    if not _is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be a power of 2, got {rot_size}")
    dev = device_of(x)
    lead = x.shape[:-1]
    out = _rotate_rows(x.reshape(-1, x.shape[-1]), rot_size, dev)
    if x.dtype in (torch.float16, torch.bfloat16):
        out = out.to(x.dtype)
    return back(out.reshape(*lead, out.shape[-1]), x)


def rotate_hessian(H, rot_size: int):
    """H_rot = R^T H R (rotation.py:156-234) for 2-D [in,in], 3-D [nb,bs,bs] or DLR dict."""
    if not _is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be a power of 2, got {rot_size}")
    if isinstance(H, dict) and H.get("format") == "dlr":
        from .hessian import dlr_to_dense
        H = dlr_to_dense(H["D"], H["U"])
    like = H
    dev = device_of(H)
    Hd = f32(H, dev)
    lib = nat.load()
    if Hd.dim() == 2:
        n = Hd.shape[0]
        if Hd.shape[0] != Hd.shape[1]:
            raise ValueError(f"Expected square Hessian, got {tuple(Hd.shape)}")
        npad = -(-n // rot_size) * rot_size
        out = torch.empty(npad, npad, device=dev, dtype=torch.float32)
        nat.check(lib.ic_rotate_hessian(Hd.data_ptr(), 1, n, n, rot_size, out.data_ptr(), None, npad,
                                        nat.stream_ptr(dev)), "rotate_hessian")
        return back(out, like)
    if Hd.dim() == 3:
        nb, bs, bs2 = Hd.shape
        if bs != bs2:
            raise ValueError(f"Expected square blocks, got block shape ({bs}, {bs2})")
        if bs % rot_size != 0:
            raise ValueError(f"Block size {bs} is not divisible by rot_size {rot_size}")
        out = torch.empty(nb, bs, bs, device=dev, dtype=torch.float32)
        nat.check(lib.ic_rotate_hessian(Hd.data_ptr(), nb, bs, bs, rot_size, out.data_ptr(), None, bs,
                                        nat.stream_ptr(dev)), "rotate_hessian")
        return back(out, like)
    raise ValueError(f"Expected 2D or 3D Hessian, got {Hd.dim()}D")
