"""numpy/scipy restatement of the reference's per-layer quantization path.

TEST INFRASTRUCTURE ONLY -- the checker for the CUDA kernels and the timed CPU
baseline of ``bench.py``.  The product package never imports this module.

Every function restates one function of ThunderFun/int_crush_converter
(``converter/<file>.py:<lines>``) in fp32 numpy arithmetic, operation by
operation, so that elementwise results are bit-identical to the reference's
torch-CPU path.  Reductions (sums, means) and BLAS/LAPACK calls (matmul,
Cholesky, inverse) follow the same algorithm but not necessarily the same
summation order as torch's CPU kernels; the golden fixtures in
``tests/golden`` pin how close that is.

Third-party arithmetic the reference delegates to torch (not under the
reference tree; torch 2.11.0 where the fixtures were generated, ``pyproject.toml`` pins
only ``torch>=2.1``):
  * ``torch.linalg.cholesky`` + ``torch.cholesky_inverse`` = LAPACK
    ``spotrf`` + ``spotri``: restated with ``scipy.linalg.lapack`` (same
    LAPACK routines, OpenBLAS build here vs MKL in torch).
  * ``torch.linspace`` (fp32): its rounding depends on torch's CPU vector
    width, so the oracle takes the table from the same call.
  * ``Tensor.round()`` = round-half-to-even = ``np.rint``.
"""

from __future__ import annotations

import math

import numpy as np
import scipy.linalg.lapack as lapack

f32 = np.float32

# converter/config.py:32-92 (constants, same values)
INT4_SCALE_DIVISOR = 7.0
INT8_SCALE_DIVISOR = 127.0
SCALE_MIN = 1e-5
SCALE_MAX = 65500.0
SCALE_FLOOR = 1e-8
DIAG_MEAN_FLOOR = 1e-6
DENOMINATOR_FLOOR = 1e-8
HINV_DIAG_FLOOR = 1e-8
ERR_CLAMP_RANGE = 100.0
SANITIZE_FLOOR = 1e-8
SANITIZE_CEIL = 1e30
SIGN_FLIP_THRESHOLD = 1e-8
CONVERGENCE_EPS = 1e-10
CONVERGENCE_IMPROVEMENT_THRESHOLD = 1e-4
SCALE_FLOOR_MULTIPLIER = 0.1
SCALE_CEIL_MULTIPLIER = 10.0
ABS_SCALE_FLOOR = 1e-8


class INT4PackingError(ValueError):
    """converter/packing.py:13-14."""


def _c(x, lo=None, hi=None):
    """torch.clamp on an fp32 array (NaN propagates, bounds cast to the dtype)."""
    x = np.asarray(x)
    if lo is not None:
        x = np.maximum(x, x.dtype.type(lo))
    if hi is not None:
        x = np.minimum(x, x.dtype.type(hi))
    return x


# ---------------------------------------------------------------------------
# rotation.py
# ---------------------------------------------------------------------------

def _is_power_of_four(n: int) -> bool:  # rotation.py:16-19
    return n >= 4 and (n & (n - 1)) == 0 and (n & 0x55555555) == n


def _is_power_of_two(n: int) -> bool:  # rotation.py:22-23
    return n > 0 and (n & (n - 1)) == 0


def make_hadamard_sylvester(n: int) -> np.ndarray:  # rotation.py:26-36
    if not _is_power_of_two(n):
        raise ValueError(f"n must be a power of 2, got {n}")
    H = np.array([[1.0]], dtype=f32)
    base = np.array([[1.0, 1.0], [1.0, -1.0]], dtype=f32)
    while H.shape[0] < n:
        H = np.kron(base, H)
    return (H * f32(1.0 / math.sqrt(n))).astype(f32)


def make_hadamard_regular(n: int) -> np.ndarray:  # rotation.py:39-62
    if not _is_power_of_four(n):
        raise ValueError(f"Regular Hadamard requires power of 4, got {n}")
    H4 = (np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]],
                   dtype=f32) / f32(2.0)).astype(f32)
    H = H4
    while H.shape[0] < n:
        H = np.kron(H, H4).astype(f32)
    return H


def _hadamard(rot_size: int) -> np.ndarray:  # rotation.py:82-92
    if _is_power_of_four(rot_size):
        return make_hadamard_regular(rot_size)
    return make_hadamard_sylvester(rot_size)


def rotate_weights(W: np.ndarray, rot_size: int) -> np.ndarray:  # rotation.py:95-125
    W = np.asarray(W, dtype=f32)
    if W.ndim != 2:
        raise ValueError(f"Expected 2D tensor, got {W.ndim}D")
    if not _is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be a power of 2, got {rot_size}")
    M, N = W.shape
    if N % rot_size:
        W = np.pad(W, ((0, 0), (0, rot_size - N % rot_size)))
    H = _hadamard(rot_size)
    G = W.shape[1] // rot_size
    return (W.reshape(M, G, rot_size) @ H.T).reshape(M, -1).astype(f32)


def rotate_activations(x: np.ndarray, rot_size: int) -> np.ndarray:  # rotation.py:128-153
    """Group-wise Hadamard of the last dimension (zero padded), any leading dims."""
    x = np.asarray(x, dtype=f32)
    if not _is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be a power of 2, got {rot_size}")
    n = x.shape[-1]
    if n % rot_size:
        x = np.pad(x, [(0, 0)] * (x.ndim - 1) + [(0, rot_size - n % rot_size)])
    lead = x.shape[:-1]
    flat = x.reshape(-1, x.shape[-1] // rot_size, rot_size)
    return (flat @ _hadamard(rot_size).T).reshape(*lead, -1).astype(f32)


def rotate_hessian(H: np.ndarray, rot_size: int) -> np.ndarray:  # rotation.py:156-248
    if not _is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be a power of 2, got {rot_size}")
    H = np.asarray(H, dtype=f32)
    R = _hadamard(rot_size)
    if H.ndim == 2:
        n = H.shape[0]
        if H.shape[0] != H.shape[1]:
            raise ValueError(f"Expected square Hessian, got {H.shape}")
        if n % rot_size:
            p = rot_size - n % rot_size
            H = np.pad(H, ((0, p), (0, p)))
            n = H.shape[0]
        nb = n // rot_size
        blocks = H.reshape(nb, rot_size, nb, rot_size).transpose(0, 2, 1, 3)
        blocks = R.T @ blocks @ R  # einsum("kp,nkl,le->npe") per block
        return blocks.transpose(0, 2, 1, 3).reshape(n, n).astype(f32)
    if H.ndim == 3:
        nb, bs, bs2 = H.shape
        if bs != bs2:
            raise ValueError("Expected square blocks")
        if bs % rot_size:
            raise ValueError(f"Block size {bs} is not divisible by rot_size {rot_size}")
        ns = bs // rot_size
        sub = H.reshape(nb, ns, rot_size, ns, rot_size).transpose(0, 1, 3, 2, 4)
        sub = R.T @ sub @ R
        return sub.transpose(0, 1, 3, 2, 4).reshape(nb, bs, bs).astype(f32)
    raise ValueError(f"Expected 2D or 3D Hessian, got {H.ndim}D")


# ---------------------------------------------------------------------------
# rounding.py
# ---------------------------------------------------------------------------

def rhaz(x: np.ndarray) -> np.ndarray:  # rounding.py:106-112
    x = np.asarray(x)
    return np.where(x >= 0, np.floor(x + x.dtype.type(0.5)), np.ceil(x - x.dtype.type(0.5)))


def invert_hessian(H: np.ndarray) -> tuple[np.ndarray, str]:  # rounding.py:19-34
    """Cholesky -> cholesky_inverse, else inv, else pinv.  Returns (Hinv, path)."""
    H = np.asarray(H, dtype=f32)
    c, info = lapack.spotrf(H, lower=1, clean=1)
    if info == 0:
        inv, info2 = lapack.spotri(c, lower=1)
        if info2 == 0:
            inv = np.tril(inv) + np.tril(inv, -1).T
            return inv.astype(f32), "cholesky"
    try:
        return np.linalg.inv(H).astype(f32), "inv"
    except np.linalg.LinAlgError:
        return np.linalg.pinv(H).astype(f32), "pinv"


def damp(H: np.ndarray, damping: float) -> np.ndarray:  # gptq.py:113-121 (damping part)
    H = np.asarray(H, dtype=f32)
    diag_mean = _c(np.mean(np.diagonal(H), dtype=f32), DIAG_MEAN_FLOOR)
    return (H + f32(damping) * diag_mean * np.eye(H.shape[0], dtype=f32)).astype(f32)


def gptq_block(W_work, Q, row_scales, H_inv, col_start, col_end, block_size,
               clamp_min, clamp_max, row_zp=None):  # rounding.py:37-103
    """In-place GPTQ column loop over columns [col_start, col_end)."""
    M = W_work.shape[0]
    n_cols = col_end - col_start
    s = row_scales.reshape(-1).astype(f32)
    zp = None if row_zp is None else row_zp.reshape(-1).astype(f32)
    for blk_start in range(0, n_cols, block_size):
        blk_end = min(blk_start + block_size, n_cols)
        E = np.zeros((M, blk_end - blk_start), dtype=f32)
        for jo in range(blk_end - blk_start):
            jl = blk_start + jo
            jg = col_start + jl
            col = W_work[:, jg].copy()
            raw = col / s + zp if zp is not None else col / s
            q = _c(rhaz(raw), clamp_min, clamp_max)
            Q[:, jg] = q.astype(np.int8)
            deq = (q - zp) * s if zp is not None else q * s
            with np.errstate(divide="ignore", invalid="ignore"):
                err = (col - deq) / H_inv[jl, jl]
            err = _c(err, -ERR_CLAMP_RANGE, ERR_CLAMP_RANGE)
            err = np.nan_to_num(err, nan=0.0, posinf=ERR_CLAMP_RANGE, neginf=-ERR_CLAMP_RANGE).astype(f32)
            E[:, jo] = err
            if jo < blk_end - blk_start - 1:
                W_work[:, jg + 1:col_start + blk_end] -= err[:, None] * H_inv[jl, jl + 1:blk_end][None, :]
        if blk_end < n_cols:
            W_work[:, col_start + blk_end:col_end] -= E @ H_inv[blk_start:blk_end, blk_end:n_cols]


# ---------------------------------------------------------------------------
# scales.py
# ---------------------------------------------------------------------------

def _pad_to_group(W, gs):  # scales.py:16-22
    if W.shape[1] % gs:
        W = np.pad(W, ((0, 0), (0, gs - W.shape[1] % gs)))
    return W


def _search_clipping_ratio(ratios, fn):  # scales.py:25-59
    best_s = best_zp = best_mse = None
    for r in ratios:
        s, zp, mse = fn(r)
        if best_s is None:
            best_s, best_zp, best_mse = s, zp, mse
        else:
            better = mse < best_mse
            best_s = np.where(better, s, best_s)
            if zp is not None:
                best_zp = np.where(better, zp, best_zp)
            best_mse = np.where(better, mse, best_mse)
    return best_s, best_zp


def calculate_scales(W, group_size=128, clipping_ratios=None):  # scales.py:62-99
    W = np.asarray(W, dtype=f32)
    if W.ndim != 2:
        raise ValueError(f"Expected 2D tensor, got {W.ndim}D")
    if clipping_ratios is not None and len(clipping_ratios) == 0:
        clipping_ratios = None
    Wp = _pad_to_group(W, group_size)
    M, N = Wp.shape
    Wg = Wp.reshape(M, N // group_size, group_size)
    mx = np.abs(Wg).max(axis=2)
    if clipping_ratios is None:
        return _c(mx / f32(INT4_SCALE_DIVISOR), SCALE_MIN, SCALE_MAX).astype(np.float16)

    def fn(r):
        cs = _c(mx * f32(r) / f32(INT4_SCALE_DIVISOR), SCALE_MIN, SCALE_MAX)
        q = _c(np.rint(Wg / cs[:, :, None]), -8, 7)
        mse = np.mean((Wg - q * cs[:, :, None]) ** 2, axis=2, dtype=f32)
        return cs, None, mse

    best, _ = _search_clipping_ratio(clipping_ratios, fn)
    return best.astype(np.float16)


def quantize_weights(W, scales, group_size=128):  # scales.py:102-123
    W = np.asarray(W, dtype=f32)
    M = W.shape[0]
    W = _pad_to_group(W, group_size)
    N = W.shape[1]
    Wg = W.reshape(M, N // group_size, group_size)
    y = Wg / np.asarray(scales).astype(f32)[:, :, None]
    return _c(rhaz(y), -8, 7).reshape(M, N).astype(np.int8)


def calculate_scales_int8(W, clipping_ratios=None):  # scales.py:126-160
    W = np.asarray(W, dtype=f32)
    if W.ndim != 2:
        raise ValueError(f"Expected 2D tensor, got {W.ndim}D")
    if clipping_ratios is not None and len(clipping_ratios) == 0:
        clipping_ratios = None
    mx = np.abs(W).max(axis=1, keepdims=True)
    if clipping_ratios is None:
        return _c(mx / f32(INT8_SCALE_DIVISOR), SCALE_MIN, SCALE_MAX).astype(np.float16)

    def fn(r):
        cs = _c(mx * f32(r) / f32(INT8_SCALE_DIVISOR), SCALE_MIN, SCALE_MAX)
        q = _c(np.rint(W / cs), -128, 127)
        mse = np.mean((W - q * cs) ** 2, axis=1, keepdims=True, dtype=f32)
        return cs, None, mse

    best, _ = _search_clipping_ratio(clipping_ratios, fn)
    return best.astype(np.float16)


def quantize_weights_int8(W, scales):  # scales.py:163-178
    W = np.asarray(W, dtype=f32)
    return _c(rhaz(W / np.asarray(scales).astype(f32)), -128, 127).astype(np.int8)


def fix_asymmetric_scale(scales, w_min, w_max, qmin, qmax):  # scales.py:184-229
    spread = f32(qmax - qmin)
    zp_raw = f32(qmin) - rhaz(w_min / scales)
    lo = zp_raw < qmin
    hi = zp_raw > qmax
    if lo.any():
        fix = _c(w_max / spread, SCALE_MIN, SCALE_MAX)
        scales = np.maximum(scales, np.where(lo, fix, scales))
    if hi.any():
        fix = _c(-w_min / spread, SCALE_MIN, SCALE_MAX)
        scales = np.maximum(scales, np.where(hi, fix, scales))
    return scales


def calculate_scales_asymmetric(W, group_size=128, clipping_ratios=None):  # scales.py:232-282
    W = np.asarray(W, dtype=f32)
    if W.ndim != 2:
        raise ValueError(f"Expected 2D tensor, got {W.ndim}D")
    if clipping_ratios is not None and len(clipping_ratios) == 0:
        clipping_ratios = None
    Wp = _pad_to_group(W, group_size)
    M, N = Wp.shape
    Wg = Wp.reshape(M, N // group_size, group_size)
    wmin = Wg.min(axis=2)
    wmax = Wg.max(axis=2)
    if clipping_ratios is None:
        s = _c((wmax - wmin) / f32(15.0), SCALE_MIN, SCALE_MAX)
        s = fix_asymmetric_scale(s, wmin, wmax, -8, 7)
        zp = _c(f32(-8) - rhaz(wmin / s), -8, 7)
        zp = np.where((wmin == 0) & (wmax == 0), f32(0), zp)
        return s.astype(np.float16), zp.astype(np.int8)

    def fn(r):
        cs = _c((wmax - wmin) * f32(r) / f32(15.0), SCALE_MIN, SCALE_MAX)
        cs = fix_asymmetric_scale(cs, wmin, wmax, -8, 7)
        czp = _c(f32(-8) - rhaz(wmin / cs), -8, 7)
        q = _c(np.rint(Wg / cs[:, :, None] + czp[:, :, None]), -8, 7)
        deq = (q - czp[:, :, None]) * cs[:, :, None]
        mse = np.mean((Wg - deq) ** 2, axis=2, dtype=f32)
        return cs, czp, mse

    s, zp = _search_clipping_ratio(clipping_ratios, fn)
    return s.astype(np.float16), zp.astype(np.int8)


def quantize_weights_asymmetric(W, scales, zero_points, group_size=128):  # scales.py:285-313
    W = np.asarray(W, dtype=f32)
    M = W.shape[0]
    W = _pad_to_group(W, group_size)
    N = W.shape[1]
    Wg = W.reshape(M, N // group_size, group_size)
    y = Wg / np.asarray(scales).astype(f32)[:, :, None] + np.asarray(zero_points).astype(f32)[:, :, None]
    return _c(rhaz(y), -8, 7).reshape(M, N).astype(np.int8)


def calculate_scales_int8_asymmetric(W, clipping_ratios=None):  # scales.py:316-361
    W = np.asarray(W, dtype=f32)
    if W.ndim != 2:
        raise ValueError(f"Expected 2D tensor, got {W.ndim}D")
    if clipping_ratios is not None and len(clipping_ratios) == 0:
        clipping_ratios = None
    wmin = W.min(axis=1, keepdims=True)
    wmax = W.max(axis=1, keepdims=True)
    if clipping_ratios is None:
        s = _c((wmax - wmin) / f32(255.0), SCALE_MIN, SCALE_MAX)
        s = fix_asymmetric_scale(s, wmin, wmax, -128, 127)
        zp = _c(f32(-128) - rhaz(wmin / s), -128, 127)
        return s.astype(np.float16), zp.astype(np.int8)

    def fn(r):
        cs = _c((wmax - wmin) * f32(r) / f32(255.0), SCALE_MIN, SCALE_MAX)
        cs = fix_asymmetric_scale(cs, wmin, wmax, -128, 127)
        czp = _c(f32(-128) - rhaz(wmin / cs), -128, 127)
        q = _c(np.rint(W / cs + czp), -128, 127)
        mse = np.mean((W - (q - czp) * cs) ** 2, axis=1, keepdims=True, dtype=f32)
        return cs, czp, mse

    s, zp = _search_clipping_ratio(clipping_ratios, fn)
    return s.astype(np.float16), zp.astype(np.int8)


def quantize_weights_int8_asymmetric(W, scales, zero_points):  # scales.py:364-384
    W = np.asarray(W, dtype=f32)
    y = W / np.asarray(scales).astype(f32) + np.asarray(zero_points).astype(f32)
    return _c(rhaz(y), -128, 127).astype(np.int8)


# ---------------------------------------------------------------------------
# packing.py
# ---------------------------------------------------------------------------

def validate_int4_range(v):  # packing.py:17-27
    v = np.asarray(v)
    if v.size == 0:
        return
    if not np.isfinite(v.astype(np.float64)).all():
        raise INT4PackingError("Tensor contains NaN or Inf values")
    if v.min() < -8 or v.max() > 7:
        raise INT4PackingError(f"Values must be in [-8, 7], got [{v.min()}, {v.max()}]")


def pack_int4(v):  # packing.py:30-46
    validate_int4_range(v)
    v = np.asarray(v).astype(np.int8)
    if v.shape[-1] % 2:
        v = np.concatenate([v, np.zeros(v.shape[:-1] + (1,), np.int8)], axis=-1)
    u = np.where(v < 0, 16 + v.astype(np.int16), v.astype(np.int16)).astype(np.uint8)
    return (u[..., 0::2] | (u[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(p, K):  # packing.py:49-66
    p = np.asarray(p, dtype=np.uint8)
    lo = (p & 0x0F).astype(np.int8)
    hi = ((p >> 4) & 0x0F).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo).astype(np.int8)
    hi = np.where(hi >= 8, hi - 16, hi).astype(np.int8)
    out = np.zeros(p.shape[:-1] + (p.shape[-1] * 2,), np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out[..., :K]


# ---------------------------------------------------------------------------
# gptq.py
# ---------------------------------------------------------------------------

def gptq_row_params(W, int_bits=4, asymmetric=False):  # gptq.py:254-317 (non-PiSO branch)
    """Per-row fp32 scales and (int8 or None) zero-points used by the loop."""
    W = np.asarray(W, dtype=f32)
    if int_bits == 4 or asymmetric:
        qmin, qmax, spread = (-8, 7, 15.0) if int_bits == 4 else (-128, 127, 255.0)
        wmin = W.min(axis=1, keepdims=True)
        wmax = W.max(axis=1, keepdims=True)
        s = _c((wmax - wmin) / f32(spread), SCALE_MIN, SCALE_MAX)
        zp_raw = f32(qmin) - rhaz(wmin / s)
        lo = zp_raw < qmin
        hi = zp_raw > qmax
        if lo.any():
            s = np.maximum(s, np.where(lo, _c(wmax / f32(spread), SCALE_MIN, SCALE_MAX), s))
        if hi.any():
            s = np.maximum(s, np.where(hi, _c(-wmin / f32(spread), SCALE_MIN, SCALE_MAX), s))
        zp = _c(f32(qmin) - rhaz(wmin / s), qmin, qmax)
        zp = np.where((wmin == 0) & (wmax == 0), f32(0), zp)
        return s.astype(f32), zp.astype(np.int8)
    s = _c(np.abs(W).max(axis=1, keepdims=True) / f32(INT8_SCALE_DIVISOR), SCALE_MIN, SCALE_MAX)
    return s.astype(f32), None


def gptq_row_params_piso(W, piso_scales, piso_zero_points, int_bits, asymmetric):  # gptq.py:210-252
    W = np.asarray(W, dtype=f32)
    s = _c(np.asarray(piso_scales, dtype=f32), SCALE_MIN, SCALE_MAX)
    wmin = W.min(axis=1, keepdims=True)
    wmax = W.max(axis=1, keepdims=True)
    zero_rows = (wmin == 0) & (wmax == 0)
    if int_bits == 4:
        if piso_zero_points is not None:
            zp = _c(np.asarray(piso_zero_points).astype(f32), -8, 7)
        else:
            s = fix_asymmetric_scale(s, wmin, wmax, -8, 7)
            zp = _c(f32(-8) - rhaz(wmin / s), -8, 7)
        zp = np.where(zero_rows, f32(0), zp)
        return s, zp.astype(np.int8)
    if asymmetric:
        s = fix_asymmetric_scale(s, wmin, wmax, -128, 127)
        zp = _c(f32(-128) - rhaz(wmin / s), -128, 127)
        zp = np.where(zero_rows, f32(0), zp)
        return s, zp.astype(np.int8)
    return s, None


def woodbury_inverse(D, U, damping=0.0):  # dlr.py:75-124
    D = np.asarray(D, f32)
    U = np.asarray(U, f32)
    r = U.shape[1]
    if damping > 0.0:
        dm = _c(np.mean(D + (U * U).sum(axis=1, dtype=f32), dtype=f32), DIAG_MEAN_FLOOR)
        Dd = D + f32(damping) * dm
    else:
        Dd = D
    Dinv = f32(1.0) / _c(Dd, 1e-12)
    Z = Dinv[:, None] * U
    Mm = np.eye(r, dtype=f32) + U.T @ Z
    Minv, _ = invert_hessian(Mm)
    return (np.diag(Dinv) - Z @ Minv @ Z.T).astype(f32)


def _result_stats(W, Q, s, zp):  # gptq.py:398-405
    deq = Q.astype(f32) * s if zp is None else (Q.astype(f32) - zp.astype(f32)) * s
    d = W - deq
    return float(np.mean(d.astype(np.float64) ** 2)), float(np.abs(d).max()) if d.size else 0.0


def prepare_hessian_cholesky(H, damping):  # gptq.py:91-110 (hessian_method="cholesky")
    """Upper factor L^T of chol(H_damped^-1); the full inverse when that Cholesky fails."""
    Hinv, p = invert_hessian(damp(H, damping))
    c, info = lapack.spotrf(Hinv, lower=1, clean=1)
    if info != 0:
        return Hinv, p
    return np.ascontiguousarray(c.T).astype(f32), p


def gptq_quantize_layer(W, hessian, block_size=128, damping=0.01, int_bits=4, asymmetric=False,
                        piso_scales=None, piso_zero_points=None, hessian_method="hinv"):  # gptq.py:137-417
    """Returns dict(quantized_W, scales(fp16), scales_f32, zero_points, mse, max_err, hinv_path).

    ``hessian_method`` "hinv" uses the damped inverse (gptq.py:113-121), "cholesky"
    its upper Cholesky factor (gptq.py:91-110); DLR dicts always use Woodbury."""
    if int_bits not in (4, 8):
        raise ValueError(f"int_bits must be 4 or 8, got {int_bits}")
    W = np.asarray(W, dtype=f32)
    if W.ndim != 2:
        raise ValueError(f"Expected 2D weight tensor, got {W.ndim}D")
    M, N = W.shape
    qmin, qmax = (-128, 127) if int_bits == 8 else (-8, 7)
    if piso_scales is not None and np.asarray(piso_scales).shape == (M, 1):
        s, zp = gptq_row_params_piso(W, piso_scales, piso_zero_points, int_bits, asymmetric)
    else:
        s, zp = gptq_row_params(W, int_bits, asymmetric)
    Q = np.zeros((M, N), np.int8)
    Ww = W.copy()
    paths = []
    if hessian_method == "cholesky":
        def prep(Hb):
            return prepare_hessian_cholesky(Hb, damping)
    elif hessian_method == "hinv":
        def prep(Hb):
            return invert_hessian(damp(Hb, damping))
    else:
        raise ValueError(f"hessian_method must be one of ['hinv', 'cholesky'], got '{hessian_method}'")
    if isinstance(hessian, dict):
        Hinv = woodbury_inverse(hessian["D"], hessian["U"], damping)
        gptq_block(Ww, Q, s, Hinv, 0, N, block_size, qmin, qmax, zp)
        paths.append("woodbury")
    else:
        hessian = np.asarray(hessian, dtype=f32)
        if hessian.ndim == 3:
            nb, bs, _ = hessian.shape
            for bi in range(nb):
                c0 = bi * bs
                c1 = min(c0 + bs, N)
                Hinv, p = prep(hessian[bi, :c1 - c0, :c1 - c0])
                paths.append(p)
                gptq_block(Ww, Q, s, Hinv, c0, c1, block_size, qmin, qmax, zp)
        elif hessian.ndim == 2:
            if hessian.shape != (N, N):
                raise ValueError(f"Hessian shape {hessian.shape} != ({N}, {N})")
            Hinv, p = prep(hessian)
            paths.append(p)
            gptq_block(Ww, Q, s, Hinv, 0, N, block_size, qmin, qmax, zp)
        else:
            raise ValueError("Expected 2D tensor, 3D tensor, or DLR dict Hessian")
    mse, max_err = _result_stats(W, Q, s, zp)
    return dict(quantized_W=Q, scales=s.astype(np.float16), scales_f32=s, zero_points=zp,
                mse=mse, max_err=max_err, hinv_path=paths)


def gptq_quantize_layer_rtn(W, int_bits=4, asymmetric=False, clipping_ratios=None,
                            piso_scales=None, piso_zero_points=None):  # gptq.py:420-533
    if int_bits not in (4, 8):
        raise ValueError(f"int_bits must be 4 or 8, got {int_bits}")
    W = np.asarray(W, dtype=f32)
    M, N = W.shape
    method = "rtn"
    if piso_scales is not None and int_bits == 8 and not asymmetric and np.asarray(piso_scales).shape == (M, 1):
        s = _c(np.asarray(piso_scales, f32), SCALE_MIN, SCALE_MAX).astype(np.float16)
        Q = quantize_weights_int8(W, s)
        zp = None
        method = "rtn_piso"
    elif piso_scales is not None and int_bits == 4 and np.asarray(piso_scales).shape == (M, 1):
        s = _c(np.asarray(piso_scales, f32), SCALE_MIN, SCALE_MAX).astype(np.float16)
        if piso_zero_points is not None:
            zp = np.asarray(piso_zero_points).astype(np.int8)
        else:
            _, zp = calculate_scales_asymmetric(W, N, clipping_ratios)
        Q = quantize_weights_asymmetric(W, s, zp, N)
        method = "rtn_piso"
    elif asymmetric:
        if int_bits == 8:
            s, zp = calculate_scales_int8_asymmetric(W, clipping_ratios)
            Q = quantize_weights_int8_asymmetric(W, s, zp)
        else:
            s, zp = calculate_scales_asymmetric(W, N, clipping_ratios)
            Q = quantize_weights_asymmetric(W, s, zp, N)
    else:
        zp = None
        if int_bits == 8:
            s = calculate_scales_int8(W, clipping_ratios)
            Q = quantize_weights_int8(W, s)
        else:
            s = calculate_scales(W, N, clipping_ratios)
            Q = quantize_weights(W, s, N)
    mse, max_err = _result_stats(W, Q[:, :N], s.astype(f32), zp)
    return dict(quantized_W=Q, scales=s, zero_points=zp, mse=mse, max_err=max_err, method_used=method)


# ---------------------------------------------------------------------------
# ldlq.py
# ---------------------------------------------------------------------------

def ldlq_round_column(col, scale_col, clamp_min, clamp_max):  # rounding.py:115-155
    ss = _c(scale_col, SCALE_FLOOR)
    q = _c(rhaz(col / ss), clamp_min, clamp_max)
    w_sign = np.where(np.abs(col) > f32(SIGN_FLIP_THRESHOLD), np.sign(col), np.sign(q))
    flip = (w_sign * np.sign(q)) < 0
    can = flip & (q > clamp_min)
    q = np.where(flip & (q == clamp_min), f32(clamp_max), q)
    q = np.where(can, -q, q)
    q = _c(q, clamp_min, clamp_max)
    return q.astype(f32), (col - q * ss).astype(f32)


def ldlq_loop_cpu(W_work, H_inv, scale_2d, Q, block_size, clamp_min, clamp_max):  # ldlq.py:369-417
    M, N = W_work.shape
    for i1 in range(0, N, block_size):
        i2 = min(i1 + block_size, N)
        bc = i2 - i1
        Hb = H_inv[i1:i2, i1:i2]
        dinv = (f32(1.0) / _c(np.diagonal(Hb).astype(f32), HINV_DIAG_FLOOR)).astype(f32)
        E = np.zeros((M, bc), f32)
        for jl in range(bc):
            j = i1 + jl
            q, e = ldlq_round_column(W_work[:, j].copy(), scale_2d[:, j], clamp_min, clamp_max)
            Q[:, j] = q.astype(np.int8)
            en = e * dinv[jl]
            E[:, jl] = en
            if jl + 1 < bc:
                W_work[:, j + 1:i2] -= en[:, None] * Hb[jl, jl + 1:bc][None, :]
        if i2 < N:
            W_work[:, i2:] -= E @ H_inv[i1:i2, i2:]
    return Q


def _sanitize_scales(s):  # ldlq.py:326-330
    if not np.isfinite(s).all():
        s = np.nan_to_num(s, nan=SANITIZE_FLOOR, posinf=SANITIZE_CEIL, neginf=SANITIZE_FLOOR)
        s = _c(s.astype(f32), SANITIZE_FLOOR)
    return s.astype(f32)


def single_ldlq_pass(W, H_inv, flat_scales, block_size, clamp_min, clamp_max):  # ldlq.py:282-366 (CPU)
    M, N = W.shape
    s2 = _sanitize_scales(flat_scales.reshape(M, N))
    Q = np.zeros((M, N), np.int8)
    ldlq_loop_cpu(W.copy(), H_inv, s2, Q, block_size, clamp_min, clamp_max)
    return np.clip(Q, clamp_min, clamp_max).astype(np.int8)


def update_ldlq_scales(W, Q, cur, flat, momentum, thr):  # ldlq.py:553-599
    Wf = W.reshape(-1)
    Qf = Q.reshape(-1).astype(f32)
    nz = Qf != 0
    wnz = np.abs(Wf) > f32(thr)
    sc = wnz & ((Wf * Qf) > 0)
    valid = nz & sc
    mism = nz & ~sc
    new = cur.copy()
    smin, smax = float(flat.min()), float(flat.max())
    floor = max(smin * SCALE_FLOOR_MULTIPLIER, ABS_SCALE_FLOOR)
    ceil = smax * SCALE_CEIL_MULTIPLIER
    if valid.any():
        comp = _c(np.abs(Wf[valid]) / np.abs(Qf[valid]), floor, ceil)
        if momentum > 0:
            new[valid] = f32(momentum) * cur[valid] + f32(1 - momentum) * comp
        else:
            new[valid] = comp
    if mism.any():
        new[mism] = _c(flat[mism], floor, ceil)
    return new.astype(f32)


def run_iterative_ldlq(W, H_inv, flat, iterations, block_size, clamp_min, clamp_max):  # ldlq.py:479-550
    M, N = W.shape
    cur = _sanitize_scales(flat.copy())
    prev_mse = float("inf")
    prev_scales = None
    Q_res = None
    for it in range(iterations):
        Qi = single_ldlq_pass(W, H_inv, cur, block_size, clamp_min, clamp_max)
        Q_res = Qi
        mse = float(np.mean(np.abs((W - Qi.astype(f32) * cur.reshape(M, N)).astype(np.float64)) ** 2))
        if not math.isfinite(mse):
            if prev_scales is not None:
                cur = prev_scales
            break
        if it > 0 and mse > prev_mse * 1.05:
            if prev_scales is not None:
                cur = prev_scales
            break
        impr = (prev_mse - mse) / (prev_mse + CONVERGENCE_EPS)
        if it > 0 and impr < CONVERGENCE_IMPROVEMENT_THRESHOLD:
            break
        prev_mse = mse
        if it < iterations - 1:
            prev_scales = cur.copy()
            cur = update_ldlq_scales(W, Qi, cur, flat, 0.3, 1e-8)
    return Q_res, cur


def greedy_local_search(W, Q, scale_2d, H, num_passes, clamp_min, clamp_max):  # greedy.py:487-541
    M, N = W.shape
    Q = Q.astype(f32).copy()
    grid = np.arange(clamp_min, clamp_max + 1, dtype=f32)
    Hd = np.diagonal(H).astype(f32)
    err = (Q * scale_2d - W).astype(f32)
    for _ in range(num_passes):
        for j in range(N):
            qo = Q[:, j].copy()
            sj = scale_2d[:, j]
            cross = err @ H[j, :] - err[:, j] * H[j, j]
            delta = (grid[None, :] - qo[:, None]) * sj[:, None]
            ne = err[:, j][:, None] + delta
            cost = ne * ne * Hd[j] + f32(2) * ne * cross[:, None]
            bi = np.argmin(cost, axis=1)
            qn = grid[bi]
            Q[:, j] = qn
            err[:, j] += (qn - qo) * sj
    return np.clip(Q, clamp_min, clamp_max).astype(np.int8)


def _fma32(a, b, c):
    """fp32 a*b + c with one rounding (the product is exact in fp64; the fp64
    sum is then rounded to fp32, a double rounding that differs from a true
    fused multiply-add only in rare halfway cases)."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(f32)


def greedy_lowrank_given(W, Q, scale_2d, H, s_k, U_k, num_passes, clamp_min, clamp_max,
                         stall=0.99):
    """The low-rank greedy search of greedy_lowrank_triton (greedy.py:384-479)
    given its decomposition (s_k, U_k): the per-column step of
    _greedy_lowrank_kernel (greedy.py:100-199, evaluated here row-vectorised
    with products and the accumulations err_lr . (s U_j) and err_lr += d U_j
    as fused multiply-adds, the candidate cost term by term), the proxy
    (err @ H * err).sum() after every pass and the stop when it improves by
    less than 1% (greedy.py:464-476).  Returns (int8 codes, passes run)."""
    W = np.asarray(W, dtype=f32)
    M, N = W.shape
    Q = np.asarray(Q, dtype=f32).copy()
    S = np.asarray(scale_2d, dtype=f32)
    H = np.asarray(H, dtype=f32)
    U = np.asarray(U_k, dtype=f32)
    SU = (U * np.asarray(s_k, dtype=f32)[None, :]).astype(f32)
    k = U.shape[1]
    Hd = np.diagonal(H).astype(f32)
    grid = np.arange(clamp_min, clamp_max + 1, dtype=f32)
    err = (Q * S - W).astype(f32)
    elr = (err.astype(np.float64) @ U.astype(np.float64)).astype(f32)
    prev = np.inf
    runs = 0
    for p in range(num_passes):
        runs += 1
        for j in range(N):
            cross = np.zeros(M, dtype=f32)
            for i in range(k):
                cross = _fma32(elr[:, i], np.full(M, SU[j, i], dtype=f32), cross)
            ej = err[:, j].copy()
            cross = (cross - (ej * Hd[j]).astype(f32)).astype(f32)
            sj = np.maximum(S[:, j], f32(1e-8))
            qo = Q[:, j].copy()
            best = np.full(M, f32(1e30), dtype=f32)
            bq = qo.copy()
            for g in grid:
                ne = (ej + ((g - qo).astype(f32) * sj).astype(f32)).astype(f32)
                cost = (((ne * ne).astype(f32) * Hd[j]).astype(f32)
                        + ((f32(2) * ne).astype(f32) * cross).astype(f32)).astype(f32)
                better = cost < best
                best = np.where(better, cost, best)
                bq = np.where(better, g, bq)
            bq = np.clip(bq, clamp_min, clamp_max).astype(f32)
            d = ((bq - qo).astype(f32) * sj).astype(f32)
            Q[:, j] = bq
            err[:, j] = (ej + d).astype(f32)
            for i in range(k):
                elr[:, i] = _fma32(d, np.full(M, U[j, i], dtype=f32), elr[:, i])
        proxy = float(((err.astype(np.float64) @ H.astype(np.float64)) * err).sum())
        if p > 0 and proxy >= prev * stall:
            break
        prev = proxy
    return np.clip(Q, clamp_min, clamp_max).astype(np.int8), runs


def _ls_scales(Q, W):  # ldlq.py:227-231, 262-265
    Qf = Q.astype(f32)
    num = (Qf * W).sum(axis=1, keepdims=True, dtype=f32)
    den = _c((Qf * Qf).sum(axis=1, keepdims=True, dtype=f32), DENOMINATOR_FLOOR)
    return _c(num / den, SCALE_MIN).astype(f32)


def ldlq_quantize_layer(W, hessian=None, block_size=128, damping=0.01, int_bits=4, iterations=1,
                        greedy_passes=0):  # ldlq.py:95-279 (2-D / weight-only)
    if int_bits not in (4, 8):
        raise ValueError(f"int_bits must be 4 or 8, got {int_bits}")
    W = np.asarray(W, dtype=f32)
    M, N = W.shape
    div = INT8_SCALE_DIVISOR if int_bits == 8 else INT4_SCALE_DIVISOR
    qmin, qmax = (-128, 127) if int_bits == 8 else (-8, 7)
    if hessian is not None:
        H = np.asarray(hessian, dtype=f32)
        Hinv, _ = invert_hessian(damp(H, damping))
    else:
        H = (W.T @ W / f32(M)).astype(f32)
        if not np.isfinite(H).all():
            s = _c(np.abs(W).max(axis=1, keepdims=True) / f32(div), SCALE_MIN, SCALE_MAX)
            q = _c(np.rint(W / s), qmin, qmax).astype(np.int8)
            mse, mx = _result_stats(W, q, s, None)
            return dict(quantized_W=q, scales=s.astype(np.float16), zero_points=None, mse=mse,
                        max_err=mx, H=H, method_used="rtn")
        H = damp(H, damping)
        Hinv, _ = invert_hessian(H)
    rs = _c(np.abs(W).max(axis=1, keepdims=True) / f32(div), SCALE_MIN)
    flat = np.broadcast_to(rs, (M, N)).reshape(-1).copy()
    if iterations > 1:
        Q, _ = run_iterative_ldlq(W, Hinv, flat, iterations, block_size, qmin, qmax)
    else:
        Q = single_ldlq_pass(W, Hinv, flat, block_size, qmin, qmax)
    if greedy_passes > 0:
        gs = _ls_scales(Q, W)
        Q = greedy_local_search(W, Q, np.broadcast_to(gs, (M, N)).astype(f32), H,
                                greedy_passes, qmin, qmax)
    fs = _ls_scales(Q, W)
    mse, mx = _result_stats(W, Q, fs, None)
    return dict(quantized_W=Q, scales=fs.astype(np.float16), scales_f32=fs, zero_points=None,
                mse=mse, max_err=mx, H=H, method_used="ldlq_cpu")


# ---------------------------------------------------------------------------
# piso.py
# ---------------------------------------------------------------------------

def torch_linspace_f32(start: float, end: float, steps: int) -> np.ndarray:
    """The fp32 ``torch.linspace`` table PiSO builds candidates from (piso.py:62-63, 135-136)."""
    import torch
    return torch.linspace(start, end, steps, dtype=torch.float32).numpy()


def piso_symmetric(W, h, num_coarse, num_fine, qmin, qmax, divisor):  # piso.py:29-94
    W = np.asarray(W, f32)
    h = np.asarray(h, f32)
    cf = torch_linspace_f32(0.5, 2.0, num_coarse)
    ff = torch_linspace_f32(0.95, 1.05, num_fine)
    sa = _c(np.abs(W).max(axis=1, keepdims=True) / f32(divisor), 1e-10)
    sc = sa * cf[None, :]
    W3 = W[:, None, :]
    rows = np.arange(W.shape[0])
    q = _c(rhaz(W3 / sc[:, :, None]), qmin, qmax)
    cost = (((W3 - q * sc[:, :, None]) ** 2) * h).sum(axis=2, dtype=f32)
    best = sc[rows, cost.argmin(axis=1)]
    sf = best[:, None] * ff[None, :]
    q = _c(rhaz(W3 / sf[:, :, None]), qmin, qmax)
    cost = (((W3 - q * sf[:, :, None]) ** 2) * h).sum(axis=2, dtype=f32)
    return sf[rows, cost.argmin(axis=1)][:, None].astype(f32)


def piso_asymmetric(W, h, num_coarse, num_fine, qmin, qmax, lo, hi):  # piso.py:97-182
    W = np.asarray(W, f32)
    h = np.asarray(h, f32)
    cf = torch_linspace_f32(lo, hi, num_coarse)
    ff = torch_linspace_f32(0.95, 1.05, num_fine)
    div = f32(qmax - qmin)
    wmin = W.min(axis=1, keepdims=True)
    wmax = W.max(axis=1, keepdims=True)
    sr = _c((wmax - wmin) / div, 1e-10)
    W3 = W[:, None, :]
    rows = np.arange(W.shape[0])

    def ev(s):
        zp = _c(rhaz(f32(qmin) - wmin[:, :, None] / s[:, :, None]), qmin, qmax)
        q = _c(rhaz(W3 / s[:, :, None] + zp), qmin, qmax)
        cost = (((W3 - (q - zp) * s[:, :, None]) ** 2) * h).sum(axis=2, dtype=f32)
        return zp[:, :, 0], cost

    sc = _c(sr * cf[None, :], 1e-10)
    _, cost = ev(sc)
    best = sc[rows, cost.argmin(axis=1)]
    sf = _c(best[:, None] * ff[None, :], 1e-10)
    zpf, cost = ev(sf)
    bi = cost.argmin(axis=1)
    return sf[rows, bi][:, None].astype(f32), zpf[rows, bi][:, None].astype(np.int8)


def compute_piso_scales_int8(W, hd, num_coarse=128, num_fine=16):  # piso.py:190-240
    W = np.asarray(W, f32)
    return piso_symmetric(W, np.asarray(hd, f32)[:W.shape[1]], num_coarse, num_fine, -128, 127, 127.0)


def compute_piso_scales_int8_asymmetric(W, hd, num_coarse=128, num_fine=16):  # piso.py:243-295
    W = np.asarray(W, f32)
    return piso_asymmetric(W, np.asarray(hd, f32)[:W.shape[1]], num_coarse, num_fine, -128, 127, 0.8, 1.2)


def compute_piso_scales_int4(W, hd, num_coarse=128, num_fine=16):  # piso.py:303-352
    W = np.asarray(W, f32)
    return piso_symmetric(W, np.asarray(hd, f32)[:W.shape[1]], num_coarse, num_fine, -8, 7, 7.0)


def compute_piso_scales_int4_asymmetric(W, hd, num_coarse=128, num_fine=16):  # piso.py:355-408
    W = np.asarray(W, f32)
    return piso_asymmetric(W, np.asarray(hd, f32)[:W.shape[1]], num_coarse, num_fine, -8, 7, 0.5, 2.0)


# ---------------------------------------------------------------------------
# Quality metric used by the parity gates
# ---------------------------------------------------------------------------

def proxy_loss(W, Q, scales, zero_points, H) -> float:
    """tr((W - deq) H (W - deq)^T) in float64 (H = the undamped Hessian)."""
    W = np.asarray(W, np.float64)
    s = np.asarray(scales, np.float64).reshape(-1, 1)
    Qf = np.asarray(Q, np.float64)
    if zero_points is not None:
        Qf = Qf - np.asarray(zero_points, np.float64).reshape(-1, 1)
    E = W - Qf * s
    return float(np.einsum("ij,ij->", E @ np.asarray(H, np.float64), E))


# ---------------------------------------------------------------- SmoothRot pre-step
def apply_smoothing_to_weight(W, s):  # smoothquant.py:54-69
    """W[:, j] * s_j (fp32)."""
    return (np.asarray(W, f32) * np.asarray(s, f32)[None, :]).astype(f32)


SMOOTHQUANT_AMAX_FLOOR = 1e-8  # config.py:148
SMOOTHQUANT_HESSIAN_FLOOR = f32(1e-8) * f32(1e-8)  # config.py:148-152
SANITIZE_CEIL = f32(1e30)  # config.py:78


def transform_hessian_for_smoothquant(H, s):  # pipeline.py:99-137 (2-D branch)
    """H[i, j] / max(s_i s_j, 1e-16), capped at 1e30 (NaN passes)."""
    s = np.asarray(s, f32)
    outer = s[None, :] * s[:, None]
    outer = np.where(outer < SMOOTHQUANT_HESSIAN_FLOOR, SMOOTHQUANT_HESSIAN_FLOOR, outer).astype(f32)
    q = (np.asarray(H, f32) / outer).astype(f32)
    return np.where(q > SANITIZE_CEIL, SANITIZE_CEIL, q).astype(f32)


def compute_smoothing_from_hessian_diag(hd, W, alpha=0.5, num_calibration_samples=128):  # smoothquant.py:72-102
    """s_j = sqrt(max(H_jj / n, floor))^alpha / max(max_i |W_ij|, floor)^(1 - alpha), fp32."""
    n = max(1, int(num_calibration_samples))
    act = np.sqrt(_c(np.asarray(hd, f32) / f32(n), SMOOTHQUANT_AMAX_FLOOR)).astype(f32)
    ws = _c(np.abs(np.asarray(W, f32)).max(axis=0), SMOOTHQUANT_AMAX_FLOOR).astype(f32)
    # the power is the library call the reference makes (torch's vectorised CPU pow):
    # numpy's pow differs from it in the last bit on a few channels
    import torch
    pa = torch.from_numpy(act).pow(alpha).numpy()
    pb = torch.from_numpy(ws).pow(1.0 - alpha).numpy()
    return (pa / pb).astype(f32)


def compute_smoothing_factors(act_amax, W, alpha=0.5):  # smoothquant.py:11-52
    """s_j = max(amax_j, floor)^alpha / max(max_i |W_ij|, floor)^(1 - alpha), fp32."""
    import torch
    act = _c(np.asarray(act_amax, f32), SMOOTHQUANT_AMAX_FLOOR).astype(f32)
    ws = _c(np.abs(np.asarray(W, f32)).max(axis=0), SMOOTHQUANT_AMAX_FLOOR).astype(f32)
    return (torch.from_numpy(act).pow(alpha).numpy() / torch.from_numpy(ws).pow(1.0 - alpha).numpy()).astype(f32)


# ---------------------------------------------------------------- PermuQuant
def channel_second_moments(W):  # permuquant.py:13-22
    return (np.asarray(W, f32) ** 2).mean(axis=0, dtype=np.float64).astype(f32)


def permuquant_order(W, act_mu2=None, alpha=0.5):  # permuquant.py:25-67
    """Channels by descending second moment (or joint key), ties by index."""
    key = channel_second_moments(W)
    if act_mu2 is not None:
        import torch
        a = torch.from_numpy(np.maximum(np.asarray(act_mu2, f32), f32(1e-12)))
        w = torch.from_numpy(np.maximum(key, f32(1e-12)))
        key = (a.pow(alpha) * w.pow(1.0 - alpha)).numpy()
    return np.argsort(-key.astype(np.float64), kind="stable")


def compute_group_quant_error(W, group_size=128, int_bits=4):  # permuquant.py:70-105
    W = np.asarray(W, f32)
    M, N = W.shape
    if int_bits == 8:
        s = calculate_scales_int8(W).astype(f32)
        q = quantize_weights_int8(W, s)
        dq = q.astype(f32) * s
    else:
        s = calculate_scales(W, group_size)
        q = quantize_weights(W, s, group_size)
        G = q.shape[1] // group_size
        dq = (q.reshape(M, G, group_size).astype(f32) * s.astype(f32)[:, :, None]).reshape(M, -1)[:, :N]
    return float(((W - dq).astype(np.float64) ** 2).sum())


def find_permutation_with_acceptance(W, act_mu2=None, alpha=0.5, group_size=128, tau=0.0,
                                     int_bits=4):  # permuquant.py:108-150
    perm = permuquant_order(W, act_mu2, alpha)
    e0 = compute_group_quant_error(W, group_size, int_bits)
    e1 = compute_group_quant_error(np.asarray(W, f32)[:, perm], group_size, int_bits)
    rel = (e0 - e1) / e0 if e0 > 0 else 0.0
    return perm, bool(rel > tau), e0, e1
