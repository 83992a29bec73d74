"""ctypes binding of ``libintcrush_b200.so`` (the C ABI in ``include/intcrush_b200.h``).

The shared library is built in-tree (``int_crush_converter_b200/csrc``) and
loaded from the package directory.  There is no fallback: if the library is
missing, or no sm_100 GPU is present, every quantization call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libintcrush_b200.so")

IC_OK = 0
IC_ERR_INVALID = -1
IC_ERR_CUDA = -2
IC_ERR_NOT_PD = -3
DEV_TIMEOUT = 1
DEV_NOT_PD = 2
DEV_BAD_SCALE = 8  # a row's fp16 scale is NaN/inf/0 (the pipeline's bad-scale condition)
IC_ERR_TIMEOUT = -4
IC_ERR_RANGE = -5
IC_ERR_UNSUPPORTED = -6
IC_ERR_WORKSPACE = -7

IC_F32, IC_F16, IC_BF16 = 0, 1, 2

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_f64 = ctypes.c_double
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/intcrush_b200.h
SIGNATURES = {
    "ic_version": (ctypes.c_char_p, []),
    "ic_last_error": (ctypes.c_char_p, []),
    "ic_device_check": (_i32, []),
    "ic_launch_count": (ctypes.c_ulonglong, []),
    "ic_inverse_graph_count": (ctypes.c_ulonglong, []),
    "ic_selftest_bounded_wait": (_i32, [ctypes.c_ulonglong, _vp]),
    "ic_device_status": (_i32, [ctypes.POINTER(ctypes.c_uint), _vp]),
    "ic_rotate_weights": (_i32, [_vp, _i32, _i64, _i64, _i64, _i32, _vp, _i64, _vp]),
    "ic_rotate_hessian": (_i32, [_vp, _i64, _i64, _i64, _i32, _vp, _vp, _i64, _vp]),
    "ic_rtn_scales": (_i32, [_vp, _i64, _i64, _i64, _i32, _i32, _i64, _vp, _i32, _vp, _vp, _vp]),
    "ic_rtn_codes": (_i32, [_vp, _i64, _i64, _i64, _i32, _i32, _i64, _vp, _vp, _vp, _i64, _vp]),
    "ic_rtn_fused": (_i32, [_vp, _i32, _i64, _i64, _i64, _i32, _i32, _i32, _vp, _i32, _vp, _vp,
                            _vp, _vp, _vp, _vp, _vp]),
    "ic_pack_int4": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp]),
    "ic_unpack_int4": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp]),
    "ic_gemm_tn": (_i32, [_i64, _i64, _i64, _f32, _vp, _vp, _i64, _vp, _vp, _i64, _f32, _vp, _vp,
                          _i64, _vp, _vp, _i64, _i32, _vp]),
    "ic_gemm_tn_tri": (_i32, [_i64, _i64, _i64, _f32, _vp, _vp, _i64, _vp, _vp, _i64, _f32, _vp, _vp,
                              _i64, _vp, _vp, _i64, _i32, _vp]),
    "ic_spd_inverse_workspace_size": (_sz, [_i64]),
    "ic_spd_inverse": (_i32, [_vp, _vp, _i64, _i64, _f32, _vp, _sz, _vp]),
    "ic_spd_cholesky": (_i32, [_vp, _vp, _i64, _i64, _vp, _sz, _vp]),
    "ic_smooth_factors": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _i32, _f32, _f32, _vp, _vp]),
    "ic_permuquant_order": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _f32, _vp, _vp, _vp]),
    "ic_group_quant_error": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _i32, _vp, _vp, _vp]),
    "ic_orthonormalize": (_i32, [_vp, _i64, _i32, _i64, _vp]),
    "ic_sym_eig": (_i32, [_vp, _i32, _i64, _vp, _vp, _i64, _vp]),
    "ic_gptq_row_params": (_i32, [_vp, _i64, _i64, _i64, _i32, _i32, _vp, _vp, _vp]),
    "ic_gptq_workspace_size": (_sz, [_i64, _i64, _i32, _i32]),
    "ic_gptq_run": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _i32, _i32, _vp, _vp,
                           _i32, _i32, _vp, _i64, _vp, _i64, _vp, _vp, _i32, _vp, _sz, _vp]),
    "ic_gptq_run_noalloc": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _i32, _i32, _vp, _vp,
                                   _i32, _i32, _vp, _i64, _vp, _i64, _vp, _vp, _i32, _vp]),
    "ic_gptq_layer_workspace_size": (_sz, [_i64, _i64, _i32]),
    "ic_gptq_layer": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
                             _f32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ic_ldlq_run": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _i64, _i32, _i32, _vp, _i64, _i32, _i32,
                           _vp, _i64, _i32, _vp, _sz, _vp]),
    "ic_ldlq_update_scales": (_i32, [_vp, _vp, _vp, _vp, _i64, _f32, _f32, _f32, _f32, _f32, _vp]),
    "ic_greedy_workspace_size": (_sz, [_i64, _i64]),
    "ic_greedy_lowrank_pass": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i32, _vp, _i64, _i64,
                                      _i32, _i32, _vp]),
    "ic_greedy_run": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i32, _i32,
                             _i32, _i32, _vp, _sz, _vp]),
    "ic_piso": (_i32, [_vp, _i64, _i64, _i64, _vp, _i32, _i32, _i32, _f32, _vp, _i32, _vp, _i32, _vp,
                       _vp, _vp]),
    "ic_finalize_stats": (_i32, [_vp, _vp, _i64, _f64, _vp, _vp]),
    "ic_transpose": (_i32, [_vp, _vp, _i64, _i64, _i64, _f32, _vp, _vp, _i64, _vp]),
    "ic_split_tf32": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp]),
}


class NotPositiveDefinite(RuntimeError):
    """The damped Hessian has a non-positive pivot (the reference's LinAlgError)."""


class DeviceTimeout(RuntimeError):
    """A bounded device-side wait gave up; the CUDA context stays usable."""


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the in-tree shared library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing: build it with `make -C int_crush_converter_b200/csrc` "
                                  "or `python -c 'import __graft_entry__ as g; g.build()'`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = _Checked(lib)
    return _lib


class _Checked:
    """The loaded library with an argument-count check on every declared entry
    point: ctypes forwards surplus arguments silently, and a pointer landing in
    the wrong slot (a stream, a workspace) would reach the driver."""

    def __init__(self, lib: ctypes.CDLL):
        self._lib = lib
        self._fns = {}
        for name, (_, args) in SIGNATURES.items():
            fn, n = getattr(lib, name), len(args)

            def call(*a, _fn=fn, _n=n, _name=name):
                if len(a) != _n:
                    raise TypeError(f"{_name} takes {_n} arguments, got {len(a)}")
                return _fn(*a)
            self._fns[name] = call

    def __getattr__(self, name):
        fns = self.__dict__.get("_fns", {})
        if name in fns:
            return fns[name]
        return getattr(self.__dict__["_lib"], name)


def last_error() -> str:
    return load().ic_last_error().decode(errors="replace")


def check(status: int, what: str = "") -> None:
    if status == IC_OK:
        return
    msg = last_error()
    if what:
        msg = f"{what}: {msg}"
    if status == IC_ERR_INVALID:
        raise ValueError(msg)
    if status == IC_ERR_RANGE:
        from .packing import INT4PackingError
        raise INT4PackingError(msg)
    if status == IC_ERR_NOT_PD:
        raise NotPositiveDefinite(msg)
    if status == IC_ERR_TIMEOUT:
        raise DeviceTimeout(msg)
    raise RuntimeError(f"libintcrush_b200 error {status}: {msg}")


_device_ok: dict[int, bool] = {}


def require_device(device: torch.device | None = None) -> torch.device:
    """The CUDA device the kernels run on; raises if there is no sm_100 GPU."""
    if not torch.cuda.is_available():
        raise RuntimeError("int_crush_converter_b200 needs a CUDA sm_100a (B200) device; none is available")
    if device is None or device.type != "cuda":
        device = torch.device("cuda", torch.cuda.current_device())
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _device_ok:
        with torch.cuda.device(idx):
            check(load().ic_device_check(), "device check")
        _device_ok[idx] = True
    return torch.device("cuda", idx)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()
