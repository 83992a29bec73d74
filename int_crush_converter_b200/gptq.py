"""GPTQ on the GPU (mirrors converter/gptq.py).

``gptq_quantize_layer`` keeps the reference's signature, validation, scale /
zero-point rules, Hessian formats (2-D, 3-D block-diagonal, DLR dict) and
``hessian_method`` options, and returns the same ``QuantizationResult``.  The
column loop, the lazy update, the inverse and the row statistics run in
libintcrush_b200.  ``quantize_gptq_layer`` is the fused device-resident path
(rotation + Hessian rotation + GPTQ + packing in one C call) that the pipeline
hook and the benchmark use.
"""

from __future__ import annotations

import torch

from . import _native as nat
from ._dev import back, device_of, f32, round4, workspace
from .config import GEMM_PASSES, SCALE_DTYPE, SCALE_MAX, SCALE_MIN, SUPERBLOCK
from .hessian import hessian_pair, inverse_pair, woodbury_inverse
from .rounding import _round_half_away_from_zero
from .scales import (
    _fix_asymmetric_scale, calculate_scales, calculate_scales_asymmetric, calculate_scales_int8,
    calculate_scales_int8_asymmetric, quantize_weights, quantize_weights_asymmetric, quantize_weights_int8,
    quantize_weights_int8_asymmetric,
)
from .types import QuantizationResult

_HESSIAN_METHODS = ("hinv", "cholesky")


def _piso_params(Wd, piso_scales, piso_zero_points, int_bits, asymmetric):  # gptq.py:210-252
    M = Wd.shape[0]
    piso = piso_scales.float().to(Wd.device)
    if piso.shape != (M, 1):
        return None
    s = piso.clamp(min=SCALE_MIN, max=SCALE_MAX)
    wmin = Wd.amin(dim=1, keepdim=True)
    wmax = Wd.amax(dim=1, keepdim=True)
    zero_rows = (wmin == 0) & (wmax == 0)
    if int_bits == 4:
        if piso_zero_points is not None:
            zp = piso_zero_points.float().to(Wd.device).clamp(-8, 7)
        else:
            s = _fix_asymmetric_scale(s, wmin, wmax, -8, 7)
            zp = (-8 - _round_half_away_from_zero(wmin / s)).clamp(-8, 7)
        return s, zp.masked_fill(zero_rows, 0).to(torch.int8).float()
    if asymmetric:
        s = _fix_asymmetric_scale(s, wmin, wmax, -128, 127)
        zp = (-128 - _round_half_away_from_zero(wmin / s)).clamp(-128, 127)
        return s, zp.masked_fill(zero_rows, 0).to(torch.int8).float()
    return s, None


def _run_loop(W_work, W0, col0, ncols, hi, lo, ld, block_size, scale, zp, qmin, qmax, Q):
    """ic_gptq_run over columns [col0, col0+ncols) of W_work (the Hinv pair covers exactly them)."""
    dev = W_work.device
    M, N = W_work.shape
    sb = max(1, SUPERBLOCK // block_size) * block_size
    lib = nat.load()
    ws = workspace(lib.ic_gptq_workspace_size(M, ncols, block_size, sb), dev)
    rsq = torch.empty(M, dtype=torch.float64, device=dev)
    rmx = torch.empty(M, dtype=torch.float32, device=dev)
    es = W_work.element_size()
    nat.check(lib.ic_gptq_run(W_work.data_ptr() + col0 * es, N, W0.data_ptr() + col0 * es, N, M, ncols,
                              hi.data_ptr(), lo.data_ptr(), ld, block_size, sb, scale.data_ptr(), nat.ptr(zp),
                              qmin, qmax, Q.data_ptr() + col0, N, None, 0, rsq.data_ptr(), rmx.data_ptr(),
                              GEMM_PASSES, ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)), "gptq_run")
    return rsq, rmx


def gptq_quantize_layer(W: torch.Tensor, hessian, block_size: int = 128, damping: float = 0.01, int_bits: int = 4,
                        asymmetric: bool = False, hessian_method: str = "hinv", piso_scales=None,
                        piso_zero_points=None) -> QuantizationResult:
    """Quantize one weight matrix with GPTQ (gptq.py:137-417).

    INT4 is always asymmetric per-row; INT8 symmetric unless ``asymmetric``.
    Scales are clamped to [SCALE_MIN, SCALE_MAX] before the loop.  Accepts a
    2-D Hessian [in, in], a 3-D block-diagonal [nb, bs, bs] one (each block
    inverted and quantized independently) or a DLR dict (Woodbury inverse).
    """
    if int_bits not in (4, 8):
        raise ValueError(f"int_bits must be 4 or 8, got {int_bits}")
    if W.dim() != 2:
        raise ValueError(f"Expected 2D weight tensor, got {W.dim()}D")
    if hessian_method not in _HESSIAN_METHODS:
        raise ValueError(f"hessian_method must be one of {list(_HESSIAN_METHODS)}, got '{hessian_method}'")
    Hsrc = hessian["D"] if isinstance(hessian, dict) else hessian
    dev = device_of(W, Hsrc)
    Wd = f32(W, dev)
    M, N = Wd.shape
    qmin, qmax = (-128, 127) if int_bits == 8 else (-8, 7)
    lib = nat.load()
    st = nat.stream_ptr(dev)

    params = None
    if piso_scales is not None:
        params = _piso_params(Wd, piso_scales, piso_zero_points, int_bits, asymmetric)
    if params is not None:
        scale = params[0].reshape(M).contiguous()
        zp = None if params[1] is None else params[1].reshape(M).contiguous()
    else:
        scale = torch.empty(M, dtype=torch.float32, device=dev)
        has_zp = int_bits == 4 or asymmetric
        zp = torch.empty(M, dtype=torch.float32, device=dev) if has_zp else None
        if M:
            nat.check(lib.ic_gptq_row_params(Wd.data_ptr(), M, N, N, int_bits, int(asymmetric), scale.data_ptr(),
                                             nat.ptr(zp), st), "gptq_row_params")

    Q = torch.zeros(M, N, dtype=torch.int8, device=dev)
    W_work = Wd.clone()
    fallbacks: list[str] = []
    stats = []

    def loop_with(Hinv_hi, Hinv_lo, ld, c0, c1):
        if M and c1 > c0:
            stats.append(_run_loop(W_work, Wd, c0, c1 - c0, Hinv_hi, Hinv_lo, ld, block_size, scale, zp,
                                   qmin, qmax, Q))

    def maybe_cholesky(hi, lo, n):
        """hessian_method="cholesky" (gptq.py:91-110): the upper factor of chol(H^-1)
        in place of H^-1, or H^-1 itself when that factorisation fails."""
        if hessian_method != "cholesky":
            return hi, lo
        fh, fl = hi.clone(), lo.clone()
        ws = workspace(lib.ic_spd_inverse_workspace_size(n), dev)
        stc = lib.ic_spd_cholesky(fh.data_ptr(), fl.data_ptr(), n, fh.shape[1], ws.data_ptr(), ws.numel(), st)
        if stc == nat.IC_ERR_NOT_PD:
            return hi, lo
        nat.check(stc, "spd_cholesky")
        return fh, fl

    if isinstance(hessian, dict):
        D = hessian["D"]
        if D.shape[0] != N:
            raise ValueError(f"DLR Hessian dim {D.shape[0]} != in_features {N}")
        Hinv = woodbury_inverse(hessian["D"], hessian["U"], damping=damping)
        from ._dev import split
        hi, lo = split(Hinv.contiguous())
        loop_with(hi, lo, hi.shape[1], 0, N)
    elif hessian.dim() == 3:
        nb, bs, _ = hessian.shape
        Hd = f32(hessian, dev)
        for bi in range(nb):
            c0 = bi * bs
            c1 = min(c0 + bs, N)
            if c1 <= c0:
                break
            blk = Hd[bi, :c1 - c0, :c1 - c0].contiguous()
            hi, lo, n = hessian_pair(blk, 0, dev, rotate=False)
            path = inverse_pair(hi, lo, n, damping, H_fallback=blk)
            if path != "cholesky":
                fallbacks.append(f"hessian_{path}")
            hi, lo = maybe_cholesky(hi, lo, n)
            loop_with(hi, lo, hi.shape[1], c0, c1)
    elif hessian.dim() == 2:
        if tuple(hessian.shape) != (N, N):
            raise ValueError(f"Hessian shape {tuple(hessian.shape)} != ({N}, {N})")
        Hd = f32(hessian, dev)
        hi, lo, n = hessian_pair(Hd, 0, dev, rotate=False)
        path = inverse_pair(hi, lo, n, damping, H_fallback=Hd)
        if path != "cholesky":
            fallbacks.append(f"hessian_{path}")
        hi, lo = maybe_cholesky(hi, lo, n)
        loop_with(hi, lo, hi.shape[1], 0, N)
    else:
        raise ValueError(f"Expected 2D tensor, 3D tensor, or DLR dict Hessian, got {type(hessian).__name__}")

    if stats and M * N:
        mse = float(sum(s[0].sum() for s in stats).item()) / (M * N)
        max_err = float(torch.stack([s[1].max() for s in stats]).max().item())
    else:
        mse, max_err = 0.0, 0.0
    zp8 = None if zp is None else zp.reshape(M, 1).to(torch.int8)
    return QuantizationResult(
        quantized_W=back(Q, W),
        scales=back(scale.reshape(M, 1).to(SCALE_DTYPE), W),
        zero_points=back(zp8, W),
        mse=mse,
        max_err=max_err,
        method_used="gptq_b200",
        fallbacks=fallbacks,
    )


def _stats(Wd, q, s, zp):
    deq = q.float() * s.float() if zp is None else (q.float() - zp.float()) * s.float()
    d = Wd - deq[:, :Wd.shape[1]]
    return d.double().pow(2).mean().item(), (d.abs().max().item() if d.numel() else 0.0)


def gptq_quantize_layer_rtn(W: torch.Tensor, int_bits: int = 4, asymmetric: bool = False, clipping_ratios=None,
                            piso_scales=None, piso_zero_points=None) -> QuantizationResult:
    """RTN fallback for layers without a Hessian (gptq.py:420-533)."""
    if int_bits not in (4, 8):
        raise ValueError(f"int_bits must be 4 or 8, got {int_bits}")
    dev = device_of(W)
    Wd = f32(W, dev)
    M, N = Wd.shape
    method = "rtn_b200"
    if piso_scales is not None and int_bits == 8 and not asymmetric and piso_scales.shape[0] == M \
            and piso_scales.shape[1] == 1:
        s = piso_scales.float().to(dev).clamp(min=SCALE_MIN, max=SCALE_MAX).to(SCALE_DTYPE)
        q, zp = quantize_weights_int8(Wd, s), None
        method = "rtn_piso_b200"
    elif piso_scales is not None and int_bits == 4 and piso_scales.shape[0] == M and piso_scales.shape[1] == 1:
        s = piso_scales.float().to(dev).clamp(min=SCALE_MIN, max=SCALE_MAX).to(SCALE_DTYPE)
        if piso_zero_points is not None:
            zp = piso_zero_points.to(dev).to(torch.int8)
        else:
            _, zp = calculate_scales_asymmetric(Wd, N, clipping_ratios=clipping_ratios)
        q = quantize_weights_asymmetric(Wd, s, zp, N)
        method = "rtn_piso_b200"
    elif asymmetric:
        if int_bits == 8:
            s, zp = calculate_scales_int8_asymmetric(Wd, clipping_ratios=clipping_ratios)
            q = quantize_weights_int8_asymmetric(Wd, s, zp)
        else:
            s, zp = calculate_scales_asymmetric(Wd, N, clipping_ratios=clipping_ratios)
            q = quantize_weights_asymmetric(Wd, s, zp, N)
    else:
        zp = None
        if int_bits == 8:
            s = calculate_scales_int8(Wd, clipping_ratios=clipping_ratios)
            q = quantize_weights_int8(Wd, s)
        else:
            s = calculate_scales(Wd, N, clipping_ratios=clipping_ratios)
            q = quantize_weights(Wd, s, N)
    mse, max_err = _stats(Wd, q, s, zp)
    return QuantizationResult(quantized_W=back(q, W), scales=back(s, W), zero_points=back(zp, W), mse=mse,
                              max_err=max_err, method_used=method, fallbacks=[])


_DT = {torch.float32: nat.IC_F32, torch.float16: nat.IC_F16, torch.bfloat16: nat.IC_BF16}


class LayerWorkspace:
    """Reusable device workspace for :func:`quantize_gptq_layer` (grows on demand)."""

    def __init__(self):
        self.buf: dict[int, torch.Tensor] = {}

    def get(self, nbytes: int, dev: torch.device) -> torch.Tensor:
        b = self.buf.get(dev.index)
        if b is None or b.numel() < nbytes:
            self.buf[dev.index] = None
            b = workspace(nbytes, dev)
            self.buf[dev.index] = b
        return b


_default_ws = LayerWorkspace()


def quantize_gptq_layer(W: torch.Tensor, H: torch.Tensor, rot_size: int = 256, int_bits: int = 4,
                        asymmetric: bool = False, block_size: int = 128, damping: float = 0.01,
                        h_rotated: bool = False, want_codes: bool = False, want_packed: bool = True,
                        out: dict | None = None, ws: LayerWorkspace | None = None, check: bool = True,
                        update_passes: int = 1, smoothing: torch.Tensor | None = None,
                        smoothing_order: str = "pipeline") -> dict:
    """Fused GPTQ layer on the GPU: pipeline.py:527-559 + 702-809 + 919-931 + 1010-1013
    (outlier sanitize |w| > 1000 -> 0, rotations, GPTQ, packing, verify).

    W fp16/bf16/fp32 [out, in] (unrotated), H fp32 [in, in] (unrotated unless
    ``h_rotated``).  Returns a dict of device tensors: ``packed`` uint8
    [out, in_pad/2] (INT4), ``codes`` int8 [out, in_pad] (if asked),
    ``scales`` fp16 [out, 1], ``zero_points`` int8 [out, 1] or None, and
    ``stats`` fp64 [mse, max_err, status] of the pipeline's verify step.  Pass
    ``out`` (a dict of preallocated tensors with those keys) to avoid
    allocations.  The device work is asynchronous on the current stream; with
    ``check`` (default) the call synchronises and raises
    :class:`NotPositiveDefinite` when the damped Hessian had no Cholesky
    factor; with ``check=False`` the caller calls :func:`check_layer` later
    (so that layers on several streams overlap).  ``update_passes`` selects the
    precision of the lazy trailing update W -= E * Hinv: 1 = TF32 products with
    fp32 accumulation (default; the north star's "FP32-accumulate"), 3 =
    3xTF32.  The Hessian inverse is 3xTF32 either way.  Measured against the
    reference on the parity aggregates both keep tr((W-Q)H(W-Q)^T) within
    0.15%.  ``smoothing`` (per-input-channel factors s, [in]) applies the
    SmoothRot pre-step the pipeline runs on FFN down layers
    (pipeline.py:547-553 + 766-774): W[:, j] * s_j and H[i, j] / (s_i s_j)
    before both rotations, fused into their loads.  ``smoothing_order``
    "pipeline" (default) gives the Hessian the sequence the reference pipeline
    actually runs for such a layer -- rotate, smooth, rotate again
    (pipeline.py:721-723 then 766-770) -- so that results match it;
    "smooth_then_rotate" rotates the smoothed Hessian once.
    """
    dev = device_of(W, H)
    Wd = W.to(dev)
    if Wd.dtype not in _DT:
        Wd = Wd.float()
    Wd = Wd.contiguous()
    Hd = f32(H, dev)
    M, N = Wd.shape
    r = rot_size if rot_size else 1
    npad = -(-N // r) * r
    has_zp = int_bits == 4 or asymmetric
    o = out or {}
    packed = o.get("packed") if want_packed and int_bits == 4 else None
    if want_packed and int_bits == 4 and packed is None:
        packed = torch.empty(M, (npad + 1) // 2, dtype=torch.uint8, device=dev)
    codes = o.get("codes") if want_codes else None
    if want_codes and codes is None:
        codes = torch.empty(M, npad, dtype=torch.int8, device=dev)
    s16 = o.get("scales")
    if s16 is None:
        s16 = torch.empty(M, 1, dtype=torch.float16, device=dev)
    zp = o.get("zero_points") if has_zp else None
    if has_zp and zp is None:
        zp = torch.empty(M, 1, dtype=torch.int8, device=dev)
    stats = o.get("stats")
    if stats is None:
        stats = torch.empty(3, dtype=torch.float64, device=dev)
    lib = nat.load()
    need = lib.ic_gptq_layer_workspace_size(M, N, rot_size)
    wbuf = (ws or _default_ws).get(need, dev)
    sm = None
    if smoothing is not None:
        sm = f32(smoothing, dev).reshape(-1).contiguous()
        if sm.numel() != N:
            raise ValueError(f"smoothing has {sm.numel()} factors for {N} input features")
    orders = {"smooth_then_rotate": 0, "pipeline": 1}
    if smoothing_order not in orders:
        raise ValueError(f"smoothing_order must be one of {list(orders)}, got {smoothing_order!r}")
    nat.check(lib.ic_gptq_layer(Wd.data_ptr(), _DT[Wd.dtype], M, N, N, Hd.data_ptr(), Hd.shape[1], nat.ptr(sm),
                                orders[smoothing_order], int(h_rotated),
                                rot_size, int_bits, int(asymmetric), block_size, float(damping), int(update_passes),
                                nat.ptr(codes),
                                nat.ptr(packed), s16.data_ptr(), nat.ptr(zp), stats.data_ptr(), wbuf.data_ptr(),
                                wbuf.numel(), nat.stream_ptr(dev)), "gptq_layer")
    res = dict(packed=packed, codes=codes, scales=s16, zero_points=zp, stats=stats)
    if check:
        check_layer(res)
    return res


def check_layer(res: dict) -> dict:
    """Raise :class:`NotPositiveDefinite` if a :func:`quantize_gptq_layer` result
    reports a Hessian without a Cholesky factor (reads ``stats[2]``; synchronises
    with the stream that produced it)."""
    status = int(res["stats"][2].item())
    if status & nat.DEV_NOT_PD:
        raise nat.NotPositiveDefinite("Hessian is not positive definite")
    if status & nat.DEV_BAD_SCALE:  # pipeline.py:933-940 logs the same condition
        import warnings
        warnings.warn("Bad scales detected (a NaN weight row): scale NaN, zero-point and codes 0 for that row",
                      stacklevel=2)
    return res


class LayerStreams:
    """Quantize independent layers concurrently on several CUDA streams.

    The reference quantizes a model's linear layers one after another
    (pipeline.py:702-809 inside the per-layer loop); layers are independent
    given their Hessians, so on the GPU they may overlap: one layer's
    latency-bound steps (the inverse's 128-wide diagonal blocks, the GPTQ
    column loop) fill the SMs another layer's tensor-core GEMMs leave idle.
    Each stream owns a :class:`LayerWorkspace`; each submitted layer goes to the
    stream with the least estimated work queued (M*N^2 + N^3).  Used as a
    context manager: entering orders the streams after the current stream,
    leaving orders the current stream after them and raises
    :class:`NotPositiveDefinite` for any layer whose Hessian had no Cholesky
    factor (the one synchronisation).
    """

    def __init__(self, n_streams: int = 4, device=None):
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.streams = [torch.cuda.Stream(dev) for _ in range(max(1, n_streams))]
        # host inputs are copied on a lane's own copy stream, ahead of the lane's
        # compute by at most two layers (prefetch over PCIe while it computes)
        self.copy_streams = [torch.cuda.Stream(dev) for _ in self.streams]
        self._done: list[list[torch.cuda.Event]] = [[] for _ in self.streams]
        self.ws = [LayerWorkspace() for _ in self.streams]
        self.load = [0.0] * len(self.streams)
        self._stats: list[torch.Tensor] = []

    def __enter__(self):
        self.fork()
        return self

    def __exit__(self, exc_type, exc, tb):
        self.join()
        if exc_type is None:
            self.check()
        return False

    def fork(self) -> None:
        """Order the streams after the work already queued on the current stream."""
        cur = torch.cuda.current_stream(self.device)
        for s in self.streams + self.copy_streams:
            s.wait_stream(cur)
        self.load = [0.0] * len(self.streams)
        self._done = [[] for _ in self.streams]

    def join(self) -> None:
        """Order the current stream after everything submitted (no host wait)."""
        cur = torch.cuda.current_stream(self.device)
        for s in self.streams + self.copy_streams:
            cur.wait_stream(s)

    def submit(self, W: torch.Tensor, H: torch.Tensor, then=None, before=None, **kw) -> dict:
        """Issue :func:`quantize_gptq_layer` (same keyword arguments) on the least
        loaded stream; host inputs are copied to the device on that stream
        (asynchronously when pinned; keep them alive until :meth:`join`).
        ``before(W_device)`` runs on that stream first and returns extra keyword
        arguments for the layer call (e.g. SmoothQuant factors computed on the
        device); ``then(result)`` runs on that stream right after (e.g. a copy of
        the outputs to host memory).  Returns the (asynchronous) result; its
        ``done`` entry is a CUDA event recorded after the layer."""
        M, N = int(W.shape[0]), int(W.shape[1])
        i = min(range(len(self.load)), key=self.load.__getitem__)
        self.load[i] += float(M) * N * N + float(N) ** 3
        s = self.streams[i]
        if not (W.is_cuda and H.is_cuda):
            cs = self.copy_streams[i]
            done = self._done[i]
            if len(done) >= 2:
                cs.wait_event(done[-2])  # at most two layers of inputs ahead of the lane
            with torch.cuda.stream(cs):
                if not W.is_cuda:
                    W = W.to(self.device, non_blocking=True)
                if not H.is_cuda:
                    H = H.to(self.device, non_blocking=True)
            s.wait_stream(cs)
        for t in (W, H):
            t.record_stream(s)
        with torch.cuda.stream(s):
            if before is not None:
                kw = dict(kw, **before(W))
            res = quantize_gptq_layer(W, H, ws=self.ws[i], check=False, **kw)
            if then is not None:
                then(res)
            ev = torch.cuda.Event()
            ev.record(s)
        res["done"] = ev
        self._done[i] = self._done[i][-1:] + [ev]
        self._stats.append(res["stats"])
        return res

    def check(self) -> None:
        """Wait for the submitted layers; raise if any reported a non-PD Hessian."""
        if not self._stats:
            return
        self.join()
        st = torch.stack([s[2] for s in self._stats]).cpu()
        self._stats = []
        bad = [i for i, v in enumerate(st.tolist()) if int(v) & nat.DEV_NOT_PD]
        if bad:
            raise nat.NotPositiveDefinite(f"Hessian is not positive definite (layers {bad} of this batch)")
