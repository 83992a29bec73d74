"""GPU parity at the benchmark configurations' own shapes.

GPTQ and LDLQ rows are independent given the (inverse) Hessian
(rounding.py:37-103 and ldlq.py:369-417 act row by row; scales and
zero-points are per row), so the CPU oracle can check a full-size layer on a
seeded subset of its rows with the full N x N Hessian: the CUDA path
quantizes the whole layer, the oracle those rows, and the two are compared on
the same rows.  Bars (the task's): scales and zero-points bit-exact,
tr((W - deq) H (W - deq)^T) over the rows within 0.5% of the oracle's; RTN
codes bit-exact or +-1 on <= 0.01%, scales within 1 fp16 ulp (the rotation's
fp32 summation order differs from the oracle's matmul); the inverse within 8x the
error of fp32 LAPACK (the reference's own arithmetic) against an fp64 inverse.

Config 3 (GPTQ INT4 rot256, block 128, damping 0.01): qkv [12288,4096],
proj [4096,4096], mlp_up [16384,4096], mlp_down [4096,16384], fp16 weights
N(0, 0.02^2), H = X^T X / 8192 with X rows N(0, diag(s^2)), s ~ LogNormal(0,1)
(generated on the GPU from a seed, then copied to the oracle).  Config 1: the 8
RTN INT4 layers [4096,4096] with 0.1% x20 outlier columns.  Config 2: RTN
INT8 rot64 with the clipping-ratio search on [3072,3072] and [12288,3072]
Student-t-tailed layers.  Config 4: LDLQ INT4 rot256, 2 iterations, 8 greedy
passes, weight-only Hessian, on [8192,8192].
"""

import numpy as np
import pytest
import torch

from oracle import cpu_ref as R
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import int_crush_converter_b200 as B

ROWS = 256
CFG3 = {"proj": (4096, 4096, 31), "qkv": (12288, 4096, 32), "mlp_up": (16384, 4096, 33), "mlp_down": (4096, 16384, 34)}


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def np_(t):
    return t.detach().cpu().numpy()


def hessian_gpu(seed: int, n: int, samples: int = 8192) -> torch.Tensor:
    """H = X^T X / samples with X rows N(0, diag(s^2)), s ~ LogNormal(0, 1), fp32 on the GPU."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    s = torch.exp(torch.randn(n, generator=g, device="cuda"))
    H = torch.zeros(n, n, device="cuda")
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for c0 in range(0, samples, 2048):
            X = torch.randn(min(2048, samples - c0), n, generator=g, device="cuda") * s
            H.addmm_(X.T, X)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    H.div_(samples)
    return 0.5 * (H + H.T)


def proxy_rows(Wr, Q, s, zp, H64):
    E = Wr.astype(np.float64) - (Q.astype(np.float64) - (0.0 if zp is None else zp.astype(np.float64))) \
        * s.astype(np.float64).reshape(-1, 1)
    return float(np.einsum("ij,ij->", E @ H64, E))


_cache: dict = {}


def cfg3_layer(name: str):
    """The layer's inputs, the oracle's results on ROWS seeded rows, and the fp64 rotated Hessian."""
    if name in _cache:
        return _cache[name]
    _cache.clear()
    M, N, seed = CFG3[name]
    W = gi.weight_outlier_cols(seed, M, N, frac=0.0, mult=1.0)  # N(0, 0.02^2), fp16-representable
    H = hessian_gpu(1000 + seed, N)
    Hn = np_(H)
    rows = np.sort(np.random.default_rng(seed).choice(M, ROWS, replace=False))
    Wr = R.rotate_weights(W[rows], 256)
    Hr = R.rotate_hessian(Hn, 256)
    Hinv, path = R.invert_hessian(R.damp(Hr, 0.01))
    assert path == "cholesky"
    s, zp = R.gptq_row_params(Wr, 4)
    Q = np.zeros(Wr.shape, np.int8)
    R.gptq_block(Wr.copy(), Q, s, Hinv, 0, N, 128, -8, 7, zp)
    H64 = Hr.astype(np.float64)
    d = dict(W=W, H=H, rows=rows, Wr=Wr, Hr=Hr, Hinv=Hinv, s=s, zp=zp, Q=Q, H64=H64,
             p_ref=proxy_rows(Wr, Q, s.astype(np.float16).astype(np.float32), zp, H64))
    _cache[name] = d
    return d


@pytest.mark.parametrize("update_passes", [1, 3])
@pytest.mark.parametrize("name", list(CFG3))
def test_config3_gptq_layer_rows_vs_oracle(name, update_passes):
    d = cfg3_layer(name)
    M, N, _ = CFG3[name]
    out = B.quantize_gptq_layer(cu(d["W"]).half(), d["H"], rot_size=256, block_size=128, damping=0.01,
                                want_codes=True, update_passes=update_passes)
    torch.cuda.synchronize()
    rows = d["rows"]
    q = np_(out["codes"])[rows]
    s16 = np_(out["scales"])[rows]
    zp = np_(out["zero_points"])[rows]
    assert np.array_equal(s16, d["s"].astype(np.float16))
    assert np.array_equal(zp, d["zp"])
    assert np.array_equal(np_(B.unpack_int4(out["packed"][torch.from_numpy(rows).cuda()], N)), q)
    p = proxy_rows(d["Wr"], q, s16.astype(np.float32), zp, d["H64"])
    assert abs(p / d["p_ref"] - 1) < 0.005, (name, update_passes, p / d["p_ref"])
    st = np_(out["stats"])
    assert st[2] == 0 and np.isfinite(st[0]) and st[0] > 0


def test_config3_inverse_n16384_accuracy():
    """The damped inverse of the mlp_down Hessian (n = 16384) against an fp64
    inverse, compared with fp32 LAPACK's error on the same matrix."""
    d = cfg3_layer("mlp_down")
    Hd = R.damp(d["Hr"], 0.01)
    Hd_gpu = cu(Hd)
    ref = torch.linalg.inv(Hd_gpu.double())  # fp64 checker only
    out, path = B.invert_dense(Hd_gpu, damping=None)
    assert path == "cholesky"
    scale = ref.abs().max().item()
    rel = (out.double() - ref).abs().max().item() / scale
    rel_lapack = (cu(d["Hinv"]).double() - ref).abs().max().item() / scale
    assert rel < max(8 * rel_lapack, 1e-5), (rel, rel_lapack)
    assert (out - out.T).abs().max().item() <= 1e-6 * out.abs().max().item()


def fp16_ulps(a, b) -> int:
    return int(np.abs(a.astype(np.float16).view(np.int16).astype(np.int32)
                      - b.astype(np.float16).view(np.int16).astype(np.int32)).max(initial=0))


def codes_close(a, b, max_frac=1e-4):
    d = np.abs(a.astype(np.int32) - b.astype(np.int32))
    return d.max(initial=0) <= 1 and np.mean(d > 0) <= max_frac


def test_config1_rtn_int4_all_layers():
    """All 8 config-1 layers through the fused RTN call."""
    ndiff = ntot = nrows_ulp = 0
    for layer in range(8):
        W = gi.weight_outlier_cols(500 + layer, 4096, 4096, frac=0.001, mult=20.0)
        out = B.rtn_quantize_fused(cu(W).half(), 256, int_bits=4)
        Wr = R.rotate_weights(W, 256)
        s = R.calculate_scales(Wr, 4096)
        q = R.quantize_weights(Wr, s, 4096)
        gs = np_(out["scales"])
        # fp32 Hadamard summation order can move a row's absmax by an fp32 ulp and
        # its fp16 scale by one ulp (the task's bar); rare
        assert fp16_ulps(gs, s) <= 1
        nrows_ulp += int(np.sum(gs != s))
        g = np_(out["codes"])
        assert codes_close(g, q)
        # given the device's scales, the oracle's codes agree up to the same
        # summation-order +-1
        assert codes_close(g, R.quantize_weights(Wr, gs, 4096))
        assert np.array_equal(np_(out["packed"]), R.pack_int4(g))
        ndiff += int(np.sum(g != q))
        ntot += q.size
    assert ndiff <= 1e-4 * ntot
    assert nrows_ulp <= 8 * 4096 * 1e-3


@pytest.mark.parametrize("M", [3072, 12288])
def test_config2_rtn_int8_clip(M):
    W = gi.weight_heavy_tail(600 + M, M, 3072)
    ratios = [0.8, 0.85, 0.9, 0.95, 1.0]
    out = B.rtn_quantize_fused(cu(W).half(), 64, int_bits=8, clipping_ratios=ratios, want_packed=False)
    Wr = R.rotate_weights(W, 64)
    s = R.calculate_scales_int8(Wr, ratios)
    q = R.quantize_weights_int8(Wr, s)
    assert fp16_ulps(np_(out["scales"]), s) <= 1
    assert codes_close(np_(out["codes"]), q)


@pytest.mark.parametrize("greedy_gemm_passes", ["3", "1"])
def test_config4_ldlq_rows_vs_oracle(monkeypatch, greedy_gemm_passes):
    """LDLQ INT4 rot256, 2 iterations, 8 greedy passes, weight-only Hessian, one
    [8192, 8192] layer; the oracle runs 128 seeded rows with the full damped
    W^T W / M.  With 2 iterations the second pass's codes are the result
    whatever the convergence checks decide (ldlq.py:479-550), so rows stay
    independent.  Both precisions of the greedy cross terms (3xTF32, the
    default, and the opt-in one-pass TF32)."""
    monkeypatch.setenv("IC_GREEDY_GEMM_PASSES", greedy_gemm_passes)
    import warnings
    M = N = 8192
    W = gi.weight_outlier_cols(700, M, N, frac=0.0005, mult=30.0, std=0.015)
    Wr_gpu = B.rotate_weights(cu(W), 256)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        r = B.ldlq_quantize_layer(Wr_gpu, None, block_size=128, damping=0.01, int_bits=4, iterations=2,
                                  greedy_passes=8)
    torch.cuda.synchronize()
    Wr = R.rotate_weights(W, 256)
    H = (Wr.T @ Wr / np.float32(M)).astype(np.float32)
    Hd = R.damp(H, 0.01)
    Hinv, _ = R.invert_hessian(Hd)
    rows = np.sort(np.random.default_rng(7).choice(M, 128, replace=False))
    Ws = Wr[rows]
    rs = np.maximum(np.abs(Ws).max(axis=1, keepdims=True) / np.float32(7.0), np.float32(1e-5)).astype(np.float32)
    flat = np.broadcast_to(rs, Ws.shape).reshape(-1).copy()
    Q, _ = R.run_iterative_ldlq(Ws, Hinv, flat, 2, 128, -8, 7)
    gs = R._ls_scales(Q, Ws)
    Q = R.greedy_local_search(Ws, Q, np.broadcast_to(gs, Ws.shape).astype(np.float32), Hd, 8, -8, 7)
    fs = R._ls_scales(Q, Ws).astype(np.float16).astype(np.float32)
    H64 = H.astype(np.float64)
    p_ref = proxy_rows(Ws, Q, fs, None, H64)
    q = np_(r.quantized_W)[rows]
    p = proxy_rows(Ws, q, np_(r.scales)[rows].astype(np.float32), None, H64)
    assert abs(p / p_ref - 1) < 0.005, p / p_ref
