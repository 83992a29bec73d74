"""Definitions of the golden-vector cases (inputs are rebuilt from seeds).

Used by ``make_golden.py`` (which runs the reference implementation on them)
and by the tests (which rebuild the same inputs and compare with the stored
outputs).
"""

from __future__ import annotations

import numpy as np

from . import inputs as gi

f32 = np.float32

RATIOS = [0.8, 0.85, 0.9, 0.95, 1.0]


def rtn_weight(case: dict) -> np.ndarray:
    M, N, seed = case["M"], case["N"], case["seed"]
    if case.get("dist") == "heavy":
        W = gi.weight_heavy_tail(seed, M, N)
    else:
        W = gi.weight_outlier_cols(seed, M, N, frac=case.get("frac", 0.004))
    # edge rows: all-zero row, constant row, single spike, all-positive, all-negative
    if M >= 8:
        W[1] = 0.0
        W[2] = 0.01
        W[3] = 0.0
        W[3, N // 3] = 0.5
        W[4] = np.abs(W[4]) + 0.05
        W[5] = -np.abs(W[5]) - 0.05
    return W


RTN_CASES = {
    "rtn4_sym_r256": dict(M=64, N=1024, seed=11, rot=256, bits=4, asym=False, ratios=None, gs=None),
    "rtn4_sym_r256_clip": dict(M=64, N=1024, seed=12, rot=256, bits=4, asym=False, ratios=RATIOS, gs=None),
    "rtn4_sym_r64_pad": dict(M=48, N=200, seed=13, rot=64, bits=4, asym=False, ratios=None, gs=None),
    "rtn4_sym_g128": dict(M=32, N=512, seed=14, rot=16, bits=4, asym=False, ratios=None, gs=128),
    "rtn4_sym_g96_clip": dict(M=32, N=500, seed=15, rot=0, bits=4, asym=False, ratios=RATIOS, gs=96),
    "rtn4_asym_r256": dict(M=64, N=768, seed=16, rot=256, bits=4, asym=True, ratios=None, gs=None),
    "rtn4_asym_r256_clip": dict(M=64, N=768, seed=17, rot=256, bits=4, asym=True, ratios=RATIOS, gs=None),
    "rtn4_asym_g64": dict(M=32, N=256, seed=18, rot=0, bits=4, asym=True, ratios=None, gs=64),
    "rtn8_sym_r64": dict(M=64, N=768, seed=19, rot=64, bits=8, asym=False, ratios=None, gs=None, dist="heavy"),
    "rtn8_sym_r64_clip": dict(M=96, N=768, seed=20, rot=64, bits=8, asym=False, ratios=RATIOS, gs=None, dist="heavy"),
    "rtn8_asym_r16": dict(M=64, N=384, seed=21, rot=16, bits=8, asym=True, ratios=None, gs=None),
    "rtn8_asym_r64_clip": dict(M=64, N=384, seed=22, rot=64, bits=8, asym=True, ratios=RATIOS, gs=None, dist="heavy"),
}

ROT_CASES = {
    "rotw_r16": dict(M=16, N=128, seed=31, rot=16),
    "rotw_r64_pad": dict(M=24, N=300, seed=32, rot=64),
    "rotw_r256": dict(M=16, N=512, seed=33, rot=256),
    "rotw_r32_sylvester": dict(M=8, N=96, seed=34, rot=32),
}

ROTH_CASES = {
    "roth_r64_pad": dict(N=200, rot=64, seed=41, nblk=None),
    "roth_r256": dict(N=512, rot=256, seed=42, nblk=None),
    "roth_3d_r64": dict(N=128, rot=64, seed=43, nblk=3),
}

GPTQ_CASES = {
    # single block: the column loop alone (bit-exact given the same Hinv)
    "gptq4_single_block": dict(M=8, N=32, seed=51, bits=4, asym=False, bs=32, nsamp=64, rot=0),
    "gptq4_r256": dict(M=64, N=512, seed=52, bits=4, asym=False, bs=128, nsamp=1024, rot=256),
    "gptq4_r64_ragged_block": dict(M=40, N=320, seed=53, bits=4, asym=False, bs=128, nsamp=512, rot=64),
    "gptq8_sym": dict(M=48, N=256, seed=54, bits=8, asym=False, bs=128, nsamp=512, rot=256),
    "gptq8_asym": dict(M=48, N=256, seed=55, bits=8, asym=True, bs=64, nsamp=512, rot=256),
    "gptq4_blockdiag": dict(M=32, N=256, seed=56, bits=4, asym=False, bs=64, nsamp=512, rot=0, nblk=2),
    "gptq4_rank_deficient": dict(M=32, N=384, seed=57, bits=4, asym=False, bs=128, nsamp=128, rot=256),
}

LDLQ_CASES = {
    "ldlq4_weight_only": dict(M=64, N=256, seed=61, bits=4, iters=1, greedy=0, bs=128, rot=256),
    "ldlq4_iter2_greedy2": dict(M=48, N=256, seed=62, bits=4, iters=2, greedy=2, bs=64, rot=256),
    "ldlq8_calib": dict(M=32, N=256, seed=63, bits=8, iters=1, greedy=0, bs=128, rot=0, calib=True),
}

GREEDY_CASES = {
    "greedy4": dict(M=32, N=128, seed=71, bits=4, passes=2),
    "greedy8": dict(M=16, N=64, seed=72, bits=8, passes=1),
}

PISO_CASES = {
    "piso_int8_sym": dict(M=32, N=512, seed=81, kind="int8"),
    "piso_int8_asym": dict(M=32, N=512, seed=82, kind="int8_asym"),
    "piso_int4_sym": dict(M=32, N=512, seed=83, kind="int4"),
    "piso_int4_asym": dict(M=32, N=512, seed=84, kind="int4_asym"),
}

PACK_CASES = {
    "pack_even": dict(M=16, K=64, seed=91),
    "pack_odd": dict(M=7, K=33, seed=92),
}

# SmoothRot pre-step (smoothquant.py:54-69, pipeline.py:99-137): the last two
# factors are tiny so that s_i s_j hits the 1e-16 floor
SMOOTH_CASES = {
    "smooth_basic": dict(M=48, N=256, seed=95),
}


def smooth_inputs(case: dict):
    M, N, seed = case["M"], case["N"], case["seed"]
    W = gi.weight_outlier_cols(seed, M, N)
    H = gi.hessian_lognormal(seed + 1, N, 2 * N)
    rng = np.random.default_rng(seed + 2)
    s = np.exp(rng.normal(0.0, 0.7, N)).astype(np.float32)
    s[-2:] = np.float32(1e-9)
    return W, H, s


LINSPACE_CASES = {
    "ls_coarse_sym": (0.5, 2.0, 128),
    "ls_coarse_asym8": (0.8, 1.2, 128),
    "ls_fine": (0.95, 1.05, 16),
    "ls_small": (0.5, 2.0, 7),
}


def gptq_inputs(case: dict):
    M, N, seed = case["M"], case["N"], case["seed"]
    W = gi.weight_outlier_cols(seed, M, N)
    H = gi.hessian_lognormal(seed + 1000, N, case["nsamp"])
    if case.get("nblk"):
        nb = case["nblk"]
        bs = N // nb
        H = np.stack([H[i * bs:(i + 1) * bs, i * bs:(i + 1) * bs] for i in range(nb)])
    return W, H


def ldlq_inputs(case: dict):
    M, N, seed = case["M"], case["N"], case["seed"]
    W = gi.weight_outlier_cols(seed, M, N, frac=0.01, mult=30.0, std=0.015)
    H = gi.hessian_lognormal(seed + 1000, N, 512) if case.get("calib") else None
    return W, H


def greedy_inputs(case: dict):
    M, N, seed = case["M"], case["N"], case["seed"]
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, N)) * 0.02).astype(f32)
    qmax = 7 if case["bits"] == 4 else 127
    s = (np.abs(W).max(axis=1, keepdims=True) / qmax).astype(f32)
    Q = np.clip(np.rint(W / s), -qmax - 1, qmax).astype(np.int8)
    H = gi.hessian_lognormal(seed + 1000, N, 256)
    H = (H + 0.01 * np.mean(np.diag(H)) * np.eye(N)).astype(f32)
    return W, Q, np.broadcast_to(s, (M, N)).astype(f32).copy(), H


def piso_inputs(case: dict):
    M, N, seed = case["M"], case["N"], case["seed"]
    W = gi.weight_outlier_cols(seed, M, N)
    rng = np.random.default_rng(seed + 7)
    hd = rng.lognormal(0.0, 1.0, size=N).astype(f32) ** 2
    return W, hd.astype(f32)


# GPTQ entry points beyond the default hinv path: the RTN fallback
# (gptq.py:420-533), PiSO scale / zero-point overrides (gptq.py:210-252),
# DLR Hessians through Woodbury (gptq.py:323-344, dlr.py:75-124) and
# hessian_method="cholesky" (gptq.py:91-110)
GPTQ_EXTRA_CASES = {
    "gx_rtn4_sym": dict(kind="rtn", M=48, N=256, seed=101, bits=4, asym=False, ratios=None),
    "gx_rtn4_asym_clip": dict(kind="rtn", M=48, N=256, seed=102, bits=4, asym=True, ratios=RATIOS),
    "gx_rtn8_sym_clip": dict(kind="rtn", M=48, N=256, seed=103, bits=8, asym=False, ratios=RATIOS),
    "gx_rtn8_asym": dict(kind="rtn", M=48, N=256, seed=104, bits=8, asym=True, ratios=None),
    "gx_rtn4_piso": dict(kind="rtn", M=48, N=256, seed=105, bits=4, asym=False, ratios=None, piso=True),
    "gx_rtn4_piso_zp": dict(kind="rtn", M=48, N=256, seed=106, bits=4, asym=False, ratios=None, piso=True,
                            piso_zp=True),
    "gx_rtn8_piso": dict(kind="rtn", M=48, N=256, seed=107, bits=8, asym=False, ratios=None, piso=True),
    "gx_gptq4_piso": dict(kind="gptq", M=48, N=256, seed=108, bits=4, asym=False, piso=True),
    "gx_gptq4_piso_zp": dict(kind="gptq", M=48, N=256, seed=109, bits=4, asym=False, piso=True, piso_zp=True),
    "gx_gptq8_piso_asym": dict(kind="gptq", M=48, N=256, seed=110, bits=8, asym=True, piso=True),
    "gx_gptq8_piso_sym": dict(kind="gptq", M=48, N=256, seed=111, bits=8, asym=False, piso=True),
    "gx_gptq4_dlr": dict(kind="dlr", M=48, N=256, seed=112, bits=4, asym=False, rank=16),
    "gx_gptq4_cholesky": dict(kind="cholesky", M=48, N=256, seed=113, bits=4, asym=False),
    "gx_gptq8_cholesky_3d": dict(kind="cholesky", M=32, N=256, seed=114, bits=8, asym=False, nblk=2),
}


def gptq_extra_inputs(case: dict):
    """W fp32 [M,N]; the Hessian (2-D, 3-D or DLR dict of numpy arrays, None for
    RTN); PiSO scales [M,1] (absmax-based, jittered) and zero-points [M,1] or None."""
    M, N, seed = case["M"], case["N"], case["seed"]
    W = gi.weight_outlier_cols(seed, M, N)
    rng = np.random.default_rng(seed + 5)
    H = None
    if case["kind"] == "dlr":
        D = (rng.lognormal(0.0, 1.0, N) ** 2).astype(f32)
        U = (rng.standard_normal((N, case["rank"])) * 0.5).astype(f32)
        H = {"format": "dlr", "D": D, "U": U}
    elif case["kind"] != "rtn":
        H = gi.hessian_lognormal(seed + 1000, N, 2 * N)
        if case.get("nblk"):
            nb = case["nblk"]
            bs = N // nb
            H = np.stack([H[i * bs:(i + 1) * bs, i * bs:(i + 1) * bs] for i in range(nb)])
    ps = pz = None
    if case.get("piso"):
        qmax = 7.0 if case["bits"] == 4 else 127.0
        base = np.abs(W).max(axis=1, keepdims=True) / qmax
        ps = (base * rng.uniform(0.7, 1.3, size=(M, 1))).astype(f32)
        if case.get("piso_zp"):
            pz = rng.integers(-3, 3, size=(M, 1)).astype(np.int8)
    return W, H, ps, pz


# rotation.rotate_activations (rotation.py:128-153): any leading dims, padding
ROTACT_CASES = {
    "ra_r64_pad_3d": dict(shape=(2, 3, 200), rot=64, seed=121),
    "ra_r256": dict(shape=(5, 512), rot=256, seed=122),
}


# SmoothQuant factors from the Hessian diagonal (smoothquant.py:72-102), the
# form config 5 (SmoothQuant alpha 0.5 with calibration Hessians) uses
SQ_CASES = {
    "sq_hdiag_a05": dict(M=48, N=256, seed=131, alpha=0.5, nsamp=8192),
    "sq_hdiag_a075": dict(M=32, N=128, seed=132, alpha=0.75, nsamp=128),
    "sq_amax_a05": dict(M=48, N=256, seed=133, alpha=0.5, nsamp=0),
}


def sq_inputs(case: dict):
    W = gi.weight_outlier_cols(case["seed"], case["M"], case["N"])
    H = gi.hessian_lognormal(case["seed"] + 1, case["N"], 2 * case["N"]) * np.float32(case["nsamp"])
    hd = np.ascontiguousarray(np.diagonal(H)).astype(f32)
    hd[:3] = 0.0  # dead channels hit the amax floor
    if not case["nsamp"]:  # per-channel activation amax instead (compute_smoothing_factors)
        hd = np.sqrt(hd).astype(f32) * f32(3.0)
    W[:, 5] = 0.0  # an all-zero weight column hits the weight floor
    return W, hd


# PermuQuant (permuquant.py:13-211): candidate order, group errors, acceptance
PQ_CASES = {
    "pq_w_g128": dict(M=64, N=512, seed=141, group=128, bits=4, joint=False),
    "pq_joint_g128": dict(M=64, N=512, seed=142, group=128, bits=4, joint=True),
    "pq_w_rowwise": dict(M=64, N=512, seed=143, group=512, bits=4, joint=False),
    "pq_w_int8": dict(M=48, N=384, seed=144, group=128, bits=8, joint=False),
}


def pq_inputs(case: dict):
    """Weights whose channel magnitudes vary (so the order and the group
    errors are far from ties) and activation second moments."""
    M, N, seed = case["M"], case["N"], case["seed"]
    rng = np.random.default_rng(seed)
    colscale = np.exp(rng.normal(0.0, 1.0, N))
    W = (rng.standard_normal((M, N)) * 0.02 * colscale).astype(np.float16).astype(f32)
    act = (rng.lognormal(0.0, 1.0, N) ** 2).astype(f32) if case["joint"] else None
    return W, act


# SVD-absorbed split (svd.py:35-75): a planted low-rank part plus noise
SVD_CASES = {
    "svd_r16": dict(M=256, N=512, seed=151, rank=16, planted=16),
    "svd_r32_wide": dict(M=192, N=640, seed=152, rank=32, planted=24),
    "svd_r8_tall": dict(M=768, N=256, seed=153, rank=8, planted=12),
}


def svd_inputs(case: dict):
    M, N, seed, k = case["M"], case["N"], case["seed"], case["planted"]
    rng = np.random.default_rng(seed)
    sv = np.geomspace(1.0, 0.05, k)
    A = rng.standard_normal((M, k)) * sv
    B = rng.standard_normal((k, N))
    W = 0.02 * (A @ B) / np.sqrt(N) * 8 + 0.002 * rng.standard_normal((M, N))
    return W.astype(np.float32)
