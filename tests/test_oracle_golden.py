"""The CPU oracle (oracle/cpu_ref.py) against golden vectors made by the reference.

These pin the oracle before it is trusted as the checker of the CUDA path.
Tolerances are the parity bar of the task: codes/packed bytes bit-exact,
scales exact; GPTQ/LDLQ through tr(E H E^T) (GPTQ-hinv is chaotic, so codes of
the larger cases differ in a few positions between any two fp32 inverses).
"""

import numpy as np
import pytest

from oracle import cpu_ref as R
from tests.golden import cases as C
from tests.golden import inputs as gi


def test_hadamard_and_rounding(golden):
    for n in (16, 64, 256):
        assert np.array_equal(R.make_hadamard_regular(n), golden[f"hadamard_{n}/H"])
    assert np.array_equal(R.rhaz(golden["kat_rhaz/x"]), golden["kat_rhaz/y"])
    for k, (a, b, n) in C.LINSPACE_CASES.items():
        assert np.array_equal(R.torch_linspace_f32(a, b, n), golden[k + "/v"])


@pytest.mark.parametrize("name", list(C.ROT_CASES))
def test_rotate_weights(golden, name):
    c = C.ROT_CASES[name]
    W = gi.weight_outlier_cols(c["seed"], c["M"], c["N"])
    assert gi.checksum(W) == str(golden[name + "/chk"])
    g = golden[name + "/Wrot"]
    np.testing.assert_allclose(R.rotate_weights(W, c["rot"]), g, rtol=0, atol=1e-6 * np.abs(g).max())


@pytest.mark.parametrize("name", list(C.ROTH_CASES))
def test_rotate_hessian(golden, name):
    c = C.ROTH_CASES[name]
    H = gi.hessian_lognormal(c["seed"], c["N"], 256)
    if c["nblk"]:
        H = np.stack([H] * c["nblk"]) * np.arange(1, c["nblk"] + 1, dtype=np.float32)[:, None, None]
    g = golden[name + "/Hrot"]
    np.testing.assert_allclose(R.rotate_hessian(H, c["rot"]), g, rtol=0, atol=1e-6 * np.abs(g).max())


def rtn_oracle(c):
    W = C.rtn_weight(c)
    Ww = R.rotate_weights(W, c["rot"]) if c["rot"] else W
    gs = c["gs"] or Ww.shape[1]
    if c["bits"] == 4 and not c["asym"]:
        s = R.calculate_scales(Ww, gs, c["ratios"])
        return Ww, s, None, R.quantize_weights(Ww, s, gs)
    if c["bits"] == 4:
        s, zp = R.calculate_scales_asymmetric(Ww, gs, c["ratios"])
        return Ww, s, zp, R.quantize_weights_asymmetric(Ww, s, zp, gs)
    if not c["asym"]:
        s = R.calculate_scales_int8(Ww, c["ratios"])
        return Ww, s, None, R.quantize_weights_int8(Ww, s)
    s, zp = R.calculate_scales_int8_asymmetric(Ww, c["ratios"])
    return Ww, s, zp, R.quantize_weights_int8_asymmetric(Ww, s, zp)


@pytest.mark.parametrize("name", list(C.RTN_CASES))
def test_rtn(golden, name):
    c = C.RTN_CASES[name]
    _, s, zp, q = rtn_oracle(c)
    assert np.array_equal(s, golden[name + "/scales"])
    assert np.array_equal(q, golden[name + "/codes"])
    if zp is not None:
        assert np.array_equal(zp, golden[name + "/zp"])
    if c["bits"] == 4:
        assert np.array_equal(R.pack_int4(q), golden[name + "/packed"])


@pytest.mark.parametrize("name", list(C.PACK_CASES))
def test_pack(golden, name):
    c = C.PACK_CASES[name]
    q = gi.codes(c["seed"], c["M"], c["K"])
    p = R.pack_int4(q)
    assert np.array_equal(p, golden[name + "/packed"])
    assert np.array_equal(R.unpack_int4(p, c["K"]), q)
    with pytest.raises(R.INT4PackingError):
        R.pack_int4(np.array([[8, 0]], np.int8))


@pytest.mark.parametrize("name", list(C.GPTQ_CASES))
def test_gptq(golden, name):
    c = C.GPTQ_CASES[name]
    W, H = C.gptq_inputs(c)
    Ww = R.rotate_weights(W, c["rot"]) if c["rot"] else W
    Hr = R.rotate_hessian(H, c["rot"]) if c["rot"] else H
    r = R.gptq_quantize_layer(Ww, Hr, c["bs"], 0.01, c["bits"], c["asym"])
    assert np.array_equal(r["scales"], golden[name + "/scales"])
    if r["zero_points"] is not None:
        assert np.array_equal(r["zero_points"], golden[name + "/zp"])
    assert np.mean(r["quantized_W"] == golden[name + "/codes"]) > 0.99
    if Hr.ndim == 2:
        p = R.proxy_loss(Ww, r["quantized_W"], r["scales"].astype(np.float32), r["zero_points"], Hr)
        assert abs(p / float(golden[name + "/proxy"]) - 1) < 0.01
    if name + "/Hinv" in golden:  # the column loop alone is bit-exact given the same Hinv
        s, zp = R.gptq_row_params(Ww, c["bits"], c["asym"])
        Q = np.zeros(Ww.shape, np.int8)
        R.gptq_block(Ww.copy(), Q, s, golden[name + "/Hinv"], 0, Ww.shape[1], c["bs"], -8, 7, zp)
        assert np.array_equal(Q, golden[name + "/codes"])


@pytest.mark.parametrize("name", list(C.LDLQ_CASES))
def test_ldlq(golden, name):
    c = C.LDLQ_CASES[name]
    W, H = C.ldlq_inputs(c)
    Ww = R.rotate_weights(W, c["rot"]) if c["rot"] else W
    Hr = None if H is None else (R.rotate_hessian(H, c["rot"]) if c["rot"] else H)
    r = R.ldlq_quantize_layer(Ww, Hr, c["bs"], 0.01, c["bits"], c["iters"], c["greedy"])
    Hp = Hr if Hr is not None else Ww.astype(np.float64).T @ Ww.astype(np.float64) / Ww.shape[0]
    p = R.proxy_loss(Ww, r["quantized_W"], r["scales"].astype(np.float32), None, Hp)
    assert abs(p / float(golden[name + "/proxy"]) - 1) < 0.005
    assert np.mean(r["quantized_W"] == golden[name + "/codes"]) > 0.99


@pytest.mark.parametrize("name", list(C.GREEDY_CASES))
def test_greedy(golden, name):
    c = C.GREEDY_CASES[name]
    W, Q, S, H = C.greedy_inputs(c)
    qm = (-8, 7) if c["bits"] == 4 else (-128, 127)
    assert np.array_equal(R.greedy_local_search(W, Q, S, H, c["passes"], *qm), golden[name + "/codes"])


@pytest.mark.parametrize("name", list(C.PISO_CASES))
def test_piso(golden, name):
    c = C.PISO_CASES[name]
    W, hd = C.piso_inputs(c)
    f = dict(int8=R.compute_piso_scales_int8, int4=R.compute_piso_scales_int4,
             int8_asym=R.compute_piso_scales_int8_asymmetric,
             int4_asym=R.compute_piso_scales_int4_asymmetric)[c["kind"]]
    o = f(W, hd)
    if isinstance(o, tuple):
        assert np.array_equal(o[0], golden[name + "/scales"])
        assert np.array_equal(o[1], golden[name + "/zp"])
    else:
        assert np.array_equal(o, golden[name + "/scales"])


@pytest.mark.parametrize("name", list(C.SMOOTH_CASES))
def test_smoothing_matches_reference(golden, name):
    W, H, s = C.smooth_inputs(C.SMOOTH_CASES[name])
    assert np.array_equal(R.apply_smoothing_to_weight(W, s), golden[name + "/W_smooth"])
    assert np.array_equal(R.transform_hessian_for_smoothquant(H, s), golden[name + "/H_smooth"])


@pytest.mark.parametrize("name", list(C.GPTQ_EXTRA_CASES))
def test_gptq_extra_entry_points(golden, name):
    """RTN fallback, PiSO overrides, DLR (Woodbury) and hessian_method='cholesky'."""
    c = C.GPTQ_EXTRA_CASES[name]
    W, H, ps, pz = C.gptq_extra_inputs(c)
    assert gi.checksum(W) == str(golden[name + "/chk"])
    if c["kind"] == "rtn":
        r = R.gptq_quantize_layer_rtn(W, c["bits"], c["asym"], c.get("ratios"), ps, pz)
    else:
        method = "cholesky" if c["kind"] == "cholesky" else "hinv"
        r = R.gptq_quantize_layer(W, H, 128, 0.01, c["bits"], c["asym"], ps, pz, hessian_method=method)
    assert np.array_equal(r["quantized_W"], golden[name + "/codes"])
    assert np.array_equal(r["scales"], golden[name + "/scales"])
    if r["zero_points"] is None:
        assert name + "/zp" not in golden.files
    else:
        assert np.array_equal(r["zero_points"], golden[name + "/zp"])
    assert abs(r["mse"] / float(golden[name + "/mse"]) - 1) < 1e-6
    if c["kind"] == "dlr":
        g = golden[name + "/Hinv"]
        np.testing.assert_allclose(R.woodbury_inverse(H["D"], H["U"], 0.01), g, rtol=0, atol=1e-5 * np.abs(g).max())


@pytest.mark.parametrize("name", list(C.ROTACT_CASES))
def test_rotate_activations(golden, name):
    c = C.ROTACT_CASES[name]
    x = np.random.default_rng(c["seed"]).standard_normal(c["shape"]).astype(np.float32)
    g = golden[name + "/y"]
    np.testing.assert_allclose(R.rotate_activations(x, c["rot"]), g, rtol=0, atol=2e-6 * np.abs(g).max())


@pytest.mark.parametrize("name", list(C.SQ_CASES))
def test_smoothing_factors_from_hessian_diag(golden, name):
    c = C.SQ_CASES[name]
    W, hd = C.sq_inputs(c)
    if c["nsamp"]:
        s = R.compute_smoothing_from_hessian_diag(hd, W, c["alpha"], c["nsamp"])
    else:
        s = R.compute_smoothing_factors(hd, W, c["alpha"])
    assert np.array_equal(s, golden[name + "/s"])


@pytest.mark.parametrize("name", list(C.PQ_CASES))
def test_permuquant(golden, name):
    """Order exact; errors within fp32-summation noise of the reference's; the
    acceptance decision equal (these cases' improvements are far from 0, or
    exactly 0 where the groups span the row)."""
    c = C.PQ_CASES[name]
    W, act = C.pq_inputs(c)
    np.testing.assert_allclose(R.channel_second_moments(W), golden[name + "/mu2"], rtol=2e-6)
    perm, acc, e0, e1 = R.find_permutation_with_acceptance(W, act, 0.5, c["group"], 0.0, c["bits"])
    assert np.array_equal(perm, golden[name + "/perm"])
    assert abs(e0 / float(golden[name + "/err"]) - 1) < 1e-5
    assert abs(e1 / float(golden[name + "/err_perm"]) - 1) < 1e-5
    assert acc == bool(golden[name + "/accepted"])


def test_lowrank_greedy_oracle_with_full_decomposition_is_the_full_rank_search():
    """The low-rank greedy restatement (greedy.py:100-199, 384-479) given every
    eigenpair of H computes the full-rank coordinate descent of the golden-pinned
    oracle (greedy.py:487-541): same codes."""
    rng = np.random.default_rng(0)
    M, N = 48, 96
    W = (rng.standard_normal((M, N)) * 0.02).astype(np.float32)
    W[:, 5] *= 30
    H = (W.T @ W / M).astype(np.float32)
    H += np.eye(N, dtype=np.float32) * np.float32(0.01 * np.diag(H).mean())
    ev, V = np.linalg.eigh(H.astype(np.float64))
    ev, V = ev[::-1].astype(np.float32), V[:, ::-1].astype(np.float32)
    s = (np.abs(W).max(1, keepdims=True) / 7).astype(np.float32)
    Q = np.clip(np.rint(W / s), -8, 7).astype(np.int8)
    S = np.ascontiguousarray(np.broadcast_to(s, (M, N)))
    q_lr, runs = R.greedy_lowrank_given(W, Q, S, H, ev, V, 2, -8, 7)
    q_full = R.greedy_local_search(W, Q, S, H, 2, -8, 7)
    assert runs == 2
    assert np.array_equal(q_lr, q_full)
