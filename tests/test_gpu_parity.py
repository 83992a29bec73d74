"""GPU parity: the CUDA path (through the C ABI / the mirrored Python API)
against the golden vectors made by the reference and against the CPU oracle.

Bars: codes / packed bytes / scales / zero-points bit-exact for rotation + RTN
+ packing (the task allows +-1 on <= 0.01% of codes where fp32 Hadamard
summation order differs; we assert that); GPTQ/LDLQ through
tr((W - deq) H (W - deq)^T) within 0.5% of the reference on the aggregate of
several layers (1% per small layer), since GPTQ-hinv is chaotic in the last
fp32 bits of Hinv; the GPTQ column loop alone bit-exact given the reference's
own Hinv.
"""

import numpy as np
import pytest
import torch

from oracle import cpu_ref as R
from tests.golden import cases as C
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import int_crush_converter_b200 as B
    from int_crush_converter_b200 import _native as nat
    from int_crush_converter_b200._dev import split


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def np_(t):
    return t.detach().cpu().numpy()


def codes_close(a, b, max_frac=1e-4):
    d = np.abs(a.astype(np.int32) - b.astype(np.int32))
    return d.max(initial=0) <= 1 and np.mean(d > 0) <= max_frac


# ---------------------------------------------------------------- GEMM
@pytest.mark.parametrize("m,n,k,passes", [(128, 128, 32, 3), (300, 200, 100, 3), (128, 256, 1024, 1),
                                          (513, 700, 260, 1), (1, 5, 7, 3), (256, 384, 2048, 3),
                                          (129, 64, 40, 3), (1000, 130, 128, 3), (768, 1024, 4096, 3),
                                          (4096, 128, 128, 3)])
def test_gemm_tn(m, n, k, passes):
    g = torch.Generator().manual_seed(m * 7 + n)
    A = torch.randn(m, k, generator=g).cuda()
    Bm = torch.randn(n, k, generator=g).cuda()
    Cm = torch.randn(m, n, generator=g).cuda()
    ah, al = split(A)
    bh, bl = split(Bm)
    D = Cm.clone()
    lib = nat.load()
    nat.check(lib.ic_gemm_tn(m, n, k, -0.5, ah.data_ptr(), al.data_ptr(), ah.shape[1], bh.data_ptr(), bl.data_ptr(),
                             bh.shape[1], 2.0, D.data_ptr(), None, n, D.data_ptr(), None, n, passes,
                             nat.stream_ptr(D.device)))
    torch.cuda.synchronize()
    ref = 2.0 * Cm.double() - 0.5 * (A.double() @ Bm.double().T)
    scale = 2.0 * Cm.double().abs() + 0.5 * (A.double().abs() @ Bm.double().abs().T)
    err = ((D.double() - ref).abs() / scale).max().item()
    assert err < (1e-5 if passes == 3 else 2e-3), err


@pytest.mark.parametrize("tri", [1, 2, 3])
@pytest.mark.parametrize("n", [384, 520])
def test_gemm_triangular(n, tri):
    """tri bit 0: only output 128-tiles on/below the diagonal are required;
    bit 1: A is upper triangular and K starts at the tile row."""
    g = torch.Generator().manual_seed(n + tri)
    A = torch.randn(n, n, generator=g)
    if tri & 2:
        A = torch.triu(A)
    A = A.cuda()
    Bm = torch.randn(n, n, generator=g).cuda()
    ah, al = split(A)
    bh, bl = split(Bm)
    D = torch.full((n, n), float("nan"), device="cuda")
    ld = ah.shape[1]
    nat.check(nat.load().ic_gemm_tn_tri(n, n, n, 1.0, ah.data_ptr(), al.data_ptr(), ld, bh.data_ptr(), bl.data_ptr(),
                                        ld, 0.0, None, None, n, D.data_ptr(), None, n, tri, nat.stream_ptr(D.device)))
    torch.cuda.synchronize()
    ref = A.double() @ Bm.double().T
    scale = A.double().abs() @ Bm.double().abs().T
    r = torch.arange(n, device="cuda")
    need = (r[None, :] // 128 <= r[:, None] // 128) if tri & 1 else torch.ones(n, n, dtype=torch.bool, device="cuda")
    err = ((D.double() - ref).abs() / scale)[need]
    assert not torch.isnan(err).any()
    assert err.max().item() < 1e-5


@pytest.mark.parametrize("tri", [0, 3])
def test_gemm_k_slabs(tri):
    """Products large enough to be split into K-slabs (m*n >= 2^26, k >= 8192),
    plain and triangular, against an fp64 product on the GPU."""
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(5 + tri)
    A = torch.randn(n, n, device="cuda", generator=g)
    if tri & 2:
        A = torch.triu(A)
    Bm = torch.randn(n, n, device="cuda", generator=g)
    ah, al = split(A)
    bh, bl = split(Bm)
    del A, Bm
    D = torch.full((n, n), float("nan"), device="cuda")
    Dl = torch.empty_like(D)
    nat.check(nat.load().ic_gemm_tn_tri(n, n, n, 1.0, ah.data_ptr(), al.data_ptr(), n, bh.data_ptr(), bl.data_ptr(),
                                        n, 0.0, None, None, n, D.data_ptr(), Dl.data_ptr(), n, tri,
                                        nat.stream_ptr(D.device)))
    torch.cuda.synchronize()
    Ad = ah.double() + al.double()
    Bd = bh.double() + bl.double()
    rows = torch.arange(0, n, 1024, device="cuda")  # sampled rows keep the fp64 check cheap
    ref = Ad[rows] @ Bd.T
    scale = Ad[rows].abs() @ Bd.abs().T
    got = D.double()[rows] + Dl.double()[rows]
    err = (got - ref).abs() / scale
    if tri & 1:
        cols = torch.arange(n, device="cuda")
        err = err[(cols[None, :] // 128) <= (rows[:, None] // 128)]
    assert not torch.isnan(err).any()
    assert err.max().item() < 1e-5


def test_gemm_cta_pair_kernel_subprocess():
    """The cta_group::2 kernel (opt-in, IC_GEMM_PAIR=1) on the GEMM cases above."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, IC_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", __file__, "-k",
                        "test_gemm_tn or test_gemm_triangular"], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def test_gemm_pair_output():
    m, n, k = 256, 128, 96
    A = torch.randn(m, k).cuda()
    Bm = torch.randn(n, k).cuda()
    ah, al = split(A)
    bh, bl = split(Bm)
    dh = torch.empty(m, n, device="cuda")
    dl = torch.empty(m, n, device="cuda")
    nat.check(nat.load().ic_gemm_tn(m, n, k, 1.0, ah.data_ptr(), al.data_ptr(), ah.shape[1], bh.data_ptr(),
                                    bl.data_ptr(), bh.shape[1], 0.0, None, None, n, dh.data_ptr(), dl.data_ptr(), n, 3,
                                    nat.stream_ptr(dh.device)))
    ref = A.double() @ Bm.double().T
    assert ((dh.double() + dl.double()) - ref).abs().max().item() < 1e-4
    # hi is TF32-exact: low 13 mantissa bits zero
    assert int((dh.view(torch.int32) & 0x1FFF).abs().max().item()) == 0


# ---------------------------------------------------------------- rotation
@pytest.mark.parametrize("name", list(C.ROT_CASES))
def test_rotate_weights(golden, name):
    c = C.ROT_CASES[name]
    W = gi.weight_outlier_cols(c["seed"], c["M"], c["N"])
    g = golden[name + "/Wrot"]
    out = np_(B.rotate_weights(cu(W), c["rot"]))
    np.testing.assert_allclose(out, g, rtol=0, atol=2e-6 * np.abs(g).max())
    out16 = np_(B.rotate_weights(cu(W).half(), c["rot"]).float())
    assert out16.shape == g.shape


@pytest.mark.parametrize("name", list(C.ROTH_CASES))
def test_rotate_hessian(golden, name):
    c = C.ROTH_CASES[name]
    H = gi.hessian_lognormal(c["seed"], c["N"], 256)
    if c["nblk"]:
        H = np.stack([H] * c["nblk"]) * np.arange(1, c["nblk"] + 1, dtype=np.float32)[:, None, None]
    g = golden[name + "/Hrot"]
    np.testing.assert_allclose(np_(B.rotate_hessian(cu(H), c["rot"])), g, rtol=0, atol=2e-6 * np.abs(g).max())


# ---------------------------------------------------------------- RTN
def _rtn_gpu(c):
    W = C.rtn_weight(c)
    Ww = B.rotate_weights(cu(W), c["rot"]) if c["rot"] else cu(W)
    gs = c["gs"] or Ww.shape[1]
    if c["bits"] == 4 and not c["asym"]:
        s = B.calculate_scales(Ww, gs, c["ratios"])
        return s, None, B.quantize_weights(Ww, s, gs)
    if c["bits"] == 4:
        s, zp = B.calculate_scales_asymmetric(Ww, gs, c["ratios"])
        return s, zp, B.quantize_weights_asymmetric(Ww, s, zp, gs)
    if not c["asym"]:
        s = B.calculate_scales_int8(Ww, c["ratios"])
        return s, None, B.quantize_weights_int8(Ww, s)
    s, zp = B.calculate_scales_int8_asymmetric(Ww, c["ratios"])
    return s, zp, B.quantize_weights_int8_asymmetric(Ww, s, zp)


@pytest.mark.parametrize("name", list(C.RTN_CASES))
def test_rtn_api(golden, name):
    c = C.RTN_CASES[name]
    s, zp, q = _rtn_gpu(c)
    assert np.array_equal(np_(s), golden[name + "/scales"])
    if zp is not None:
        assert np.array_equal(np_(zp), golden[name + "/zp"])
    assert codes_close(np_(q), golden[name + "/codes"])


@pytest.mark.parametrize("name", [k for k, c in C.RTN_CASES.items() if c["gs"] is None])
def test_rtn_fused(golden, name):
    c = C.RTN_CASES[name]
    W = C.rtn_weight(c)
    out = B.rtn_quantize_fused(cu(W), c["rot"], c["bits"], c["asym"], c["ratios"])
    assert np.array_equal(np_(out["scales"]), golden[name + "/scales"])
    if c["asym"]:
        assert np.array_equal(np_(out["zero_points"]), golden[name + "/zp"])
    assert codes_close(np_(out["codes"]), golden[name + "/codes"])
    if c["bits"] == 4:
        assert np.mean(np_(out["packed"]) != golden[name + "/packed"]) <= 2e-4
    # verify statistics match a recomputation from the outputs
    Wr = R.rotate_weights(W, c["rot"]) if c["rot"] else W
    s = golden[name + "/scales"].astype(np.float32)
    q = golden[name + "/codes"].astype(np.float32)
    zp = golden[name + "/zp"].astype(np.float32) if c["asym"] else 0.0
    mse = np.mean((Wr - (q - zp) * s).astype(np.float64) ** 2)
    assert abs(np_(out["stats"])[0] / mse - 1) < 1e-3


# ---------------------------------------------------------------- packing
@pytest.mark.parametrize("name", list(C.PACK_CASES))
def test_pack(golden, name):
    c = C.PACK_CASES[name]
    q = gi.codes(c["seed"], c["M"], c["K"])
    p = B.pack_int4(cu(q))
    assert np.array_equal(np_(p), golden[name + "/packed"])
    assert np.array_equal(np_(B.unpack_int4(p, c["K"])), q)


def test_pack_range_error():
    with pytest.raises(B.INT4PackingError):
        B.pack_int4(cu(np.array([[3, 8]], np.int8)))
    with pytest.raises(B.INT4PackingError):
        B.pack_int4(torch.tensor([[1.0, float("nan")]], device="cuda"))
    assert B.pack_int4(torch.zeros(0, 4, dtype=torch.int8, device="cuda")).shape == (0, 2)


# ---------------------------------------------------------------- inverse
@pytest.mark.parametrize("n,ns", [(100, 400), (128, 512), (384, 1024), (1000, 3000), (2048, 1024)])
def test_spd_inverse(n, ns):
    H = gi.hessian_lognormal(n, n, ns)
    Hd = R.damp(H, 0.01).astype(np.float64)
    ref = np.linalg.inv(Hd)
    out, path = B.invert_dense(cu(H), damping=0.01)
    assert path == "cholesky"
    out = np_(out).astype(np.float64)
    rel = np.abs(out - ref).max() / np.abs(ref).max()
    lapack, _ = R.invert_hessian(R.damp(H, 0.01))  # fp32 LAPACK, the reference's own arithmetic
    rel_lapack = np.abs(lapack - ref).max() / np.abs(ref).max()
    assert rel < max(8 * rel_lapack, 1e-5), (rel, rel_lapack)
    assert np.abs(out - out.T).max() <= 1e-6 * np.abs(out).max()


def test_not_pd_falls_back():
    H = -np.eye(40, dtype=np.float32)
    out, path = B.invert_dense(cu(H), damping=None)
    assert path == "inv"
    np.testing.assert_allclose(np_(out), -np.eye(40), atol=1e-6)


# ---------------------------------------------------------------- GPTQ
def test_gptq_loop_exact_given_reference_hinv(golden):
    name = "gptq4_single_block"
    c = C.GPTQ_CASES[name]
    W, _ = C.gptq_inputs(c)
    Hinv = golden[name + "/Hinv"]
    s, zp = R.gptq_row_params(W, 4)
    Wd = cu(W)
    Ww = Wd.clone()
    hh, hl = split(cu(Hinv))
    Q = torch.zeros(W.shape, dtype=torch.int8, device="cuda")
    lib = nat.load()
    M, N = W.shape
    ws = torch.empty(lib.ic_gptq_workspace_size(M, N, c["bs"], c["bs"]), dtype=torch.uint8, device="cuda")
    sc = cu(s.reshape(-1))
    zz = cu(zp.reshape(-1).astype(np.float32))
    nat.check(lib.ic_gptq_run(Ww.data_ptr(), N, Wd.data_ptr(), N, M, N, hh.data_ptr(), hl.data_ptr(), hh.shape[1],
                              c["bs"], c["bs"], sc.data_ptr(), zz.data_ptr(), -8, 7, Q.data_ptr(), N, None, 0, None,
                              None, 3, ws.data_ptr(), ws.numel(), nat.stream_ptr(Q.device)))
    assert np.array_equal(np_(Q), golden[name + "/codes"])


@pytest.mark.parametrize("name", list(C.GPTQ_CASES))
def test_gptq_api(golden, name):
    c = C.GPTQ_CASES[name]
    W, H = C.gptq_inputs(c)
    Ww = R.rotate_weights(W, c["rot"]) if c["rot"] else W
    Hr = R.rotate_hessian(H, c["rot"]) if c["rot"] else H
    r = B.gptq_quantize_layer(cu(Ww), cu(Hr), block_size=c["bs"], int_bits=c["bits"], asymmetric=c["asym"])
    assert r.method_used == "gptq_b200"
    assert np.array_equal(np_(r.scales), golden[name + "/scales"])
    if r.zero_points is not None:
        assert np.array_equal(np_(r.zero_points), golden[name + "/zp"])
    q = np_(r.quantized_W)
    assert np.mean(q == golden[name + "/codes"]) > 0.97
    zp = None if r.zero_points is None else np_(r.zero_points)
    if Hr.ndim == 2:
        p = R.proxy_loss(Ww, q, np_(r.scales).astype(np.float32), zp, Hr)
        assert abs(p / float(golden[name + "/proxy"]) - 1) < 0.01
    assert abs(r.mse / float(golden[name + "/mse"]) - 1) < 0.01


def test_gptq_cpu_tensors_roundtrip(golden):
    c = C.GPTQ_CASES["gptq8_sym"]
    W, H = C.gptq_inputs(c)
    r = B.gptq_quantize_layer(torch.from_numpy(W), torch.from_numpy(H), block_size=128, int_bits=8)
    assert r.quantized_W.device.type == "cpu" and r.quantized_W.dtype == torch.int8
    assert r.scales.dtype == torch.float16 and r.scales.shape == (W.shape[0], 1)
    assert r.zero_points is None


def test_gptq_block_size_not_multiple_of_4():
    W = gi.weight_outlier_cols(5, 16, 64)
    H = gi.hessian_lognormal(6, 64, 256)
    ref = R.gptq_quantize_layer(W, H, 10, 0.01, 4)
    r = B.gptq_quantize_layer(cu(W), cu(H), block_size=10)
    p = R.proxy_loss(W, np_(r.quantized_W), ref["scales"].astype(np.float32), ref["zero_points"], H)
    pr = R.proxy_loss(W, ref["quantized_W"], ref["scales"].astype(np.float32), ref["zero_points"], H)
    assert abs(p / pr - 1) < 0.02


@pytest.mark.parametrize("update_passes,M,N,layers", [(1, 256, 1024, 4), (3, 256, 1024, 4), (1, 512, 2048, 2)])
def test_gptq_aggregate_proxy_vs_oracle(update_passes, M, N, layers):
    """Several mid-size layers: sum of tr(E H E^T) within 0.5% of the oracle's,
    for both precisions of the trailing update."""
    tot_gpu = tot_ref = 0.0
    for seed in range(layers):
        W = gi.weight_outlier_cols(100 + seed, M, N)
        H = gi.hessian_lognormal(200 + seed, N, 2 * N)
        Wr = R.rotate_weights(W, 256)
        Hr = R.rotate_hessian(H, 256)
        ref = R.gptq_quantize_layer(Wr, Hr, 128, 0.01, 4)
        out = B.quantize_gptq_layer(cu(W).half(), cu(H), rot_size=256, want_codes=True,
                                    update_passes=update_passes)
        q = np_(out["codes"])
        assert np.array_equal(np_(out["scales"]), ref["scales"])
        assert np.array_equal(np_(B.unpack_int4(out["packed"], N)), q)
        tot_gpu += R.proxy_loss(Wr, q, ref["scales"].astype(np.float32), ref["zero_points"], Hr)
        tot_ref += R.proxy_loss(Wr, ref["quantized_W"], ref["scales"].astype(np.float32), ref["zero_points"], Hr)
    assert abs(tot_gpu / tot_ref - 1) < 0.005, tot_gpu / tot_ref


def test_gptq_layer_not_pd_reported():
    """A Hessian without a Cholesky factor: the asynchronous call reports it in
    stats[2], the checked call raises, and the C call without stats returns
    IC_ERR_NOT_PD."""
    M, N = 64, 256
    W = cu(gi.weight_outlier_cols(5, M, N)).half()
    H = -torch.eye(N, device="cuda")
    out = B.quantize_gptq_layer(W, H, rot_size=256, check=False)
    torch.cuda.synchronize()
    assert int(out["stats"][2].item()) & nat.DEV_NOT_PD
    with pytest.raises(nat.NotPositiveDefinite):
        B.quantize_gptq_layer(W, H, rot_size=256)
    lib = nat.load()
    ws = torch.empty(lib.ic_gptq_layer_workspace_size(M, N, 256), dtype=torch.uint8, device="cuda")
    packed = torch.empty(M, N // 2, dtype=torch.uint8, device="cuda")
    s16 = torch.empty(M, dtype=torch.float16, device="cuda")
    zp = torch.empty(M, dtype=torch.int8, device="cuda")
    st = lib.ic_gptq_layer(W.data_ptr(), nat.IC_F16, M, N, N, H.data_ptr(), N, None, 0, 0, 256, 4, 0, 128, 0.01, 1, None,
                           packed.data_ptr(), s16.data_ptr(), zp.data_ptr(), None, ws.data_ptr(), ws.numel(),
                           nat.stream_ptr(W.device))
    assert st == nat.IC_ERR_NOT_PD
    # a good Hessian afterwards is unaffected
    Hg = cu(gi.hessian_lognormal(6, N, 2 * N))
    assert int(B.quantize_gptq_layer(W, Hg, rot_size=256)["stats"][2].item()) == 0


def test_gptq_layers_on_streams_match_serial():
    """Layers issued through LayerStreams (two streams, own workspaces, host and
    device inputs) give the same codes, scales and statistics as the same
    layers issued one after another; a non-PD Hessian among them raises at exit."""
    shapes = [(256, 1024), (512, 512), (128, 2048)]
    ins = [(cu(gi.weight_outlier_cols(30 + i, m, n)).half(), cu(gi.hessian_lognormal(40 + i, n, 2 * n)))
           for i, (m, n) in enumerate(shapes)]
    serial = [B.quantize_gptq_layer(W, H, rot_size=256, want_codes=True) for W, H in ins]
    pool = B.LayerStreams(2)
    with pool:
        par = [pool.submit(W if i % 2 else W.cpu().pin_memory(), H, rot_size=256, want_codes=True)
               for i, (W, H) in enumerate(ins)]
    for a, b in zip(serial, par):
        assert torch.equal(a["codes"], b["codes"])
        assert torch.equal(a["packed"], b["packed"])
        assert torch.equal(a["scales"], b["scales"])
        assert torch.equal(a["stats"], b["stats"])
    with pytest.raises(nat.NotPositiveDefinite):
        with pool:
            pool.submit(*ins[0], rot_size=256)
            pool.submit(ins[1][0], -torch.eye(512, device="cuda"), rot_size=256)


def test_layer_streams_callbacks_and_errors():
    """Four lanes with pinned host inputs, twice through one pool: results match
    the serial call, ``then`` runs on the lane's stream after the layer (a copy
    to pinned host memory), and an invalid argument raises without leaving the
    pool unusable."""
    shapes = [(256, 1024), (512, 512), (128, 2048), (384, 1024), (256, 512), (512, 1024)]
    ins = [(cu(gi.weight_outlier_cols(60 + i, m, n)).half(), cu(gi.hessian_lognormal(70 + i, n, 2 * n)))
           for i, (m, n) in enumerate(shapes)]
    serial = [B.quantize_gptq_layer(W, H, rot_size=256) for W, H in ins]
    host = [torch.empty(r["packed"].shape, dtype=torch.uint8).pin_memory() for r in serial]
    pool = B.LayerStreams(4)
    for _ in range(2):
        for h in host:
            h.zero_()
        with pool:
            par = [pool.submit(W.cpu().pin_memory(), H.cpu().pin_memory(), rot_size=256,
                               then=lambda o, h=h: h.copy_(o["packed"], non_blocking=True))
                   for (W, H), h in zip(ins, host)]
        torch.cuda.synchronize()
        for a, b, h in zip(serial, par, host):
            assert torch.equal(a["packed"], b["packed"])
            assert torch.equal(a["stats"], b["stats"])
            assert torch.equal(a["packed"].cpu(), h)
    with pytest.raises(ValueError, match="int_bits"):
        with pool:
            pool.submit(*ins[0], rot_size=256, int_bits=5)
    with pool:
        again = pool.submit(*ins[1], rot_size=256)
    assert torch.equal(again["packed"], serial[1]["packed"])


def test_bounded_wait_times_out_and_context_survives():
    """Failure path without a GPU fault: a kernel waits on an mbarrier that
    nothing arrives on through the library's bounded wait; after the limit it
    records DEV_TIMEOUT in the device status word and returns, the host reads
    the bit, and the context runs a parity-checked call afterwards."""
    import ctypes
    lib = nat.load()
    st = nat.stream_ptr(torch.device("cuda", 0))
    f = ctypes.c_uint(0)
    nat.check(lib.ic_device_status(ctypes.byref(f), st))  # clear
    with pytest.raises(ValueError):
        nat.check(lib.ic_selftest_bounded_wait(10, st))
    nat.check(lib.ic_selftest_bounded_wait(20_000_000, st))  # 20 ms
    nat.check(lib.ic_device_status(ctypes.byref(f), st))
    assert f.value & nat.DEV_TIMEOUT
    nat.check(lib.ic_device_status(ctypes.byref(f), st))
    assert f.value == 0  # read-and-clear
    W, H = cu(gi.weight_outlier_cols(80, 256, 512)).half(), cu(gi.hessian_lognormal(81, 512, 1024))
    a = B.quantize_gptq_layer(W, H, rot_size=256)
    b = B.quantize_gptq_layer(W, H, rot_size=256)
    assert torch.equal(a["packed"], b["packed"]) and int(a["stats"][2].item()) == 0
    nat.check(lib.ic_device_status(ctypes.byref(f), st))
    assert f.value == 0


@pytest.mark.parametrize("M,N,bits,asym", [(300, 512, 4, False), (257, 384, 8, False), (130, 256, 8, True)])
def test_row_sharded_layer_equals_one_gpu(M, N, bits, asym):
    """Row sharding of one layer: the rows quantized in slices against the same
    H^-1 pair, concatenated, equal the one-GPU layer bit for bit (codes,
    scales, zero-points); the public entry at world size 1 is the one-GPU
    layer; a slice of no rows is handled."""
    from int_crush_converter_b200 import sharding as S
    from int_crush_converter_b200.hessian import hessian_pair, inverse_pair
    W = cu(gi.weight_outlier_cols(90 + M, M, N))
    H = cu(gi.hessian_lognormal(91 + N, N, 2 * N))
    ref = B.gptq_quantize_layer(W, H, int_bits=bits, asymmetric=asym)
    one = S.gptq_quantize_layer_row_sharded(W, H, int_bits=bits, asymmetric=asym)
    assert torch.equal(one.quantized_W, ref.quantized_W)
    assert torch.equal(one.scales, ref.scales)
    assert (one.zero_points is None) == (ref.zero_points is None)
    if ref.zero_points is not None:
        assert torch.equal(one.zero_points, ref.zero_points)
    assert one.mse == pytest.approx(ref.mse, rel=1e-12) and one.max_err == ref.max_err
    hi, lo, n = hessian_pair(H, 0, W.device, rotate=False)
    assert inverse_pair(hi, lo, n, 0.01, H_fallback=H) == "cholesky"
    for world in (2, 3):
        parts = [S._quantize_rows(W, hi, lo, *S.row_slice(M, r, world), 128, bits, asym) for r in range(world)]
        assert torch.equal(torch.cat([p[0] for p in parts]), ref.quantized_W)
        assert torch.equal(torch.cat([p[1] for p in parts]).half().reshape(M, 1), ref.scales)
        sq = sum(float(p[3]) for p in parts)
        assert sq / (M * N) == pytest.approx(ref.mse, rel=1e-12)
        assert max(float(p[4]) for p in parts) == ref.max_err
    empty = S._quantize_rows(W, hi, lo, 5, 5, 128, bits, asym)
    assert empty[0].shape == (0, N) and float(empty[3]) == 0.0


# ---------------------------------------------------------------- LDLQ / greedy / PiSO
@pytest.mark.parametrize("name", list(C.LDLQ_CASES))
def test_ldlq(golden, name):
    c = C.LDLQ_CASES[name]
    W, H = C.ldlq_inputs(c)
    Ww = R.rotate_weights(W, c["rot"]) if c["rot"] else W
    Hr = None if H is None else (R.rotate_hessian(H, c["rot"]) if c["rot"] else H)
    r = B.ldlq_quantize_layer(cu(Ww), None if Hr is None else cu(Hr), block_size=c["bs"], int_bits=c["bits"],
                              iterations=c["iters"], greedy_passes=c["greedy"])
    Hp = Hr if Hr is not None else Ww.astype(np.float64).T @ Ww.astype(np.float64) / Ww.shape[0]
    p = R.proxy_loss(Ww, np_(r.quantized_W), np_(r.scales).astype(np.float32), None, Hp)
    # 32-64 row layers: single-seed chaos of the error feedback reaches ~1.5%
    assert abs(p / float(golden[name + "/proxy"]) - 1) < 0.02


@pytest.mark.parametrize("iters,greedy", [(1, 0), (2, 1)])
def test_ldlq_aggregate_proxy_vs_oracle(iters, greedy):
    """Weight-only LDLQ on four 256x512 layers: summed tr(E H E^T) within 0.5% of the oracle's."""
    tg = tr = 0.0
    for seed in range(4):
        W = gi.weight_outlier_cols(300 + seed, 256, 512, frac=0.01, mult=30.0, std=0.015)
        Wr = R.rotate_weights(W, 256)
        ref = R.ldlq_quantize_layer(Wr, None, 128, 0.01, 4, iters, greedy)
        r = B.ldlq_quantize_layer(cu(Wr), None, block_size=128, iterations=iters, greedy_passes=greedy)
        Hp = Wr.astype(np.float64).T @ Wr.astype(np.float64) / Wr.shape[0]
        tg += R.proxy_loss(Wr, np_(r.quantized_W), np_(r.scales).astype(np.float32), None, Hp)
        tr += R.proxy_loss(Wr, ref["quantized_W"], ref["scales"].astype(np.float32), None, Hp)
    assert abs(tg / tr - 1) < 0.005, tg / tr


@pytest.mark.parametrize("name", list(C.GREEDY_CASES))
def test_greedy(golden, name):
    c = C.GREEDY_CASES[name]
    W, Q, S, H = C.greedy_inputs(c)
    qm = (-8, 7) if c["bits"] == 4 else (-128, 127)
    out = np_(B.greedy_local_search(cu(W), cu(Q), cu(S), cu(H), c["passes"], *qm))
    g = golden[name + "/codes"]
    assert np.mean(out == g) > 0.99
    pg = R.proxy_loss(W, g, np.ones((W.shape[0], 1)), None, H)  # scales are per-element here
    E_g = g.astype(np.float64) * S - W
    E_o = out.astype(np.float64) * S - W
    assert np.einsum("ij,ij->", E_o @ H, E_o) <= np.einsum("ij,ij->", E_g @ H, E_g) * 1.005
    del pg


@pytest.mark.parametrize("name", list(C.PISO_CASES))
def test_piso(golden, name):
    c = C.PISO_CASES[name]
    W, hd = C.piso_inputs(c)
    f = dict(int8=B.compute_piso_scales_int8, int4=B.compute_piso_scales_int4,
             int8_asym=B.compute_piso_scales_int8_asymmetric, int4_asym=B.compute_piso_scales_int4_asymmetric)[c["kind"]]
    o = f(cu(W), cu(hd))
    if isinstance(o, tuple):
        assert np.mean(np_(o[0]) == golden[name + "/scales"]) >= 0.95
        assert np.mean(np_(o[1]) == golden[name + "/zp"]) >= 0.95
    else:
        assert np.mean(np_(o) == golden[name + "/scales"]) >= 0.95


def test_sharded_layers_world1_match_serial():
    """sharding.quantize_layers_sharded (the multi-GPU entry, here one rank) gives
    the serial results for every layer."""
    from int_crush_converter_b200 import sharding as S
    layers = {f"l{i}": (cu(gi.weight_outlier_cols(60 + i, m, n)).half(), cu(gi.hessian_lognormal(70 + i, n, 2 * n)))
              for i, (m, n) in enumerate([(256, 512), (128, 1024), (384, 256)])}
    got = S.quantize_layers_sharded(layers, 0, 1, streams=2, rot_size=256)
    assert set(got) == set(layers)
    for k, (W, H) in layers.items():
        ref = B.quantize_gptq_layer(W, H, rot_size=256)
        assert torch.equal(ref["packed"], got[k]["packed"])
        assert torch.equal(ref["scales"], got[k]["scales"])


@pytest.mark.parametrize("bs", [64, 96])
def test_gptq_layer_block_sizes_vs_oracle(bs):
    """The fused layer at block sizes that divide 128 (Hinv's upper tiles are not
    written) and that do not (they are mirrored): proxy within 1% of the oracle."""
    M, N = 256, 1024
    W = gi.weight_outlier_cols(80 + bs, M, N)
    H = gi.hessian_lognormal(90 + bs, N, 2 * N)
    Wr = R.rotate_weights(W, 256)
    Hr = R.rotate_hessian(H, 256)
    ref = R.gptq_quantize_layer(Wr, Hr, bs, 0.01, 4)
    out = B.quantize_gptq_layer(cu(W).half(), cu(H), rot_size=256, block_size=bs, want_codes=True)
    q = np_(out["codes"])
    assert np.array_equal(np_(out["scales"]), ref["scales"])
    p = R.proxy_loss(Wr, q, ref["scales"].astype(np.float32), ref["zero_points"], Hr)
    pr = R.proxy_loss(Wr, ref["quantized_W"], ref["scales"].astype(np.float32), ref["zero_points"], Hr)
    assert abs(p / pr - 1) < 0.01, p / pr


@pytest.mark.parametrize("bits,asym,N,dtype,h_rot", [
    (8, False, 1024, "half", False),     # INT8 codes, no packing
    (4, True, 1024, "half", False),      # asymmetric INT4
    (4, False, 1000, "half", False),     # ragged width: zero padding to 1024
    (4, False, 768, "bfloat16", False),  # bf16 weights
    (4, False, 512, "half", True),       # Hessian passed already rotated
])
def test_gptq_layer_variants_vs_oracle(bits, asym, N, dtype, h_rot):
    """Fused layer call across the pipeline's variants: scales and zero-points
    equal to the oracle's, packed bytes equal to the codes, proxy within 1%."""
    M = 192
    W = gi.weight_outlier_cols(300 + N + bits, M, N)
    H = gi.hessian_lognormal(400 + N + bits, N, 2 * N)
    Wt = torch.from_numpy(W).to(getattr(torch, dtype))
    Wq = Wt.float().numpy()  # the values the device sees
    Wr = R.rotate_weights(Wq, 256)
    Hr = R.rotate_hessian(H, 256)
    ref = R.gptq_quantize_layer(Wr, Hr, 128, 0.01, bits, asymmetric=asym)
    out = B.quantize_gptq_layer(Wt.cuda(), cu(Hr if h_rot else H), rot_size=256, int_bits=bits,
                                asymmetric=asym, h_rotated=h_rot, want_codes=True)
    q = np_(out["codes"])
    npad = Wr.shape[1]
    assert q.shape == (M, npad)
    assert np.array_equal(np_(out["scales"]), ref["scales"])
    if ref["zero_points"] is not None and out["zero_points"] is not None:
        assert np.array_equal(np_(out["zero_points"]).reshape(-1), np.asarray(ref["zero_points"]).reshape(-1))
    if bits == 4:
        assert np.array_equal(np_(B.unpack_int4(out["packed"], npad)), q)
    p = R.proxy_loss(Wr, q, ref["scales"].astype(np.float32), ref["zero_points"], Hr)
    pr = R.proxy_loss(Wr, ref["quantized_W"], ref["scales"].astype(np.float32), ref["zero_points"], Hr)
    assert abs(p / pr - 1) < 0.01, p / pr


def test_fused_calls_sanitize_outliers_like_the_pipeline():
    """pipeline.py:527-537 zeroes |w| > 1000 before rotating; the fused layer
    calls do the same (the plain rotate_weights mirror does not)."""
    M, N = 128, 512
    W = gi.weight_outlier_cols(500, M, N)
    W[3, 7] = 5000.0
    W[10, 100] = -2000.0
    W[20, 300] = np.inf
    Ws = np.where(np.abs(W) > 1000.0, 0.0, W).astype(np.float32)
    H = gi.hessian_lognormal(501, N, 2 * N)
    Wr = R.rotate_weights(Ws, 256)
    Hr = R.rotate_hessian(H, 256)
    ref = R.gptq_quantize_layer(Wr, Hr, 128, 0.01, 4)
    out = B.quantize_gptq_layer(cu(W), cu(H), rot_size=256, want_codes=True)
    assert np.array_equal(np_(out["scales"]), ref["scales"])
    rt = B.rtn_quantize_fused(cu(W), 256, int_bits=4)
    s_ref = R.calculate_scales(Wr, Wr.shape[1])
    assert np.array_equal(np_(rt["scales"]).reshape(-1), np.asarray(s_ref).reshape(-1))
    assert np.isfinite(np_(B.rotate_weights(cu(Ws), 256))).all()
    assert not np.isfinite(np_(B.rotate_weights(cu(W), 256))).all()  # the mirror keeps the reference's semantics


def test_smoothing_mirrors_match_golden(golden):
    W, H, s = C.smooth_inputs(C.SMOOTH_CASES["smooth_basic"])
    assert np.array_equal(np_(B.apply_smoothing_to_weight(cu(W), cu(s))), golden["smooth_basic/W_smooth"])
    assert np.array_equal(np_(B._transform_hessian_for_smoothquant(cu(H), cu(s))), golden["smooth_basic/H_smooth"])


@pytest.mark.parametrize("order", ["smooth_then_rotate", "pipeline"])
def test_gptq_layer_with_smoothrot_vs_oracle(order):
    """The fused SmoothRot pre-step (W * s and H / (s_i s_j) in the rotation
    loads) against the oracle's smooth -> rotate -> GPTQ; with order
    "pipeline" the Hessian takes the reference pipeline's own sequence for a
    SmoothRot layer, rotate -> smooth -> rotate (pipeline.py:721-723, 766-770)."""
    M, N = 256, 1024
    W = gi.weight_outlier_cols(600, M, N)
    H = gi.hessian_lognormal(601, N, 2 * N)
    s = np.exp(np.random.default_rng(602).normal(0.0, 0.5, N)).astype(np.float32)
    Wr = R.rotate_weights(R.apply_smoothing_to_weight(W, s), 256)
    if order == "pipeline":
        Hr = R.rotate_hessian(R.transform_hessian_for_smoothquant(R.rotate_hessian(H, 256), s), 256)
    else:
        Hr = R.rotate_hessian(R.transform_hessian_for_smoothquant(H, s), 256)
    ref = R.gptq_quantize_layer(Wr, Hr, 128, 0.01, 4)
    out = B.quantize_gptq_layer(cu(W), cu(H), rot_size=256, want_codes=True,
                                smoothing=cu(s), smoothing_order=order)
    q = np_(out["codes"])
    assert np.array_equal(np_(out["scales"]), ref["scales"])
    p = R.proxy_loss(Wr, q, ref["scales"].astype(np.float32), ref["zero_points"], Hr)
    pr = R.proxy_loss(Wr, ref["quantized_W"], ref["scales"].astype(np.float32), ref["zero_points"], Hr)
    assert abs(p / pr - 1) < 0.01, p / pr
