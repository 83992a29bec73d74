"""The reference's GPU low-rank greedy search (greedy_lowrank_triton,
greedy.py:384-479) on this path: the randomized decomposition against an exact
eigendecomposition, one device pass sequence against the oracle restatement
given the same decomposition, the full-rank fallback, and the LDLQ option.

Bars: the leading eigenvalues within 1e-4 relative and their eigenvectors
aligned to 1e-4; codes >= 99.9% equal to the oracle's (the device sums
err_lr . (s U_j) in fp32 from a 3xTF32 projection, the oracle in fp64 then
fp32, so near-ties may split) with the same number of passes, and the proxy
tr(E H E^T) within 0.1%."""

import numpy as np
import pytest
import torch

from oracle import cpu_ref as R

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import int_crush_converter_b200 as B
    from int_crush_converter_b200 import greedy as G


def _problem(M, N, spikes, seed):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, N)) * 0.015).astype(np.float32)
    cols = rng.choice(N, spikes, replace=False)
    W[:, cols] *= 30.0
    H = (W.T.astype(np.float64) @ W.astype(np.float64) / M).astype(np.float32)
    H += np.eye(N, dtype=np.float32) * np.float32(0.01 * np.diag(H).mean())
    s = (np.abs(W).max(1, keepdims=True) / 7).astype(np.float32)
    Q = np.clip(np.rint(W / s), -8, 7).astype(np.int8)
    S = np.ascontiguousarray(np.broadcast_to(s, (M, N)))
    return W, H, Q, S


def test_lowrank_decomposition_matches_eigh():
    W, H, _, _ = _problem(256, 512, 4, 1)
    s_k, U_k, k, ok = G.lowrank_decompose(torch.from_numpy(H).cuda(), 0.01)
    ev, V = np.linalg.eigh(H.astype(np.float64))
    ev, V = ev[::-1], V[:, ::-1]
    k_ref = int((ev > ev[0] * 0.01).sum())
    assert ok and k == k_ref == 4
    s = s_k.cpu().numpy().astype(np.float64)
    assert np.max(np.abs(s - ev[:k]) / ev[:k]) < 1e-4
    align = np.abs(U_k.cpu().numpy().astype(np.float64).T @ V[:, :k])
    assert np.max(np.abs(np.diag(align) - 1.0)) < 1e-4


def test_lowrank_passes_vs_oracle_same_decomposition():
    W, H, Q, S = _problem(384, 1024, 6, 2)
    Hc = torch.from_numpy(H).cuda()
    s_k, U_k, k, ok = G.lowrank_decompose(Hc, 0.01)
    assert ok
    dec = (s_k.cpu().numpy(), U_k.cpu().numpy())
    q_dev, k_dev, used = G.greedy_lowrank(torch.from_numpy(W).cuda(), torch.from_numpy(Q).cuda(),
                                          torch.from_numpy(S).cuda(), Hc, 8, -8, 7, decomposition=dec)
    torch.cuda.synchronize()
    assert used and k_dev == k
    q_ref, runs = R.greedy_lowrank_given(W, Q, S, H, dec[0], dec[1], 8, -8, 7)
    assert G.greedy_lowrank.passes_run == runs
    q = q_dev.cpu().numpy()
    assert np.mean(q == q_ref) >= 0.999

    def proxy(codes):
        E = codes.astype(np.float64) * S - W
        return float(((E @ H.astype(np.float64)) * E).sum())

    assert abs(proxy(q) / proxy(q_ref) - 1) < 1e-3
    assert proxy(q) < proxy(Q)


def test_lowrank_falls_back_to_full_rank():
    rng = np.random.default_rng(3)
    M, N = 128, 256
    W = (rng.standard_normal((M, N)) * 0.02).astype(np.float32)
    H = np.eye(N, dtype=np.float32) + np.float32(1e-3) * np.ones((N, N), dtype=np.float32)  # flat spectrum
    s = (np.abs(W).max(1, keepdims=True) / 7).astype(np.float32)
    Q = np.clip(np.rint(W / s), -8, 7).astype(np.int8)
    S = np.ascontiguousarray(np.broadcast_to(s, (M, N)))
    q, k, used = G.greedy_lowrank(torch.from_numpy(W).cuda(), torch.from_numpy(Q).cuda(),
                                  torch.from_numpy(S).cuda(), torch.from_numpy(H).cuda(), 2, -8, 7)
    assert not used
    q_full = B.greedy.greedy_local_search(torch.from_numpy(W).cuda(), torch.from_numpy(Q).cuda(),
                                          torch.from_numpy(S).cuda(), torch.from_numpy(H).cuda(), 2, -8, 7)
    assert torch.equal(q.cpu(), q_full.cpu())


def test_ldlq_with_lowrank_greedy():
    """ldlq_quantize_layer(greedy_lowrank=True) takes the low-rank search
    (the weight-only Hessian of a layer with outlier columns has a few
    dominant eigenpairs): same result layout and a weight error of the same
    order as the full-rank search's (the two searches differ: the low-rank one
    sees the Hessian's off-diagonal part only through its leading
    eigenpairs)."""
    W, _, _, _ = _problem(512, 1024, 4, 4)
    Wc = torch.from_numpy(W).cuda()
    full = B.ldlq_quantize_layer(Wc, None, int_bits=4, iterations=1, greedy_passes=4, greedy_lowrank=False)
    low = B.ldlq_quantize_layer(Wc, None, int_bits=4, iterations=1, greedy_passes=4, greedy_lowrank=True)
    assert low.quantized_W.shape == full.quantized_W.shape and low.quantized_W.dtype == torch.int8
    assert low.scales.shape == full.scales.shape and low.fallbacks == full.fallbacks
    assert np.isfinite(low.mse) and low.mse <= full.mse * 1.5
