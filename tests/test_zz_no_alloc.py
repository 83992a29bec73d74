"""ic_gptq_run_noalloc: the GPTQ column loop for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc: their device memory is owned (and capped)
by another allocator, or an allocation is not acceptable on their
latency-critical path.  This entry point keeps its scratch in a static device
array inside the library instead of a caller workspace.  The test calls it
through the C ABI twice in a row and checks both results against the regular
workspace entry point, ic_gptq_run, on the same inputs (the loop is
deterministic, so codes and statistics must match exactly), and checks that an
oversized shape is rejected with a clear error.  It sits in a file of its own
that pytest collects last.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(M, N, seed):
    from tests.golden import inputs as gi
    import int_crush_converter_b200 as B
    from int_crush_converter_b200._dev import split
    W = torch.from_numpy(gi.weight_outlier_cols(seed, M, N)).cuda()
    H = torch.from_numpy(gi.hessian_lognormal(seed + 1, N, 2 * N)).cuda()
    Hinv, _ = B.invert_dense(H, damping=0.01)
    hi, lo = split(Hinv.contiguous())
    return W, hi, lo


def _run(fn_name, W, hi, lo, bs, sb, ws=None):
    from int_crush_converter_b200 import _native as nat
    lib = nat.load()
    M, N = W.shape
    scale = torch.empty(M, device="cuda")
    zp = torch.empty(M, device="cuda")
    nat.check(lib.ic_gptq_row_params(W.data_ptr(), M, N, N, 4, 0, scale.data_ptr(), zp.data_ptr(),
                                     nat.stream_ptr(W.device)))
    Wk = W.clone()
    Q = torch.zeros(M, N, dtype=torch.int8, device="cuda")
    rsq = torch.empty(M, dtype=torch.float64, device="cuda")
    rmx = torch.empty(M, dtype=torch.float32, device="cuda")
    args = [Wk.data_ptr(), N, W.data_ptr(), N, M, N, hi.data_ptr(), lo.data_ptr(), hi.shape[1], bs, sb,
            scale.data_ptr(), zp.data_ptr(), -8, 7, Q.data_ptr(), N, None, 0, rsq.data_ptr(), rmx.data_ptr(), 3]
    if fn_name == "ic_gptq_run":
        args += [ws.data_ptr(), ws.numel()]
    status = getattr(lib, fn_name)(*args, nat.stream_ptr(W.device))
    nat.check(status, fn_name)
    torch.cuda.synchronize()
    return Q.cpu().numpy(), rsq.sum().item(), rmx.max().item()


def test_noalloc_matches_workspace_entry_twice():
    from int_crush_converter_b200 import _native as nat
    lib = nat.load()
    # the last case has a block size that is not a multiple of 4, which carves
    # the staging slices of the far update from the array as well
    for (M, N, bs, sb, seed) in [(512, 1024, 128, 512, 3), (300, 640, 64, 256, 4), (300, 640, 6, 6, 5)]:
        W, hi, lo = _inputs(M, N, seed)
        ws = torch.empty(lib.ic_gptq_workspace_size(M, N, bs, sb), dtype=torch.uint8, device="cuda")
        ref = _run("ic_gptq_run", W, hi, lo, bs, sb, ws)
        for _ in range(2):  # the shared scratch keeps the previous call's contents
            got = _run("ic_gptq_run_noalloc", W, hi, lo, bs, sb)
            assert np.array_equal(got[0], ref[0])
            assert got[1] == ref[1] and got[2] == ref[2]


def test_noalloc_rejects_oversized_shape():
    from int_crush_converter_b200 import _native as nat
    lib = nat.load()
    M, N = 65536, 2048
    assert lib.ic_gptq_workspace_size(M, N, 128, 1024) > (32 << 20)
    status = lib.ic_gptq_run_noalloc(None, N, None, N, M, N, None, None, N, 128, 1024, None, None, -8, 7,
                                     None, N, None, 0, None, None, 3, nat.stream_ptr(torch.device("cuda")))
    assert status == nat.IC_ERR_UNSUPPORTED
    assert "scratch" in nat.last_error()
    # empty and negative shapes: nothing to do, the same answer as the workspace entry point
    for m, n in [(0, N), (-3, N), (4, -1)]:
        args = [None, N, None, N, m, n, None, None, N, 128, 1024, None, None, -8, 7, None, N, None, 0, None,
                None, 3]
        scale = torch.empty(4, device="cuda")
        args[11] = scale.data_ptr()
        a = lib.ic_gptq_run_noalloc(*args, nat.stream_ptr(torch.device("cuda")))
        b = lib.ic_gptq_run(*args, None, 0, nat.stream_ptr(torch.device("cuda")))
        assert a == b == nat.IC_OK
