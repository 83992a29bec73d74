"""The fused-RTN kernels against each other, each selected in a child process
with IC_RTN_FAST: the paired kernel (default; two chunks per thread on the
packed fp32 pair instructions), the fast kernel (=1; one scale per row,
rot 16 / 64 / 256, deferred Hadamard scaling, shared-memory transpose) and the
register kernel (=0).  Codes, packed bytes, scales, zero-points and verify
statistics must be bit-identical on every mode (INT4/INT8,
symmetric/asymmetric, clipping-ratio search incl. small ratios, padding, outliers above the
sanitize clamp, NaN rows, fp16/bf16/fp32 inputs)."""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RATIOS = [0.8, 0.85, 0.9, 0.95, 1.0]
CASES = [
    # (M, N, rot, bits, asym, ratios, dtype)
    (64, 4096, 256, 4, False, None, "half"),
    (64, 4096, 256, 4, True, None, "bfloat16"),
    (48, 1000, 256, 4, False, RATIOS, "float"),
    (96, 3072, 64, 8, False, RATIOS, "half"),
    (32, 3072, 64, 8, True, RATIOS, "half"),
    (40, 200, 64, 4, False, None, "half"),
    (40, 512, 16, 8, True, None, "float"),
    (16, 4096, 16, 4, True, RATIOS, "half"),
    (48, 3072, 64, 8, False, RATIOS, "bfloat16"),
    (24, 2048, 256, 4, False, RATIOS, "half"),
    (24, 1024, 64, 8, True, None, "float"),
    # ratios small enough that |v / s| exceeds the range of the uncorrected quotient
    (32, 3072, 64, 8, False, [0.3, 0.6, 1.0], "half"),
    (32, 4096, 256, 8, True, [0.5, 1.0], "half"),
]

CHILD = r"""
import sys, numpy as np, torch
sys.path.insert(0, {root!r})
import int_crush_converter_b200 as B
from tests.golden import inputs as gi
out = {{}}
for k, (M, N, rot, bits, asym, ratios, dt) in enumerate({cases!r}):
    W = gi.weight_heavy_tail(900 + k, M, N)
    W[1] = 0.0
    W[2, 3] = 1500.0          # zeroed by the outlier sanitize
    W[3, 7] = float("nan")    # a NaN row
    W[4] = -np.abs(W[4]) - 0.01
    Wt = torch.from_numpy(W).cuda().to(getattr(torch, dt))
    o = B.rtn_quantize_fused(Wt, rot, int_bits=bits, asymmetric=asym, clipping_ratios=ratios,
                             want_codes=True, want_packed=(bits == 4))
    torch.cuda.synchronize()
    for key in ("codes", "packed", "scales", "zero_points"):
        if o[key] is not None:
            t = o[key].cpu()
            out[f"{{k}}/{{key}}"] = (t.view(torch.int16) if t.dtype == torch.float16 else t).numpy()
    out[f"{{k}}/stats"] = o["stats"].cpu().numpy()
np.savez({path!r}, **out)
"""


def _run(mode: str, path: str):
    env = dict(os.environ)
    env.pop("IC_RTN_FAST", None)
    if mode:
        env["IC_RTN_FAST"] = mode
    code = CHILD.format(root=ROOT, cases=CASES, path=path)
    subprocess.run([sys.executable, "-c", code], env=env, check=True, cwd=ROOT)
    return np.load(path)


@pytest.mark.parametrize("mode", ["", "1"])
def test_rtn_kernels_bit_identical_to_register_kernel(tmp_path, mode):
    a = _run(mode, str(tmp_path / "a.npz"))
    b = _run("0", str(tmp_path / "regs.npz"))
    assert sorted(a.files) == sorted(b.files)
    for k in a.files:
        x, y = a[k], b[k]
        if k.endswith("stats"):
            both_nan = np.isnan(x) & np.isnan(y)
            assert np.array_equal(x[~both_nan], y[~both_nan]), (k, x, y)
        else:
            assert np.array_equal(x, y), k
