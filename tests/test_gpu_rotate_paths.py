"""The rot = 256 row rotation on two groups per 16-lane team (packed fp32
pairs, shared-memory transpose; the default) against the one-group register
kernel (IC_ROT_PAIR=0), each in a child process: weights in fp16 / bf16 / fp32
with ragged widths, 2-D Hessians with padding rows, a 3-D block-diagonal
Hessian, and whole GPTQ layers with outliers above the sanitize clamp and the
SmoothRot pre-step (weight and Hessian smoothing fused into the rotations).
Every output must be bit-identical."""

import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys, numpy as np, torch
sys.path.insert(0, {root!r})
import int_crush_converter_b200 as B
from int_crush_converter_b200 import _native as nat
lib = nat.load()
st = nat.stream_ptr(torch.device("cuda"))
g = torch.Generator(device="cuda").manual_seed(17)
out = {{}}
codes = {{"float": 0, "half": 1, "bfloat16": 2}}
for k, (M, N, dt) in enumerate([(64, 4096, "half"), (48, 1000, "bfloat16"), (40, 16384, "float"), (33, 512, "half")]):
    W = (torch.randn(M, N, device="cuda", generator=g) * 0.02).to(getattr(torch, dt))
    npad = (N + 255) // 256 * 256
    o = torch.full((M, npad), float("nan"), device="cuda")
    nat.check(lib.ic_rotate_weights(W.data_ptr(), codes[dt], M, N, N, 256, o.data_ptr(), npad, st), "rotw")
    out[f"w{{k}}"] = o.cpu().numpy()
for k, n in enumerate([300, 1024, 4096]):
    X = torch.randn(2 * n, n, device="cuda", generator=g)
    H = X.T @ X / (2 * n)
    npad = (n + 255) // 256 * 256
    hi = torch.full((npad, npad), float("nan"), device="cuda")
    lo = torch.full((npad, npad), float("nan"), device="cuda")
    nat.check(lib.ic_rotate_hessian(H.data_ptr(), 1, n, n, 256, hi.data_ptr(), lo.data_ptr(), npad, st), "roth")
    out[f"h{{k}}"] = np.stack([hi.cpu().numpy(), lo.cpu().numpy()])
H3 = torch.randn(3, 512, 512, device="cuda", generator=g)
H3 = H3 @ H3.transpose(1, 2)
hi = torch.empty(3, 512, 512, device="cuda")
lo = torch.empty(3, 512, 512, device="cuda")
nat.check(lib.ic_rotate_hessian(H3.data_ptr(), 3, 512, 512, 256, hi.data_ptr(), lo.data_ptr(), 512, st), "roth3")
out["h3d"] = np.stack([hi.cpu().numpy(), lo.cpu().numpy()])
for k, (M, N) in enumerate([(256, 1024), (128, 768)]):
    W = torch.randn(M, N, device="cuda", generator=g) * 0.02
    W[3, 5] = 2000.0  # zeroed by the outlier sanitize
    X = torch.randn(2 * N, N, device="cuda", generator=g) * torch.exp(torch.randn(N, device="cuda", generator=g))
    H = X.T @ X / (2 * N)
    s = torch.exp(torch.randn(N, device="cuda", generator=g) * 0.5)
    r = B.quantize_gptq_layer(W.half(), H, 256, want_codes=True, smoothing=s)
    torch.cuda.synchronize()
    out[f"g{{k}}_codes"] = r["codes"].cpu().numpy()
    out[f"g{{k}}_scales"] = r["scales"].cpu().view(torch.int16).numpy()
np.savez({path!r}, **out)
"""


def _run(mode: str, path: str):
    env = dict(os.environ)
    env.pop("IC_ROT_PAIR", None)
    if mode:
        env["IC_ROT_PAIR"] = mode
    subprocess.run([sys.executable, "-c", CHILD.format(root=ROOT, path=path)], env=env, check=True, cwd=ROOT)
    return np.load(path)


def test_rotate_pair_kernel_bit_identical(tmp_path):
    a = _run("", str(tmp_path / "pair.npz"))
    b = _run("0", str(tmp_path / "regs.npz"))
    assert sorted(a.files) == sorted(b.files)
    for k in a.files:
        x, y = a[k], b[k]
        assert not np.isnan(x).any(), k
        assert np.array_equal(x.view(np.uint8), y.view(np.uint8)), k
