"""The reference pipeline (converter.pipeline.quantize_model) run unchanged with
this package installed in place of its per-layer functions
(int_crush_converter_b200.pipeline_hook), against the same pipeline on its
own CPU code in a child process that sees no GPU.

A tiny synthetic DiT-style model (FFN pairs that SmoothRot detects, an
attention layer, a width that rotation pads) and a calibration dict (Hessians,
per-channel activation amax, sample count) go through three configurations:
GPTQ INT4 rot256 with SmoothQuant (SmoothRot on the FFN down layers), RTN
INT8 rot64 with the clipping-ratio search, and LDLQ INT4 rot256 with 2
iterations and a greedy pass.  The outputs must have the same tensors (names,
dtypes, shapes) and metadata; GPTQ / RTN scales and SmoothRot factors within
1 fp16 ulp; RTN codes equal up to
+-1 on <= 0.1%; per-layer MSE of the pipeline's quality report within 2% for
GPTQ / LDLQ (small single layers; the aggregate bar of the other tests is
0.5%) and 1e-4 for RTN.  Needs the reference installed under baseline/_ref.
"""

import json
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "converter")),
                                 reason="the reference is not installed under baseline/_ref")]

SHAPES = {
    "double_blocks.0.img_mlp.0.weight": (512, 256),
    "double_blocks.0.img_mlp.2.weight": (256, 512),
    "double_blocks.0.img_attn.qkv.weight": (768, 256),
    "double_blocks.0.img_attn.proj.weight": (256, 384),  # padded to 512 by rotation
    "single_blocks.0.linear1.weight": (512, 256),
    "single_blocks.0.linear2.weight": (256, 512),
}

CONFIGS = {
    "gptq_int4_smoothrot": dict(rot_size=256, quant_method="gptq", int_bits=4, smoothquant=True, smooth_alpha=0.5),
    "rtn_int8_clip": dict(rot_size=64, quant_method="rtn", int_bits=8, clipping_ratios=[0.8, 0.85, 0.9, 0.95, 1.0]),
    "ldlq_int4": dict(rot_size=256, quant_method="ldlq", int_bits=4, ldlq_iterations=2, greedy_passes=1),
}

RUN = r"""
import json, sys, torch
sys.path.insert(0, {ref!r})
sys.path.insert(0, {root!r})
import converter.pipeline as P
from converter.types import QuantizeConfig
P.load_calibration = lambda path: torch.load(path)
if {hook!r}:
    from int_crush_converter_b200 import pipeline_hook
    pipeline_hook.install(P)
P.quantize_model(QuantizeConfig(**json.loads({cfg!r})))
"""


def _model(tmp):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(11)
    sd, hess, amax = {}, {}, {}
    for name, (m, n) in SHAPES.items():
        W = torch.randn(m, n, generator=g) * 0.02
        W[:, int(torch.randint(0, n, (1,), generator=g))] *= 20.0
        sd[name] = W.half()
        X = torch.randn(1024, n, generator=g) * torch.exp(torch.randn(n, generator=g))
        hess[name[:-len(".weight")]] = X.T @ X / 1024
        amax[name[:-len(".weight")]] = X.abs().amax(0)
    mp = os.path.join(tmp, "model.in.safetensors")
    save_file(sd, mp)
    cp = os.path.join(tmp, "cal.pt")
    torch.save({"hessians": hess, "amax_per_channel": amax, "metadata": {"num_samples": 1024}}, cp)
    return mp, cp


def _run(tmp, tag, cfg, hook):
    out = os.path.join(tmp, tag)
    full = dict(cfg, output_dir=out, quality_report_path=os.path.join(out, "report.json"))
    code = RUN.format(ref=REF, root=ROOT, hook=hook, cfg=json.dumps(full))
    env = dict(os.environ)
    if not hook:
        env["CUDA_VISIBLE_DEVICES"] = ""  # the reference's own CPU code path
    subprocess.run([sys.executable, "-c", code], env=env, check=True, cwd=ROOT)
    return out


def _load(out):
    from safetensors import safe_open
    tensors, meta = {}, {}
    with safe_open(os.path.join(out, "model.safetensors"), "pt") as f:
        meta = f.metadata()
        for k in f.keys():
            tensors[k] = f.get_tensor(k)
    report = json.load(open(os.path.join(out, "report.json")))
    return tensors, meta, report


def _layer_mse(report):
    layers = report["layers"] if isinstance(report, dict) and "layers" in report else report
    return {r["name"]: r for r in layers}


@pytest.mark.parametrize("tag", list(CONFIGS))
def test_reference_pipeline_with_the_b200_path(tmp_path, tag):
    tmp = str(tmp_path)
    mp, cp = _model(tmp)
    cfg = dict(CONFIGS[tag], input_path=mp, calibration_path=cp)
    ref_t, ref_m, ref_r = _load(_run(tmp, "ref", cfg, False))
    got_t, got_m, got_r = _load(_run(tmp, "b200", cfg, True))
    assert sorted(got_t) == sorted(ref_t)
    assert got_m == ref_m
    for k, r in ref_t.items():
        g = got_t[k]
        assert g.dtype == r.dtype and g.shape == r.shape, k
        # GPTQ and RTN scales come from the weights alone; LDLQ's are least-squares
        # fits to its codes (ldlq.py:262-265), covered by the MSE check below
        if (k.endswith("_scale") and tag != "ldlq_int4") or k.endswith("_smoothrot_factors"):
            ulp = (g.view(torch.int16).int() - r.view(torch.int16).int()).abs().max().item()
            assert ulp <= 1, (k, ulp)
        elif tag == "rtn_int8_clip" and g.dtype == torch.int8 and k.endswith(".weight"):
            d = (g.int() - r.int()).abs()
            assert d.max().item() <= 1 and d.float().mean().item() <= 1e-3, k
    rm, gm = _layer_mse(ref_r), _layer_mse(got_r)
    assert sorted(rm) == sorted(gm)
    tol = 1e-4 if tag == "rtn_int8_clip" else 0.02
    for name in rm:
        assert gm[name]["method"].endswith("_b200") or gm[name]["method"] == rm[name]["method"], name
        a, b = gm[name]["mse"], rm[name]["mse"]
        assert abs(a / b - 1) < tol, (name, a, b)
    # the FFN down layers went through SmoothRot on both sides
    assert any(k.endswith("_smoothrot_factors") for k in ref_t) == (tag == "gptq_int4_smoothrot")
