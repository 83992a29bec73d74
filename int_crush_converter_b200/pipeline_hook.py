"""Install the B200 path into the reference pipeline (converter/pipeline.py).

The pipeline's per-layer loop (pipeline.py:511-1113) calls the per-layer
functions by the names it imported at module level (pipeline.py:18-47).
:func:`install` rebinds those names in the pipeline module to this package's
functions -- same signatures, arguments, returns and errors -- so that
``converter.pipeline.quantize_model`` and the CLI run unchanged on the GPU;
:func:`uninstall` restores the previous bindings.  Everything else in the
pipeline (safetensors I/O, calibration loading, SmoothRot pair detection, the
PermuQuant decision, the bad-scale repair, output layout and metadata) stays
the reference's own code.
"""

from __future__ import annotations

import importlib

# names pipeline.py imports and calls per layer, with their home in this package
HOOKED = (
    "rotate_weights", "rotate_hessian",
    "calculate_scales", "quantize_weights", "calculate_scales_int8", "quantize_weights_int8",
    "calculate_scales_asymmetric", "quantize_weights_asymmetric", "calculate_scales_int8_asymmetric",
    "quantize_weights_int8_asymmetric",
    "pack_int4",
    "gptq_quantize_layer", "gptq_quantize_layer_rtn",
    "ldlq_quantize_layer",
    "compute_piso_scales_int8", "compute_piso_scales_int4_asymmetric",
    "compute_smoothing_factors", "compute_smoothing_from_hessian_diag", "apply_smoothing_to_weight",
    "sweep_alpha", "decompose_weight",
)


def install(pipeline=None) -> dict:
    """Rebind the per-layer functions of ``pipeline`` (default: the importable
    ``converter.pipeline``) to this package's; returns the previous bindings."""
    import int_crush_converter_b200 as B
    if pipeline is None:
        pipeline = importlib.import_module("converter.pipeline")
    saved = {}
    for name in HOOKED:
        if hasattr(pipeline, name):
            saved[name] = getattr(pipeline, name)
            setattr(pipeline, name, getattr(B, name))
    return saved


def uninstall(saved: dict, pipeline=None) -> None:
    """Restore the bindings :func:`install` returned."""
    if pipeline is None:
        pipeline = importlib.import_module("converter.pipeline")
    for name, fn in saved.items():
        setattr(pipeline, name, fn)
