"""B200-native (sm_100a) per-layer weight-quantization path of int_crush_converter.

The public functions mirror the reference's ``converter`` API (same names,
arguments, return types and errors) and run hand-written CUDA kernels from
``libintcrush_b200.so`` (C ABI: ``include/intcrush_b200.h``).  There is no CPU
path: without an sm_100 GPU or without the built library, calls raise.
"""

from .gptq import gptq_quantize_layer, gptq_quantize_layer_rtn, quantize_gptq_layer, check_layer, LayerWorkspace, LayerStreams
from .greedy import greedy_local_search, greedy_local_search_pytorch
from .hessian import dlr_to_dense, invert_dense, woodbury_inverse
from .ldlq import ldlq_quantize_layer
from .packing import INT4PackingError, pack_int4, unpack_int4, validate_int4_range
from .piso import (
    compute_piso_scales_int4, compute_piso_scales_int4_asymmetric, compute_piso_scales_int8,
    compute_piso_scales_int8_asymmetric,
)
from .rotation import (
    clear_hadamard_cache, get_hadamard, make_hadamard_regular, make_hadamard_sylvester, rotate_activations,
    rotate_hessian, rotate_weights,
)
from .rounding import _invert_hessian, _round_half_away_from_zero
from .scales import (
    calculate_scales, calculate_scales_asymmetric, calculate_scales_int8, calculate_scales_int8_asymmetric,
    quantize_weights, quantize_weights_asymmetric, quantize_weights_int8, quantize_weights_int8_asymmetric,
    rtn_quantize_fused,
)
from .types import QuantizationResult

__version__ = "0.1.0"
from .smoothquant import (  # noqa: E402,F401
    apply_smoothing_to_weight, _transform_hessian_for_smoothquant, compute_smoothing_factors,
    compute_smoothing_from_hessian_diag,
)
from .permuquant import (  # noqa: E402,F401
    channel_second_moments, compute_group_quant_error, find_permutation_joint, find_permutation_weight,
    find_permutation_with_acceptance, sweep_alpha,
)
from .svd import SVDResult, decompose_weight  # noqa: E402,F401
