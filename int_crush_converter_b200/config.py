"""Numeric constants of the quantization path.

Same values as the reference's ``converter/config.py`` (lines 32-189), so that
results here and there agree; restated because this package runs without the
reference installed.
"""

import torch

INT4_SCALE_DIVISOR = 7.0
INT8_SCALE_DIVISOR = 127.0
SCALE_DTYPE = torch.float16
SCALE_MIN = 1e-5
SCALE_MAX = 65500.0
SCALE_FLOOR = 1e-8
DIAG_MEAN_FLOOR = 1e-6
DENOMINATOR_FLOOR = 1e-8
HINV_DIAG_FLOOR = 1e-8
ERR_CLAMP_RANGE = 100.0
SANITIZE_FLOOR = 1e-8
SANITIZE_CEIL = 1e30
WEIGHT_OUTLIER_CLAMP = 1000.0
SIGN_FLIP_THRESHOLD = 1e-8
CONVERGENCE_EPS = 1e-10
CONVERGENCE_IMPROVEMENT_THRESHOLD = 1e-4
SCALE_FLOOR_MULTIPLIER = 0.1
SCALE_CEIL_MULTIPLIER = 10.0
ABS_SCALE_FLOOR = 1e-8
SCALE_MOMENTUM = 0.3             # ldlq.py:503
MSE_DIVERGENCE_THRESHOLD = 1.05  # ldlq.py:504
W_NONZERO_THRESHOLD = 1e-8       # ldlq.py:505

# Tensor-core passes of the lazy GPTQ/LDLQ update and the greedy cross terms:
# 3 = 3xTF32 (~fp32 accurate, default), 1 = plain TF32 with fp32 accumulation.
GEMM_PASSES = 3
# Tensor-core passes of the greedy local search's cross terms E @ H[:, block]:
# 3xTF32 by default (the codes follow the reference's fp32 search); 1 = plain
# TF32 with fp32 accumulation, faster, with more near-ties broken the other
# way (environment variable IC_GREEDY_GEMM_PASSES overrides).
GREEDY_GEMM_PASSES = 3
# Columns per super-block of the two-level lazy update (multiple of the block size).
SUPERBLOCK = 1024

# Low-rank greedy (greedy.py:293-381, config.py:124-137)
EIGENVALUE_FLOOR = 1e-12
STALL_THRESHOLD = 0.99
LOWRANK_MAX_RANK_FRAC = 0.3
LOWRANK_MAX_K = 512
# Sketch width of the low-rank decomposition here: the small eigenproblem runs in
# one CTA's shared memory (ic_sym_eig), which bounds it at 64 columns.
LOWRANK_SKETCH = 64
