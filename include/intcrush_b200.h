/*
 * libintcrush_b200 -- C ABI of the B200 (sm_100a) per-layer weight-quantization
 * path of int_crush_converter.
 *
 * Conventions
 *  - All pointers are DEVICE pointers unless stated otherwise; sizes are
 *    element counts; leading dimensions (ld*) are in elements; matrices are
 *    row-major.  Every call is asynchronous on `stream` (a cudaStream_t passed
 *    as void*) except where it says it synchronises.
 *  - Return value: IC_OK (0) or a negative ic_status; ic_last_error() gives a
 *    message for the calling thread's last failure.
 *  - Nothing here allocates device memory except the one-time 4-byte status
 *    word per device; scratch comes from a caller workspace whose size the
 *    matching *_workspace_size function returns.
 *  - Reference citations are file:line inside ThunderFun/int_crush_converter.
 */
#ifndef INTCRUSH_B200_H
#define INTCRUSH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  IC_OK = 0,
  IC_ERR_INVALID = -1,     /* bad argument (maps to ValueError)                 */
  IC_ERR_CUDA = -2,        /* CUDA runtime / driver error                       */
  IC_ERR_NOT_PD = -3,      /* Hessian not positive definite (take general inv)  */
  IC_ERR_TIMEOUT = -4,     /* a bounded device-side wait gave up               */
  IC_ERR_RANGE = -5,       /* INT4 packing: value outside [-8,7]                */
  IC_ERR_UNSUPPORTED = -6, /* shape/option outside what the kernels implement   */
  IC_ERR_WORKSPACE = -7    /* workspace too small                               */
} ic_status;

/* input element types */
enum { IC_F32 = 0, IC_F16 = 1, IC_BF16 = 2 };

const char* ic_version(void);
const char* ic_last_error(void);
/* IC_OK if the current device is sm_100 (B200 class); IC_ERR_UNSUPPORTED otherwise */
int ic_device_check(void);
/* Number of kernels this library has launched in the process (all devices);
 * the benchmark uses it to count its own launches inside a timed region. */
unsigned long long ic_launch_count(void);
/* Number of Hessian-inverse CUDA graphs this library has instantiated in the
 * process (each costs milliseconds of host time; a count that still grows in
 * steady state means the replay cache misses). */
unsigned long long ic_inverse_graph_count(void);
/* Failure-path self-test (no reference counterpart): launches one thread that
 * waits on an mbarrier nothing arrives on, through the same bounded wait every
 * kernel of the library uses; after `limit_ns` (0.1 ms .. 2 s) it gives up,
 * sets DEV_TIMEOUT in the device status word (read it with
 * ic_device_status) and returns, leaving the context usable.  Asynchronous
 * on `stream`. */
int ic_selftest_bounded_wait(unsigned long long limit_ns, void* stream);
/* Reads and clears the device status word (bit0 timeout, bit1 not-PD,
 * bit2 INT4 range).  Synchronises `stream`. */
int ic_device_status(unsigned* flags_out, void* stream);

/* ---------------------------------------------------------------- rotation */
/* Group-wise Hadamard rotation of the in_features dimension.
 * Replaces rotation.rotate_weights (converter/rotation.py:95-125) and
 * _apply_hadamard (rotation.py:82-92).  rot: power of two 2..1024 (regular
 * Hadamard H4^{kron k}/2^k for powers of four, rotation.py:39-62; Sylvester
 * otherwise, rotation.py:26-36); rot == 0 copies/upcasts.  out: fp32
 * [M, npad], npad = N rounded up to a multiple of rot (zero padding). */
int ic_rotate_weights(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, int rot,
                      float* out, int64_t ldo, void* stream);

/* H_rot = R^T H R of a 2-D [n,n] Hessian (nbatch = 1, zero padding to npad)
 * or of nbatch block-diagonal [n,n] blocks (n % rot == 0).  Replaces
 * rotation.rotate_hessian / _transform_hessian_blocks (rotation.py:156-248).
 * Output rows have leading dimension npad.  If out_lo != NULL the result is
 * a TF32 hi/lo pair (hi + lo == the fp32 value), the layout the inverse uses. */
int ic_rotate_hessian(const float* H, int64_t nbatch, int64_t n, int64_t ldh, int rot,
                      float* out_hi, float* out_lo, int64_t npad, void* stream);

/* -------------------------------------------------------------------- RTN */
/* Per-group scales (and zero-points) with optional clipping-ratio search.
 * bits 4: calculate_scales / calculate_scales_asymmetric (converter/scales.py:62-99,
 * 232-282); bits 8: calculate_scales_int8 / _int8_asymmetric (scales.py:126-160,
 * 316-361; group_size must equal N).  W fp32 [M, N], N a multiple of
 * group_size (the caller pads).  scales fp16 [M, N/group_size]; zp int8
 * (asymmetric only).  ratios: HOST array of nratios floats, or NULL. */
int ic_rtn_scales(const float* W, int64_t M, int64_t N, int64_t ldw, int bits, int asym,
                  int64_t group_size, const float* ratios, int nratios,
                  uint16_t* scales_f16, int8_t* zp, void* stream);

/* Codes from given fp16 scales: quantize_weights / _asymmetric / _int8 /
 * _int8_asymmetric (converter/scales.py:102-123, 163-178, 285-313, 364-384). */
int ic_rtn_codes(const float* W, int64_t M, int64_t N, int64_t ldw, int bits, int asym,
                 int64_t group_size, const uint16_t* scales_f16, const int8_t* zp,
                 int8_t* codes, int64_t ldc, void* stream);

/* Fused single pass over each row: load W (fp16/bf16/fp32), zero |w| > 1000
 * (the pipeline's outlier sanitize, pipeline.py:527-537), rotate (rot as in
 * ic_rotate_weights), per-row scale search, round-half-away, clamp, write int8
 * codes [M, npad] and/or packed INT4 [M, ceil(npad/2)], fp16 scales [M], int8
 * zp [M], and the verify statistics of pipeline.py:919-931 per row (sum of
 * squared error, fp64; max |error|) against the rotated weights.  This is
 * pipeline.py:547-559 + 890-917 + 1010-1013 for one RTN layer.  Any output
 * may be NULL. */
int ic_rtn_fused(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, int rot, int bits,
                 int asym, const float* ratios, int nratios, int8_t* codes, uint8_t* packed,
                 uint16_t* scales_f16, int8_t* zp, double* row_sqerr, float* row_maxerr,
                 void* stream);

/* ---------------------------------------------------------------- packing */
/* pack_int4 (converter/packing.py:30-46): two's-complement nibbles, low nibble
 * = even column, odd K padded with 0.  Range check of validate_int4_range
 * (packing.py:17-27): IC_ERR_RANGE if any code is outside [-8,7]
 * (synchronises to read the check). */
int ic_pack_int4(const int8_t* codes, int64_t M, int64_t K, int64_t ldc, uint8_t* packed,
                 int64_t ldp, void* stream);
/* unpack_int4 (packing.py:49-66) */
int ic_unpack_int4(const uint8_t* packed, int64_t M, int64_t K, int64_t ldp, int8_t* codes,
                   int64_t ldc, void* stream);

/* ------------------------------------------------------ dense contraction */
/* D = beta*C + alpha * A * B^T on the tcgen05 tensor cores (TMA-fed, TMEM
 * accumulators).  A [m,k] and B [n,k] row-major with k contiguous, 16-byte
 * aligned, lda/ldb multiples of 4.  passes = 3: operands are TF32 hi/lo pairs
 * and the product is hi*hi + hi*lo + lo*hi (3xTF32, ~fp32 accuracy);
 * passes = 1: plain TF32 with fp32 accumulation.  C/D plain fp32 when
 * c_lo/d_lo are NULL, else hi/lo pairs.  D may alias C.  Replaces the torch
 * matmuls of gptq_triton.py:178-180, rounding.py:102-103, ldlq.py:413,
 * greedy.py:519 and the GEMMs inside the LAPACK inverse. */
int ic_gemm_tn(int64_t m, int64_t n, int64_t k, float alpha, const float* a_hi,
               const float* a_lo, int64_t lda, const float* b_hi, const float* b_lo, int64_t ldb,
               float beta, const float* c_hi, const float* c_lo, int64_t ldc, float* d_hi,
               float* d_lo, int64_t ldd, int passes, void* stream);

/* 3xTF32 ic_gemm_tn restricted by triangular structure, as the inverse uses
 * it (no direct counterpart in the reference, whose LAPACK call hides these
 * products): tri bit 0 computes only the output 128-tiles on or below the
 * diagonal (others are left unspecified); bit 1 declares A upper triangular
 * (row i zero left of column i), so each tile's K loop starts at its first
 * row. */
int ic_gemm_tn_tri(int64_t m, int64_t n, int64_t k, float alpha, const float* a_hi,
                   const float* a_lo, int64_t lda, const float* b_hi, const float* b_lo,
                   int64_t ldb, float beta, const float* c_hi, const float* c_lo, int64_t ldc,
                   float* d_hi, float* d_lo, int64_t ldd, int tri, void* stream);

/* ---------------------------------------------------- Hessian preparation */
/* Damping + inverse of an SPD Hessian held as a TF32 hi/lo pair [n,n] (in
 * place, ldh a multiple of 4): H <- (H + damping*max(mean(diag H),1e-6)*I)^-1.
 * Replaces gptq._prepare_hinv (converter/gptq.py:113-121) and the Cholesky
 * branch of rounding._invert_hessian (rounding.py:19-34).  Only the lower
 * triangle of H is read; the result is full and symmetric.  Returns
 * IC_ERR_NOT_PD (after synchronising) when a pivot is not positive; the
 * caller then takes the reference's general-inverse branch.  damping < 0
 * skips the damping step. */
size_t ic_spd_inverse_workspace_size(int64_t n);
int ic_spd_inverse(float* h_hi, float* h_lo, int64_t n, int64_t ldh, float damping,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Lower Cholesky factor L of an SPD matrix held as a TF32 hi/lo pair [n,n]
 * (in place, lower triangle read), returned as its symmetric completion: the
 * lower triangle holds L and the strictly upper triangle L^T, so that row j
 * right of the diagonal is row j of the upper factor U = L^T.  With A = the
 * damped inverse this is the "cholesky" Hessian method of gptq._prepare_hessian
 * (converter/gptq.py:91-110: torch.linalg.cholesky(H^-1).T), in the layout the
 * GPTQ column loop (ic_gptq_run) reads.  Workspace: ic_spd_inverse_workspace_size(n).
 * Synchronises; IC_ERR_NOT_PD when a pivot is not positive (the reference then
 * keeps the full inverse). */
int ic_spd_cholesky(float* h_hi, float* h_lo, int64_t n, int64_t ldh, void* workspace,
                    size_t workspace_bytes, void* stream);

/* SmoothQuant factors of one layer (converter/smoothquant.py:11-52 and 72-102):
 * s_j = a_j^alpha / max(max_i |W[i,j]|, 1e-8)^(1-alpha) with
 *   mode 0: a_j = max(act[j * act_stride], 1e-8)            (per-channel activation amax)
 *   mode 1: a_j = sqrt(max(act[j * act_stride] / nsamp, 1e-8)) (Hessian diagonal; pass the
 *           Hessian itself with act_stride = ldh + 1)
 * W: fp16/bf16/fp32 [M, N] (unrotated, as the pipeline's W_down.float()).  out fp32 [N].
 * powf may differ from torch's CPU pow in the last bit. */
int ic_smooth_factors(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, const float* act,
                      int64_t act_stride, int mode, float alpha, float nsamp, float* out, void* stream);

/* PermuQuant candidate order (converter/permuquant.py:13-67): key[j] = the second
 * moment mean_i W[i,j]^2 of input channel j (fp64 sum, fp32 result), or with
 * act_mu2 != NULL the joint key max(act_mu2[j],1e-12)^alpha *
 * max(key[j],1e-12)^(1-alpha); perm int32 [N] = channels by descending key,
 * ties by index (a stable argsort(descending=True)).  W fp16/bf16/fp32 [M, N]. */
int ic_permuquant_order(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, const float* act_mu2,
                        float alpha, float* key, int32_t* perm, void* stream);

/* compute_group_quant_error (converter/permuquant.py:70-105) of W, or of
 * W[:, perm] when perm != NULL (inv_scratch int32 [N] then receives the
 * inverse permutation): RTN with fp16 per-group scales (bits 4: group_size,
 * absmax/7; bits 8: per row, absmax/127), round-half-away codes, and per row
 * the sum of squared errors, each term exact in fp64, summed in the original
 * column order (so with groups spanning the row a permutation gives the same
 * sums bit for bit).  row_err fp64 [M]. */
int ic_group_quant_error(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, const int32_t* perm,
                         int64_t group_size, int bits, int32_t* inv_scratch, double* row_err, void* stream);

/* --------------------------------------- SVD-absorbed split (svd.py:35-75) */
/* The small dense steps of the randomized low-rank SVD that
 * svd.decompose_weight calls (torch.svd_lowrank, q = rank, niter = 2); its
 * products run on ic_gemm_tn.  ic_orthonormalize: the columns of X [m, q]
 * (row-major, leading dimension ldx, 1 <= q <= min(m, 64)) made orthonormal in
 * place (classical Gram-Schmidt applied twice, fp64 sums) -- the range finder's QR.
 * ic_sym_eig: eigenvalues (descending) and eigenvectors (columns of V) of a
 * symmetric q x q matrix, q <= 64, by cyclic Jacobi -- the SVD of the
 * projected matrix through B B^T. */
int ic_orthonormalize(float* X, int64_t m, int q, int64_t ldx, void* stream);
int ic_sym_eig(const float* A, int q, int64_t lda, float* evals, float* V, int64_t ldv, void* stream);

/* ------------------------------------------------------------------- GPTQ */
/* Per-row scale / zero-point preparation of gptq_quantize_layer
 * (converter/gptq.py:254-317): bits 4 -> asymmetric range scales with the
 * zero-point clamp fix; bits 8 -> symmetric absmax/127, or asymmetric.
 * W fp32 [M,N]; scale fp32 [M]; zp fp32 [M] (written when bits == 4 or asym). */
int ic_gptq_row_params(const float* W, int64_t M, int64_t N, int64_t ldw, int bits, int asym,
                       float* scale, float* zp, void* stream);

/* The GPTQ column loop over columns [0, N) of W_work (mutated):
 * rounding._gptq_block (converter/rounding.py:37-103) with the reference's
 * per-column arithmetic (eager intra-block update, error clamp +-100,
 * NaN -> 0) and the lazy inter-block update as tcgen05 GEMMs (two-level:
 * near updates inside a super-block of `superblock` columns, one far update
 * per super-block).  Hinv: TF32 hi/lo pair [N,N] (symmetric, ldh % 4 == 0).
 * scale fp32 [M]; zp fp32 [M] or NULL (symmetric).  Outputs (any may be
 * NULL): codes int8, packed uint8 (INT4, even block size), row_sqerr fp64 [M]
 * and row_maxerr fp32 [M] of (W0 - dequant(codes, scale)). */
size_t ic_gptq_workspace_size(int64_t M, int64_t N, int block_size, int superblock);
int ic_gptq_run(float* W_work, int64_t ldw, const float* W0, int64_t ldw0, int64_t M, int64_t N,
                const float* hinv_hi, const float* hinv_lo, int64_t ldh, int block_size,
                int superblock, const float* scale, const float* zp, int qmin, int qmax,
                int8_t* codes, int64_t ldq, uint8_t* packed, int64_t ldp, double* row_sqerr,
                float* row_maxerr, int gemm_passes, void* workspace, size_t workspace_bytes,
                void* stream);

/* Same as ic_gptq_run, for callers that cannot allocate device memory (their
 * device memory is owned and capped by another allocator, or an allocation is
 * not acceptable on their latency-critical path).  No counterpart in the
 * reference (the reference allocates with torch).  Takes no workspace: its
 * scratch is a static device array of IC_NOALLOC_SCRATCH_BYTES per GPU that
 * lives until the process exits; shapes whose ic_gptq_workspace_size exceeds
 * it are rejected with IC_ERR_UNSUPPORTED.  Calls no cudaMalloc/cudaFree.  The
 * first call on a device looks up the array's address (make it before any
 * stream capture).  All calls share the array, so calls that overlap on the
 * GPU race; serialise them. */
#define IC_NOALLOC_SCRATCH_BYTES (32u << 20)
int ic_gptq_run_noalloc(float* W_work, int64_t ldw, const float* W0, int64_t ldw0, int64_t M,
                        int64_t N, const float* hinv_hi, const float* hinv_lo, int64_t ldh,
                        int block_size, int superblock, const float* scale, const float* zp,
                        int qmin, int qmax, int8_t* codes, int64_t ldq, uint8_t* packed,
                        int64_t ldp, double* row_sqerr, float* row_maxerr, int gemm_passes,
                        void* stream);

/* One whole GPTQ layer as pipeline.py:527-559 + 702-809 + 919-931 + 1010-1013
 * run it: zero |w| > 1000 (outlier sanitize), rotate W (fp16/bf16/fp32) and
 * H, row params, damping, inverse,
 * column loop, pack, verify statistics.  smoothing (fp32 [N_in] or NULL):
 * the SmoothRot pre-step of pipeline.py:547-553 + 766-774, W[:, j] * s_j and
 * H[i,j] / max(s_i s_j, 1e-16) capped at 1e30 (pipeline.py:99-137), fused
 * into the rotation loads (needs 16 <= rot <= 512).  smooth_order (with smoothing): 0
 * smooths H and rotates it once (R^T diag(1/s) H diag(1/s) R, the Hessian of the
 * smoothed-then-rotated weights); 1 follows the pipeline's own sequence for a
 * SmoothRot layer, which rotates H before smoothing and again after it
 * (pipeline.py:721-723 then 766-770: R^T diag(1/s) (R^T H R) diag(1/s) R; needs
 * N_in % rot == 0).  H fp32 [N_in, N_in] (already in the
 * rotated space when h_rotated != 0).  Outputs: packed uint8 [M, npad/2]
 * (bits 4) and/or codes int8 [M, npad]; scales_f16 [M]; zp int8 [M] (bits 4
 * or asym).  With stats (fp64 [3] = {mse, max_err, status}: the pipeline's
 * verify statistics and the layer's status bits: 2 = Hessian not positive
 * definite, 8 = a row's fp16 scale is NaN, infinite or zero, the condition on
 * which the pipeline repairs scales, pipeline.py:935-1007; for the only
 * reachable case, a NaN weight, the outputs already equal the repaired ones:
 * NaN scale, zero-point 0, codes 0) the call does not synchronise and the caller checks stats[2]
 * (the reference then takes its inv/pinv branch); with stats == NULL it
 * synchronises once and returns IC_ERR_NOT_PD.  update_passes: the lazy
 * trailing update W -= E * Hinv (rounding.py:100-103) as 1 = TF32 products
 * with fp32 accumulation or 3 = 3xTF32 (fp32-class); the Hessian inverse is
 * always 3xTF32.  Both keep tr((W-Q)H(W-Q)^T) within 0.15% of the reference
 * on the parity aggregates; 1 does a third of the update's tensor work. */
size_t ic_gptq_layer_workspace_size(int64_t M, int64_t N_in, int rot);
int ic_gptq_layer(const void* W, int dtype, int64_t M, int64_t N_in, int64_t ldw, const float* H,
                  int64_t ldh, const float* smoothing, int smooth_order, int h_rotated, int rot, int bits,
                  int asym, int block_size,
                  float damping, int update_passes, int8_t* codes, uint8_t* packed, uint16_t* scales_f16,
                  int8_t* zp, double* stats, void* workspace, size_t workspace_bytes,
                  void* stream);

/* ------------------------------------------------------------------- LDLQ */
/* The LDLQ column loop (ldlq._ldlq_loop_cpu, converter/ldlq.py:369-417, with
 * rounding._ldlq_round_column, rounding.py:115-155): per-element scales
 * scale2d fp32 [M,N] (floored at 1e-8), sign-flip correction, error times
 * 1/max(Hinv[j,j],1e-8), lazy inter-block GEMM update.  W_work mutated. */
int ic_ldlq_run(float* W_work, int64_t ldw, int64_t M, int64_t N, const float* hinv_hi,
                const float* hinv_lo, int64_t ldh, int block_size, int superblock,
                const float* scale2d, int64_t lds, int qmin, int qmax, int8_t* codes,
                int64_t ldq, int gemm_passes, void* workspace, size_t workspace_bytes,
                void* stream);

/* Scale refinement between LDLQ iterations (ldlq._update_ldlq_scales,
 * converter/ldlq.py:553-599), elementwise over `count` contiguous elements;
 * floor/ceil computed by the caller as the reference does. */
int ic_ldlq_update_scales(const float* W, const int8_t* Q, float* cur, const float* flat,
                          int64_t count, float momentum, float one_minus_momentum,
                          float floor_v, float ceil_v, float nonzero_thr, void* stream);

/* --------------------------------------------------------- greedy search */
/* greedy.greedy_local_search_pytorch (converter/greedy.py:487-541):
 * coordinate descent over [qmin,qmax] minimising tr(E H E^T), E = Q*s - W.
 * Cross terms err * H[blk,:]^T per 128-column block on the tensor cores plus
 * exact in-block rank-1 corrections.  Q int8 [M,N] updated in place; H fp32
 * [N,N] as a hi/lo pair (ldh % 4 == 0).  gemm_passes: 3 = cross terms in
 * 3xTF32, 1 = one TF32 pass with fp32 accumulation (the products read h_hi
 * alone, the in-block terms still the exact pair; more near-ties broken the
 * other way). */
size_t ic_greedy_workspace_size(int64_t M, int64_t N);
int ic_greedy_run(const float* W, int64_t ldw, int8_t* Q, int64_t ldq, const float* scale2d,
                  int64_t lds, const float* h_hi, const float* h_lo, int64_t ldh, int64_t M,
                  int64_t N, int passes, int qmin, int qmax, int gemm_passes, void* workspace,
                  size_t workspace_bytes, void* stream);

/* One pass of the low-rank greedy search (converter/greedy.py:100-199, launched
 * per 64 columns by greedy_lowrank_triton, greedy.py:384-479): H ~ U_k
 * diag(s_k) U_k^T plus the exact diagonal.  Per row, for every column in
 * order: cross = err_lr . (s_k * U_k[j]) - err_j H_jj, candidates in
 * [qmin,qmax] ascending with cost ne^2 H_jj + 2 ne cross (strict < against
 * 1e30), then err_j and err_lr += delta U_k[j].  err fp32 [M,N] (Q*s - W),
 * Q int8, err_lr fp32 [M,k] = err U_k, all updated in place; hdiag [N]; U and
 * SU = s_k * U fp32 [N,k] row-major; 1 <= k <= 64. */
int ic_greedy_lowrank_pass(float* err, int64_t lde, int8_t* Q, int64_t ldq, const float* scale2d,
                           int64_t lds, const float* hdiag, const float* U, const float* SU, int k,
                           float* err_lr, int64_t M, int64_t N, int qmin, int qmax, void* stream);

/* -------------------------------------------------------------------- PiSO */
/* PiSO per-row scale search (converter/piso.py:29-182): coarse candidates
 * base*coarse[i], then fine candidates best*fine[i]; cost sum_d h_d (w_d -
 * deq_d)^2; first minimum wins.  coarse/fine: HOST fp32 factor tables (the
 * reference builds them with torch.linspace, piso.py:62-63/135-136).
 * asym = 0: base = max|w|/divisor; asym = 1: base = (max-min)/(qmax-qmin) with
 * a per-candidate zero-point.  scales fp32 [M]; zp int8 [M] (asym). */
int ic_piso(const float* W, int64_t M, int64_t N, int64_t ldw, const float* hdiag, int asym,
            int qmin, int qmax, float divisor, const float* coarse, int ncoarse,
            const float* fine, int nfine, float* scales, int8_t* zp, void* stream);

/* ------------------------------------------------------------- utilities */
/* stats[2] = {sum(row_sqerr)/count, max(row_maxerr)} (fp64) */
int ic_finalize_stats(const double* row_sqerr, const float* row_maxerr, int64_t M,
                      double count, double* stats, void* stream);
/* out = alpha * in^T on hi/lo pairs (lo pointers may be NULL) */
int ic_transpose(const float* in_hi, const float* in_lo, int64_t rows, int64_t cols,
                 int64_t ldi, float alpha, float* out_hi, float* out_lo, int64_t ldo,
                 void* stream);
/* fp32 -> TF32 hi/lo pair (out_lo may be NULL) */
int ic_split_tf32(const float* in, int64_t rows, int64_t cols, int64_t ldi, float* out_hi,
                  float* out_lo, int64_t ldo, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* INTCRUSH_B200_H */
