// SmoothQuant factors of one layer on the GPU: compute_smoothing_factors
// (converter/smoothquant.py:11-52, per-channel activation amax) and
// compute_smoothing_from_hessian_diag (smoothquant.py:72-102), the two forms
// the pipeline's SmoothRot pre-pass uses (pipeline.py:362-415).
//
// Pass 1 reduces max_i |W[i,j]| per column (one thread per column, a slab of
// rows per CTA, coalesced along the row; slabs combine with an integer
// atomicMax, exact for non-negative floats and NaN-propagating like torch's
// amax); pass 2 applies the formula per column.
#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int COLS = 256;       // columns (threads) per CTA
constexpr int SLAB = 512;       // rows per CTA

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
  if constexpr (sizeof(T) == 4) return *p;
  else if constexpr (std::is_same<T, __half>::value) return __half2float(*p);
  else return __bfloat162float(*p);
}

template <typename T>
__global__ void __launch_bounds__(COLS) colmax_kernel(const T* __restrict__ W, int64_t M, int64_t N, int64_t ldw,
                                                      float* __restrict__ out) {
  const int64_t j = (int64_t)blockIdx.x * COLS + threadIdx.x;
  if (j >= N) return;
  const int64_t r0 = (int64_t)blockIdx.y * SLAB, r1 = min(M, r0 + SLAB);
  float m = 0.f;
  bool nan = false;
  for (int64_t r = r0; r < r1; ++r) {
    const float v = fabsf(ld_f(W + r * ldw + j));
    nan |= (v != v);
    m = fmaxf(m, v);
  }
  const int bits = nan ? 0x7fc00000 : __float_as_int(m);
  atomicMax(reinterpret_cast<int*>(out) + j, bits);
}

__global__ void factors_kernel(const float* __restrict__ act, int64_t stride, int64_t N, int mode, float alpha,
                               float beta, float nsamp, float* __restrict__ out) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= N) return;
  const float floor_v = 1e-8f;  // config.SMOOTHQUANT_AMAX_FLOOR
  float a = act[j * stride];
  if (mode == 1) a = sqrtf(fmaxf(__fdiv_rn(a, nsamp), floor_v));
  else a = fmaxf(a, floor_v);
  const float w = fmaxf(out[j], floor_v);
  out[j] = __fdiv_rn(powf(a, alpha), powf(w, beta));
}

}  // namespace

int smooth_factors(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, const float* act,
                   int64_t act_stride, int mode, float alpha, float nsamp, float* out, cudaStream_t st) {
  if (N <= 0) return IC_OK;
  if (M < 0 || ldw < N) return fail(IC_ERR_INVALID, "smooth_factors: bad shape");
  if (!W || !act || !out) return fail(IC_ERR_INVALID, "smooth_factors: null pointer");
  if (mode != 0 && mode != 1) return fail(IC_ERR_INVALID, "smooth_factors: mode must be 0 (amax) or 1 (Hessian)");
  if (mode == 1 && !(nsamp >= 1.f)) return fail(IC_ERR_INVALID, "smooth_factors: nsamp must be >= 1");
  if (act_stride < 1) return fail(IC_ERR_INVALID, "smooth_factors: act_stride must be >= 1");
  IC_CUDA(cudaMemsetAsync(out, 0, (size_t)N * 4, st));
  if (M > 0) {
    dim3 grid((unsigned)cdiv(N, COLS), (unsigned)cdiv(M, SLAB));
    if (grid.y > 65535u) return fail(IC_ERR_UNSUPPORTED, "smooth_factors: too many rows");
    switch (dtype) {
      case IC_F32: colmax_kernel<float><<<grid, COLS, 0, st>>>((const float*)W, M, N, ldw, out); break;
      case IC_F16: colmax_kernel<__half><<<grid, COLS, 0, st>>>((const __half*)W, M, N, ldw, out); break;
      case IC_BF16: colmax_kernel<__nv_bfloat16><<<grid, COLS, 0, st>>>((const __nv_bfloat16*)W, M, N, ldw, out); break;
      default: return fail(IC_ERR_INVALID, "smooth_factors: unknown dtype %d", dtype);
    }
    IC_CHECK_LAUNCH();
  }
  const float beta = (float)(1.0 - (double)alpha);
  factors_kernel<<<(unsigned)cdiv(N, 256), 256, 0, st>>>(act, act_stride, N, mode, alpha, beta, nsamp, out);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

}  // namespace ic

extern "C" int ic_smooth_factors(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, const float* act,
                                 int64_t act_stride, int mode, float alpha, float nsamp, float* out, void* stream) {
  return ic::smooth_factors(W, dtype, M, N, ldw, act, act_stride, mode, alpha, nsamp, out, (cudaStream_t)stream);
}
