// PermuQuant on the GPU (converter/permuquant.py): the candidate channel
// order and the quantization errors its acceptance rule compares.
//
// order_kernel: per input channel j the second moment mean_i W[i,j]^2
// (permuquant.py:13-22), optionally the joint criterion
// act^alpha * w^(1-alpha) (permuquant.py:43-67), then the descending order
// by rank counting: channel j's position is the number of channels with a
// larger key, ties broken by index (a stable descending sort).
//
// group_err_kernel: compute_group_quant_error (permuquant.py:70-105) of W or of
// W[:, perm] without forming the permuted matrix: one CTA per row, the row in
// shared memory; per group (of the permuted layout) the INT4 scale
// clamp(max|w| / 7, 1e-5, 65500) in fp16 (scales.py:62-99) or, for INT8, one
// per row (absmax / 127, scales.py:126-160); per element the code
// clamp(rhaz(w / s)) and the squared error, exact in fp64, summed over the
// row in the ORIGINAL column order.  With groups that span the row the
// permuted errors are then bit-identical to the unpermuted ones, as they are
// in exact arithmetic, so the acceptance rule's strict comparison sees no
// difference (the reference compares two fp32 sums of the same numbers in
// different orders there).
#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  if constexpr (sizeof(T) == 4) return *p;
  else if constexpr (std::is_same<T, __half>::value) return __half2float(*p);
  else return __bfloat162float(*p);
}

// moments[j] = sum_i W[i,j]^2 / M (fp64 accumulation, rounded to fp32)
template <typename T>
__global__ void moments_kernel(const T* __restrict__ W, int64_t M, int64_t N, int64_t ldw, float* __restrict__ mom) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= N) return;
  double s = 0.0;
  for (int64_t i = 0; i < M; ++i) {
    const double v = (double)ldf(W + i * ldw + j);
    s += v * v;
  }
  mom[j] = (float)(s / (double)M);
}

__global__ void key_kernel(float* __restrict__ key, const float* __restrict__ act, int64_t N, float alpha,
                           float beta) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= N || !act) return;
  const float w = fmaxf(key[j], 1e-12f), a = fmaxf(act[j], 1e-12f);
  key[j] = __fmul_rn(powf(a, alpha), powf(w, beta));
}

// perm[rank(j)] = j, rank = #{k : key_k > key_j or (key_k == key_j and k < j)}; NaN keys last
__global__ void rank_kernel(const float* __restrict__ key, int64_t N, int32_t* __restrict__ perm) {
  __shared__ float tile[1024];
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const float kj = j < N ? key[j] : 0.f;
  const bool nj = kj != kj;
  int64_t r = 0;
  for (int64_t t0 = 0; t0 < N; t0 += 1024) {
    __syncthreads();
    for (int i = threadIdx.x; i < 1024; i += blockDim.x) tile[i] = (t0 + i < N) ? key[t0 + i] : 0.f;
    __syncthreads();
    const int lim = (int)(N - t0 < 1024 ? N - t0 : 1024);
    for (int i = 0; i < lim; ++i) {
      const float kk = tile[i];
      const int64_t k = t0 + i;
      const bool nk = kk != kk;
      bool before;
      if (nj) before = nk ? (k < j) : true;       // NaN keys sort after every number
      else before = nk ? false : (kk > kj || (kk == kj && k < j));
      r += before ? 1 : 0;
    }
  }
  if (j < N) perm[r] = (int32_t)j;
}

template <typename T>
__global__ void __launch_bounds__(256) group_err_kernel(const T* __restrict__ W, int64_t N, int64_t ldw,
                                                        const int32_t* __restrict__ inv, int gs, int bits,
                                                        double* __restrict__ row_err) {
  extern __shared__ float sm[];
  float* row = sm;                      // [N] the row in original order
  float* sc = sm + N;                   // [ngroups] fp16-rounded scales
  __shared__ double red[8];
  const int64_t r = blockIdx.x;
  const int ngroups = (int)((N + gs - 1) / gs);
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x) row[c] = ldf(W + r * ldw + c);
  for (int g = threadIdx.x; g < ngroups; g += blockDim.x) sc[g] = 0.f;
  __syncthreads();
  // per-group absmax of the permuted layout: element c sits at position inv[c]
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x) {
    const int64_t p = inv ? inv[c] : c;
    const float a = fabsf(row[c]);
    atomicMax(reinterpret_cast<int*>(sc) + p / gs, a != a ? 0x7fc00000 : __float_as_int(a));
  }
  __syncthreads();
  const float div = bits == 8 ? 127.f : 7.f;
  for (int g = threadIdx.x; g < ngroups; g += blockDim.x)
    sc[g] = __half2float(__float2half_rn(clampf(__fdiv_rn(sc[g], div), 1e-5f, 65500.f)));
  __syncthreads();
  const float qmin = bits == 8 ? -128.f : -8.f, qmax = bits == 8 ? 127.f : 7.f;
  double acc = 0.0;
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x) {
    const int64_t p = inv ? inv[c] : c;
    const float s = sc[p / gs];
    const float w = row[c];
    const float q = clampf(rhaz(__fdiv_rn(w, s)), qmin, qmax);
    const float d = __fsub_rn(w, __fmul_rn(q, s));
    acc += (double)d * (double)d;
  }
  acc = warp_sum_d(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    row_err[r] = t;
  }
}

__global__ void invert_perm_kernel(const int32_t* __restrict__ perm, int64_t N, int32_t* __restrict__ inv) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p < N) inv[perm[p]] = (int32_t)p;
}

}  // namespace
}  // namespace ic

using namespace ic;

extern "C" int ic_permuquant_order(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, const float* act_mu2,
                                   float alpha, float* key, int32_t* perm, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (N <= 0) return IC_OK;
  if (M <= 0 || ldw < N || !W || !key || !perm) return fail(IC_ERR_INVALID, "permuquant_order: bad arguments");
  if (N > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "permuquant_order: too many channels");
  const unsigned g = (unsigned)cdiv(N, 256);
  switch (dtype) {
    case IC_F32: moments_kernel<float><<<g, 256, 0, st>>>((const float*)W, M, N, ldw, key); break;
    case IC_F16: moments_kernel<__half><<<g, 256, 0, st>>>((const __half*)W, M, N, ldw, key); break;
    case IC_BF16: moments_kernel<__nv_bfloat16><<<g, 256, 0, st>>>((const __nv_bfloat16*)W, M, N, ldw, key); break;
    default: return fail(IC_ERR_INVALID, "permuquant_order: unknown dtype %d", dtype);
  }
  IC_CHECK_LAUNCH();
  if (act_mu2) {
    key_kernel<<<g, 256, 0, st>>>(key, act_mu2, N, alpha, (float)(1.0 - (double)alpha));
    IC_CHECK_LAUNCH();
  }
  rank_kernel<<<g, 256, 0, st>>>(key, N, perm);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

extern "C" int ic_group_quant_error(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, const int32_t* perm,
                                    int64_t group_size, int bits, int32_t* inv_scratch, double* row_err,
                                    void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (M <= 0 || N <= 0) return IC_OK;
  if (bits != 4 && bits != 8) return fail(IC_ERR_INVALID, "int_bits must be 4 or 8, got %d", bits);
  if (!W || !row_err || ldw < N) return fail(IC_ERR_INVALID, "group_quant_error: bad arguments");
  if (perm && !inv_scratch) return fail(IC_ERR_INVALID, "group_quant_error: a permutation needs inv_scratch [N]");
  const int64_t gs = bits == 8 ? N : (group_size > 0 ? group_size : N);
  const int64_t ngroups = cdiv(N, gs);
  const size_t smem = (size_t)(N + ngroups) * 4;
  if (smem > 200 * 1024) return fail(IC_ERR_UNSUPPORTED, "group_quant_error: row of %lld too long", (long long)N);
  if (M > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "group_quant_error: too many rows");
  const int32_t* inv = nullptr;
  if (perm) {
    invert_perm_kernel<<<(unsigned)cdiv(N, 256), 256, 0, st>>>(perm, N, inv_scratch);
    IC_CHECK_LAUNCH();
    inv = inv_scratch;
  }
  static std::atomic<unsigned long long> attr{0};
  IC_TRY(once_per_device(attr, [&]() -> int {
      IC_CUDA(cudaFuncSetAttribute(group_err_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      IC_CUDA(cudaFuncSetAttribute(group_err_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      IC_CUDA(cudaFuncSetAttribute(group_err_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   200 * 1024));
      return IC_OK;
    }));
  switch (dtype) {
    case IC_F32: group_err_kernel<float><<<(unsigned)M, 256, smem, st>>>((const float*)W, N, ldw, inv, (int)gs, bits, row_err); break;
    case IC_F16: group_err_kernel<__half><<<(unsigned)M, 256, smem, st>>>((const __half*)W, N, ldw, inv, (int)gs, bits, row_err); break;
    case IC_BF16:
      group_err_kernel<__nv_bfloat16><<<(unsigned)M, 256, smem, st>>>((const __nv_bfloat16*)W, N, ldw, inv, (int)gs, bits,
                                                                     row_err);
      break;
    default: return fail(IC_ERR_INVALID, "group_quant_error: unknown dtype %d", dtype);
  }
  IC_CHECK_LAUNCH();
  return IC_OK;
}
