// PiSO per-row scale search (converter/piso.py:29-182): one CTA per row, the
// row and the Hessian diagonal in shared memory, every candidate scale costed
// as sum_d h_d (w_d - dequant_d)^2 with a CTA reduction; the first minimum
// wins (torch.argmin).  Coarse candidates are base * coarse[i]; the fine
// candidates are (coarse winner) * fine[i], and the fine winner is the result.
#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int NT = 256;
constexpr int MAXC = 512;
constexpr int64_t MAXN = 24576;

struct PArgs {
  const float* W;
  int64_t N, ldw;
  const float* h;
  int asym;
  float qmin, qmax, divisor;
  float coarse[MAXC];
  int nc;
  float fine[64];
  int nf;
  float* scales;
  int8_t* zp;
};

__device__ float block_sum(float v, float* red) {
  for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < NT / 32; ++w) r = __fadd_rn(r, red[w]);
  return r;
}

__device__ float cost_of(const float* w, const float* h, int64_t N, float s, float zp, bool asym, float qmin,
                         float qmax, float* red) {
  float part = 0.f;
  for (int64_t i = threadIdx.x; i < N; i += NT) {
    const float x = w[i];
    float y = __fdiv_rn(x, s);
    if (asym) y = __fadd_rn(y, zp);
    const float q = clampf(rhaz(y), qmin, qmax);
    const float deq = asym ? __fmul_rn(__fsub_rn(q, zp), s) : __fmul_rn(q, s);
    const float e = __fsub_rn(x, deq);
    part = __fadd_rn(part, __fmul_rn(__fmul_rn(e, e), h[i]));
  }
  return block_sum(part, red);
}

__global__ void __launch_bounds__(NT) piso_kernel(const __grid_constant__ PArgs a) {
  extern __shared__ float sm[];
  __shared__ float red[32];
  __shared__ float r3[3][8];
  float* w = sm;
  float* h = sm + a.N;
  const int64_t row = blockIdx.x;
  float amax = 0.f, mn = __int_as_float(0x7f800000), mx = __int_as_float(0xff800000);
  for (int64_t i = threadIdx.x; i < a.N; i += NT) {
    const float v = a.W[row * a.ldw + i];
    w[i] = v;
    h[i] = a.h[i];
    amax = nmax(amax, fabsf(v));
    mn = nmin(mn, v);
    mx = nmax(mx, v);
  }
  for (int o = 16; o; o >>= 1) {
    amax = nmax(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    mn = nmin(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = nmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if ((threadIdx.x & 31) == 0) {
    r3[0][threadIdx.x >> 5] = amax;
    r3[1][threadIdx.x >> 5] = mn;
    r3[2][threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  amax = r3[0][0];
  mn = r3[1][0];
  mx = r3[2][0];
  for (int i = 1; i < NT / 32; ++i) {
    amax = nmax(amax, r3[0][i]);
    mn = nmin(mn, r3[1][i]);
    mx = nmax(mx, r3[2][i]);
  }
  const bool asym = a.asym != 0;
  const float base = asym ? clamp_lo(__fdiv_rn(__fsub_rn(mx, mn), a.divisor), 1e-10f)
                          : clamp_lo(__fdiv_rn(amax, a.divisor), 1e-10f);
  auto zp_for = [&](float s) {
    return asym ? clampf(rhaz(__fsub_rn(a.qmin, __fdiv_rn(mn, s))), a.qmin, a.qmax) : 0.f;
  };
  float best_cost = 0.f, best_s = base;
  for (int i = 0; i < a.nc; ++i) {
    float s = __fmul_rn(base, a.coarse[i]);
    if (asym) s = clamp_lo(s, 1e-10f);
    const float c = cost_of(w, h, a.N, s, zp_for(s), asym, a.qmin, a.qmax, red);
    if (i == 0 || c < best_cost) {
      best_cost = c;
      best_s = s;
    }
  }
  float fs = best_s, fz = zp_for(best_s), fbest = 0.f;
  for (int i = 0; i < a.nf; ++i) {
    float s = __fmul_rn(best_s, a.fine[i]);
    if (asym) s = clamp_lo(s, 1e-10f);
    const float z = zp_for(s);
    const float c = cost_of(w, h, a.N, s, z, asym, a.qmin, a.qmax, red);
    if (i == 0 || c < fbest) {
      fbest = c;
      fs = s;
      fz = z;
    }
  }
  if (threadIdx.x == 0) {
    a.scales[row] = fs;
    if (asym && a.zp) a.zp[row] = (int8_t)fz;
  }
}

}  // namespace
}  // namespace ic

using namespace ic;

extern "C" int ic_piso(const float* W, int64_t M, int64_t N, int64_t ldw, const float* hdiag, int asym, int qmin,
                       int qmax, float divisor, const float* coarse, int ncoarse, const float* fine, int nfine,
                       float* scales, int8_t* zp, void* stream) {
  if (M <= 0 || N <= 0) return IC_OK;
  if (N > MAXN) return fail(IC_ERR_UNSUPPORTED, "piso: in_features %lld > %lld", (long long)N, (long long)MAXN);
  if (ncoarse < 1 || ncoarse > MAXC || nfine < 1 || nfine > 64)
    return fail(IC_ERR_UNSUPPORTED, "piso: candidate counts out of range");
  if (M > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "piso: too many rows");
  PArgs h{};  // the candidate tables travel in the kernel's parameter block
  h.W = W; h.N = N; h.ldw = ldw; h.h = hdiag; h.asym = asym; h.qmin = (float)qmin; h.qmax = (float)qmax;
  h.divisor = divisor; h.nc = ncoarse; h.nf = nfine; h.scales = scales; h.zp = zp;
  for (int i = 0; i < ncoarse; ++i) h.coarse[i] = coarse[i];
  for (int i = 0; i < nfine; ++i) h.fine[i] = fine[i];
  static std::atomic<unsigned long long> attr{0};
  IC_TRY(once_per_device(attr, [&]() -> int {
      IC_CUDA(cudaFuncSetAttribute(piso_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(MAXN * 8)));
      return IC_OK;
    }));
  piso_kernel<<<(unsigned)M, NT, (size_t)N * 8, (cudaStream_t)stream>>>(h);
  IC_CHECK_LAUNCH();
  return IC_OK;
}
