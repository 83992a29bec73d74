// Shared-memory group Hadamard used by the rotation and RTN kernels.
//
// The regular Hadamard H_r = H4^{kron k}/2^k (r = 4^k) is applied as k radix-4
// butterfly stages, one per base-4 digit of the in-group index (all Kronecker
// factors are the same symmetric H4, so the stages commute); other powers of
// two use the Sylvester matrix as radix-2 stages followed by the 1/sqrt(r)
// normalisation.
#pragma once
#include "common.cuh"

namespace ic {

__host__ __device__ inline bool is_pow4(int n) {
  return n >= 4 && (n & (n - 1)) == 0 && (n & 0x55555555) == n;
}

// H4/2 applied to (x0,x1,x2,x3): rows +++-, ++-+, +-++, -+++ (rotation.py:51-56)
__device__ __forceinline__ void h4(float& x0, float& x1, float& x2, float& x3) {
  const float p = __fadd_rn(x0, x1), m = __fsub_rn(x0, x1);
  const float P = __fadd_rn(x2, x3), Mm = __fsub_rn(x2, x3);
  x0 = __fmul_rn(__fadd_rn(p, Mm), 0.5f);
  x1 = __fmul_rn(__fsub_rn(p, Mm), 0.5f);
  x2 = __fmul_rn(__fadd_rn(m, P), 0.5f);
  x3 = __fmul_rn(__fsub_rn(P, m), 0.5f);
}

// In-place group Hadamard on shared memory, executed by the whole CTA.  There
// are `nvec` vectors of `len` elements (len % rot == 0; each run of `rot`
// consecutive elements is one group); element e of vector v is s[v*vs + e*es].
__device__ inline void hadamard_smem(float* s, int len, int rot, int es, int nvec, int vs) {
  if (rot <= 1) return;
  if (is_pow4(rot)) {
    const int per = len / 4;
    for (int st = 1; st < rot; st *= 4) {
      for (int i = threadIdx.x; i < per * nvec; i += blockDim.x) {
        const int v = i / per, b = i % per;
        const int base = (b / st) * 4 * st + (b % st);
        float* p0 = s + v * vs + base * es;
        const int d = st * es;
        float a0 = p0[0], a1 = p0[d], a2 = p0[2 * d], a3 = p0[3 * d];
        h4(a0, a1, a2, a3);
        p0[0] = a0;
        p0[d] = a1;
        p0[2 * d] = a2;
        p0[3 * d] = a3;
      }
      __syncthreads();
    }
  } else {
    const int per = len / 2;
    for (int st = 1; st < rot; st *= 2) {
      for (int i = threadIdx.x; i < per * nvec; i += blockDim.x) {
        const int v = i / per, b = i % per;
        const int base = (b / st) * 2 * st + (b % st);
        float* p0 = s + v * vs + base * es;
        const int d = st * es;
        const float a0 = p0[0], a1 = p0[d];
        p0[0] = __fadd_rn(a0, a1);
        p0[d] = __fsub_rn(a0, a1);
      }
      __syncthreads();
    }
    const float c = (float)(1.0 / sqrt((double)rot));  // fp32(1/sqrt(n)), rotation.py:36
    for (int i = threadIdx.x; i < len * nvec; i += blockDim.x) {
      float* p = s + (i / len) * vs + (i % len) * es;
      *p = __fmul_rn(*p, c);
    }
    __syncthreads();
  }
}

}  // namespace ic
