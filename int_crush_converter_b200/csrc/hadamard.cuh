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

// s[0, len) <- fp32 of src[c0 + i] for c0 + i < N, zero beyond (the padding);
// 16-byte vector loads when the source row allows them.
template <typename T>
__device__ inline void load_row_smem(const T* __restrict__ src, int64_t c0, int64_t N, int len, float* s) {
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte load
  const bool vec = ((reinterpret_cast<uintptr_t>(src + c0) & 15) == 0) && (len % V == 0);
  if (vec) {
    for (int i = threadIdx.x * V; i < len; i += blockDim.x * V) {
      const int64_t c = c0 + i;
      if (c + V <= N) {
        const uint4 raw = *reinterpret_cast<const uint4*>(src + c);
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int u = 0; u < V; ++u) s[i + u] = load_as_f32(e + u);
      } else {
#pragma unroll
        for (int u = 0; u < V; ++u) s[i + u] = (c + u < N) ? load_as_f32(src + c + u) : 0.f;
      }
    }
  } else {
    for (int i = threadIdx.x; i < len; i += blockDim.x) {
      const int64_t c = c0 + i;
      s[i] = c < N ? load_as_f32(src + c) : 0.f;
    }
  }
}

// dst[0, len) <- s[0, len), float4 stores when dst is 16-byte aligned
__device__ inline void store_row_smem(const float* s, int len, float* __restrict__ dst) {
  if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0 && len % 4 == 0) {
    for (int i = threadIdx.x * 4; i < len; i += blockDim.x * 4)
      *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(s + i);
  } else {
    for (int i = threadIdx.x; i < len; i += blockDim.x) dst[i] = s[i];
  }
}

__host__ __device__ inline int ilog2(int v) {
  int l = 0;
  while ((1 << (l + 1)) <= v) ++l;
  return l;
}

// In-place group Hadamard on shared memory, executed by the whole CTA.  There
// are `nvec` vectors of `len` elements (len % rot == 0; each run of `rot`
// consecutive elements is one group); element e of vector v is s[v*vs + e*es].
// All strides of the butterfly index are powers of two: shifts and masks, no
// integer division.
__device__ inline void hadamard_smem(float* s, int len, int rot, int es, int nvec, int vs) {
  if (rot <= 1) return;
  const bool p4 = is_pow4(rot);
  const int radix = p4 ? 4 : 2;
  const int per = len / radix;  // butterflies per vector and stage
  // vector index of a butterfly: i / per (per is a power of two whenever nvec > 1)
  const int per_lg = ilog2(per);
  const bool per_pow2 = (1 << per_lg) == per;
  const int total = per * nvec;
  for (int st = 1, lg = 0; st < rot; st *= radix, lg += (p4 ? 2 : 1)) {
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      int v = 0, b = i;
      if (nvec > 1) {
        v = per_pow2 ? (i >> per_lg) : i / per;
        b = per_pow2 ? (i & (per - 1)) : i - v * per;
      }
      const int base = p4 ? (((b >> lg) << (lg + 2)) | (b & (st - 1))) : (((b >> lg) << (lg + 1)) | (b & (st - 1)));
      float* p0 = s + v * vs + base * es;
      const int d = st * es;
      if (p4) {
        float a0 = p0[0], a1 = p0[d], a2 = p0[2 * d], a3 = p0[3 * d];
        h4(a0, a1, a2, a3);
        p0[0] = a0;
        p0[d] = a1;
        p0[2 * d] = a2;
        p0[3 * d] = a3;
      } else {
        const float a0 = p0[0], a1 = p0[d];
        p0[0] = __fadd_rn(a0, a1);
        p0[d] = __fsub_rn(a0, a1);
      }
    }
    __syncthreads();
  }
  if (!p4) {
    const float c = (float)(1.0 / sqrt((double)rot));  // fp32(1/sqrt(n)), rotation.py:36
    const int len_lg = ilog2(len);
    const bool len_pow2 = (1 << len_lg) == len;
    for (int i = threadIdx.x; i < len * nvec; i += blockDim.x) {
      const int v = len_pow2 ? (i >> len_lg) : i / len;
      float* p = s + v * vs + (i - v * len) * es;
      *p = __fmul_rn(*p, c);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Register-resident group Hadamard for 16 <= rot <= 512 on a row held in
// shared memory (len % rot == 0), executed by the whole CTA.  A group is
// spread over L = rot/16 lanes, 16 consecutive elements per lane: the two
// (radix-4) or four (radix-2) lowest index digits are butterflies inside a
// lane's registers, the higher digits cross lanes with shfl_xor.  The stages
// run in the same digit order with the same fp32 operations as hadamard_smem,
// so the result is bit-identical; each element is read and written once.
__host__ __device__ inline bool hadamard_regs_ok(int rot) {
  return rot >= 16 && rot <= 512 && (rot & (rot - 1)) == 0;
}

// radix-4 digit across lanes: lane digit k of partner lanes l ^ (t*m), t = 1..3.
// out_k = ((a_k + a_{k^1}) + (a_{k^2} - a_{k^3})) / 2 equals output k of h4()
// for every k, operation for operation.
__device__ __forceinline__ void cross4(float (&v)[16], int m) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float a1 = __shfl_xor_sync(0xffffffffu, v[j], m);
    const float a2 = __shfl_xor_sync(0xffffffffu, v[j], 2 * m);
    const float a3 = __shfl_xor_sync(0xffffffffu, v[j], 3 * m);
    v[j] = __fmul_rn(__fadd_rn(__fadd_rn(v[j], a1), __fsub_rn(a2, a3)), 0.5f);
  }
}
// radix-2 digit across lanes: the lower index takes a + b, the upper a - b
__device__ __forceinline__ void cross2(float (&v)[16], int m, bool upper) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float o = __shfl_xor_sync(0xffffffffu, v[j], m);
    v[j] = upper ? __fsub_rn(o, v[j]) : __fadd_rn(v[j], o);
  }
}

// The group Hadamard of 16 consecutive elements per lane, L = rot/16 lanes per
// group (lane l of the group holds elements 16l .. 16l+15), all lanes of the
// warp taking part (shfl_xor).  16 <= rot <= 512.
// H4 without its factor 1/2, and cross4 likewise: the factors of all stages
// are applied at once at the end (a power of two, so every intermediate is the
// scaled twin of the per-stage result and the output is bit-identical).
__device__ __forceinline__ void h4_unscaled(float& x0, float& x1, float& x2, float& x3) {
  const float p = __fadd_rn(x0, x1), m = __fsub_rn(x0, x1);
  const float P = __fadd_rn(x2, x3), Mm = __fsub_rn(x2, x3);
  x0 = __fadd_rn(p, Mm);
  x1 = __fsub_rn(p, Mm);
  x2 = __fadd_rn(m, P);
  x3 = __fsub_rn(P, m);
}
__device__ __forceinline__ void cross4_unscaled(float (&v)[16], int m) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float a1 = __shfl_xor_sync(0xffffffffu, v[j], m);
    const float a2 = __shfl_xor_sync(0xffffffffu, v[j], 2 * m);
    const float a3 = __shfl_xor_sync(0xffffffffu, v[j], 3 * m);
    v[j] = __fadd_rn(__fadd_rn(v[j], a1), __fsub_rn(a2, a3));
  }
}

__device__ __forceinline__ void hadamard_regs16(float (&v)[16], int rot, int l) {
  const int L = rot / 16;
  const bool p4 = is_pow4(rot);
  if (p4) {
#pragma unroll
    for (int q = 0; q < 4; ++q) h4_unscaled(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
    for (int q = 0; q < 4; ++q) h4_unscaled(v[q], v[4 + q], v[8 + q], v[12 + q]);
    float scale = 0.25f;
    for (int m = 1; m < L; m <<= 2) {
      cross4_unscaled(v, m);
      scale *= 0.5f;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __fmul_rn(v[j], scale);
  } else {
#pragma unroll
    for (int st = 1; st < 16; st <<= 1) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j & st) continue;
        const float a0 = v[j], a1 = v[j + st];
        v[j] = __fadd_rn(a0, a1);
        v[j + st] = __fsub_rn(a0, a1);
      }
    }
    for (int m = 1; m < L; m <<= 1) cross2(v, m, (l & m) != 0);
    const float c = (float)(1.0 / sqrt((double)rot));  // fp32(1/sqrt(n)), rotation.py:36
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __fmul_rn(v[j], c);
  }
}

__device__ inline void hadamard_row_regs(float* s, int len, int rot) {
  const int L = rot / 16;      // lanes per group
  const int gpw = 32 / L;      // groups per warp pass
  const int ngroups = len / rot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int l = lane & (L - 1);
  for (int g0 = warp * gpw; g0 < ngroups; g0 += nw * gpw) {
    const int g = g0 + lane / L;
    const bool act = g < ngroups;
    float v[16];
    float4* p = reinterpret_cast<float4*>(s + (int64_t)(act ? g : 0) * rot + 16 * l);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 t = act ? p[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 * q] = t.x;
      v[4 * q + 1] = t.y;
      v[4 * q + 2] = t.z;
      v[4 * q + 3] = t.w;
    }
    hadamard_regs16(v, rot, l);
    if (act) {
#pragma unroll
      for (int q = 0; q < 4; ++q) p[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  }
  __syncthreads();
}

// group Hadamard of one contiguous row in shared memory (16-byte aligned)
__device__ inline void hadamard_row(float* s, int len, int rot) {
  if (hadamard_regs_ok(rot) && len % rot == 0) hadamard_row_regs(s, len, rot);
  else hadamard_smem(s, len, rot, 1, 1, 0);
}

}  // namespace ic
