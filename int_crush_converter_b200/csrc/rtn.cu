// Round-to-nearest quantization: per-group scale search, codes, INT4 packing
// and the pipeline's verify statistics, one CTA per weight row with the
// (optionally rotated) row resident in shared memory, so HBM sees each weight
// once: read fp16/bf16/fp32, write codes + scales.
//
// Arithmetic follows converter/scales.py operation by operation (fp32 IEEE,
// no contraction): scale = clamp(stat * ratio / divisor), fp16 storage,
// candidate MSE with round-half-even (Tensor.round), final codes with
// round-half-away-from-zero, strict-< ratio selection (first ratio wins ties).
#include <cstdlib>

#include "common.cuh"
#include "hadamard.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int NT = 256;
constexpr int MAX_RATIOS = 32;
constexpr int64_t MAX_ROW = 49152;  // fp32 elements of one row in shared memory

struct RtnArgs {
  const void* W;
  int dtype;
  int64_t N, ldw, npad, gs;
  int rot, bits, asym, G, nratios, given, zero_group_zp0;
  float ratios[MAX_RATIOS];
  float clamp;  // > 0: |w| > clamp zeroed on load (the pipeline's outlier sanitize)
  const uint16_t* in_scales;
  const int8_t* in_zp;
  uint16_t* scales;
  int8_t* zp;
  int8_t* codes;
  int64_t ldc;
  uint8_t* packed;
  int64_t ldp;
  double* row_sqerr;
  float* row_maxerr;
};

// Reduction over a "team": the whole CTA (CTA=true) or one warp.
template <bool CTA>
struct Team {
  float* red;  // >= 32 floats of shared scratch (CTA teams only)
  __device__ int rank() const { return CTA ? (int)threadIdx.x : (int)(threadIdx.x & 31); }
  __device__ int size() const { return CTA ? (int)blockDim.x : 32; }
  template <typename Op>
  __device__ float reduce(float v, Op op) const {
    for (int o = 16; o; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (!CTA) return v;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = op(r, red[w]);
    return r;
  }
};

struct OpMax { __device__ float operator()(float a, float b) const { return nmax(a, b); } };
struct OpMin { __device__ float operator()(float a, float b) const { return nmin(a, b); } };
struct OpSum { __device__ float operator()(float a, float b) const { return __fadd_rn(a, b); } };

__device__ __forceinline__ float clamp_scale(float s) { return clampf(s, 1e-5f, 65500.f); }

// converter/scales.py:184-229
__device__ __forceinline__ float fix_asym(float s, float wmin, float wmax, float qmin, float qmax) {
  const float spread = qmax - qmin;
  const float zr = __fsub_rn(qmin, rhaz(__fdiv_rn(wmin, s)));
  if (zr < qmin) s = fmaxf(s, clamp_scale(__fdiv_rn(wmax, spread)));
  if (zr > qmax) s = fmaxf(s, clamp_scale(__fdiv_rn(-wmin, spread)));
  return s;
}

template <bool CTA>
__device__ void process_group(const float* x, int len, const RtnArgs& a, int64_t row, int g, Team<CTA> team,
                              double& sq_acc, float& max_acc) {
  const float qmin = a.bits == 4 ? -8.f : -128.f;
  const float qmax = a.bits == 4 ? 7.f : 127.f;
  const int t = team.rank(), T = team.size();
  float s = 0.f, zp = 0.f;
  uint16_t s16;
  if (a.given) {
    s16 = a.in_scales[row * a.G + g];
    zp = a.asym ? (float)a.in_zp[row * a.G + g] : 0.f;
  } else {
    float amax = 0.f, wmin = __int_as_float(0x7f800000), wmax = __int_as_float(0xff800000);
    for (int i = t; i < len; i += T) {
      const float v = x[i];
      amax = nmax(amax, fabsf(v));
      wmin = nmin(wmin, v);
      wmax = nmax(wmax, v);
    }
    if (a.asym) {
      wmin = team.reduce(wmin, OpMin());
      wmax = team.reduce(wmax, OpMax());
    } else {
      amax = team.reduce(amax, OpMax());
    }
    const float div = a.asym ? (qmax - qmin) : (a.bits == 4 ? 7.f : 127.f);
    if (a.nratios == 0) {
      if (a.asym) {
        s = clamp_scale(__fdiv_rn(__fsub_rn(wmax, wmin), div));
        s = fix_asym(s, wmin, wmax, qmin, qmax);
        zp = clampf(__fsub_rn(qmin, rhaz(__fdiv_rn(wmin, s))), qmin, qmax);
        if (a.zero_group_zp0 && wmin == 0.f && wmax == 0.f) zp = 0.f;
      } else {
        s = clamp_scale(__fdiv_rn(amax, div));
      }
    } else {
      float best_mse = 0.f;
      for (int r = 0; r < a.nratios; ++r) {
        const float ratio = a.ratios[r];
        float cs, czp = 0.f;
        if (a.asym) {
          cs = clamp_scale(__fdiv_rn(__fmul_rn(__fsub_rn(wmax, wmin), ratio), div));
          cs = fix_asym(cs, wmin, wmax, qmin, qmax);
          czp = clampf(__fsub_rn(qmin, rhaz(__fdiv_rn(wmin, cs))), qmin, qmax);
        } else {
          cs = clamp_scale(__fdiv_rn(__fmul_rn(amax, ratio), div));
        }
        float part = 0.f;
        for (int i = t; i < len; i += T) {
          const float v = x[i];
          float y = __fdiv_rn(v, cs);
          if (a.asym) y = __fadd_rn(y, czp);
          const float q = clampf(rintf(y), qmin, qmax);
          const float deq = a.asym ? __fmul_rn(__fsub_rn(q, czp), cs) : __fmul_rn(q, cs);
          const float e = __fsub_rn(v, deq);
          part = __fadd_rn(part, __fmul_rn(e, e));
        }
        const float mse = __fdiv_rn(team.reduce(part, OpSum()), (float)len);
        if (r == 0 || mse < best_mse) {
          best_mse = mse;
          s = cs;
          zp = czp;
        }
      }
    }
    s16 = __half_as_ushort(__float2half_rn(s));
    if (t == 0) {
      if (a.scales) a.scales[row * a.G + g] = s16;
      if (a.zp && a.asym) a.zp[row * a.G + g] = (int8_t)zp;
    }
  }
  if (!(a.codes || a.packed || a.row_sqerr || a.row_maxerr)) return;
  const float sf = __half2float(__ushort_as_half(s16));
  const int64_t col0 = (int64_t)g * a.gs;
  // two adjacent columns per step so a thread owns whole packed bytes
  for (int i = 2 * t; i < len; i += 2 * T) {
    float qv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (i + u >= len) {
        qv[u] = 0.f;
        continue;
      }
      const float v = x[i + u];
      float y = __fdiv_rn(v, sf);
      if (a.asym) y = __fadd_rn(y, zp);
      const float q = clampf(rhaz(y), qmin, qmax);
      qv[u] = q;
      if (a.codes) a.codes[row * a.ldc + col0 + i + u] = (int8_t)q;
      // verify statistics over the rotated, padded W_work (pipeline.py:919-931)
      const float deq = a.asym ? __fmul_rn(__fsub_rn(q, zp), sf) : __fmul_rn(q, sf);
      const float d = __fsub_rn(v, deq);
      sq_acc += (double)d * (double)d;
      max_acc = nmax(max_acc, fabsf(d));
    }
    if (a.packed) {
      const int lo = (int)qv[0] & 15, hi = (int)qv[1] & 15;
      a.packed[row * a.ldp + (col0 + i) / 2] = (uint8_t)(lo | (hi << 4));
    }
  }
}

__global__ void __launch_bounds__(NT) rtn_row_kernel(const RtnArgs a) {
  extern __shared__ __align__(16) float row_s[];
  __shared__ float red[32];
  __shared__ double red_d[32];
  const int64_t row = blockIdx.x;
  if (a.dtype == IC_F16)
    load_row_smem(reinterpret_cast<const __half*>(a.W) + row * a.ldw, 0, a.N, (int)a.npad, row_s);
  else if (a.dtype == IC_BF16)
    load_row_smem(reinterpret_cast<const __nv_bfloat16*>(a.W) + row * a.ldw, 0, a.N, (int)a.npad, row_s);
  else
    load_row_smem(reinterpret_cast<const float*>(a.W) + row * a.ldw, 0, a.N, (int)a.npad, row_s);
  __syncthreads();
  if (a.clamp > 0.f) {
    for (int64_t i = threadIdx.x; i < a.npad; i += NT) row_s[i] = fabsf(row_s[i]) > a.clamp ? 0.f : row_s[i];
    __syncthreads();
  }
  if (a.rot > 1) hadamard_row(row_s, (int)a.npad, a.rot);
  double sq = 0.0;
  float mx = 0.f;
  if (a.G == 1) {
    Team<true> team{red};
    process_group<true>(row_s, (int)a.npad, a, row, 0, team, sq, mx);
  } else {
    Team<false> team{nullptr};
    for (int g = threadIdx.x >> 5; g < a.G; g += NT / 32)
      process_group<false>(row_s + (int64_t)g * a.gs, (int)a.gs, a, row, g, team, sq, mx);
  }
  if (a.row_sqerr || a.row_maxerr) {
    sq = warp_sum_d(sq);
    for (int o = 16; o; o >>= 1) mx = nmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
      red_d[threadIdx.x >> 5] = sq;
      red[threadIdx.x >> 5] = mx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double s = 0.0;
      float m = 0.f;
      for (int w = 0; w < NT / 32; ++w) {
        s += red_d[w];
        m = nmax(m, red[w]);
      }
      if (a.row_sqerr) a.row_sqerr[row] = s;
      if (a.row_maxerr) a.row_maxerr[row] = m;
    }
  }
}

// ---------------------------------------------------------------------------
// Register-only path for a per-row scale (G == 1), 16 <= rot <= 512 (or no
// rotation), npad <= 16 * NT: one CTA per row, lane ch of the CTA owns
// elements 16ch .. 16ch+15 of the row in registers from the load to the
// stores (no shared-memory copy of the row).  The XU pipe (reciprocal,
// conversions, floor) bounded the shared-memory kernel, so the per-element
// work here is ALU/FMA only:
//   * x / s through RN(1/s) with one FMA correction; a quotient that lands
//     within a few ulps of a rounding boundary of the code is recomputed with
//     the IEEE division, so the codes equal the shared-memory kernel's;
//   * round-half-away with an exact magic-number floor (|y| < 2^22);
//   * verify statistics as fp32 partial sums per lane (16 terms), fp64 across.
// The clip-ratio search keeps the IEEE division and round-half-even of the
// reference (its candidate MSEs decide the scale).
__device__ __forceinline__ float floor_small(float y) {  // 0 <= y < 2^22
  const float r = __fsub_rn(__fadd_rn(y, 8388608.f), 8388608.f);  // RN(y)
  return r > y ? __fsub_rn(r, 1.f) : r;
}
__device__ __forceinline__ float rhaz_fast(float x) {
  const float a = fabsf(x);
  if (!(a < 4194304.f)) return rhaz(x);  // large or NaN
  return copysignf(floor_small(__fadd_rn(a, 0.5f)), x);
}
// v / s rounded as __fdiv_rn(v, s) wherever it can change the code
__device__ __forceinline__ float code_arg(float v, float s, float rs, float z, bool has_z) {
  const float q0 = __fmul_rn(v, rs);
  const float q = __fmaf_rn(__fmaf_rn(-q0, s, v), rs, q0);
  float y = has_z ? __fadd_rn(q, z) : q;
  // The corrected quotient is within an ulp of RN(v / s); a margin of 2^-14
  // around the boundaries covers that up to |y| < 512 (ulp <= 2^-15), past
  // every code of INT4 and INT8 (also with a zero-point), so only quotients
  // that clamp to the end of the range anyway skip the check.
  const float a = fabsf(y);
  if (a < 512.f) {
    const float t = __fadd_rn(a, 0.5f);
    const float d = __fsub_rn(t, floor_small(t));
    if (d < 0x1p-14f || d > 1.f - 0x1p-14f) {
      y = __fdiv_rn(v, s);
      if (has_z) y = __fadd_rn(y, z);
    }
  }
  return y;
}

// two's-complement bits of an integer-valued float in [-2^22, 2^22] without
// the conversion unit: x + 1.5*2^23 holds x in its low mantissa bits
__device__ __forceinline__ uint32_t small_int_bits(float x) {
  return (uint32_t)__float_as_int(__fadd_rn(x, 12582912.f)) - 0x4B400000u;
}

template <typename Op>
__device__ __forceinline__ float cta_reduce(float v, Op op, float* red) {
  for (int o = 16; o; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = op(r, red[w]);
  return r;
}

template <typename T>
__global__ void __launch_bounds__(NT) rtn_regs_kernel(const RtnArgs a) {
  __shared__ float red[32];
  __shared__ double red_d[32];
  const int64_t row = blockIdx.x;
  const int ch = threadIdx.x;
  const int64_t c0 = (int64_t)ch * 16;
  const bool act = c0 < a.npad;
  const float qmin = a.bits == 4 ? -8.f : -128.f;
  const float qmax = a.bits == 4 ? 7.f : 127.f;

  float v[16];
  const T* src = reinterpret_cast<const T*>(a.W) + row * a.ldw + c0;
  constexpr int V = 16 / sizeof(T);
  if (act && c0 + 16 <= a.N && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < 16 / V; ++q) {
      const uint4 raw = reinterpret_cast<const uint4*>(src)[q];
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int u = 0; u < V; ++u) v[q * V + u] = load_as_f32(e + u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = (act && c0 + j < a.N) ? load_as_f32(src + j) : 0.f;
  }
  if (a.clamp > 0.f) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = fabsf(v[j]) > a.clamp ? 0.f : v[j];
  }
  if (a.rot > 1) hadamard_regs16(v, a.rot, ch & (a.rot / 16 - 1));

  // ---- per-row scale (converter/scales.py, as process_group) ----
  float s = 0.f, zp = 0.f;
  {
    float amax = 0.f, wmin = __int_as_float(0x7f800000), wmax = __int_as_float(0xff800000);
    if (act) {
      if (a.asym) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          wmin = nmin(wmin, v[j]);
          wmax = nmax(wmax, v[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) amax = nmax(amax, fabsf(v[j]));
      }
    }
    if (a.asym) {
      wmin = cta_reduce(wmin, OpMin(), red);
      wmax = cta_reduce(wmax, OpMax(), red);
    } else {
      amax = cta_reduce(amax, OpMax(), red);
    }
    const float div = a.asym ? (qmax - qmin) : (a.bits == 4 ? 7.f : 127.f);
    if (a.nratios == 0) {
      if (a.asym) {
        s = clamp_scale(__fdiv_rn(__fsub_rn(wmax, wmin), div));
        s = fix_asym(s, wmin, wmax, qmin, qmax);
        zp = clampf(__fsub_rn(qmin, rhaz(__fdiv_rn(wmin, s))), qmin, qmax);
        if (a.zero_group_zp0 && wmin == 0.f && wmax == 0.f) zp = 0.f;
      } else {
        s = clamp_scale(__fdiv_rn(amax, div));
      }
    } else {
      float best_mse = 0.f;
      for (int r = 0; r < a.nratios; ++r) {
        const float ratio = a.ratios[r];
        float cs, czp = 0.f;
        if (a.asym) {
          cs = clamp_scale(__fdiv_rn(__fmul_rn(__fsub_rn(wmax, wmin), ratio), div));
          cs = fix_asym(cs, wmin, wmax, qmin, qmax);
          czp = clampf(__fsub_rn(qmin, rhaz(__fdiv_rn(wmin, cs))), qmin, qmax);
        } else {
          cs = clamp_scale(__fdiv_rn(__fmul_rn(amax, ratio), div));
        }
        float part = 0.f;
        if (act) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float y = __fdiv_rn(v[j], cs);
            if (a.asym) y = __fadd_rn(y, czp);
            const float q = clampf(rintf(y), qmin, qmax);
            const float deq = a.asym ? __fmul_rn(__fsub_rn(q, czp), cs) : __fmul_rn(q, cs);
            const float e = __fsub_rn(v[j], deq);
            part = __fadd_rn(part, __fmul_rn(e, e));
          }
        }
        const float mse = __fdiv_rn(cta_reduce(part, OpSum(), red), (float)a.npad);
        if (r == 0 || mse < best_mse) {
          best_mse = mse;
          s = cs;
          zp = czp;
        }
      }
    }
  }
  const uint16_t s16 = __half_as_ushort(__float2half_rn(s));
  if (threadIdx.x == 0) {
    if (a.scales) a.scales[row] = s16;
    if (a.zp && a.asym) a.zp[row] = (int8_t)zp;
  }

  // ---- codes, packing, verify statistics ----
  const float sf = __half2float(__ushort_as_half(s16));
  const float rs = __frcp_rn(sf);
  float part = 0.f, mx = 0.f;
  float q[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    q[j] = clampf(rhaz_fast(code_arg(v[j], sf, rs, zp, a.asym != 0)), qmin, qmax);
    const float deq = a.asym ? __fmul_rn(__fsub_rn(q[j], zp), sf) : __fmul_rn(q[j], sf);
    const float d = __fsub_rn(v[j], deq);
    part = __fmaf_rn(d, d, part);
    mx = nmax(mx, fabsf(d));
  }
  if (act) {
    if (a.codes) {
      int8_t* dst = a.codes + row * a.ldc + c0;
      uint32_t w4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        w4[i] = (small_int_bits(q[4 * i]) & 255u) | ((small_int_bits(q[4 * i + 1]) & 255u) << 8) |
                ((small_int_bits(q[4 * i + 2]) & 255u) << 16) | ((small_int_bits(q[4 * i + 3]) & 255u) << 24);
      if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) dst[j] = (int8_t)q[j];
      }
    }
    if (a.packed) {
      uint8_t* dst = a.packed + row * a.ldp + c0 / 2;
      uint32_t p2[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 16; ++j) p2[j >> 3] |= (small_int_bits(q[j]) & 15u) << (4 * (j & 7));
      if ((reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(p2[0], p2[1]);
      } else {
#pragma unroll
        for (int b = 0; b < 8; ++b) dst[b] = (uint8_t)(p2[b >> 2] >> (8 * (b & 3)));
      }
    }
  } else {
    part = 0.f;
    mx = 0.f;
  }
  if (a.row_sqerr || a.row_maxerr) {
    double sq = warp_sum_d((double)part);
    for (int o = 16; o; o >>= 1) mx = nmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
      red_d[threadIdx.x >> 5] = sq;
      red[threadIdx.x >> 5] = mx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      float m = 0.f;
      for (int w = 0; w < NT / 32; ++w) {
        t += red_d[w];
        m = nmax(m, red[w]);
      }
      if (a.row_sqerr) a.row_sqerr[row] = t;
      if (a.row_maxerr) a.row_maxerr[row] = m;
    }
  }
}

// ---------------------------------------------------------------------------
// Fast path for the common shape of the fused RTN call: one scale per row,
// a regular (power-of-four) rotation of 16, 64 or 256, rows of at most 4096
// elements.  Same results as rtn_regs_kernel, fewer instructions per weight:
//   * the Hadamard's 1/2 per radix-4 stage is deferred: the butterflies run on
//     2^k-scaled values (k = log4(rot)); every quantity the kernel derives from
//     them (absmax, quotients against the 2^k-scaled scale, errors, squared
//     errors) is the unscaled one times a power of two, exactly, so codes,
//     scales and statistics are bit-identical;
//   * for rot 256 the two cross-lane digits go through one shared-memory
//     transpose (16 stores + 4 vector loads per lane) instead of 6 shuffles per
//     element, and the codes come back through a byte transpose for packing;
//   * NaN-propagating max as one max.NaN instruction;
//   * round-half-away-from-zero and the check for quotients next to a rounding
//     boundary fused (floor by a round-down add of 1.5 * 2^23);
//   * the clipping-ratio search takes the FMA-corrected quotient and its
//     round-half-even by the same magic add, and falls back to the IEEE
//     division only for quotients within 2^-14 of a tie.
__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float min_nan(float a, float b) {
  float d;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
// y = RN(v / s) for the code's round-half-away, from rs = RN(1/s): corrected
// quotient, then exact IEEE division when |y| + 1/2 lies within 2^-14 of an
// integer (the only quotients whose code the last ulp can change).  Returns
// the rounded magnitude floor(|y| + 1/2) as a float and y itself.
__device__ __forceinline__ float fast_rhaz(float v, float s, float rs, float z, bool has_z) {
  const float q0 = __fmul_rn(v, rs);
  float y = __fmaf_rn(__fmaf_rn(-q0, s, v), rs, q0);
  if (has_z) y = __fadd_rn(y, z);
  const float t = __fadd_rn(fabsf(y), 0.5f);
  float fl = __fsub_rn(__fadd_rd(t, 12582912.f), 12582912.f);  // floor(t), t < 2^22
  const float d = __fsub_rn(t, fl);
  if (!(t < 4194304.f) || d < 0x1p-14f || d > 1.f - 0x1p-14f) {
    y = __fdiv_rn(v, s);
    if (has_z) y = __fadd_rn(y, z);
    return rhaz(y);
  }
  return copysignf(fl, y);
}
// round-half-even of RN(v / s) (Tensor.round in the clip search), same scheme
__device__ __forceinline__ float fast_rint_div(float v, float s, float rs, float z, bool has_z) {
  const float q0 = __fmul_rn(v, rs);
  float y = __fmaf_rn(__fmaf_rn(-q0, s, v), rs, q0);
  if (has_z) y = __fadd_rn(y, z);
  const float r = __fsub_rn(__fadd_rn(y, 12582912.f), 12582912.f);  // RN-even, |y| < 2^22
  const float d = fabsf(__fsub_rn(y, r));
  if (!(fabsf(y) < 4194304.f) || d > 0.5f - 0x1p-14f) {
    y = __fdiv_rn(v, s);
    if (has_z) y = __fadd_rn(y, z);
    return rintf(y);
  }
  return r;
}

template <typename T, int ROT>
__global__ void __launch_bounds__(NT) rtn_fast_kernel(const RtnArgs a) {
  constexpr int K = ROT == 256 ? 4 : (ROT == 64 ? 3 : 2);  // radix-4 stages
  constexpr float DESCALE = ROT == 256 ? 0.0625f : (ROT == 64 ? 0.125f : 0.25f);
  constexpr float UP = 1.f / DESCALE;
  constexpr int TP = 16 * 16 + 16;  // transpose stride per 16-lane group (floats)
  __shared__ __align__(16) float tr[(NT / 16) * TP];
  __shared__ float red[32];
  __shared__ double red_d[32];
  const int64_t row = blockIdx.x;
  const int ch = threadIdx.x;
  const int64_t c0 = (int64_t)ch * 16;
  const bool act = c0 < a.npad;
  const bool has_z = a.asym != 0;
  const float qmin = a.bits == 4 ? -8.f : -128.f;
  const float qmax = a.bits == 4 ? 7.f : 127.f;

  float v[16];
  const T* src = reinterpret_cast<const T*>(a.W) + row * a.ldw + c0;
  constexpr int V = 16 / sizeof(T);
  if (act && c0 + 16 <= a.N && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < 16 / V; ++q) {
      const uint4 raw = reinterpret_cast<const uint4*>(src)[q];
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int u = 0; u < V; ++u) v[q * V + u] = load_as_f32(e + u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = (act && c0 + j < a.N) ? load_as_f32(src + j) : 0.f;
  }
  if (a.clamp > 0.f) {  // outlier sanitize; the select loop only when a weight exceeds the clamp
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) m = fmaxf(m, fabsf(v[j]));
    if (m > a.clamp) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = fabsf(v[j]) > a.clamp ? 0.f : v[j];
    }
  }
  // ---- group Hadamard, scaled by 2^K ----
#pragma unroll
  for (int q = 0; q < 4; ++q) h4_unscaled(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
  for (int q = 0; q < 4; ++q) h4_unscaled(v[q], v[4 + q], v[8 + q], v[12 + q]);
  const int lane16 = ch & 15;
  float* trg = tr + (ch >> 4) * TP;
  if (ROT == 64) cross4_unscaled(v, 1);
  if (ROT == 256) {
    // lane l (of the group's 16) holds in-group elements 16 l + j.  Transpose so
    // that lane t holds elements 16 l' + t for l' = 0..15: its 16 values then
    // span the two high digits.  Element (l, j) goes to row j of the group's
    // tile at column chunk ((l >> 2) + (j >> 1)) & 3 (a skew that keeps both
    // the scalar stores and the vector loads free of bank conflicts).
    const int lq = lane16 >> 2, lr = lane16 & 3;
    int off[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) off[k] = (((lq + k) & 3) << 2) + lr;
#pragma unroll
    for (int j = 0; j < 16; ++j) trg[j * 16 + off[(j >> 1) & 3]] = v[j];
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 t = *reinterpret_cast<const float4*>(trg + lane16 * 16 + ((((c + (lane16 >> 1)) & 3)) << 2));
      v[4 * c] = t.x;
      v[4 * c + 1] = t.y;
      v[4 * c + 2] = t.z;
      v[4 * c + 3] = t.w;
    }
    // v[4c + u] = element (l' = 4c + u, j = lane16): digits l' & 3 (u) and l' >> 2 (c)
#pragma unroll
    for (int c = 0; c < 4; ++c) h4_unscaled(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
#pragma unroll
    for (int u = 0; u < 4; ++u) h4_unscaled(v[u], v[4 + u], v[8 + u], v[12 + u]);
  }
  (void)K;

  // ---- per-row scale (converter/scales.py), on the scaled values ----
  float s = 0.f, zp = 0.f;
  {
    float amax = 0.f, wmin = __int_as_float(0x7f800000), wmax = __int_as_float(0xff800000);
    if (act) {
      if (has_z) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          wmin = min_nan(wmin, v[j]);
          wmax = max_nan(wmax, v[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) amax = max_nan(amax, fabsf(v[j]));
      }
    }
    if (has_z) {
      wmin = __fmul_rn(cta_reduce(wmin, OpMin(), red), DESCALE);
      wmax = __fmul_rn(cta_reduce(wmax, OpMax(), red), DESCALE);
    } else {
      amax = __fmul_rn(cta_reduce(amax, OpMax(), red), DESCALE);
    }
    const float div = has_z ? (qmax - qmin) : (a.bits == 4 ? 7.f : 127.f);
    if (a.nratios == 0) {
      if (has_z) {
        s = clamp_scale(__fdiv_rn(__fsub_rn(wmax, wmin), div));
        s = fix_asym(s, wmin, wmax, qmin, qmax);
        zp = clampf(__fsub_rn(qmin, rhaz(__fdiv_rn(wmin, s))), qmin, qmax);
        if (a.zero_group_zp0 && wmin == 0.f && wmax == 0.f) zp = 0.f;
      } else {
        s = clamp_scale(__fdiv_rn(amax, div));
      }
    } else {
      float best_mse = 0.f;
      for (int r = 0; r < a.nratios; ++r) {
        const float ratio = a.ratios[r];
        float cs, czp = 0.f;
        if (has_z) {
          cs = clamp_scale(__fdiv_rn(__fmul_rn(__fsub_rn(wmax, wmin), ratio), div));
          cs = fix_asym(cs, wmin, wmax, qmin, qmax);
          czp = clampf(__fsub_rn(qmin, rhaz(__fdiv_rn(wmin, cs))), qmin, qmax);
        } else {
          cs = clamp_scale(__fdiv_rn(__fmul_rn(amax, ratio), div));
        }
        const float csk = __fmul_rn(cs, UP), rcs = __frcp_rn(csk);
        float part = 0.f;
        if (act) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float q = clampf(fast_rint_div(v[j], csk, rcs, czp, has_z), qmin, qmax);
            const float deq = has_z ? __fmul_rn(__fsub_rn(q, czp), csk) : __fmul_rn(q, csk);
            const float e = __fsub_rn(v[j], deq);
            part = __fadd_rn(part, __fmul_rn(e, e));
          }
        }
        // the common 2^2K factor does not change which candidate wins
        const float mse = __fdiv_rn(cta_reduce(part, OpSum(), red), (float)a.npad);
        if (r == 0 || mse < best_mse) {
          best_mse = mse;
          s = cs;
          zp = czp;
        }
      }
    }
  }
  const uint16_t s16 = __half_as_ushort(__float2half_rn(s));
  if (threadIdx.x == 0) {
    if (a.scales) a.scales[row] = s16;
    if (a.zp && a.asym) a.zp[row] = (int8_t)zp;
  }

  // ---- codes, verify statistics (scaled), packing ----
  const float sk = __fmul_rn(__half2float(__ushort_as_half(s16)), UP);
  const float rs = __frcp_rn(sk);
  float part = 0.f, mx = 0.f;
  uint32_t cb[4] = {0u, 0u, 0u, 0u};  // the 16 codes as bytes, in register order
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float q = clampf(fast_rhaz(v[j], sk, rs, zp, has_z), qmin, qmax);
    const float deq = has_z ? __fmul_rn(__fsub_rn(q, zp), sk) : __fmul_rn(q, sk);
    const float d = __fsub_rn(v[j], deq);
    part = __fmaf_rn(d, d, part);
    mx = max_nan(mx, fabsf(d));
    cb[j >> 2] |= (small_int_bits(q) & 255u) << (8 * (j & 3));
  }
  if (ROT == 256) {
    // back to row order: byte (l', j) of the group's 16 x 16 code tile
    __syncwarp();
    uint8_t* tb = reinterpret_cast<uint8_t*>(trg);
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int u = 0; u < 4; ++u) tb[(4 * c + u) * 16 + lane16] = (uint8_t)(cb[c] >> (8 * u));
    __syncwarp();
    const uint4 t = *reinterpret_cast<const uint4*>(tb + lane16 * 16);
    cb[0] = t.x;
    cb[1] = t.y;
    cb[2] = t.z;
    cb[3] = t.w;
  }
  if (act) {
    if (a.codes) {
      int8_t* dst = a.codes + row * a.ldc + c0;
      if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(cb[0], cb[1], cb[2], cb[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) dst[j] = (int8_t)(cb[j >> 2] >> (8 * (j & 3)));
      }
    }
    if (a.packed) {
      uint32_t p2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        // bytes b0..b7 (two words) -> nibbles: (b0 & 15) | (b1 & 15) << 4 | ...
        uint32_t x = cb[2 * h] & 0x0F0F0F0Fu, y = cb[2 * h + 1] & 0x0F0F0F0Fu;
        x = (x | (x >> 4)) & 0x00FF00FFu;
        y = (y | (y >> 4)) & 0x00FF00FFu;
        p2[h] = __byte_perm(x, y, 0x6420);
      }
      uint8_t* dst = a.packed + row * a.ldp + c0 / 2;
      if ((reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(p2[0], p2[1]);
      } else {
#pragma unroll
        for (int b = 0; b < 8; ++b) dst[b] = (uint8_t)(p2[b >> 2] >> (8 * (b & 3)));
      }
    }
  } else {
    part = 0.f;
    mx = 0.f;
  }
  if (a.row_sqerr || a.row_maxerr) {
    double sq = warp_sum_d((double)part);
    for (int o = 16; o; o >>= 1) mx = max_nan(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
      red_d[threadIdx.x >> 5] = sq;
      red[threadIdx.x >> 5] = mx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      float m = 0.f;
      for (int w = 0; w < NT / 32; ++w) {
        t += red_d[w];
        m = nmax(m, red[w]);
      }
      if (a.row_sqerr) a.row_sqerr[row] = t * (double)DESCALE * (double)DESCALE;
      if (a.row_maxerr) a.row_maxerr[row] = __fmul_rn(m, DESCALE);
    }
  }
}

// ---------------------------------------------------------------------------
// Paired fast path (rows of 1024 * k <= 4096 elements): each thread owns two
// chunks of 16 elements that sit at the same position of two groups half a
// row apart (columns 16t.. and npad/2 + 16t..), so every per-element operation
// of the two chunks is the same instruction on different data: they run as
// the sm_100 packed fp32 pair instructions (add/sub/mul/fma .f32x2, IEEE
// round-to-nearest per lane like the scalar ones, so results stay
// bit-identical), halving the instruction count of the butterflies, the
// quotients, the rounding and the statistics.  One CTA of npad/32 threads per
// row; otherwise the same algorithm as rtn_fast_kernel.
typedef unsigned long long f2;
__device__ __forceinline__ f2 pk(float a, float b) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float lo_of(f2 r) { return __uint_as_float((uint32_t)(r & 0xffffffffull)); }
__device__ __forceinline__ float hi_of(f2 r) { return __uint_as_float((uint32_t)(r >> 32)); }
__device__ __forceinline__ uint32_t lo_of_bits(f2 r) { return (uint32_t)(r & 0xffffffffull); }
__device__ __forceinline__ uint32_t hi_of_bits(f2 r) { return (uint32_t)(r >> 32); }
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 add2_rm(f2 a, f2 b) {
  f2 d;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ void h4p(f2& x0, f2& x1, f2& x2, f2& x3) {
  const f2 p = add2(x0, x1), m = sub2(x0, x1), P = add2(x2, x3), Mm = sub2(x2, x3);
  x0 = add2(p, Mm);
  x1 = sub2(p, Mm);
  x2 = add2(m, P);
  x3 = sub2(P, m);
}
__device__ __forceinline__ float clamp_nan(float x, float lo, float hi) { return min_nan(max_nan(x, lo), hi); }
constexpr float MAGIC = 12582912.f;  // 1.5 * 2^23

template <typename T, int ROT>
__global__ void __launch_bounds__(128) rtn_pair_kernel(const RtnArgs a) {
  constexpr float DESCALE = ROT == 256 ? 0.0625f : (ROT == 64 ? 0.125f : 0.25f);
  constexpr float UP = 1.f / DESCALE;
  __shared__ __align__(16) f2 tr[(128 / 16) * 256];  // one 16 x 16 tile of pairs per 16-lane group
  __shared__ float red[8];
  __shared__ double red_d[8];
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x, nt = blockDim.x;
  const int64_t half = a.npad / 2;
  const int64_t ca = (int64_t)t * 16, cb = half + ca;
  const bool has_z = a.asym != 0;
  const float qmin = a.bits == 4 ? -8.f : -128.f;
  const float qmax = a.bits == 4 ? 7.f : 127.f;

  f2 v[16];
  {
    float x[16], y[16];
    const T* src = reinterpret_cast<const T*>(a.W) + row * a.ldw;
    constexpr int V = 16 / sizeof(T);
    const bool fa = ca + 16 <= a.N && (reinterpret_cast<uintptr_t>(src + ca) & 15) == 0;
    const bool fb = cb + 16 <= a.N && (reinterpret_cast<uintptr_t>(src + cb) & 15) == 0;
    if (fa) {
#pragma unroll
      for (int q = 0; q < 16 / V; ++q) {
        const uint4 raw = reinterpret_cast<const uint4*>(src + ca)[q];
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int u = 0; u < V; ++u) x[q * V + u] = load_as_f32(e + u);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = ca + j < a.N ? load_as_f32(src + ca + j) : 0.f;
    }
    if (fb) {
#pragma unroll
      for (int q = 0; q < 16 / V; ++q) {
        const uint4 raw = reinterpret_cast<const uint4*>(src + cb)[q];
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int u = 0; u < V; ++u) y[q * V + u] = load_as_f32(e + u);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) y[j] = cb + j < a.N ? load_as_f32(src + cb + j) : 0.f;
    }
    if (a.clamp > 0.f) {
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) m = fmaxf(m, fmaxf(fabsf(x[j]), fabsf(y[j])));
      if (m > a.clamp) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          x[j] = fabsf(x[j]) > a.clamp ? 0.f : x[j];
          y[j] = fabsf(y[j]) > a.clamp ? 0.f : y[j];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = pk(x[j], y[j]);
  }
  // ---- group Hadamard on the pairs, scaled by 2^K ----
#pragma unroll
  for (int q = 0; q < 4; ++q) h4p(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
  for (int q = 0; q < 4; ++q) h4p(v[q], v[4 + q], v[8 + q], v[12 + q]);
  const int lane16 = t & 15;
  f2* trg = tr + (t >> 4) * 256;
  if (ROT == 64) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const f2 a1 = __shfl_xor_sync(0xffffffffu, v[j], 1);
      const f2 a2 = __shfl_xor_sync(0xffffffffu, v[j], 2);
      const f2 a3 = __shfl_xor_sync(0xffffffffu, v[j], 3);
      v[j] = add2(add2(v[j], a1), sub2(a2, a3));
    }
  }
  if (ROT == 256) {
    // as rtn_fast_kernel, with 8-byte elements: element (l, j) goes to row j,
    // pair slot 2 * (((l >> 1) + j) & 7) + (l & 1); lane t then reads row t as
    // eight 16-byte chunks starting at chunk t (a rotation that keeps each
    // quarter-warp's 128-bit loads on distinct banks)
#pragma unroll
    for (int j = 0; j < 16; ++j) trg[j * 16 + 2 * (((lane16 >> 1) + j) & 7) + (lane16 & 1)] = v[j];
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 w = *reinterpret_cast<const uint4*>(trg + lane16 * 16 + 2 * ((c + lane16) & 7));
      // slot c' = (c + t) & 7 holds l' = 2c'' with c'' = (c' - t) & 7 = c
      v[2 * c] = ((f2)w.y << 32) | w.x;
      v[2 * c + 1] = ((f2)w.w << 32) | w.z;
    }
    // v[l'] = element (l', j = lane16): digits l' & 3 and l' >> 2
#pragma unroll
    for (int c = 0; c < 4; ++c) h4p(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
#pragma unroll
    for (int u = 0; u < 4; ++u) h4p(v[u], v[4 + u], v[8 + u], v[12 + u]);
  }

  // ---- per-row scale on the scaled values (both chunks belong to the row) ----
  float s = 0.f, zp = 0.f;
  {
    const float div = has_z ? (qmax - qmin) : (a.bits == 4 ? 7.f : 127.f);
    const int w = t >> 5, nw = nt >> 5;
    float amax = 0.f, wmin = __int_as_float(0x7f800000), wmax = __int_as_float(0xff800000);
    if (has_z) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        wmin = min_nan(wmin, min_nan(lo_of(v[j]), hi_of(v[j])));
        wmax = max_nan(wmax, max_nan(lo_of(v[j]), hi_of(v[j])));
      }
      float r0, r1;
      asm("redux.sync.min.NaN.f32 %0, %1, 0xffffffff;" : "=f"(r0) : "f"(wmin));
      asm("redux.sync.max.NaN.f32 %0, %1, 0xffffffff;" : "=f"(r1) : "f"(wmax));
      if ((t & 31) == 0) {
        red[w] = r0;
        red[4 + w] = r1;
      }
      __syncthreads();
      wmin = red[0];
      wmax = red[4];
      for (int k = 1; k < nw; ++k) {
        wmin = nmin(wmin, red[k]);
        wmax = nmax(wmax, red[4 + k]);
      }
      wmin = __fmul_rn(wmin, DESCALE);
      wmax = __fmul_rn(wmax, DESCALE);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) amax = max_nan(amax, max_nan(fabsf(lo_of(v[j])), fabsf(hi_of(v[j]))));
      float r0;
      asm("redux.sync.max.abs.NaN.f32 %0, %1, 0xffffffff;" : "=f"(r0) : "f"(amax));
      if ((t & 31) == 0) red[w] = r0;
      __syncthreads();
      amax = red[0];
      for (int k = 1; k < nw; ++k) amax = nmax(amax, red[k]);
      amax = __fmul_rn(amax, DESCALE);
    }
    if (a.nratios == 0) {
      if (has_z) {
        s = clamp_scale(__fdiv_rn(__fsub_rn(wmax, wmin), div));
        s = fix_asym(s, wmin, wmax, qmin, qmax);
        zp = clampf(__fsub_rn(qmin, rhaz(__fdiv_rn(wmin, s))), qmin, qmax);
        if (a.zero_group_zp0 && wmin == 0.f && wmax == 0.f) zp = 0.f;
      } else {
        s = clamp_scale(__fdiv_rn(amax, div));
      }
    } else {
      float best_mse = 0.f;
      for (int r = 0; r < a.nratios; ++r) {
        const float ratio = a.ratios[r];
        float cs, czp = 0.f;
        if (has_z) {
          cs = clamp_scale(__fdiv_rn(__fmul_rn(__fsub_rn(wmax, wmin), ratio), div));
          cs = fix_asym(cs, wmin, wmax, qmin, qmax);
          czp = clampf(__fsub_rn(qmin, rhaz(__fdiv_rn(wmin, cs))), qmin, qmax);
        } else {
          cs = clamp_scale(__fdiv_rn(__fmul_rn(amax, ratio), div));
        }
        const float csk = __fmul_rn(cs, UP), rcs = __frcp_rn(csk);
        const f2 S = pk(csk, csk), RS = pk(rcs, rcs), Z = pk(czp, czp);
        const f2 M2 = pk(MAGIC, MAGIC);
        const float THR = has_z ? 0x1p-13f : 0x1p-14f;
        f2 part2 = 0ull;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          // y = v * RN(1/s) (+ z), uncorrected: within 3 * 2^-24 * |v/s| of the
          // IEEE quotient, and a code can only change while |v/s| <= 2^8 + 1
          // (beyond, both roundings clamp alike), so y is within 4.6e-5 of the
          // reference's RN(v/s) (+ z) there; a fractional part within THR of
          // .5 takes the exact division
          f2 y = mul2(v[j], RS);
          if (has_z) y = add2(y, Z);
          // round-half-even by the magic add (|y| stays far below 2^22 here:
          // |v| <= the row's absmax and cs >= absmax * 0.8 / 127 up to the
          // scale clamp; a NaN fails the test below and takes the exact path)
          f2 rq = sub2(add2(y, M2), M2);
          const f2 dy = sub2(y, rq);
          float r0 = lo_of(rq), r1 = hi_of(rq);
          if (!(fabsf(lo_of(dy)) <= 0.5f - THR)) {
            float e = __fdiv_rn(lo_of(v[j]), csk);
            if (has_z) e = __fadd_rn(e, czp);
            r0 = rintf(e);
          }
          if (!(fabsf(hi_of(dy)) <= 0.5f - THR)) {
            float e = __fdiv_rn(hi_of(v[j]), csk);
            if (has_z) e = __fadd_rn(e, czp);
            r1 = rintf(e);
          }
          const f2 q = pk(clamp_nan(r0, qmin, qmax), clamp_nan(r1, qmin, qmax));
          const f2 deq = has_z ? mul2(sub2(q, Z), S) : mul2(q, S);
          const f2 e = sub2(v[j], deq);
          part2 = add2(part2, mul2(e, e));
        }
        // the same fp32 sum as rtn_fast_kernel: a chunk's 16 terms in order, a
        // warp's chunks by an xor tree, then the warps in order -- chunk-a warps
        // first (columns [0, npad/2)), then chunk-b warps
        float tot;
        {
          f2 x = part2;
          for (int o = 16; o; o >>= 1) x = add2(x, __shfl_xor_sync(0xffffffffu, x, o));
          const int nw = nt >> 5;
          __syncthreads();
          if ((t & 31) == 0) {
            red[t >> 5] = lo_of(x);
            red[nw + (t >> 5)] = hi_of(x);
          }
          __syncthreads();
          tot = red[0];
          for (int k = 1; k < 2 * nw; ++k) tot = __fadd_rn(tot, red[k]);
        }
        const float mse = __fdiv_rn(tot, (float)a.npad);
        if (r == 0 || mse < best_mse) {
          best_mse = mse;
          s = cs;
          zp = czp;
        }
      }
    }
  }
  const uint16_t s16 = __half_as_ushort(__float2half_rn(s));
  if (t == 0) {
    if (a.scales) a.scales[row] = s16;
    if (a.zp && a.asym) a.zp[row] = (int8_t)zp;
  }

  // ---- codes, statistics, packing ----
  const float sk = __fmul_rn(__half2float(__ushort_as_half(s16)), UP);
  const float rsk = __frcp_rn(sk);
  const f2 S = pk(sk, sk), RS = pk(rsk, rsk), Z = pk(zp, zp);
  const f2 HALF = pk(0.5f, 0.5f), M2 = pk(MAGIC, MAGIC);
  const float THR = has_z ? 0x1p-13f : 0x1p-14f;  // as in the clip search
  f2 part2 = 0ull;
  float mx = 0.f;
  uint32_t ca4[4] = {0u, 0u, 0u, 0u}, cb4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    // uncorrected quotient, as in the clip search
    f2 y = mul2(v[j], RS);
    if (has_z) y = add2(y, Z);
    const f2 ay = pk(fabsf(lo_of(y)), fabsf(hi_of(y)));
    const f2 tt = add2(ay, HALF);
    const f2 fl = sub2(add2_rm(tt, M2), M2);  // floor(|y| + 1/2)
    const f2 d = sub2(tt, fl);
    float q0 = copysignf(lo_of(fl), lo_of(y)), q1 = copysignf(hi_of(fl), hi_of(y));
    // |y| + 1/2 near an integer (d near 0 or 1): the exact division decides.
    // |y| is bounded by the scale (|v| <= absmax, s >= absmax / 7.x, or the
    // asymmetric range); a NaN passes the test and stays NaN as rhaz(NaN).
    const f2 dh = sub2(d, HALF);
    if (fabsf(lo_of(dh)) > 0.5f - THR) {
      float e = __fdiv_rn(lo_of(v[j]), sk);
      if (has_z) e = __fadd_rn(e, zp);
      q0 = rhaz(e);
    }
    if (fabsf(hi_of(dh)) > 0.5f - THR) {
      float e = __fdiv_rn(hi_of(v[j]), sk);
      if (has_z) e = __fadd_rn(e, zp);
      q1 = rhaz(e);
    }
    const f2 q = pk(clamp_nan(q0, qmin, qmax), clamp_nan(q1, qmin, qmax));
    const f2 deq = has_z ? mul2(sub2(q, Z), S) : mul2(q, S);
    const f2 e = sub2(v[j], deq);
    part2 = fma2(e, e, part2);
    mx = max_nan(mx, max_nan(fabsf(lo_of(e)), fabsf(hi_of(e))));
    const f2 bits = add2(q, M2);  // low byte = two's-complement code
    ca4[j >> 2] |= ((uint32_t)lo_of_bits(bits) & 255u) << (8 * (j & 3));
    cb4[j >> 2] |= ((uint32_t)hi_of_bits(bits) & 255u) << (8 * (j & 3));
  }
  if (ROT == 256) {
    // codes back to row order through a 16 x 16 tile of 16-bit (chunk a, chunk b) pairs
    __syncwarp();
    uint16_t* tb = reinterpret_cast<uint16_t*>(trg);
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int u = 0; u < 4; ++u)
        tb[(4 * c + u) * 16 + lane16] =
            (uint16_t)(((ca4[c] >> (8 * u)) & 255u) | (((cb4[c] >> (8 * u)) & 255u) << 8));
    __syncwarp();
    const uint4 w0 = *reinterpret_cast<const uint4*>(tb + lane16 * 16);
    const uint4 w1 = *reinterpret_cast<const uint4*>(tb + lane16 * 16 + 8);
    const uint32_t wd[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      ca4[k] = __byte_perm(wd[2 * k], wd[2 * k + 1], 0x6420);
      cb4[k] = __byte_perm(wd[2 * k], wd[2 * k + 1], 0x7531);
    }
  }
  const int64_t cols[2] = {ca, cb};
  const uint32_t* cw[2] = {ca4, cb4};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t* c4 = cw[h];
    if (a.codes) {
      int8_t* dst = a.codes + row * a.ldc + cols[h];
      if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(c4[0], c4[1], c4[2], c4[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) dst[j] = (int8_t)(c4[j >> 2] >> (8 * (j & 3)));
      }
    }
    if (a.packed) {
      uint32_t p2[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        uint32_t x = c4[2 * k] & 0x0F0F0F0Fu, y = c4[2 * k + 1] & 0x0F0F0F0Fu;
        x = (x | (x >> 4)) & 0x00FF00FFu;
        y = (y | (y >> 4)) & 0x00FF00FFu;
        p2[k] = __byte_perm(x, y, 0x6420);
      }
      uint8_t* dst = a.packed + row * a.ldp + cols[h] / 2;
      if ((reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(p2[0], p2[1]);
      } else {
#pragma unroll
        for (int b = 0; b < 8; ++b) dst[b] = (uint8_t)(p2[b >> 2] >> (8 * (b & 3)));
      }
    }
  }
  if (a.row_sqerr || a.row_maxerr) {
    // as rtn_fast_kernel: a chunk's 16 squared errors in fp32, chunks of a warp
    // by an fp64 xor tree, warps in order (chunk-a warps first)
    const double sa = warp_sum_d((double)lo_of(part2)), sb = warp_sum_d((double)hi_of(part2));
    float m;
    asm("redux.sync.max.abs.NaN.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(mx));
    const int nw = nt >> 5;
    __syncthreads();
    if ((t & 31) == 0) {
      red_d[t >> 5] = sa;
      red_d[nw + (t >> 5)] = sb;
      red[t >> 5] = m;
    }
    __syncthreads();
    if (t == 0) {
      double tt = 0.0;
      float mm = 0.f;
      for (int k = 0; k < 2 * nw; ++k) tt += red_d[k];
      for (int k = 0; k < nw; ++k) mm = nmax(mm, red[k]);
      if (a.row_sqerr) a.row_sqerr[row] = tt * (double)DESCALE * (double)DESCALE;
      if (a.row_maxerr) a.row_maxerr[row] = __fmul_rn(mm, DESCALE);
    }
  }
}

template <int ROT>
void launch_rtn_pair(const RtnArgs& a, int64_t M, cudaStream_t st) {
  const unsigned threads = (unsigned)(a.npad / 32);
  switch (a.dtype) {
    case IC_F16: rtn_pair_kernel<__half, ROT><<<(unsigned)M, threads, 0, st>>>(a); break;
    case IC_BF16: rtn_pair_kernel<__nv_bfloat16, ROT><<<(unsigned)M, threads, 0, st>>>(a); break;
    default: rtn_pair_kernel<float, ROT><<<(unsigned)M, threads, 0, st>>>(a); break;
  }
}

template <int ROT>
void launch_rtn_fast(const RtnArgs& a, int64_t M, cudaStream_t st) {
  switch (a.dtype) {
    case IC_F16: rtn_fast_kernel<__half, ROT><<<(unsigned)M, NT, 0, st>>>(a); break;
    case IC_BF16: rtn_fast_kernel<__nv_bfloat16, ROT><<<(unsigned)M, NT, 0, st>>>(a); break;
    default: rtn_fast_kernel<float, ROT><<<(unsigned)M, NT, 0, st>>>(a); break;
  }
}

__global__ void pack_kernel(const int8_t* __restrict__ codes, int64_t M, int64_t K, int64_t ldc,
                            uint8_t* __restrict__ packed, int64_t ldp, unsigned* flags) {
  const int64_t kp = (K + 1) / 2;
  const int64_t total = M * kp;
  bool bad = false;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / kp, b = i % kp;
    const int c0 = codes[r * ldc + 2 * b];
    const int c1 = (2 * b + 1 < K) ? codes[r * ldc + 2 * b + 1] : 0;
    bad |= (c0 < -8 || c0 > 7 || c1 < -8 || c1 > 7);
    packed[r * ldp + b] = (uint8_t)((c0 & 15) | ((c1 & 15) << 4));
  }
  if (bad) atomicOr(flags, DEV_RANGE);
}

__global__ void unpack_kernel(const uint8_t* __restrict__ packed, int64_t M, int64_t K, int64_t ldp,
                              int8_t* __restrict__ codes, int64_t ldc) {
  const int64_t total = M * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K, c = i % K;
    const int b = packed[r * ldp + c / 2];
    const int v = (c & 1) ? (b >> 4) & 15 : b & 15;
    codes[r * ldc + c] = (int8_t)(v >= 8 ? v - 16 : v);
  }
}

// IC_RTN_FAST=0 selects the previous register kernel (A/B and parity checks)
bool fast_off() {
  static const bool off = [] {
    const char* e = getenv("IC_RTN_FAST");
    return e && e[0] == '0';
  }();
  return off;
}

// IC_RTN_FAST=1 selects rtn_fast_kernel over the paired kernel (A/B checks)
bool pair_on() {
  static const bool on = [] {
    const char* e = getenv("IC_RTN_FAST");
    return !(e && (e[0] == '0' || e[0] == '1'));
  }();
  return on;
}

int launch_rtn(RtnArgs& a, int64_t M, cudaStream_t st) {
  if (M == 0 || a.npad == 0) return IC_OK;
  if (M > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "rtn: too many rows");
  if (a.G == 1 && !a.given && a.npad <= 4096 && a.npad % 1024 == 0 && pair_on() &&
      (a.rot == 16 || a.rot == 64 || a.rot == 256)) {
    if (a.rot == 256) launch_rtn_pair<256>(a, M, st);
    else if (a.rot == 64) launch_rtn_pair<64>(a, M, st);
    else launch_rtn_pair<16>(a, M, st);
    IC_CHECK_LAUNCH();
    return IC_OK;
  }
  if (a.G == 1 && !a.given && a.npad <= 16 * NT && a.npad % 16 == 0 && !fast_off() &&
      (a.rot == 16 || a.rot == 64 || a.rot == 256)) {
    if (a.rot == 256) launch_rtn_fast<256>(a, M, st);
    else if (a.rot == 64) launch_rtn_fast<64>(a, M, st);
    else launch_rtn_fast<16>(a, M, st);
    IC_CHECK_LAUNCH();
    return IC_OK;
  }
  if (a.G == 1 && !a.given && a.npad <= 16 * NT && a.npad % 16 == 0 && (a.rot <= 1 || hadamard_regs_ok(a.rot))) {
    switch (a.dtype) {
      case IC_F16: rtn_regs_kernel<__half><<<(unsigned)M, NT, 0, st>>>(a); break;
      case IC_BF16: rtn_regs_kernel<__nv_bfloat16><<<(unsigned)M, NT, 0, st>>>(a); break;
      default: rtn_regs_kernel<float><<<(unsigned)M, NT, 0, st>>>(a); break;
    }
    IC_CHECK_LAUNCH();
    return IC_OK;
  }
  if (a.npad > MAX_ROW)
    return fail(IC_ERR_UNSUPPORTED, "rtn: row of %lld elements exceeds %lld", (long long)a.npad, (long long)MAX_ROW);
  if (M > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "rtn: too many rows");
  static std::atomic<unsigned long long> attr{0};
  IC_TRY(once_per_device(attr, [&]() -> int {
      IC_CUDA(cudaFuncSetAttribute(rtn_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(MAX_ROW * 4)));
      return IC_OK;
    }));
  rtn_row_kernel<<<(unsigned)M, NT, (size_t)a.npad * 4, st>>>(a);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

int fill_ratios(RtnArgs& a, const float* ratios, int nratios) {
  if (nratios < 0 || nratios > MAX_RATIOS)
    return fail(IC_ERR_UNSUPPORTED, "rtn: at most %d clipping ratios", MAX_RATIOS);
  a.nratios = ratios ? nratios : 0;
  for (int i = 0; i < a.nratios; ++i) a.ratios[i] = ratios[i];
  return IC_OK;
}

int64_t grid_elems(int64_t n) { return std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 256), 148 * 32)); }

}  // namespace
}  // namespace ic

using namespace ic;

extern "C" int ic_rtn_scales(const float* W, int64_t M, int64_t N, int64_t ldw, int bits, int asym,
                             int64_t group_size, const float* ratios, int nratios, uint16_t* scales_f16,
                             int8_t* zp, void* stream) {
  if (bits != 4 && bits != 8) return fail(IC_ERR_INVALID, "int_bits must be 4 or 8, got %d", bits);
  if (group_size <= 0 || N % group_size) return fail(IC_ERR_INVALID, "rtn_scales: N must be a multiple of group_size");
  if (bits == 8 && group_size != N) return fail(IC_ERR_INVALID, "rtn_scales: INT8 scales are per row");
  if (asym && !zp) return fail(IC_ERR_INVALID, "rtn_scales: asymmetric needs a zero-point output");
  RtnArgs a{};
  a.W = W; a.dtype = IC_F32; a.N = N; a.ldw = ldw; a.npad = N; a.gs = group_size;
  a.rot = 0; a.bits = bits; a.asym = asym; a.G = (int)(N / group_size); a.given = 0;
  a.zero_group_zp0 = (bits == 4);
  a.scales = scales_f16; a.zp = zp;
  IC_TRY(fill_ratios(a, ratios, nratios));
  return launch_rtn(a, M, (cudaStream_t)stream);
}

extern "C" int ic_rtn_codes(const float* W, int64_t M, int64_t N, int64_t ldw, int bits, int asym,
                            int64_t group_size, const uint16_t* scales_f16, const int8_t* zp, int8_t* codes,
                            int64_t ldc, void* stream) {
  if (bits != 4 && bits != 8) return fail(IC_ERR_INVALID, "int_bits must be 4 or 8, got %d", bits);
  if (group_size <= 0 || N % group_size) return fail(IC_ERR_INVALID, "rtn_codes: N must be a multiple of group_size");
  if (asym && !zp) return fail(IC_ERR_INVALID, "rtn_codes: asymmetric needs zero-points");
  RtnArgs a{};
  a.W = W; a.dtype = IC_F32; a.N = N; a.ldw = ldw; a.npad = N; a.gs = group_size;
  a.rot = 0; a.bits = bits; a.asym = asym; a.G = (int)(N / group_size); a.given = 1;
  a.in_scales = scales_f16; a.in_zp = zp; a.codes = codes; a.ldc = ldc;
  return launch_rtn(a, M, (cudaStream_t)stream);
}

extern "C" int ic_rtn_fused(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, int rot, int bits,
                            int asym, const float* ratios, int nratios, int8_t* codes, uint8_t* packed,
                            uint16_t* scales_f16, int8_t* zp, double* row_sqerr, float* row_maxerr,
                            void* stream) {
  if (bits != 4 && bits != 8) return fail(IC_ERR_INVALID, "int_bits must be 4 or 8, got %d", bits);
  if (rot != 0 && (rot < 2 || rot > 1024 || (rot & (rot - 1))))
    return fail(IC_ERR_INVALID, "rot_size must be a power of 2, got %d", rot);
  if (packed && bits != 4) return fail(IC_ERR_INVALID, "rtn_fused: packing is INT4 only");
  if (dtype != IC_F32 && dtype != IC_F16 && dtype != IC_BF16) return fail(IC_ERR_INVALID, "rtn_fused: dtype");
  const int r = rot ? rot : 1;
  RtnArgs a{};
  a.W = W; a.dtype = dtype; a.N = N; a.ldw = ldw; a.npad = cdiv(N, r) * r; a.gs = a.npad;
  a.rot = rot; a.bits = bits; a.asym = asym; a.G = 1; a.given = 0;
  a.zero_group_zp0 = (bits == 4);
  a.clamp = WEIGHT_OUTLIER_CLAMP;
  a.scales = scales_f16; a.zp = zp; a.codes = codes; a.ldc = a.npad; a.packed = packed;
  a.ldp = (a.npad + 1) / 2; a.row_sqerr = row_sqerr; a.row_maxerr = row_maxerr;
  IC_TRY(fill_ratios(a, ratios, nratios));
  return launch_rtn(a, M, (cudaStream_t)stream);
}

extern "C" int ic_pack_int4(const int8_t* codes, int64_t M, int64_t K, int64_t ldc, uint8_t* packed, int64_t ldp,
                            void* stream) {
  if (M == 0 || K == 0) return IC_OK;
  cudaStream_t st = (cudaStream_t)stream;
  unsigned* flags = device_flags();
  if (!flags) return fail(IC_ERR_CUDA, "device status word unavailable");
  unsigned before = 0;
  IC_TRY(read_and_clear_flags(&before, st));
  pack_kernel<<<(int)grid_elems(M * ((K + 1) / 2)), 256, 0, st>>>(codes, M, K, ldc, packed, ldp, flags);
  IC_CHECK_LAUNCH();
  unsigned after = 0;
  IC_TRY(read_and_clear_flags(&after, st));
  if (after & DEV_RANGE) return fail(IC_ERR_RANGE, "Values must be in [-8, 7]");
  return IC_OK;
}

extern "C" int ic_unpack_int4(const uint8_t* packed, int64_t M, int64_t K, int64_t ldp, int8_t* codes, int64_t ldc,
                              void* stream) {
  if (M == 0 || K == 0) return IC_OK;
  unpack_kernel<<<(int)grid_elems(M * K), 256, 0, (cudaStream_t)stream>>>(packed, M, K, ldp, codes, ldc);
  IC_CHECK_LAUNCH();
  return IC_OK;
}
