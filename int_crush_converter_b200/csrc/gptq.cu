// GPTQ / LDLQ column loop: rounding._gptq_block (converter/rounding.py:37-103)
// and ldlq._ldlq_loop_cpu (converter/ldlq.py:369-417).
//
// Intra-block kernel: one thread per weight row (a CTA owns 128 rows), the
// block's <= 128 columns in four groups of 32.  The block's Hinv and the
// CTA's block of W live in shared memory; the current group's 32 weights of
// the row sit in registers.  Inside a group every column is quantized and its
// normalised error applied at once to the group's later columns; then the
// group's 32 errors are applied to the block's later columns, column by
// column in ascending order.  Every weight therefore sees exactly the
// reference's sequence of fp32 operations (w_k <- w_k - e_j * Hinv[j,k], a
// rounded multiply then a rounded subtract).  Rows are independent, so no
// thread ever waits for another after the loads.
//
// Inter-block update as tensor-core GEMMs, two-level.  Inside a super-block
// (1024 columns) the update is left-looking: before a block is quantized its
// 128 columns take W[:, blk] -= E[:, sb:blk] * Hinv[sb:blk, blk] in one GEMM
// whose K is everything processed so far in the super-block (the sum the
// reference's lazy inter-block update, rounding.py:100-103, forms block by
// block, with one rounding instead of one per block).  After the super-block, one "far"
// update W[:, after] -= E_sb * Hinv[sb, after] with K = super-block width
// covers every later column, so the fp32 W_work read-modify-write traffic is
// divided by super-block / block.
#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int GROUP = 32;
constexpr int MAXB = 128;
constexpr int ROWS = 128;  // weight rows (threads) per CTA of the block kernel

struct BlockArgs {
  float* W;
  int64_t ldw;
  const float* W0;
  int64_t ldw0;
  int64_t M, i1;
  int bc;
  const float* h_hi;
  const float* h_lo;
  int64_t ldh;
  const float* scale;
  const float* zp;
  const float* stat_scale;
  const float* scale2d;
  int64_t lds;
  float qmin, qmax;
  int8_t* codes;
  int64_t ldq;
  uint8_t* packed;
  int64_t ldp;
  float* e_hi;
  float* e_lo;
  int64_t lde;
  double* row_sqerr;
  float* row_maxerr;
  int vec;  // W and Hinv rows of this block are 16-byte aligned
  unsigned* flags;  // device status word (DEV_TIMEOUT if a bounded wait gives up)
};

// Packed pairs of fp32 (low = first) and the sm_100 two-wide fp32 operations;
// each half is rounded to nearest exactly as the scalar __fmul_rn / __fsub_rn.
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t sub_f32x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// Bulk global -> shared copies (cp.async.bulk, no multicast) completing on an
// mbarrier, and a bounded wait on it.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "{\n .reg .u64 g;\n cvta.to.global.u64 g, %1;\n"
      " cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [g], %2, [%3];\n}\n" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, unsigned* flags) {
  return mbar_wait_bounded(bar, parity, flags, 1000000000ull);  // 1 s
}

// Compact Hinv block: row j keeps columns [32*(j/32), 128) only (the serial
// part reads its group's diagonal block, the apply part the columns after it).
constexpr int HS_FLOATS = GROUP * (MAXB + (MAXB - GROUP) + (MAXB - 2 * GROUP) + (MAXB - 3 * GROUP));
// weight staging row stride: 132 floats = 528 bytes, so the float4 accesses of
// a quarter-warp (8 threads, 8 different rows) fall in 8 different 16-byte
// bank groups
constexpr int WLD = MAXB + 4;
constexpr uint32_t BULK_BYTES = (uint32_t)(ROWS * MAXB * 4 + 2 * HS_FLOATS * 4);
__device__ __forceinline__ int hs_index(int j, int c) {
  const int G = j >> 5;
  const int base = GROUP * (MAXB * G - 16 * G * (G - 1));  // sum of the earlier groups' rows
  return base + (j - G * GROUP) * (MAXB - G * GROUP) + (c - G * GROUP);
}

template <bool LDLQ>
__global__ void __launch_bounds__(ROWS) block_kernel(const BlockArgs a) {
  extern __shared__ __align__(16) float smem[];
  // Hinv block (exact fp32), row j = error column j, compact: only columns from
  // the start of row j's group on are ever read (HS_FLOATS = 32 x (128+96+64+32))
  float* hs = smem;
  float* wst = hs + HS_FLOATS;            // [ROWS][WLD] the CTA's weight rows of the block, row-major
  float* lost = wst + ROWS * WLD;         // lo halves of the compact Hinv block (bulk path)
  float* dinv = lost + HS_FLOATS;         // [MAXB] LDLQ: 1/max(Hinv[j,j],1e-8)
  uint64_t* bar = reinterpret_cast<uint64_t*>(dinv + MAXB);

  const int t = threadIdx.x;
  const int bc = a.bc;
  const int64_t r = (int64_t)blockIdx.x * ROWS + t;
  const bool rv = r < a.M;
  const int64_t rr = rv ? r : a.M - 1;  // clamp loads for the tail rows

  if (a.vec && bc == MAXB) {
    // full 128 x 128 block: every byte in flight at once as bulk copies, one
    // weight row and one compact Hinv row (hi and lo) per thread, all
    // completing on one mbarrier; then hi + lo summed in place
    const uint32_t mb = smem_addr(bar);
    if (t == 0) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mb));
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mb), "r"(BULK_BYTES)
                   : "memory");
    }
    __syncthreads();
    bulk_g2s(smem_addr(wst + t * WLD), a.W + rr * a.ldw + a.i1, MAXB * 4, mb);
    const int c0 = (t >> 5) * GROUP;
    const int64_t ho = (a.i1 + t) * a.ldh + a.i1 + c0;
    const uint32_t len = (uint32_t)(MAXB - c0) * 4;
    bulk_g2s(smem_addr(hs + hs_index(t, c0)), a.h_hi + ho, len, mb);
    bulk_g2s(smem_addr(lost + hs_index(t, c0)), a.h_lo + ho, len, mb);
    bool ok = bar_wait(mb, 0, a.flags);
    if (!__syncthreads_and(ok)) {
      if (!ok) bar_wait(mb, 0, nullptr);  // give the copies in flight (bounded) time to land
      return;
    }
    float4* h4 = reinterpret_cast<float4*>(hs);
    const float4* l4 = reinterpret_cast<const float4*>(lost);
#pragma unroll 4
    for (int i = t; i < HS_FLOATS / 4; i += ROWS) {
      const float4 h = h4[i], l = l4[i];
      h4[i] = make_float4(__fadd_rn(h.x, l.x), __fadd_rn(h.y, l.y), __fadd_rn(h.z, l.z), __fadd_rn(h.w, l.w));
    }
  } else {
    for (int j = 0; j < bc; ++j)
      for (int k = (j & ~(GROUP - 1)) + t; k < bc; k += ROWS) {
        const int64_t o = (a.i1 + j) * a.ldh + a.i1 + k;
        hs[hs_index(j, k)] = __fadd_rn(a.h_hi[o], a.h_lo[o]);
      }
    const float* wrow = a.W + rr * a.ldw + a.i1;
    for (int c = 0; c < bc; ++c) wst[t * WLD + c] = wrow[c];
  }
  __syncthreads();
  if (LDLQ)
    for (int j = t; j < bc; j += ROWS) dinv[j] = __fdiv_rn(1.0f, fmaxf(hs[hs_index(j, j)], 1e-8f));
  if (LDLQ) __syncthreads();

  const float s = LDLQ ? 1.f : a.scale[rr];
  const float z = (!LDLQ && a.zp) ? a.zp[rr] : 0.f;
  const bool has_zp = !LDLQ && a.zp != nullptr;
  const bool want_stats = !LDLQ && (a.row_sqerr || a.row_maxerr) && a.W0 != nullptr;
  const float sst = (!LDLQ && a.stat_scale) ? a.stat_scale[rr] : s;
  double sq_tot = 0.0;
  float mx = 0.f;
  const int ng = (bc + GROUP - 1) / GROUP;

#pragma unroll 1
  for (int G = 0; G < ng; ++G) {
    const int cb = G * GROUP;  // first block-local column of the group
    const float* hg = hs + hs_index(cb, cb);  // row cb of the group's compact rows, stride hstride
    const int hstride = MAXB - cb;
    float w[GROUP], ev[GROUP];
    float sc[LDLQ ? GROUP : 1];
    {
      const float4* wr = reinterpret_cast<const float4*>(wst + t * WLD + cb);
#pragma unroll
      for (int c4 = 0; c4 < GROUP / 4; ++c4) {
        const float4 q4 = wr[c4];
        w[4 * c4] = q4.x;
        w[4 * c4 + 1] = q4.y;
        w[4 * c4 + 2] = q4.z;
        w[4 * c4 + 3] = q4.w;
      }
    }
#pragma unroll
    for (int c = 0; c < GROUP; ++c) {
      if (cb + c >= bc) w[c] = 0.f;  // columns past a ragged block's end (unset staging)
      if (LDLQ) sc[c] = (cb + c < bc) ? fmaxf(a.scale2d[rr * a.lds + a.i1 + cb + c], 1e-8f) : 1.f;
    }
    // the group's columns in order, each error applied at once to the group's later columns
#pragma unroll 32
    for (int c = 0; c < GROUP; ++c) {
      const int j = cb + c;
      ev[c] = 0.f;
      if (j < bc) {
        const float x = w[c];
        float q, e;
        if (!LDLQ) {
          float raw = __fdiv_rn(x, s);
          if (has_zp) raw = __fadd_rn(raw, z);
          q = clampf(rhaz(raw), a.qmin, a.qmax);
          const float deq = has_zp ? __fmul_rn(__fsub_rn(q, z), s) : __fmul_rn(q, s);
          e = __fdiv_rn(__fsub_rn(x, deq), hg[c * hstride + c]);
          e = clampf(e, -100.f, 100.f);  // ERR_CLAMP_RANGE
          if (e != e) e = 0.f;           // nan_to_num
        } else {
          // rounding._ldlq_round_column (rounding.py:115-155)
          const float ss = sc[c];
          q = clampf(rhaz(__fdiv_rn(x, ss)), a.qmin, a.qmax);
          const float qs = (q > 0.f) ? 1.f : (q < 0.f ? -1.f : 0.f);
          const float xs = (x > 0.f) ? 1.f : (x < 0.f ? -1.f : 0.f);
          const float wsg = fabsf(x) > 1e-8f ? xs : qs;
          const bool flip = wsg * qs < 0.f;
          const bool can = flip && (q > a.qmin);
          if (flip && q == a.qmin) q = a.qmax;
          if (can) q = -q;
          q = clampf(q, a.qmin, a.qmax);
          e = __fmul_rn(__fsub_rn(x, __fmul_rn(q, ss)), dinv[j]);
        }
        w[c] = q;  // the weight itself is no longer needed
        ev[c] = e;
#pragma unroll 31
        for (int c2 = c + 1; c2 < GROUP; ++c2)
          if (cb + c2 < bc) w[c2] = __fsub_rn(w[c2], __fmul_rn(e, hg[c * hstride + c2]));
      }
    }

    // ---- outputs of the group (w[] holds the codes) ----
    const int nvalid = min(GROUP, bc - cb);
    if (rv) {
      const int64_t col = a.i1 + cb;
      if (a.codes) {
        int8_t* dst = a.codes + r * a.ldq + col;
        if (nvalid == GROUP && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            pk[i] = ((uint32_t)(uint8_t)(int8_t)w[4 * i]) | ((uint32_t)(uint8_t)(int8_t)w[4 * i + 1] << 8) |
                    ((uint32_t)(uint8_t)(int8_t)w[4 * i + 2] << 16) |
                    ((uint32_t)(uint8_t)(int8_t)w[4 * i + 3] << 24);
          reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        } else {
#pragma unroll
          for (int c = 0; c < GROUP; ++c)
            if (c < nvalid) dst[c] = (int8_t)w[c];
        }
      }
      if (a.packed) {  // col is even (packing here needs an even block size)
        uint8_t* dst = a.packed + r * a.ldp + col / 2;
        if (nvalid == GROUP && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
          uint32_t pk[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t v = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) v |= ((uint32_t)((int)w[8 * i + k] & 15)) << (4 * k);
            pk[i] = v;
          }
          *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        } else {
#pragma unroll
          for (int c = 0; c < GROUP; c += 2)
            if (c < nvalid) {
              const int lo = (int)w[c] & 15;
              const int hi = (c + 1 < nvalid) ? ((int)w[c + 1] & 15) : 0;
              dst[c / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
      }
      if (a.e_hi) {
        float* dh = a.e_hi + r * a.lde + cb;
        float* dl = a.e_lo ? a.e_lo + r * a.lde + cb : nullptr;
        if (nvalid == GROUP && dl && ((reinterpret_cast<uintptr_t>(dh) | reinterpret_cast<uintptr_t>(dl)) & 15) == 0) {
#pragma unroll
          for (int c = 0; c < GROUP; c += 4) {
            float4 h, l;
            split_tf32(ev[c], h.x, l.x);
            split_tf32(ev[c + 1], h.y, l.y);
            split_tf32(ev[c + 2], h.z, l.z);
            split_tf32(ev[c + 3], h.w, l.w);
            *reinterpret_cast<float4*>(dh + c) = h;
            *reinterpret_cast<float4*>(dl + c) = l;
          }
        } else {
#pragma unroll
          for (int c = 0; c < GROUP; ++c)
            if (c < nvalid) {
              const float h = to_tf32(ev[c]);
              dh[c] = h;
              if (dl) dl[c] = __fsub_rn(ev[c], h);
            }
        }
      }
      if (want_stats) {
        double sq = 0.0;
        const float* w0 = a.W0 + r * a.ldw0 + col;
#pragma unroll
        for (int c = 0; c < GROUP; ++c)
          if (c < nvalid) {
            const float deq = has_zp ? __fmul_rn(__fsub_rn(w[c], z), sst) : __fmul_rn(w[c], sst);
            const float d = __fsub_rn(w0[c], deq);
            sq += (double)d * (double)d;
            mx = nmax(mx, fabsf(d));
          }
        sq_tot += sq;
      }
    }

    // ---- this group's errors into the block's later columns, in column order ----
    const int cend = (bc + 3) & ~3;  // columns past bc are scratch (never read back)
#pragma unroll 1
    for (int c2 = cb + GROUP; c2 < cend; c2 += 4) {
      float4* wc = reinterpret_cast<float4*>(wst + t * WLD + c2);
      // two columns per packed f32x2 operation (each half rounded as the scalar op)
      const float4 w4 = *wc;
      uint64_t v01 = pack2(w4.x, w4.y), v23 = pack2(w4.z, w4.w);
#pragma unroll
      for (int j = 0; j < GROUP; ++j) {
        const ulonglong2 h = *reinterpret_cast<const ulonglong2*>(hg + j * hstride + (c2 - cb));
        const uint64_t e2 = pack2(ev[j], ev[j]);
        v01 = sub_f32x2(v01, mul_f32x2(e2, h.x));
        v23 = sub_f32x2(v23, mul_f32x2(e2, h.y));
      }
      float4 o4;
      unpack2(v01, o4.x, o4.y);
      unpack2(v23, o4.z, o4.w);
      *wc = o4;
    }
  }
  if (want_stats && rv) {
    if (a.row_sqerr) a.row_sqerr[r] += sq_tot;
    if (a.row_maxerr) a.row_maxerr[r] = nmax(a.row_maxerr[r], mx);
  }
}

constexpr size_t BLOCK_SMEM = (size_t)HS_FLOATS * 4 * 2 + (size_t)ROWS * WLD * 4 + MAXB * 4 + 16;

// ---- per-row scale / zero-point preparation (converter/gptq.py:254-317) ----
__global__ void __launch_bounds__(256) row_params_kernel(const float* __restrict__ W, int64_t N, int64_t ldw,
                                                         int bits, int asym, float* __restrict__ scale,
                                                         float* __restrict__ zp) {
  __shared__ float r0[8], r1[8], r2[8];
  const int64_t row = blockIdx.x;
  const float* w = W + row * ldw;
  float amax = 0.f, mn = __int_as_float(0x7f800000), mx = __int_as_float(0xff800000);
  for (int64_t i = threadIdx.x; i < N; i += blockDim.x) {
    const float v = w[i];
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
    r0[threadIdx.x >> 5] = amax;
    r1[threadIdx.x >> 5] = mn;
    r2[threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) {
    r0[0] = nmax(r0[0], r0[i]);
    r1[0] = nmin(r1[0], r1[i]);
    r2[0] = nmax(r2[0], r2[i]);
  }
  amax = r0[0];
  mn = r1[0];
  mx = r2[0];
  if (bits == 4 || asym) {
    const float qmin = bits == 4 ? -8.f : -128.f, qmax = bits == 4 ? 7.f : 127.f;
    const float spread = bits == 4 ? 15.f : 255.f;
    float s = clampf(__fdiv_rn(__fsub_rn(mx, mn), spread), 1e-5f, 65500.f);
    const float zr = __fsub_rn(qmin, rhaz(__fdiv_rn(mn, s)));
    const bool lo = zr < qmin, hi = zr > qmax;  // both from the unadjusted scale
    if (lo) s = fmaxf(s, clampf(__fdiv_rn(mx, spread), 1e-5f, 65500.f));
    if (hi) s = fmaxf(s, clampf(__fdiv_rn(-mn, spread), 1e-5f, 65500.f));
    float z = clampf(__fsub_rn(qmin, rhaz(__fdiv_rn(mn, s))), qmin, qmax);
    if (mn == 0.f && mx == 0.f) z = 0.f;
    scale[row] = s;
    if (zp) zp[row] = z;
  } else {
    scale[row] = clampf(__fdiv_rn(amax, 127.f), 1e-5f, 65500.f);
  }
}

__global__ void fill_kernel_d(double* p, int64_t n, double v) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}
__global__ void fill_kernel_f(float* p, int64_t n, float v) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// copy a [rows x cols] block of a hi/lo pair into an aligned buffer (ldo)
__global__ void copy_pair_kernel(const float* __restrict__ ih, const float* __restrict__ il, int64_t rows,
                                 int64_t cols, int64_t ldi, float* __restrict__ oh, float* __restrict__ ol,
                                 int64_t ldo) {
  const int64_t total = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    oh[r * ldo + c] = ih[r * ldi + c];
    if (ol) ol[r * ldo + c] = il[r * ldi + c];
  }
}

__global__ void stats_kernel(const double* __restrict__ sq, const float* __restrict__ mx, int64_t M, double count,
                             double* out, const unsigned* status) {
  __shared__ double rs[32];
  __shared__ float rm[32];
  double s = 0.0;
  float m = 0.f;
  for (int64_t i = threadIdx.x; i < M; i += blockDim.x) {
    if (sq) s += sq[i];
    if (mx) m = nmax(m, mx[i]);
  }
  s = warp_sum_d(s);
  for (int o = 16; o; o >>= 1) m = nmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) {
    rs[threadIdx.x >> 5] = s;
    rm[threadIdx.x >> 5] = m;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) {
      rs[0] += rs[i];
      rm[0] = nmax(rm[0], rm[i]);
    }
    out[0] = count > 0 ? rs[0] / count : 0.0;
    out[1] = (double)rm[0];
    if (status) out[2] = (double)*status;
  }
}

// fp16 scales and int8 zero-points of the layer.  A row whose stored scale is
// NaN, infinite or zero (only a NaN weight in the row can cause one: the scale
// is clamped to [1e-5, 65500]) sets DEV_BAD_SCALE in `status`: the pipeline's
// verify step flags such a layer and "repairs" its rows (pipeline.py:935-1007),
// which for a NaN row reproduces the NaN scale, and zero zero-point and codes
// (torch converts NaN to int8 0, as the conversions here do).
__global__ void params_out_kernel(const float* __restrict__ s, const float* __restrict__ z, int64_t M,
                                  uint16_t* __restrict__ s16, int8_t* __restrict__ z8, float* __restrict__ s16f,
                                  unsigned* status) {
  bool bad = false;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M; i += (int64_t)gridDim.x * blockDim.x) {
    const __half h = __float2half_rn(s[i]);
    const float hf = __half2float(h);
    bad |= !(fabsf(hf) < INFINITY) || hf == 0.f;
    if (s16) s16[i] = __half_as_ushort(h);
    if (s16f) s16f[i] = hf;
    if (z8 && z) z8[i] = z[i] != z[i] ? (int8_t)0 : (int8_t)z[i];
  }
  if (bad && status) atomicOr(status, DEV_BAD_SCALE);
}

// converter/ldlq.py:553-599, elementwise (floor/ceil from the caller)
__global__ void ldlq_update_kernel(const float* __restrict__ W, const int8_t* __restrict__ Q, float* __restrict__ cur,
                                   const float* __restrict__ flat, int64_t n, float mom, float one_minus, float lo,
                                   float hi, float thr) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float q = (float)Q[i];
    if (q == 0.f) continue;
    const float w = W[i];
    if (fabsf(w) > thr && __fmul_rn(w, q) > 0.f) {
      const float comp = clampf(__fdiv_rn(fabsf(w), fabsf(q)), lo, hi);
      cur[i] = mom > 0.f ? __fadd_rn(__fmul_rn(mom, cur[i]), __fmul_rn(one_minus, comp)) : comp;
    } else {
      cur[i] = clampf(flat[i], lo, hi);
    }
  }
}

int grid1(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 256), 148 * 8)); }

struct LoopArgs {
  float* W;
  int64_t ldw;
  const float* W0;
  int64_t ldw0;
  int64_t M, N;
  const float* h_hi;
  const float* h_lo;
  int64_t ldh;
  int B, SB;
  const float* scale;
  const float* zp;
  const float* stat_scale;
  const float* scale2d;
  int64_t lds;
  int qmin, qmax;
  int8_t* codes;
  int64_t ldq;
  uint8_t* packed;
  int64_t ldp;
  double* row_sqerr;
  float* row_maxerr;
  int passes;
  bool ldlq;
};

size_t loop_ws(int64_t M, int64_t N, int B, int SB) {
  const int sb = (B % 4) ? B : SB;
  const int64_t lde = (sb + 3) & ~3;
  const size_t e = (size_t)M * lde * 4 * 2 + 512;
  const size_t h = (B % 4) ? (size_t)N * ((B + 3) & ~3) * 4 * 2 + 512 : 0;
  return e + h + 1024;
}

int run_loop(const LoopArgs& L, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (L.B <= 0 || L.B > MAXB) return fail(IC_ERR_UNSUPPORTED, "block_size must be in [1, %d], got %d", MAXB, L.B);
  if (L.SB < L.B || L.SB % L.B) return fail(IC_ERR_INVALID, "superblock must be a multiple of block_size");
  if (L.M <= 0 || L.N <= 0) return IC_OK;
  if (L.M > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "too many rows");
  if (L.ldh % 4) return fail(IC_ERR_INVALID, "Hinv leading dimension must be a multiple of 4");
  if (L.packed && (L.B % 2)) return fail(IC_ERR_UNSUPPORTED, "in-loop packing needs an even block size");
  if (ws_bytes < loop_ws(L.M, L.N, L.B, L.SB)) return fail(IC_ERR_WORKSPACE, "gptq: workspace too small");
  unsigned* flags = device_flags();
  if (!flags) return fail(IC_ERR_CUDA, "device status word unavailable");
  const int SB = (L.B % 4) ? L.B : L.SB;
  const int64_t lde = (SB + 3) & ~3;
  Carver cv(ws, ws_bytes);
  float* e_hi = cv.take<float>((size_t)L.M * lde);
  float* e_lo = cv.take<float>((size_t)L.M * lde);
  const int64_t ldb2 = (L.B + 3) & ~3;
  float* hb_hi = nullptr;
  float* hb_lo = nullptr;
  if (L.B % 4) {
    hb_hi = cv.take<float>((size_t)L.N * ldb2);
    hb_lo = cv.take<float>((size_t)L.N * ldb2);
  }
  static std::atomic<unsigned long long> attr{0};
  IC_TRY(once_per_device(attr, [&]() -> int {
      IC_CUDA(cudaFuncSetAttribute(block_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BLOCK_SMEM));
      IC_CUDA(cudaFuncSetAttribute(block_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BLOCK_SMEM));
      return IC_OK;
    }));
  if (L.row_sqerr) fill_kernel_d<<<grid1(L.M), 256, 0, st>>>(L.row_sqerr, L.M, 0.0);
  if (L.row_maxerr) fill_kernel_f<<<grid1(L.M), 256, 0, st>>>(L.row_maxerr, L.M, 0.f);
  IC_CHECK_LAUNCH();
  const unsigned nblk = (unsigned)cdiv(L.M, ROWS);
  for (int64_t sb = 0; sb < L.N; sb += SB) {
    const int64_t sbe = std::min<int64_t>(sb + SB, L.N);
    for (int64_t i1 = sb; i1 < sbe; i1 += L.B) {
      const int64_t i2 = std::min<int64_t>(i1 + L.B, L.N);
      if (i1 > sb) {  // left-looking near update: this block's columns take the super-block's earlier errors
        IC_TRY(gemm_tn(L.M, i2 - i1, i1 - sb, -1.f, e_hi, e_lo, lde, L.h_hi + i1 * L.ldh + sb,
                       L.h_lo + i1 * L.ldh + sb, L.ldh, 1.f, L.W + i1, nullptr, L.ldw, L.W + i1, nullptr, L.ldw,
                       L.passes, st));
      }
      BlockArgs a{};
      a.W = L.W; a.ldw = L.ldw; a.W0 = L.W0; a.ldw0 = L.ldw0; a.M = L.M; a.i1 = i1; a.bc = (int)(i2 - i1);
      a.h_hi = L.h_hi; a.h_lo = L.h_lo; a.ldh = L.ldh; a.scale = L.scale; a.zp = L.zp;
      a.stat_scale = L.stat_scale; a.scale2d = L.scale2d; a.lds = L.lds;
      a.qmin = (float)L.qmin; a.qmax = (float)L.qmax; a.codes = L.codes; a.ldq = L.ldq;
      a.packed = L.packed; a.ldp = L.ldp; a.e_hi = e_hi + (i1 - sb); a.e_lo = e_lo + (i1 - sb);
      a.lde = lde; a.row_sqerr = L.row_sqerr; a.row_maxerr = L.row_maxerr;
      a.vec = ((L.ldw | L.ldh | i1) & 3) == 0 && (reinterpret_cast<uintptr_t>(L.W) & 15) == 0 &&
              (reinterpret_cast<uintptr_t>(L.h_hi) & 15) == 0 && (reinterpret_cast<uintptr_t>(L.h_lo) & 15) == 0;
      a.flags = flags;
      if (L.ldlq) block_kernel<true><<<nblk, ROWS, BLOCK_SMEM, st>>>(a);
      else block_kernel<false><<<nblk, ROWS, BLOCK_SMEM, st>>>(a);
      IC_CHECK_LAUNCH();
    }
    if (sbe < L.N) {  // far update: everything after the super-block, K = super-block width
      const float* bh = L.h_hi + sbe * L.ldh + sb;
      const float* bl = L.h_lo + sbe * L.ldh + sb;
      int64_t ldb = L.ldh;
      if (sb % 4) {  // unaligned column offset (block_size % 4 != 0): stage the slice
        copy_pair_kernel<<<grid1((L.N - sbe) * (sbe - sb)), 256, 0, st>>>(bh, bl, L.N - sbe, sbe - sb, L.ldh,
                                                                           hb_hi, hb_lo, ldb2);
        IC_CHECK_LAUNCH();
        bh = hb_hi;
        bl = hb_lo;
        ldb = ldb2;
      }
      IC_TRY(gemm_tn(L.M, L.N - sbe, sbe - sb, -1.f, e_hi, e_lo, lde, bh, bl, ldb, 1.f, L.W + sbe, nullptr, L.ldw,
                     L.W + sbe, nullptr, L.ldw, L.passes, st));
    }
  }
  return IC_OK;
}

// ------------------------------------------------------------ whole layer
struct LayerWs {
  float *W0, *Wk, *Hh, *Hl, *scale, *zp, *sscale, *rmx;
  double* rsq;
  unsigned* status;
  void* loop;
  size_t loop_bytes;
  void* inv;
  size_t inv_bytes;
};
constexpr int LAYER_SB = 1024;
int64_t round4(int64_t x) { return (x + 3) & ~int64_t(3); }

size_t layer_ws(int64_t M, int64_t N_in, int rot, LayerWs* out, void* base, size_t cap) {
  const int r = rot > 0 ? rot : 1;
  const int64_t npad = cdiv(N_in, r) * r;
  const int64_t ldw = round4(npad);
  Carver cv(base, cap);
  LayerWs w{};
  // The Hessian pair, the status word and the inverse's scratch come first, at
  // offsets that depend on the input width alone: the inverse's replayed graph
  // is keyed on these addresses, so layers of one width that share a workspace
  // (qkv, proj and mlp_up of a block) reuse one graph instead of instantiating
  // one per output width (10-80 ms of host time each, during which no stream
  // is fed).
  w.Hh = cv.take<float>((size_t)npad * ldw);
  w.Hl = cv.take<float>((size_t)npad * ldw);
  w.status = cv.take<unsigned>(1);
  w.inv_bytes = spd_inverse_ws(npad);
  w.inv = cv.take<char>(w.inv_bytes);
  w.W0 = cv.take<float>((size_t)M * ldw);
  w.Wk = cv.take<float>((size_t)M * ldw);
  w.scale = cv.take<float>(M);
  w.zp = cv.take<float>(M);
  w.sscale = cv.take<float>(M);
  w.rmx = cv.take<float>(M);
  w.rsq = cv.take<double>(M);
  w.loop_bytes = loop_ws(M, npad, 128, LAYER_SB);
  w.loop = cv.take<char>(w.loop_bytes);
  if (out) *out = w;
  return cv.off + 256;
}

}  // namespace

int finalize_stats(const double* row_sqerr, const float* row_maxerr, int64_t M, double count, double* stats,
                   cudaStream_t st) {
  stats_kernel<<<1, 1024, 0, st>>>(row_sqerr, row_maxerr, M, count, stats, nullptr);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

}  // namespace ic

using namespace ic;

extern "C" int ic_gptq_row_params(const float* W, int64_t M, int64_t N, int64_t ldw, int bits, int asym, float* scale,
                                  float* zp, void* stream) {
  if (bits != 4 && bits != 8) return fail(IC_ERR_INVALID, "int_bits must be 4 or 8, got %d", bits);
  if (M <= 0) return IC_OK;
  if (M > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "too many rows");
  row_params_kernel<<<(unsigned)M, 256, 0, (cudaStream_t)stream>>>(W, N, ldw, bits, asym, scale, zp);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

extern "C" size_t ic_gptq_workspace_size(int64_t M, int64_t N, int block_size, int superblock) {
  if (block_size <= 0) return 0;
  if (M < 0) M = 0;  // empty shapes need no scratch (the loop returns before using any)
  if (N < 0) N = 0;
  if (superblock < block_size) superblock = block_size;
  return loop_ws(M, N, block_size, superblock);
}

extern "C" int ic_gptq_run(float* W_work, int64_t ldw, const float* W0, int64_t ldw0, int64_t M, int64_t N,
                           const float* hinv_hi, const float* hinv_lo, int64_t ldh, int block_size, int superblock,
                           const float* scale, const float* zp, int qmin, int qmax, int8_t* codes, int64_t ldq,
                           uint8_t* packed, int64_t ldp, double* row_sqerr, float* row_maxerr, int gemm_passes,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (!scale) return fail(IC_ERR_INVALID, "gptq_run: scale required");
  LoopArgs L{};
  L.W = W_work; L.ldw = ldw; L.W0 = W0; L.ldw0 = ldw0; L.M = M; L.N = N; L.h_hi = hinv_hi; L.h_lo = hinv_lo;
  L.ldh = ldh; L.B = block_size; L.SB = superblock < block_size ? block_size : superblock;
  L.scale = scale; L.zp = zp; L.qmin = qmin; L.qmax = qmax; L.codes = codes; L.ldq = ldq;
  L.packed = packed; L.ldp = ldp; L.row_sqerr = row_sqerr; L.row_maxerr = row_maxerr;
  L.passes = gemm_passes; L.ldlq = false;
  return run_loop(L, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int ic_ldlq_run(float* W_work, int64_t ldw, int64_t M, int64_t N, const float* hinv_hi,
                           const float* hinv_lo, int64_t ldh, int block_size, int superblock, const float* scale2d,
                           int64_t lds, int qmin, int qmax, int8_t* codes, int64_t ldq, int gemm_passes,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (!scale2d) return fail(IC_ERR_INVALID, "ldlq_run: scale2d required");
  LoopArgs L{};
  L.W = W_work; L.ldw = ldw; L.M = M; L.N = N; L.h_hi = hinv_hi; L.h_lo = hinv_lo; L.ldh = ldh;
  L.B = block_size; L.SB = superblock < block_size ? block_size : superblock;
  L.scale2d = scale2d; L.lds = lds; L.qmin = qmin; L.qmax = qmax; L.codes = codes; L.ldq = ldq;
  L.passes = gemm_passes; L.ldlq = true;
  return run_loop(L, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int ic_ldlq_update_scales(const float* W, const int8_t* Q, float* cur, const float* flat, int64_t count,
                                     float momentum, float one_minus_momentum, float floor_v, float ceil_v,
                                     float nonzero_thr, void* stream) {
  if (count <= 0) return IC_OK;
  ldlq_update_kernel<<<grid1(count), 256, 0, (cudaStream_t)stream>>>(W, Q, cur, flat, count, momentum,
                                                                      one_minus_momentum, floor_v, ceil_v, nonzero_thr);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

extern "C" int ic_finalize_stats(const double* row_sqerr, const float* row_maxerr, int64_t M, double count,
                                 double* stats, void* stream) {
  return finalize_stats(row_sqerr, row_maxerr, M, count, stats, (cudaStream_t)stream);
}

extern "C" size_t ic_gptq_layer_workspace_size(int64_t M, int64_t N_in, int rot) {
  return layer_ws(M, N_in, rot, nullptr, nullptr, 0);
}

extern "C" int ic_gptq_layer(const void* W, int dtype, int64_t M, int64_t N_in, int64_t ldw_in, const float* H,
                             int64_t ldh_in, const float* smoothing, int smooth_order, int h_rotated, int rot, int bits,
                             int asym, int block_size, float damping,
                             int update_passes,
                             int8_t* codes, uint8_t* packed, uint16_t* scales_f16, int8_t* zp_out, double* stats,
                             void* workspace, size_t workspace_bytes, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (bits != 4 && bits != 8) return fail(IC_ERR_INVALID, "int_bits must be 4 or 8, got %d", bits);
  if (update_passes != 1 && update_passes != 3) return fail(IC_ERR_INVALID, "update_passes must be 1 or 3");
  if (block_size <= 0 || block_size > MAXB) return fail(IC_ERR_UNSUPPORTED, "block_size must be in [1,%d]", MAXB);
  if (bits == 4 && packed && block_size % 2) return fail(IC_ERR_UNSUPPORTED, "gptq_layer: odd block size with packing");
  const int r = rot > 0 ? rot : 1;
  const int64_t npad = cdiv(N_in, r) * r;
  const int64_t ldw = round4(npad);
  LayerWs w{};
  const size_t need = layer_ws(M, N_in, rot, &w, workspace, workspace_bytes);
  if (workspace_bytes < need)
    return fail(IC_ERR_WORKSPACE, "gptq_layer: workspace too small (%zu < %zu)", workspace_bytes, need);
  if (h_rotated && N_in != npad) return fail(IC_ERR_INVALID, "pre-rotated Hessian needs in_features % rot_size == 0");
  IC_TRY(rotate_weights(W, dtype, M, N_in, ldw_in, rot, w.W0, ldw, st, WEIGHT_OUTLIER_CLAMP, smoothing));
  IC_CUDA(cudaMemcpyAsync(w.Wk, w.W0, (size_t)M * ldw * 4, cudaMemcpyDeviceToDevice, st));
  if (smooth_order != 0 && smooth_order != 1) return fail(IC_ERR_INVALID, "smooth_order must be 0 or 1");
  if (h_rotated || r <= 1) {
    IC_TRY(split_tf32(H, npad, npad, ldh_in, w.Hh, w.Hl, ldw, st, smoothing));
  } else if (smoothing && smooth_order == 1) {
    // The pipeline's own order for a SmoothRot layer (pipeline.py:721-723, then
    // 766-770): rotate H, smooth the rotated matrix, rotate again.  The first
    // rotation lands in the inverse's scratch (its U pair holds npad x ldw floats
    // and is written only later, by the inverse).
    if (npad != N_in) return fail(IC_ERR_UNSUPPORTED, "smooth_order 1 needs in_features % rot_size == 0");
    float* tmp = static_cast<float*>(w.inv);
    IC_TRY(rotate_hessian(H, 1, N_in, ldh_in, rot, tmp, nullptr, npad, ldw, st));
    IC_TRY(rotate_hessian(tmp, 1, npad, ldw, rot, w.Hh, w.Hl, npad, ldw, st, smoothing));
  } else {
    IC_TRY(rotate_hessian(H, 1, N_in, ldh_in, rot, w.Hh, w.Hl, npad, ldw, st, smoothing));
  }
  const bool has_zp = bits == 4 || asym;
  IC_TRY(ic_gptq_row_params(w.W0, M, npad, ldw, bits, asym, w.scale, has_zp ? w.zp : nullptr, st));
  // With stats the call stays asynchronous: the inverse's not-positive-definite bit (and the
  // bad-scale bit) land in stats[2].  Without stats it synchronises once to return IC_ERR_NOT_PD.
  IC_CUDA(cudaMemsetAsync(w.status, 0, sizeof(unsigned), st));
  params_out_kernel<<<grid1(M), 256, 0, st>>>(w.scale, has_zp ? w.zp : nullptr, M, scales_f16,
                                               has_zp ? zp_out : nullptr, w.sscale, w.status);
  IC_CHECK_LAUNCH();
  // The column loop reads Hinv's lower 128-tiles and its diagonal blocks; when
  // the block size divides 128 no block straddles a tile, so the upper tiles
  // are never read and the mirror pass is skipped.
  IC_TRY(spd_inverse(w.Hh, w.Hl, npad, ldw, damping, w.inv, w.inv_bytes, st, w.status, 128 % block_size != 0));
  LoopArgs L{};
  L.W = w.Wk; L.ldw = ldw; L.W0 = w.W0; L.ldw0 = ldw; L.M = M; L.N = npad; L.h_hi = w.Hh; L.h_lo = w.Hl;
  L.ldh = ldw; L.B = block_size; L.SB = (LAYER_SB / block_size) * block_size;
  L.scale = w.scale; L.zp = has_zp ? w.zp : nullptr; L.stat_scale = w.sscale;
  L.qmin = bits == 4 ? -8 : -128; L.qmax = bits == 4 ? 7 : 127;
  L.codes = codes; L.ldq = npad; L.packed = bits == 4 ? packed : nullptr;
  L.ldp = (npad + 1) / 2; L.row_sqerr = w.rsq; L.row_maxerr = w.rmx; L.passes = update_passes; L.ldlq = false;
  IC_TRY(run_loop(L, w.loop, w.loop_bytes, st));
  if (stats) {
    stats_kernel<<<1, 1024, 0, st>>>(w.rsq, w.rmx, M, (double)M * (double)npad, stats, w.status);
    IC_CHECK_LAUNCH();
    return IC_OK;
  }
  unsigned f = 0;
  IC_CUDA(cudaMemcpyAsync(&f, w.status, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  IC_CUDA(cudaStreamSynchronize(st));
  if (f & DEV_NOT_PD) return fail(IC_ERR_NOT_PD, "Hessian is not positive definite");
  return IC_OK;
}
