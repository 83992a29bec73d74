// Group-wise Hadamard rotation (ConvRot) of weights and Hessians: the row
// (or a 32-column strip of rot rows) being rotated lives in shared memory,
// so HBM sees each element once per pass.
#include <math.h>
#include <stdlib.h>

#include "common.cuh"
#include "hadamard.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int ROT_CHUNK = 8192;  // columns per CTA for the row rotation

template <typename T>
__global__ void __launch_bounds__(256) rotate_rows_kernel(const T* __restrict__ W, int64_t N, int64_t ldw,
                                                          int rot, float* __restrict__ out, int64_t ldo,
                                                          int64_t npad, float clamp) {
  __shared__ __align__(16) float s[ROT_CHUNK];
  const int64_t row = blockIdx.x;
  const int64_t c0 = (int64_t)blockIdx.y * ROT_CHUNK;
  const int len = (int)((npad - c0) < ROT_CHUNK ? (npad - c0) : ROT_CHUNK);
  load_row_smem(W + row * ldw, c0, N, len, s);
  if (clamp > 0.f)
    for (int i = threadIdx.x; i < len; i += blockDim.x) s[i] = fabsf(s[i]) > clamp ? 0.f : s[i];
  __syncthreads();
  hadamard_row(s, len, rot);
  store_row_smem(s, len, out + row * ldo + c0);
}

// torch semantics of (H / s_outer.clamp(min=1e-16)).clamp(max=1e30): NaN passes
__device__ __forceinline__ float smooth_hessian(float h, float si, float sj) {
  float p = __fmul_rn(sj, si);
  p = p < 1e-16f ? 1e-16f : p;
  const float q = __fdiv_rn(h, p);
  return q > 1e30f ? 1e30f : q;
}

// Register-only row rotation for 16 <= rot <= 512: every warp streams groups
// global -> registers -> butterflies -> global with no shared memory and no
// barrier, 32/L groups per warp pass (L = rot/16 lanes per group, 16
// consecutive elements per lane).  Rows are `nb` batches of `rows` rows of
// which the first `valid` exist in the source (the rest are zero padding);
// columns >= N are zero padding.  Same operations as hadamard_smem.
template <typename T>
__global__ void __launch_bounds__(256) rotate_regs_kernel(const T* __restrict__ src, int64_t N, int64_t ld,
                                                          int64_t bstride, int64_t rows, int64_t valid, int64_t nb,
                                                          int rot, float* __restrict__ out, int64_t ldo,
                                                          int64_t ostride, int64_t npad, float clamp,
                                                          const float* __restrict__ smw,
                                                          const float* __restrict__ smh) {
  const int L = rot / 16, gpw = 32 / L;
  const int lane = threadIdx.x & 31, l = lane & (L - 1);
  const int64_t ngr = npad / rot;                    // groups per row
  const int64_t tasks = cdiv(nb * rows * ngr, (int64_t)gpw);
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  constexpr int V = 16 / sizeof(T);
  for (int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < tasks; task += warps) {
    const int64_t g = task * gpw + lane / L;          // global group index
    const bool act = g < nb * rows * ngr;
    const int64_t rg = act ? g / ngr : 0;             // batch-row
    const int64_t col = (act ? g - rg * ngr : 0) * rot + 16 * l;
    const int64_t b = rg / rows, r = rg - b * rows;
    float v[16];
    const T* p = src + b * bstride + r * ld + col;
    if (act && r < valid && col + 16 <= N && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
      for (int q = 0; q < 16 / V; ++q) {
        const uint4 raw = reinterpret_cast<const uint4*>(p)[q];
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int u = 0; u < V; ++u) v[q * V + u] = load_as_f32(e + u);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = (act && r < valid && col + j < N) ? load_as_f32(p + j) : 0.f;
    }
    if (clamp > 0.f) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = fabsf(v[j]) > clamp ? 0.f : v[j];
    }
    if (smw && act) {  // SmoothQuant: W[:, j] * s_j (smoothquant.py:54-69)
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (col + j < N) v[j] = __fmul_rn(v[j], smw[col + j]);
    }
    if (smh && act && r < valid) {  // H / max(s_i s_j, 1e-16), capped at 1e30 (pipeline.py:99-137)
      const float si = smh[r];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (col + j < N) v[j] = smooth_hessian(v[j], si, smh[col + j]);
    }
    hadamard_regs16(v, rot, l);
    if (act) {
      float* o = out + b * ostride + r * ldo + col;
      if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          reinterpret_cast<float4*>(o)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = v[j];
      }
    }
  }
}

// rot = 256 with two groups per 16-lane team: lane l holds chunk l (16
// elements) of two neighbouring groups of a row as fp32 pairs, so every
// butterfly of both groups is one packed .f32x2 instruction; the two lane
// digits go through one 16 x 16 shared-memory transpose of pairs instead of
// shuffles.  Same stage order and fp32 operations as rotate_regs_kernel
// (digits of the element index inside the chunk, then of the chunk index;
// the factor 1/16 once at the end): bit-identical output.  Rows are `nb`
// batches of `rows` rows of which the first `valid` exist in the source;
// columns >= N are zero padding; npad % 512 == 0.
typedef unsigned long long f2;
__device__ __forceinline__ f2 pk2(float a, float b) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float lo2(f2 r) { return __uint_as_float((uint32_t)(r & 0xffffffffull)); }
__device__ __forceinline__ float hi2(f2 r) { return __uint_as_float((uint32_t)(r >> 32)); }
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
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
__device__ __forceinline__ void h4pair(f2& x0, f2& x1, f2& x2, f2& x3) {
  const f2 p = add2(x0, x1), m = sub2(x0, x1), P = add2(x2, x3), Mm = sub2(x2, x3);
  x0 = add2(p, Mm);
  x1 = sub2(p, Mm);
  x2 = add2(m, P);
  x3 = sub2(P, m);
}

// 16 elements of one chunk as fp32 (zero past N or for padding rows)
template <typename T>
__device__ __forceinline__ void load_chunk16(const T* p, bool in_row, int64_t col, int64_t N, float (&x)[16]) {
  constexpr int V = 16 / sizeof(T);
  if (in_row && col + 16 <= N && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < 16 / V; ++q) {
      const uint4 raw = reinterpret_cast<const uint4*>(p)[q];
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int u = 0; u < V; ++u) x[q * V + u] = load_as_f32(e + u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = (in_row && col + j < N) ? load_as_f32(p + j) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rotate_pair256_kernel(const T* __restrict__ src, int64_t N, int64_t ld,
                                                             int64_t bstride, int64_t rows, int64_t valid,
                                                             int64_t nb, float* __restrict__ out, int64_t ldo,
                                                             int64_t ostride, int64_t npad, float clamp,
                                                             const float* __restrict__ smw,
                                                             const float* __restrict__ smh) {
  __shared__ __align__(16) f2 tr[16][256];  // one 16 x 16 tile of pairs per 16-lane team
  const int team = threadIdx.x >> 4, l = threadIdx.x & 15;
  f2* tile = tr[team];
  const int64_t pairs_per_row = npad / 512;
  const int64_t tasks = nb * rows * pairs_per_row;
  const int64_t teams = (int64_t)gridDim.x * (blockDim.x >> 4);
  for (int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 4) + team; task - (team & 1) < tasks; task += teams) {
    // every lane of the warp runs the same number of iterations (the transpose
    // needs the whole half-warp), tasks past the end compute zeros
    const bool act = task < tasks;
    const int64_t rg = act ? task / pairs_per_row : 0;  // batch-row
    const int64_t j = act ? task - rg * pairs_per_row : 0;
    const int64_t b = rg / rows, r = rg - b * rows;
    const int64_t ca = j * 512 + 16 * l, cb = ca + 256;  // chunk l of groups 2j and 2j + 1
    const bool in_row = act && r < valid;
    f2 v[16];
    {
      float x[16], y[16];
      const T* rowp = src + b * bstride + r * ld;
      load_chunk16(rowp + ca, in_row, ca, N, x);
      load_chunk16(rowp + cb, in_row, cb, N, y);
      if (clamp > 0.f) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          x[e] = fabsf(x[e]) > clamp ? 0.f : x[e];
          y[e] = fabsf(y[e]) > clamp ? 0.f : y[e];
        }
      }
      if (smw && act) {  // SmoothQuant: W[:, c] * s_c (smoothquant.py:54-69)
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          if (ca + e < N) x[e] = __fmul_rn(x[e], smw[ca + e]);
          if (cb + e < N) y[e] = __fmul_rn(y[e], smw[cb + e]);
        }
      }
      if (smh && in_row) {  // H / max(s_i s_j, 1e-16), capped at 1e30 (pipeline.py:99-137)
        const float si = smh[r];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          if (ca + e < N) x[e] = smooth_hessian(x[e], si, smh[ca + e]);
          if (cb + e < N) y[e] = smooth_hessian(y[e], si, smh[cb + e]);
        }
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = pk2(x[e], y[e]);
    }
    // digits of the element index inside the chunk
#pragma unroll
    for (int q = 0; q < 4; ++q) h4pair(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
    for (int q = 0; q < 4; ++q) h4pair(v[q], v[4 + q], v[8 + q], v[12 + q]);
    // transpose: element (l, e) to row e, pair slot 2 * (((l >> 1) + e) & 7) + (l & 1);
    // lane l then reads row l (element index l inside every chunk) as eight
    // 16-byte chunks starting at chunk l (distinct banks per quarter-warp)
    __syncwarp();
#pragma unroll
    for (int e = 0; e < 16; ++e) tile[e * 16 + 2 * (((l >> 1) + e) & 7) + (l & 1)] = v[e];
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 w = *reinterpret_cast<const uint4*>(tile + l * 16 + 2 * ((c + l) & 7));
      v[2 * c] = ((f2)w.y << 32) | w.x;
      v[2 * c + 1] = ((f2)w.w << 32) | w.z;
    }
    // v[c] = element l of chunk c: digits of the chunk index
#pragma unroll
    for (int c = 0; c < 4; ++c) h4pair(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
#pragma unroll
    for (int u = 0; u < 4; ++u) h4pair(v[u], v[4 + u], v[8 + u], v[12 + u]);
    if (act) {
      const f2 S = pk2(0.0625f, 0.0625f);
      float* o = out + b * ostride + r * ldo + j * 512 + l;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const f2 y = mul2(v[c], S);
        o[16 * c] = lo2(y);
        o[256 + 16 * c] = hi2(y);
      }
    }
  }
}

// IC_ROT_PAIR=0 keeps rot = 256 on rotate_regs_kernel (A/B checks)
bool rot_pair_on() {
  static const bool on = [] {
    const char* e = getenv("IC_ROT_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename T>
void launch_rotate_regs(const T* src, int64_t N, int64_t ld, int64_t bstride, int64_t rows, int64_t valid,
                        int64_t nb, int rot, float* out, int64_t ldo, int64_t ostride, int64_t npad,
                        cudaStream_t st, float clamp = 0.f, const float* smw = nullptr,
                        const float* smh = nullptr) {
  if (rot == 256 && npad % 512 == 0 && rot_pair_on()) {
    const int64_t tasks = nb * rows * (npad / 512);
    const unsigned grid = (unsigned)std::min<int64_t>(cdiv(tasks, 16), 148 * 8);
    rotate_pair256_kernel<T><<<grid, 256, 0, st>>>(src, N, ld, bstride, rows, valid, nb, out, ldo, ostride, npad,
                                                   clamp, smw, smh);
    return;
  }
  const int64_t tasks = cdiv(nb * rows * (npad / rot), (int64_t)(32 / (rot / 16)));
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(tasks, 8), 148 * 16);
  rotate_regs_kernel<T><<<grid, 256, 0, st>>>(src, N, ld, bstride, rows, valid, nb, rot, out, ldo, ostride, npad,
                                               clamp, smw, smh);
}

// Row pass of R^T H R: every row of H gets the group Hadamard along its
// columns (H R).  Rows >= n and columns >= n are the zero padding.
__global__ void __launch_bounds__(256) hess_rows_kernel(const float* __restrict__ H, int64_t n, int64_t ldh,
                                                        int64_t bstride, int rot, float* __restrict__ out,
                                                        int64_t npad, int64_t ldo, int64_t ostride) {
  __shared__ __align__(16) float s[ROT_CHUNK];
  const int64_t row = blockIdx.x;
  const int64_t b = blockIdx.z;
  const int64_t c0 = (int64_t)blockIdx.y * ROT_CHUNK;
  const int len = (int)((npad - c0) < ROT_CHUNK ? (npad - c0) : ROT_CHUNK);
  if (row < n) {
    load_row_smem(H + b * bstride + row * ldh, c0, n, len, s);
  } else {
    for (int i = threadIdx.x; i < len; i += blockDim.x) s[i] = 0.f;
  }
  __syncthreads();
  hadamard_row(s, len, rot);
  store_row_smem(s, len, out + b * ostride + row * ldo + c0);
}

// Column pass: R^T along the row index within each group of `rot` rows, for a
// strip of 32 columns; writes a TF32 hi/lo pair when lo != NULL.
constexpr int COLS = 32;
__global__ void __launch_bounds__(256) hess_cols_kernel(float* __restrict__ hi, float* __restrict__ lo,
                                                        int64_t npad, int64_t ldo, int64_t ostride, int rot) {
  extern __shared__ float tile[];  // [rot][COLS+1]
  const int64_t b = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.y * rot;
  const int64_t c0 = (int64_t)blockIdx.x * COLS;
  float* base = hi + b * ostride;
  for (int i = threadIdx.x; i < rot * COLS; i += blockDim.x) {
    const int r = i / COLS, c = i % COLS;
    tile[r * (COLS + 1) + c] = (c0 + c < npad) ? base[(r0 + r) * ldo + c0 + c] : 0.f;
  }
  __syncthreads();
  hadamard_smem(tile, rot, rot, COLS + 1, COLS, 1);
  for (int i = threadIdx.x; i < rot * COLS; i += blockDim.x) {
    const int r = i / COLS, c = i % COLS;
    if (c0 + c >= npad) continue;
    const float v = tile[r * (COLS + 1) + c];
    const int64_t idx = b * ostride + (r0 + r) * ldo + c0 + c;
    if (lo) {
      const float h = to_tf32(v);
      hi[idx] = h;
      lo[idx] = __fsub_rn(v, h);
    } else {
      hi[idx] = v;
    }
  }
}

// Column pass for rot = 256 (radix 4, four digits of the row index within a
// group), a strip of 32 columns per CTA of 512 threads, one column per lane.
// Thread (w, c) first holds rows 16w + i (i = 0..15: digits 0 and 1) and
// applies those two stages in registers; one transpose through shared memory
// gives it rows w + 16j (j: digits 2 and 3) for the last two stages, which it
// writes straight out (rows of a lane set stay column-coalesced).  Same
// stage order and fp32 operations as hess_cols_kernel: bit-identical.
constexpr int COLS_R = 32;
__global__ void __launch_bounds__(512) hess_cols256_kernel(float* __restrict__ hi, float* __restrict__ lo,
                                                           int64_t npad, int64_t ldo, int64_t ostride) {
  __shared__ float tile[256][COLS_R + 1];
  const int c = threadIdx.x & 31, w = threadIdx.x >> 5;  // w = 0..15
  const int64_t b = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.y * 256;
  const int64_t col = (int64_t)blockIdx.x * COLS_R + c;
  const bool cv = col < npad;
  float* base = hi + b * ostride + r0 * ldo + col;
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = cv ? base[(int64_t)(16 * w + i) * ldo] : 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) h4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);  // digit 0
#pragma unroll
  for (int q = 0; q < 4; ++q) h4(v[q], v[4 + q], v[8 + q], v[12 + q]);  // digit 1
#pragma unroll
  for (int i = 0; i < 16; ++i) tile[16 * w + i][c] = v[i];
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = tile[w + 16 * j][c];
#pragma unroll
  for (int q = 0; q < 4; ++q) h4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);  // digit 2
#pragma unroll
  for (int q = 0; q < 4; ++q) h4(v[q], v[4 + q], v[8 + q], v[12 + q]);  // digit 3
  if (!cv) return;
  float* lbase = lo ? lo + b * ostride + r0 * ldo + col : nullptr;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int64_t o = (int64_t)(w + 16 * j) * ldo;
    if (lbase) {
      const float h = to_tf32(v[j]);
      base[o] = h;
      lbase[o] = __fsub_rn(v[j], h);
    } else {
      base[o] = v[j];
    }
  }
}

__global__ void split_kernel(const float* __restrict__ in, int64_t rows, int64_t cols, int64_t ldi,
                             float* __restrict__ hi, float* __restrict__ lo, int64_t ldo,
                             const float* __restrict__ smh) {
  const int64_t total = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    float v = in[r * ldi + c];
    if (smh) v = smooth_hessian(v, smh[r], smh[c]);
    const float h = to_tf32(v);
    hi[r * ldo + c] = h;
    if (lo) lo[r * ldo + c] = __fsub_rn(v, h);
  }
}

bool rot_ok(int rot) { return rot == 0 || (rot >= 2 && rot <= 1024 && (rot & (rot - 1)) == 0); }

}  // namespace

int rotate_weights(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, int rot, float* out,
                   int64_t ldo, cudaStream_t st, float clamp, const float* smooth) {
  if (!rot_ok(rot)) return fail(IC_ERR_INVALID, "rot_size must be a power of 2, got %d", rot);
  if (M < 0 || N < 0 || ldw < N) return fail(IC_ERR_INVALID, "rotate_weights: bad shape");
  const int r = rot ? rot : 1;
  const int64_t npad = cdiv(N, r) * r;
  if (ldo < npad) return fail(IC_ERR_INVALID, "rotate_weights: ldo < padded width");
  if (M == 0 || npad == 0) return IC_OK;
  if (M > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "rotate_weights: too many rows");
  if (hadamard_regs_ok(r)) {
    switch (dtype) {
      case IC_F32: launch_rotate_regs((const float*)W, N, ldw, 0, M, M, 1, r, out, ldo, 0, npad, st, clamp, smooth); break;
      case IC_F16: launch_rotate_regs((const __half*)W, N, ldw, 0, M, M, 1, r, out, ldo, 0, npad, st, clamp, smooth); break;
      case IC_BF16:
        launch_rotate_regs((const __nv_bfloat16*)W, N, ldw, 0, M, M, 1, r, out, ldo, 0, npad, st, clamp, smooth);
        break;
      default: return fail(IC_ERR_INVALID, "rotate_weights: unknown dtype %d", dtype);
    }
    IC_CHECK_LAUNCH();
    return IC_OK;
  }
  if (smooth) return fail(IC_ERR_UNSUPPORTED, "rotate_weights: smoothing needs 16 <= rot_size <= 512");
  dim3 grid((unsigned)M, (unsigned)cdiv(npad, ROT_CHUNK));
  switch (dtype) {
    case IC_F32: rotate_rows_kernel<float><<<grid, 256, 0, st>>>((const float*)W, N, ldw, r, out, ldo, npad, clamp); break;
    case IC_F16: rotate_rows_kernel<__half><<<grid, 256, 0, st>>>((const __half*)W, N, ldw, r, out, ldo, npad, clamp); break;
    case IC_BF16:
      rotate_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)W, N, ldw, r, out, ldo, npad, clamp);
      break;
    default: return fail(IC_ERR_INVALID, "rotate_weights: unknown dtype %d", dtype);
  }
  IC_CHECK_LAUNCH();
  return IC_OK;
}

int rotate_hessian(const float* H, int64_t nbatch, int64_t n, int64_t ldh, int rot, float* out_hi,
                   float* out_lo, int64_t npad, int64_t ldo, cudaStream_t st, const float* smooth) {
  if (!rot_ok(rot)) return fail(IC_ERR_INVALID, "rot_size must be a power of 2, got %d", rot);
  const int r = rot ? rot : 1;
  if (nbatch < 1 || n <= 0 || ldh < n) return fail(IC_ERR_INVALID, "rotate_hessian: bad shape");
  if (npad != cdiv(n, r) * r) return fail(IC_ERR_INVALID, "rotate_hessian: npad mismatch");
  if (ldo < npad) return fail(IC_ERR_INVALID, "rotate_hessian: ldo < npad");
  if (nbatch > 1 && n % r)
    return fail(IC_ERR_INVALID, "Block size %lld is not divisible by rot_size %d", (long long)n, rot);
  if (npad > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "rotate_hessian: too large");
  const int64_t ostride = npad * ldo;
  if (smooth && (!hadamard_regs_ok(r) || nbatch != 1))
    return fail(IC_ERR_UNSUPPORTED, "rotate_hessian: smoothing needs a 2-D Hessian and 16 <= rot_size <= 512");
  if (hadamard_regs_ok(r)) {
    launch_rotate_regs(H, n, ldh, n * ldh, npad, n, nbatch, r, out_hi, ldo, ostride, npad, st, 0.f, nullptr, smooth);
  } else {
    dim3 g1((unsigned)npad, (unsigned)cdiv(npad, ROT_CHUNK), (unsigned)nbatch);
    hess_rows_kernel<<<g1, 256, 0, st>>>(H, n, ldh, n * ldh, r, out_hi, npad, ldo, ostride);
  }
  IC_CHECK_LAUNCH();
  if (r == 256) {
    dim3 g2((unsigned)cdiv(npad, COLS_R), (unsigned)(npad / 256), (unsigned)nbatch);
    hess_cols256_kernel<<<g2, 512, 0, st>>>(out_hi, out_lo, npad, ldo, ostride);
    IC_CHECK_LAUNCH();
  } else if (r > 1) {
    const size_t sm = (size_t)r * (COLS + 1) * 4;
    if (sm > 48 * 1024)
      IC_CUDA(cudaFuncSetAttribute(hess_cols_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    dim3 g2((unsigned)cdiv(npad, COLS), (unsigned)(npad / r), (unsigned)nbatch);
    hess_cols_kernel<<<g2, 256, sm, st>>>(out_hi, out_lo, npad, ldo, ostride, r);
    IC_CHECK_LAUNCH();
  } else if (out_lo) {
    IC_TRY(split_tf32(out_hi, nbatch * npad, npad, ldo, out_hi, out_lo, ldo, st));
  }
  return IC_OK;
}

int split_tf32(const float* in, int64_t rows, int64_t cols, int64_t ldi, float* hi, float* lo, int64_t ldo,
               cudaStream_t st, const float* smooth) {
  if (rows <= 0 || cols <= 0) return IC_OK;
  const int64_t total = rows * cols;
  const int blocks = (int)std::min<int64_t>(cdiv(total, 256), 148 * 16);
  split_kernel<<<blocks, 256, 0, st>>>(in, rows, cols, ldi, hi, lo, ldo, smooth);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

}  // namespace ic

extern "C" int ic_rotate_weights(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, int rot,
                                 float* out, int64_t ldo, void* stream) {
  return ic::rotate_weights(W, dtype, M, N, ldw, rot, out, ldo, (cudaStream_t)stream);
}
extern "C" int ic_rotate_hessian(const float* H, int64_t nbatch, int64_t n, int64_t ldh, int rot,
                                 float* out_hi, float* out_lo, int64_t npad, void* stream) {
  return ic::rotate_hessian(H, nbatch, n, ldh, rot, out_hi, out_lo, npad, npad, (cudaStream_t)stream);
}
extern "C" int ic_split_tf32(const float* in, int64_t rows, int64_t cols, int64_t ldi, float* out_hi,
                             float* out_lo, int64_t ldo, void* stream) {
  return ic::split_tf32(in, rows, cols, ldi, out_hi, out_lo, ldo, (cudaStream_t)stream);
}
