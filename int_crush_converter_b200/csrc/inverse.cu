// Damped inverse of an SPD Hessian on the GPU, replacing gptq._prepare_hinv
// (converter/gptq.py:113-121) + the Cholesky branch of rounding._invert_hessian
// (rounding.py:19-34: torch.linalg.cholesky + torch.cholesky_inverse).
//
// Same algorithm family as LAPACK potrf + potri, recursive and GEMM-rich:
//   1. L = chol(H), recursive:      L11 = chol(A11); L21 = A21 L11^-T (recursive
//      triangular solve); A22 -= L21 L21^T; L22 = chol(A22)
//   2. U = L^-T (upper), recursive: U12 = (-U11 L21^T) L22^-T
//   3. H^-1 = U U^T
// Every O(n^3) step is D = beta*C + alpha*A*B^T on the tcgen05 tensor cores in
// 3xTF32 (matrices held as TF32 hi/lo pairs whose sum is the exact fp32
// value).  Only the 128 x 128 diagonal blocks are factored in shared memory;
// their explicit inverses serve the leaves of the triangular solves.  Only
// the lower triangle of H is read.  A non-positive pivot sets DEV_NOT_PD.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int BASE = 128;

// H += lambda*I, lambda = damping * max(mean(diag H), 1e-6)  (gptq.py:118-119)
__global__ void __launch_bounds__(1024) damp_kernel(float* hi, float* lo, int64_t n, int64_t ld, float damping) {
  __shared__ double red[32];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += (double)hi[i * ld + i] + (double)lo[i * ld + i];
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float mean = fmaxf((float)(red[0] / (double)n), 1e-6f);
  const float lam = __fmul_rn(damping, mean);
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = __fadd_rn(__fadd_rn(hi[i * ld + i], lo[i * ld + i]), lam);
    const float h = to_tf32(v);
    hi[i * ld + i] = h;
    lo[i * ld + i] = __fsub_rn(v, h);
  }
}

__device__ __forceinline__ void put_pair(float* hi, float* lo, int64_t idx, float v) {
  const float h = to_tf32(v);
  hi[idx] = h;
  lo[idx] = __fsub_rn(v, h);
}

// Cholesky of one n x n (n <= 128) diagonal block (lower triangle read), in
// place (lower L, upper zeroed), plus its explicit inverse Linv (lower) written
// to the slot [128 x 128].  Blocked in 32-wide panels inside one CTA:
//   factor the 32 x 32 diagonal block (one warp, rows in lanes, shuffles),
//   solve the panel rows below it by substitution (one thread per row),
//   update the trailing lower triangle (16 warps, one dot product per element);
// then Linv by 32-blocks: the four diagonal blocks inverted in parallel (one
// warp each, one column per lane), the off-diagonal blocks by distance from
// the diagonal.  Padding (n < 128) is an identity block.
constexpr int LDS = BASE + 1;
constexpr size_t BASE_SMEM = (size_t)(2 * BASE * LDS + 3 * 32 * 33) * 4;

// One diagonal of 32-blocks of Linv at distance D below the main one (4 - D
// blocks, 2 (4 - D) elements per thread, every slot used):
// X[I][J] = -X[I][I] * sum_{K=J}^{I-1} L[I][K] X[K][J], I = J + D.
template <int D>
__device__ __forceinline__ void offdiag_round(const float* a, float* x, float* tb, int tid) {
  constexpr int NB = 4 - D, U = 2 * NB;
  float acc[U];
#pragma unroll
  for (int u = 0; u < U; ++u) acc[u] = 0.f;
#pragma unroll 4
  for (int kk = 0; kk < 32 * D; ++kk) {  // T = sum_K L[I][K] X[K][J]
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = tid + 512 * u;
      const int J = e >> 10, rr = (e >> 5) & 31, cc = e & 31, I = J + D;
      acc[u] = fmaf(a[(32 * I + rr) * LDS + 32 * J + kk], x[(32 * J + kk) * LDS + 32 * J + cc], acc[u]);
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int e = tid + 512 * u;
    tb[(e >> 10) * 32 * 33 + ((e >> 5) & 31) * 33 + (e & 31)] = acc[u];
    acc[u] = 0.f;
  }
  __syncthreads();
#pragma unroll 4
  for (int t = 0; t < 32; ++t) {  // X[I][J] = -X[I][I] T  (X[I][I] lower triangular)
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = tid + 512 * u;
      const int J = e >> 10, rr = (e >> 5) & 31, cc = e & 31, I = J + D;
      if (t <= rr) acc[u] = fmaf(x[(32 * I + rr) * LDS + 32 * I + t], tb[J * 32 * 33 + t * 33 + cc], acc[u]);
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int e = tid + 512 * u;
    const int J = e >> 10, rr = (e >> 5) & 31, cc = e & 31, I = J + D;
    x[(32 * I + rr) * LDS + 32 * J + cc] = -acc[u];
  }
  __syncthreads();
}

__global__ void __launch_bounds__(512) chol_base_kernel(float* hi, float* lo, int n, int64_t ld, float* ihi,
                                                        float* ilo, unsigned* flags) {
  extern __shared__ float sm[];
  float* a = sm;                   // [128][LDS]  A -> L
  float* x = sm + BASE * LDS;      // [128][LDS]  Linv
  float* tb = sm + 2 * BASE * LDS;  // [3][32][33] scratch blocks
  __shared__ int bad;
  __shared__ float rdiag[32];  // 1 / L[p0+k][p0+k] of the current panel
  __shared__ __align__(16) float colbuf[64];  // the panel's current column, double-buffered
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) bad = 0;
  if (n == BASE && (ld & 3) == 0 && ((reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo)) & 15) == 0) {
    // full block: float4 loads, 8 in flight per thread
#pragma unroll
    for (int it = 0; it < BASE * BASE / 4 / 512; ++it) {
      const int idx = it * 512 + tid;
      const int i = idx >> 5, j4 = (idx & 31) << 2;
      const float4 h = *reinterpret_cast<const float4*>(hi + (int64_t)i * ld + j4);
      const float4 l = *reinterpret_cast<const float4*>(lo + (int64_t)i * ld + j4);
      float* d = a + i * LDS + j4;
      d[0] = (i >= j4) ? __fadd_rn(h.x, l.x) : 0.f;
      d[1] = (i >= j4 + 1) ? __fadd_rn(h.y, l.y) : 0.f;
      d[2] = (i >= j4 + 2) ? __fadd_rn(h.z, l.z) : 0.f;
      d[3] = (i >= j4 + 3) ? __fadd_rn(h.w, l.w) : 0.f;
      float* dx = x + i * LDS + j4;
      dx[0] = dx[1] = dx[2] = dx[3] = 0.f;
    }
  } else {
    for (int idx = tid; idx < BASE * BASE; idx += blockDim.x) {
      const int i = idx >> 7, j = idx & 127;
      float v;
      if (i < n && j < n) v = (i >= j) ? __fadd_rn(hi[(int64_t)i * ld + j], lo[(int64_t)i * ld + j]) : 0.f;
      else v = (i == j) ? 1.f : 0.f;
      a[i * LDS + j] = v;
      x[i * LDS + j] = 0.f;
    }
  }
  __syncthreads();
  for (int p0 = 0; p0 < BASE; p0 += 32) {
    // (1) 32 x 32 diagonal block, one warp: lane i holds row p0+i
    if (warp == 0) {
      float row[32];
#pragma unroll 32
      for (int j = 0; j < 32; ++j) row[j] = (j <= lane) ? a[(p0 + lane) * LDS + p0 + j] : 0.f;
#pragma unroll 32
      for (int k = 0; k < 32; ++k) {
        float d = __shfl_sync(0xffffffffu, row[k], k);
        if (!(d > 0.f) || !isfinite(d)) {
          if (lane == 0) bad = 1;
          d = 1.f;
        }
        // 1/sqrt(d) from the hardware estimate refined by one Newton-Raphson
        // step, r <- r (3 - d r^2) / 2: L[k][k] = d r and 1/L[k][k] = r, one
        // serial operation per column instead of a square root and a division
        float rd = rsqrtf(d);
        rd = __fmul_rn(rd, __fmaf_rn(-0.5f * d, __fmul_rn(rd, rd), 1.5f));
        if (lane == k) rdiag[k] = rd;
        const float l = (lane > k) ? __fmul_rn(row[k], rd) : (lane == k ? __fmul_rn(d, rd) : 0.f);
        row[k] = l;
        // the column to every lane through shared memory (broadcast loads,
        // vectorisable) rather than 31 - k shuffles; two buffers alternate
        float* colk = colbuf + (k & 1) * 32;
        colk[lane] = l;
        __syncwarp();
#pragma unroll 31
        for (int j = k + 1; j < 32; ++j) {
          const float lj = colk[j];
          if (lane >= j) row[j] = fmaf(-l, lj, row[j]);
        }
      }
#pragma unroll 32
      for (int j = 0; j < 32; ++j)
        if (j <= lane) a[(p0 + lane) * LDS + p0 + j] = row[j];
    }
    __syncthreads();
    // (2) rows below: L21 = A21 L11^-T by forward substitution, one thread per row
    const int r = p0 + 32 + tid;
    if (r < BASE) {
      float xr[32];
#pragma unroll 32
      for (int k = 0; k < 32; ++k) {
        float s = a[r * LDS + p0 + k];
#pragma unroll 31
        for (int t = 0; t < k; ++t) s = fmaf(-xr[t], a[(p0 + k) * LDS + p0 + t], s);
        xr[k] = __fmul_rn(s, rdiag[k]);
      }
#pragma unroll 32
      for (int k = 0; k < 32; ++k) a[r * LDS + p0 + k] = xr[k];
    }
    __syncthreads();
    // (3) trailing update of the lower triangle: a[i][j] -= sum_t L[i][p0+t] L[j][p0+t]
    for (int i = p0 + 32 + warp; i < BASE; i += 16) {
      for (int j = p0 + 32 + lane; j <= i; j += 32) {
        float s = a[i * LDS + j];
#pragma unroll 32
        for (int t = 0; t < 32; ++t) s = fmaf(-a[i * LDS + p0 + t], a[j * LDS + p0 + t], s);
        a[i * LDS + j] = s;
      }
    }
    __syncthreads();
  }
  // Linv, diagonal 32-blocks: warp w inverts block w, lane c computes column c
  if (warp < 4) {
    const int b0 = warp * 32, c = lane;
    float xc[32];
#pragma unroll 32
    for (int i = 0; i < 32; ++i) {
      float s = (i == c) ? 1.f : 0.f;
#pragma unroll 31
      for (int t = 0; t < i; ++t) s = fmaf(-a[(b0 + i) * LDS + b0 + t], xc[t], s);
      xc[i] = (i >= c) ? __fdiv_rn(s, a[(b0 + i) * LDS + b0 + i]) : 0.f;
    }
#pragma unroll 32
    for (int i = 0; i < 32; ++i) x[(b0 + i) * LDS + b0 + c] = xc[i];
  }
  __syncthreads();
  // off-diagonal blocks X[I][J] = -X[I][I] * sum_{K=J}^{I-1} L[I][K] X[K][J], by distance d = I - J
  offdiag_round<1>(a, x, tb, tid);
  offdiag_round<2>(a, x, tb, tid);
  offdiag_round<3>(a, x, tb, tid);
  for (int idx = tid; idx < BASE * BASE; idx += blockDim.x) {
    const int i = idx >> 7, j = idx & 127;
    if (i < n && j < n) put_pair(hi, lo, (int64_t)i * ld + j, (i >= j) ? a[i * LDS + j] : 0.f);
    put_pair(ihi, ilo, idx, (i < n && j < n && j <= i) ? x[i * LDS + j] : 0.f);
  }
  if (tid == 0 && bad) atomicOr(flags, DEV_NOT_PD);
}

// out = alpha * in^T on hi/lo pairs (32x32 tiles through shared memory)
__global__ void transpose_kernel(const float* __restrict__ ih, const float* __restrict__ il, int64_t rows,
                                 int64_t cols, int64_t ldi, float alpha, float* __restrict__ oh,
                                 float* __restrict__ ol, int64_t ldo) {
  __shared__ float t[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t r = r0 + dy, c = c0 + threadIdx.x;
    float v = 0.f;
    if (r < rows && c < cols) {
      v = ih[r * ldi + c];
      if (il) v = __fadd_rn(v, il[r * ldi + c]);
    }
    t[dy][threadIdx.x] = v;
  }
  __syncthreads();
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t orow = c0 + dy, ocol = r0 + threadIdx.x;  // out is [cols x rows]
    if (orow < cols && ocol < rows) {
      const float v = __fmul_rn(alpha, t[threadIdx.x][dy]);
      if (ol) put_pair(oh, ol, orow * ldo + ocol, v);
      else oh[orow * ldo + ocol] = v;
    }
  }
}

// Fill the strictly-upper 128-tiles of a symmetric pair from its lower tiles.
__global__ void mirror_kernel(float* __restrict__ hi, float* __restrict__ lo, int64_t n, int64_t ld) {
  const int64_t bi = blockIdx.y, bj = blockIdx.x;  // 32 x 32 destination tile (row bi, col bj)
  if (bj / 4 <= bi / 4) return;                      // not in a strictly-upper 128-tile
  __shared__ float th[32][33], tl[32][33];
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t r = bj * 32 + dy, c = bi * 32 + threadIdx.x;  // source tile (bj, bi) in the lower part
    if (r < n && c < n) {
      th[dy][threadIdx.x] = hi[r * ld + c];
      tl[dy][threadIdx.x] = lo[r * ld + c];
    }
  }
  __syncthreads();
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t r = bi * 32 + dy, c = bj * 32 + threadIdx.x;
    if (r < n && c < n) {
      hi[r * ld + c] = th[threadIdx.x][dy];
      lo[r * ld + c] = tl[threadIdx.x][dy];
    }
  }
}

// Symmetric completion of a lower triangle: H[r][c] = H[c][r] for every c > r
// (32 x 32 tiles through shared memory; only tiles on or above the diagonal run).
__global__ void sym_from_lower_kernel(float* __restrict__ hi, float* __restrict__ lo, int64_t n, int64_t ld) {
  const int64_t bi = blockIdx.y, bj = blockIdx.x;
  if (bj < bi) return;
  __shared__ float th[32][33], tl[32][33];
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t r = bj * 32 + dy, c = bi * 32 + threadIdx.x;  // source tile (bj, bi)
    if (r < n && c < n) {
      th[dy][threadIdx.x] = hi[r * ld + c];
      tl[dy][threadIdx.x] = lo[r * ld + c];
    }
  }
  __syncthreads();
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t r = bi * 32 + dy, c = bj * 32 + threadIdx.x;
    if (r < n && c < n && c > r) {
      hi[r * ld + c] = th[threadIdx.x][dy];
      lo[r * ld + c] = tl[threadIdx.x][dy];
    }
  }
}

struct Pair {
  float* hi;
  float* lo;
  Pair at(int64_t r, int64_t c, int64_t ld) const { return {hi + r * ld + c, lo + r * ld + c}; }
};

struct Ctx {
  Pair H;        // factor / result, leading dimension ld
  int64_t ld;
  Pair U;        // L^-T, leading dimension ld
  Pair Linv;     // ceil(n/128) slots of [128 x 128]
  Pair T;        // trsm leaf scratch [n x 128]
  unsigned* flags;
  cudaStream_t st;
  Pair slot(int64_t off) const { return Linv.at((off / BASE) * BASE, 0, BASE); }
};

// dynamic shared memory opt-in of the base kernel, once per device
int chol_prepare() {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  IC_CUDA(cudaGetDevice(&dev));
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load() & bit) return IC_OK;
  IC_CUDA(cudaFuncSetAttribute(chol_base_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BASE_SMEM));
  done.fetch_or(bit);
  return IC_OK;
}

int64_t split_point(int64_t n) { return std::max<int64_t>((n / 2 / BASE) * BASE, BASE); }

int gemm3(const Ctx& c, int64_t m, int64_t n, int64_t k, float alpha, Pair A, int64_t lda, Pair B, int64_t ldb,
          float beta, Pair D, int64_t ldd, bool c_is_d, int tri = 0) {
  return gemm_tn(m, n, k, alpha, A.hi, A.lo, lda, B.hi, B.lo, ldb, beta, c_is_d ? D.hi : nullptr,
                 c_is_d ? D.lo : nullptr, ldd, D.hi, D.lo, ldd, 3, c.st, tri);
}

// X [m x n] (leading dimension ldx) <- X * L^-T, L = the factor's diagonal block at off (size n)
int trsm_rec(const Ctx& c, Pair X, int64_t m, int64_t ldx, int64_t off, int64_t n) {
  if (m <= 0 || n <= 0) return IC_OK;
  if (n <= BASE) {
    // In place: with n <= 128 the product has a single column tile, so the CTA
    // that overwrites a row block is the only one that reads it, and it has
    // read all of it (all K) before its epilogue writes.
    return gemm3(c, m, n, n, 1.f, X, ldx, c.slot(off), BASE, 0.f, X, ldx, false);
  }
  const int64_t n1 = split_point(n), n2 = n - n1;
  IC_TRY(trsm_rec(c, X, m, ldx, off, n1));
  // X2 -= X1 * L21^T
  IC_TRY(gemm3(c, m, n2, n1, -1.f, X, ldx, c.H.at(off + n1, off, c.ld), c.ld, 1.f, X.at(0, n1, ldx), ldx, true));
  return trsm_rec(c, X.at(0, n1, ldx), m, ldx, off + n1, n2);
}

// lower Cholesky factor of the diagonal block at off (size n), in place
int chol_rec(const Ctx& c, int64_t off, int64_t n) {
  if (n <= BASE) {
    Pair A = c.H.at(off, off, c.ld), S = c.slot(off);
    IC_TRY(chol_prepare());
    chol_base_kernel<<<1, 512, BASE_SMEM, c.st>>>(A.hi, A.lo, (int)n, c.ld, S.hi, S.lo, c.flags);
    IC_CHECK_LAUNCH();
    return IC_OK;
  }
  const int64_t n1 = split_point(n), n2 = n - n1;
  IC_TRY(chol_rec(c, off, n1));
  Pair A21 = c.H.at(off + n1, off, c.ld);
  IC_TRY(trsm_rec(c, A21, n2, c.ld, off, n1));  // L21 = A21 L11^-T
  // only the lower triangle of A22 is ever read again: skip its strictly-upper tiles
  IC_TRY(gemm3(c, n2, n2, n1, -1.f, A21, c.ld, A21, c.ld, 1.f, c.H.at(off + n1, off + n1, c.ld), c.ld, true, 1));
  return chol_rec(c, off + n1, n2);
}

// U block at (off, off) of size n <- L^-T (upper triangular)
int invt_rec(const Ctx& c, int64_t off, int64_t n) {
  if (n <= BASE) {
    Pair S = c.slot(off), Ub = c.U.at(off, off, c.ld);
    dim3 grid((unsigned)cdiv(n, 32), (unsigned)cdiv(n, 32));
    transpose_kernel<<<grid, dim3(32, 8), 0, c.st>>>(S.hi, S.lo, n, n, BASE, 1.f, Ub.hi, Ub.lo, c.ld);
    IC_CHECK_LAUNCH();
    return IC_OK;
  }
  const int64_t n1 = split_point(n), n2 = n - n1;
  IC_TRY(invt_rec(c, off, n1));
  IC_TRY(invt_rec(c, off + n1, n2));
  Pair U12 = c.U.at(off, off + n1, c.ld);
  // U12 = (-U11 L21^T) L22^-T
  // U11 is upper triangular: row i of it is zero left of column i
  IC_TRY(gemm3(c, n1, n2, n1, -1.f, c.U.at(off, off, c.ld), c.ld, c.H.at(off + n1, off, c.ld), c.ld, 0.f, U12,
               c.ld, false, 2));
  return trsm_rec(c, U12, n1, c.ld, off + n1, n2);
}

size_t ws_layout(int64_t n, int64_t ld, Ctx* c, void* base, size_t cap) {
  Carver cv(base, cap);
  const size_t usz = (size_t)n * ld;
  const size_t nslot = (size_t)cdiv(n, BASE);
  Pair U{cv.take<float>(usz), cv.take<float>(usz)};
  Pair L{cv.take<float>(nslot * BASE * BASE), cv.take<float>(nslot * BASE * BASE)};
  Pair T{cv.take<float>((size_t)n * BASE), cv.take<float>((size_t)n * BASE)};
  if (c) {
    c->U = U;
    c->Linv = L;
    c->T = T;
  }
  return cv.off + 1024;
}

}  // namespace

size_t spd_inverse_ws(int64_t n) { return ws_layout(n, (n + 3) & ~int64_t(3), nullptr, nullptr, 0); }

int transpose(const float* in_hi, const float* in_lo, int64_t rows, int64_t cols, int64_t ldi, float alpha,
              float* out_hi, float* out_lo, int64_t ldo, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return IC_OK;
  dim3 grid((unsigned)cdiv(cols, 32), (unsigned)cdiv(rows, 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(in_hi, in_lo, rows, cols, ldi, alpha, out_hi, out_lo, ldo);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

namespace {

// Everything the inverse enqueues, on c.st.
int inverse_body(const Ctx& c, int64_t n, float damping, bool full) {
  if (damping >= 0.f) {
    damp_kernel<<<1, 1024, 0, c.st>>>(c.H.hi, c.H.lo, n, c.ld, damping);
    IC_CHECK_LAUNCH();
  }
  IC_CUDA(cudaMemsetAsync(c.U.hi, 0, (size_t)n * c.ld * 4, c.st));
  IC_CUDA(cudaMemsetAsync(c.U.lo, 0, (size_t)n * c.ld * 4, c.st));
  IC_TRY(chol_rec(c, 0, n));
  IC_TRY(invt_rec(c, 0, n));
  // H^-1 = U U^T: lower tiles only, K from the tile row (U is upper triangular), then mirror
  IC_TRY(gemm3(c, n, n, n, 1.f, c.U, c.ld, c.U, c.ld, 0.f, c.H, c.ld, false, 3));
  if (!full) return IC_OK;  // lower 128-tiles (diagonal tiles complete) suffice for the GPTQ loop
  dim3 grid((unsigned)cdiv(n, 32), (unsigned)cdiv(n, 32));
  mirror_kernel<<<grid, dim3(32, 8), 0, c.st>>>(c.H.hi, c.H.lo, n, c.ld);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

// The recursion issues ~n/128 * 14 kernels (about 2000 at n = 16384), each
// small one short; issued one by one they fill the launch queue and block the
// host thread, which then cannot feed other streams.  The asynchronous inverse
// is therefore captured once per (device, n, ld, buffers, damping, status word)
// into a CUDA graph and replayed with a single launch.  The cache holds up to
// MAX_GRAPHS executables; evicting one synchronises the device first.
struct InvGraph {
  int dev;
  int64_t n, ld;
  const void *hh, *hl, *ws, *status;
  size_t ws_bytes;
  float damping;
  bool full;
  cudaGraphExec_t exec;
  unsigned long long kernels, used;
  bool same(const InvGraph& o) const {
    return dev == o.dev && n == o.n && ld == o.ld && hh == o.hh && hl == o.hl && ws == o.ws &&
           status == o.status && ws_bytes == o.ws_bytes && damping == o.damping && full == o.full;
  }
};
constexpr size_t MAX_GRAPHS = 32;
std::mutex g_graph_mu;
std::vector<InvGraph> g_graphs;
unsigned long long g_tick = 0;
std::atomic<unsigned long long> g_instantiated{0};
cudaStream_t g_capture[64] = {nullptr};

bool graphs_enabled() {
  static const bool on = [] {
    const char* e = getenv("IC_GRAPHS");
    return !(e && e[0] == '0');
  }();
  return on;
}

int inverse_graph(const Ctx& c, int64_t n, float damping, void* ws, size_t ws_bytes, bool full) {
  InvGraph key{};
  IC_CUDA(cudaGetDevice(&key.dev));
  key.n = n; key.ld = c.ld; key.hh = c.H.hi; key.hl = c.H.lo; key.ws = ws; key.status = c.flags;
  key.ws_bytes = ws_bytes; key.damping = damping; key.full = full;
  std::lock_guard<std::mutex> lock(g_graph_mu);
  for (auto& g : g_graphs) {
    if (g.same(key)) {
      g.used = ++g_tick;
      IC_CUDA(cudaGraphLaunch(g.exec, c.st));
      add_launches(g.kernels);
      return IC_OK;
    }
  }
  // set-up that must not happen inside a capture
  IC_TRY(gemm_prepare());
  IC_TRY(chol_prepare());
  if (key.dev < 0 || key.dev >= 64) return fail(IC_ERR_UNSUPPORTED, "device index %d", key.dev);
  if (!g_capture[key.dev]) IC_CUDA(cudaStreamCreateWithFlags(&g_capture[key.dev], cudaStreamNonBlocking));
  Ctx cc = c;
  cc.st = g_capture[key.dev];
  IC_CUDA(cudaStreamBeginCapture(cc.st, cudaStreamCaptureModeThreadLocal));
  const int r = inverse_body(cc, n, damping, full);
  cudaGraph_t graph = nullptr;
  const cudaError_t e = cudaStreamEndCapture(cc.st, &graph);
  if (r != IC_OK) {
    if (graph) cudaGraphDestroy(graph);
    return r;
  }
  if (e != cudaSuccess || !graph)
    return fail(IC_ERR_CUDA, "spd_inverse: stream capture failed: %s", cudaGetErrorString(e));
  // kernels in the graph (the library's launch counter also counts other host
  // threads' launches made during the capture)
  size_t nodes = 0;
  unsigned long long kernels = 0;
  if (cudaGraphGetNodes(graph, nullptr, &nodes) == cudaSuccess && nodes) {
    std::vector<cudaGraphNode_t> list(nodes);
    if (cudaGraphGetNodes(graph, list.data(), &nodes) == cudaSuccess)
      for (size_t i = 0; i < nodes; ++i) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(list[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
      }
  }
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ei != cudaSuccess) return fail(IC_ERR_CUDA, "spd_inverse: graph instantiation failed: %s", cudaGetErrorString(ei));
  ++g_instantiated;
  key.exec = exec;
  key.kernels = kernels;
  key.used = ++g_tick;
  if (g_graphs.size() >= MAX_GRAPHS) {
    size_t lru = 0;
    for (size_t i = 1; i < g_graphs.size(); ++i)
      if (g_graphs[i].used < g_graphs[lru].used) lru = i;
    IC_CUDA(cudaDeviceSynchronize());
    cudaGraphExecDestroy(g_graphs[lru].exec);
    g_graphs.erase(g_graphs.begin() + (std::ptrdiff_t)lru);
  }
  g_graphs.push_back(key);
  IC_CUDA(cudaGraphLaunch(exec, c.st));
  return IC_OK;
}

}  // namespace

int spd_inverse(float* h_hi, float* h_lo, int64_t n, int64_t ldh, float damping, void* ws, size_t ws_bytes,
                cudaStream_t st, unsigned* status, bool full) {
  if (n <= 0) return IC_OK;
  if (!h_hi || !h_lo) return fail(IC_ERR_INVALID, "spd_inverse: hi/lo pair required");
  if (ldh % 4) return fail(IC_ERR_INVALID, "spd_inverse: ld must be a multiple of 4");
  // Without a status word the call is synchronous and reports through the device's flag word;
  // with one, a non-positive pivot is or-ed into *status and nothing is read back.
  unsigned* flags = status ? status : device_flags();
  if (!flags) return fail(IC_ERR_CUDA, "device status word unavailable");
  Ctx c{};
  c.H = Pair{h_hi, h_lo};
  c.ld = ldh;
  c.flags = flags;
  c.st = st;
  // the workspace holds U with the caller's leading dimension
  const size_t need = ws_layout(n, ldh, &c, ws, ws_bytes);
  if (ws_bytes < need) return fail(IC_ERR_WORKSPACE, "spd_inverse: workspace too small (%zu < %zu)", ws_bytes, need);
  if (status) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    IC_CUDA(cudaStreamIsCapturing(st, &cs));
    if (graphs_enabled() && cs == cudaStreamCaptureStatusNone) return inverse_graph(c, n, damping, ws, ws_bytes, full);
    return inverse_body(c, n, damping, full);
  }
  unsigned prev = 0;
  IC_TRY(read_and_clear_flags(&prev, st));
  IC_TRY(inverse_body(c, n, damping, full));
  unsigned f = 0;
  IC_TRY(read_and_clear_flags(&f, st));
  if (f & DEV_TIMEOUT) return fail(IC_ERR_TIMEOUT, "spd_inverse: a tensor-core wait timed out");
  if (f & DEV_NOT_PD) return fail(IC_ERR_NOT_PD, "Hessian is not positive definite");
  return IC_OK;
}

int spd_cholesky(float* h_hi, float* h_lo, int64_t n, int64_t ldh, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (n <= 0) return IC_OK;
  if (!h_hi || !h_lo) return fail(IC_ERR_INVALID, "spd_cholesky: hi/lo pair required");
  if (ldh % 4) return fail(IC_ERR_INVALID, "spd_cholesky: ld must be a multiple of 4");
  unsigned* flags = device_flags();
  if (!flags) return fail(IC_ERR_CUDA, "device status word unavailable");
  Ctx c{};
  c.H = Pair{h_hi, h_lo};
  c.ld = ldh;
  c.flags = flags;
  c.st = st;
  const size_t need = ws_layout(n, ldh, &c, ws, ws_bytes);
  if (ws_bytes < need) return fail(IC_ERR_WORKSPACE, "spd_cholesky: workspace too small (%zu < %zu)", ws_bytes, need);
  IC_TRY(gemm_prepare());
  unsigned prev = 0;
  IC_TRY(read_and_clear_flags(&prev, st));
  IC_TRY(chol_rec(c, 0, n));
  dim3 grid((unsigned)cdiv(n, 32), (unsigned)cdiv(n, 32));
  sym_from_lower_kernel<<<grid, dim3(32, 8), 0, st>>>(h_hi, h_lo, n, ldh);
  IC_CHECK_LAUNCH();
  unsigned f = 0;
  IC_TRY(read_and_clear_flags(&f, st));
  if (f & DEV_TIMEOUT) return fail(IC_ERR_TIMEOUT, "spd_cholesky: a tensor-core wait timed out");
  if (f & DEV_NOT_PD) return fail(IC_ERR_NOT_PD, "matrix is not positive definite");
  return IC_OK;
}

}  // namespace ic

extern "C" int ic_spd_cholesky(float* h_hi, float* h_lo, int64_t n, int64_t ldh, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return ic::spd_cholesky(h_hi, h_lo, n, ldh, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" size_t ic_spd_inverse_workspace_size(int64_t n) { return ic::spd_inverse_ws(n); }
extern "C" int ic_spd_inverse(float* h_hi, float* h_lo, int64_t n, int64_t ldh, float damping, void* workspace,
                              size_t workspace_bytes, void* stream) {
  return ic::spd_inverse(h_hi, h_lo, n, ldh, damping, workspace, workspace_bytes, (cudaStream_t)stream);
}
extern "C" int ic_transpose(const float* in_hi, const float* in_lo, int64_t rows, int64_t cols, int64_t ldi,
                            float alpha, float* out_hi, float* out_lo, int64_t ldo, void* stream) {
  return ic::transpose(in_hi, in_lo, rows, cols, ldi, alpha, out_hi, out_lo, ldo, (cudaStream_t)stream);
}

extern "C" unsigned long long ic_inverse_graph_count(void) { return ic::g_instantiated.load(); }
