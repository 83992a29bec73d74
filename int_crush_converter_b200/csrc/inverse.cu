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
#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int BASE = 128;
constexpr int LDS = BASE + 1;
constexpr size_t BASE_SMEM = (size_t)2 * BASE * LDS * 4;

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
// to the slot [128 x 128].  Inner products accumulate in fp64.
__global__ void __launch_bounds__(512) chol_base_kernel(float* hi, float* lo, int n, int64_t ld, float* ihi,
                                                        float* ilo, unsigned* flags) {
  extern __shared__ float sm[];
  float* a = sm;             // [BASE][LDS]  L
  float* x = sm + BASE * LDS;  // [BASE][LDS]  Linv
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  for (int idx = threadIdx.x; idx < n * n; idx += blockDim.x) {
    const int i = idx / n, j = idx % n;
    a[i * LDS + j] = i >= j ? __fadd_rn(hi[i * ld + j], lo[i * ld + j]) : 0.f;
  }
  __syncthreads();
  // left-looking column Cholesky: column k computed after columns < k
  for (int k = 0; k < n; ++k) {
    // diagonal
    if (threadIdx.x < 32) {
      double s = 0.0;
      for (int t = threadIdx.x; t < k; t += 32) s += (double)a[k * LDS + t] * a[k * LDS + t];
      s = warp_sum_d(s);
      if (threadIdx.x == 0) {
        const double d = (double)a[k * LDS + k] - s;
        if (!(d > 0.0) || !isfinite(d)) {
          bad = 1;
          a[k * LDS + k] = 1.f;
        } else {
          a[k * LDS + k] = (float)sqrt(d);
        }
      }
    }
    __syncthreads();
    const float dkk = a[k * LDS + k];
    // column below the diagonal: one warp per row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int i = k + 1 + warp; i < n; i += nw) {
      double s = 0.0;
      for (int t = lane; t < k; t += 32) s += (double)a[i * LDS + t] * a[k * LDS + t];
      s = warp_sum_d(s);
      if (lane == 0) a[i * LDS + k] = (float)(((double)a[i * LDS + k] - s) / (double)dkk);
    }
    __syncthreads();
  }
  // Linv: forward substitution, one thread per column c of the identity
  for (int c = threadIdx.x; c < n; c += blockDim.x) {
    for (int i = 0; i < n; ++i) {
      if (i < c) {
        x[i * LDS + c] = 0.f;
        continue;
      }
      double s = (i == c) ? 1.0 : 0.0;
      for (int t = c; t < i; ++t) s -= (double)a[i * LDS + t] * x[t * LDS + c];
      x[i * LDS + c] = (float)(s / (double)a[i * LDS + i]);
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < n * n; idx += blockDim.x) {
    const int i = idx / n, j = idx % n;
    put_pair(hi, lo, (int64_t)i * ld + j, i >= j ? a[i * LDS + j] : 0.f);
  }
  for (int idx = threadIdx.x; idx < BASE * BASE; idx += blockDim.x) {
    const int i = idx / BASE, j = idx % BASE;
    put_pair(ihi, ilo, idx, (i < n && j < n) ? x[i * LDS + j] : 0.f);
  }
  if (threadIdx.x == 0 && bad) atomicOr(flags, DEV_NOT_PD);
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

// copy a [rows x cols] hi/lo block (ldi -> ldo)
__global__ void copy_pair_kernel(const float* __restrict__ ih, const float* __restrict__ il, int64_t rows,
                                 int64_t cols, int64_t ldi, float* __restrict__ oh, float* __restrict__ ol,
                                 int64_t ldo) {
  const int64_t total = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    oh[r * ldo + c] = ih[r * ldi + c];
    ol[r * ldo + c] = il[r * ldi + c];
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

int64_t split_point(int64_t n) { return std::max<int64_t>((n / 2 / BASE) * BASE, BASE); }

int gemm3(const Ctx& c, int64_t m, int64_t n, int64_t k, float alpha, Pair A, int64_t lda, Pair B, int64_t ldb,
          float beta, Pair D, int64_t ldd, bool c_is_d) {
  return gemm_tn(m, n, k, alpha, A.hi, A.lo, lda, B.hi, B.lo, ldb, beta, c_is_d ? D.hi : nullptr,
                 c_is_d ? D.lo : nullptr, ldd, D.hi, D.lo, ldd, 3, c.st);
}

// X [m x n] (leading dimension ldx) <- X * L^-T, L = the factor's diagonal block at off (size n)
int trsm_rec(const Ctx& c, Pair X, int64_t m, int64_t ldx, int64_t off, int64_t n) {
  if (m <= 0 || n <= 0) return IC_OK;
  if (n <= BASE) {
    IC_TRY(gemm3(c, m, n, n, 1.f, X, ldx, c.slot(off), BASE, 0.f, c.T, BASE, false));
    const int blocks = (int)std::min<int64_t>(cdiv(m * n, 256), 148 * 16);
    copy_pair_kernel<<<blocks, 256, 0, c.st>>>(c.T.hi, c.T.lo, m, n, BASE, X.hi, X.lo, ldx);
    IC_CHECK_LAUNCH();
    return IC_OK;
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
    chol_base_kernel<<<1, 512, BASE_SMEM, c.st>>>(A.hi, A.lo, (int)n, c.ld, S.hi, S.lo, c.flags);
    IC_CHECK_LAUNCH();
    return IC_OK;
  }
  const int64_t n1 = split_point(n), n2 = n - n1;
  IC_TRY(chol_rec(c, off, n1));
  Pair A21 = c.H.at(off + n1, off, c.ld);
  IC_TRY(trsm_rec(c, A21, n2, c.ld, off, n1));  // L21 = A21 L11^-T
  IC_TRY(gemm3(c, n2, n2, n1, -1.f, A21, c.ld, A21, c.ld, 1.f, c.H.at(off + n1, off + n1, c.ld), c.ld, true));
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
  IC_TRY(gemm3(c, n1, n2, n1, -1.f, c.U.at(off, off, c.ld), c.ld, c.H.at(off + n1, off, c.ld), c.ld, 0.f, U12,
               c.ld, false));
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

int spd_inverse(float* h_hi, float* h_lo, int64_t n, int64_t ldh, float damping, void* ws, size_t ws_bytes,
                cudaStream_t st) {
  if (n <= 0) return IC_OK;
  if (!h_hi || !h_lo) return fail(IC_ERR_INVALID, "spd_inverse: hi/lo pair required");
  if (ldh % 4) return fail(IC_ERR_INVALID, "spd_inverse: ld must be a multiple of 4");
  unsigned* flags = device_flags();
  if (!flags) return fail(IC_ERR_CUDA, "device status word unavailable");
  Ctx c{};
  c.H = Pair{h_hi, h_lo};
  c.ld = ldh;
  c.flags = flags;
  c.st = st;
  // the workspace holds U with the caller's leading dimension
  const size_t need = ws_layout(n, ldh, &c, ws, ws_bytes);
  if (ws_bytes < need) return fail(IC_ERR_WORKSPACE, "spd_inverse: workspace too small (%zu < %zu)", ws_bytes, need);
  static bool attr = false;
  if (!attr) {
    IC_CUDA(cudaFuncSetAttribute(chol_base_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BASE_SMEM));
    attr = true;
  }
  unsigned prev = 0;
  IC_TRY(read_and_clear_flags(&prev, st));
  if (damping >= 0.f) {
    damp_kernel<<<1, 1024, 0, st>>>(h_hi, h_lo, n, ldh, damping);
    IC_CHECK_LAUNCH();
  }
  IC_CUDA(cudaMemsetAsync(c.U.hi, 0, (size_t)n * ldh * 4, st));
  IC_CUDA(cudaMemsetAsync(c.U.lo, 0, (size_t)n * ldh * 4, st));
  IC_TRY(chol_rec(c, 0, n));
  IC_TRY(invt_rec(c, 0, n));
  // H^-1 = U U^T
  IC_TRY(gemm3(c, n, n, n, 1.f, c.U, ldh, c.U, ldh, 0.f, c.H, ldh, false));
  unsigned f = 0;
  IC_TRY(read_and_clear_flags(&f, st));
  if (f & DEV_TIMEOUT) return fail(IC_ERR_TIMEOUT, "spd_inverse: a tensor-core wait timed out");
  if (f & DEV_NOT_PD) return fail(IC_ERR_NOT_PD, "Hessian is not positive definite");
  return IC_OK;
}

}  // namespace ic

extern "C" size_t ic_spd_inverse_workspace_size(int64_t n) { return ic::spd_inverse_ws(n); }
extern "C" int ic_spd_inverse(float* h_hi, float* h_lo, int64_t n, int64_t ldh, float damping, void* workspace,
                              size_t workspace_bytes, void* stream) {
  return ic::spd_inverse(h_hi, h_lo, n, ldh, damping, workspace, workspace_bytes, (cudaStream_t)stream);
}
extern "C" int ic_transpose(const float* in_hi, const float* in_lo, int64_t rows, int64_t cols, int64_t ldi,
                            float alpha, float* out_hi, float* out_lo, int64_t ldo, void* stream) {
  return ic::transpose(in_hi, in_lo, rows, cols, ldi, alpha, out_hi, out_lo, ldo, (cudaStream_t)stream);
}
