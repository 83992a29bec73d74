// Damped inverse of an SPD Hessian on the GPU, replacing gptq._prepare_hinv
// (converter/gptq.py:113-121) + the Cholesky branch of rounding._invert_hessian
// (rounding.py:19-34).
//
// H = [A B; B^T D] is inverted by the block Schur-complement recursion
//   Ai = A^-1, Ct = B^T Ai, S = D - B^T Ai B, Si = S^-1,
//   H^-1 = [Ai + C Si C^T, -C Si; -Si C^T, Si]   (C = Ct^T)
// which is block LDL^T elimination without pivoting (stable for SPD).  All
// O(n^3) work is D = beta*C + alpha*A*B^T products on the tcgen05 tensor
// cores in 3xTF32; matrices are held as TF32 hi/lo pairs whose sum is the
// exact fp32 value.  Only the lower triangle of the input is ever read (as
// LAPACK's lower Cholesky does).  Diagonal blocks of <= 128 are inverted in
// shared memory by Gauss-Jordan elimination; a non-positive pivot sets
// DEV_NOT_PD.
#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int BASE = 128;
constexpr size_t GJ_SMEM = (size_t)(BASE * (BASE + 1) + 2 * BASE) * 4;

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

// In-place Gauss-Jordan inverse of one n x n (n <= 128) SPD block, read from
// the lower triangle, written back full and symmetric.
__global__ void __launch_bounds__(512) gj_inverse_kernel(float* hi, float* lo, int n, int64_t ld, unsigned* flags) {
  extern __shared__ float gj_smem[];
  float(*a)[BASE + 1] = reinterpret_cast<float(*)[BASE + 1]>(gj_smem);
  float* colk = gj_smem + BASE * (BASE + 1);
  float* rowk = colk + BASE;
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  for (int idx = threadIdx.x; idx < n * n; idx += blockDim.x) {
    const int i = idx / n, j = idx % n;
    const int r = i >= j ? i : j, c = i >= j ? j : i;
    a[i][j] = __fadd_rn(hi[r * ld + c], lo[r * ld + c]);
  }
  __syncthreads();
  for (int k = 0; k < n; ++k) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      colk[i] = a[i][k];
      rowk[i] = a[k][i];
    }
    __syncthreads();
    const float piv = colk[k];
    if (!(piv > 0.f) || !isfinite(piv)) {
      if (threadIdx.x == 0) bad = 1;
    }
    const float inv = 1.0f / piv;
    for (int idx = threadIdx.x; idx < n * n; idx += blockDim.x) {
      const int i = idx / n, j = idx % n;
      float v;
      if (i == k && j == k) v = inv;
      else if (i == k) v = rowk[j] * inv;
      else if (j == k) v = -colk[i] * inv;
      else v = a[i][j] - colk[i] * (rowk[j] * inv);
      a[i][j] = v;
    }
    __syncthreads();
  }
  for (int idx = threadIdx.x; idx < n * n; idx += blockDim.x) {
    const int i = idx / n, j = idx % n;
    const float v = 0.5f * (a[i][j] + a[j][i]);
    const float h = to_tf32(v);
    hi[i * ld + j] = h;
    lo[i * ld + j] = __fsub_rn(v, h);
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
      if (ol) {
        const float h = to_tf32(v);
        oh[orow * ldo + ocol] = h;
        ol[orow * ldo + ocol] = __fsub_rn(v, h);
      } else {
        oh[orow * ldo + ocol] = v;
      }
    }
  }
}

// out = alpha * in on hi/lo pairs
__global__ void scale_copy_kernel(const float* __restrict__ ih, const float* __restrict__ il, int64_t rows,
                                  int64_t cols, int64_t ldi, float alpha, float* __restrict__ oh,
                                  float* __restrict__ ol, int64_t ldo) {
  const int64_t total = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const float v = __fmul_rn(alpha, __fadd_rn(ih[r * ldi + c], il[r * ldi + c]));
    const float h = to_tf32(v);
    oh[r * ldo + c] = h;
    ol[r * ldo + c] = __fsub_rn(v, h);
  }
}

struct Pair {
  float* hi;
  float* lo;
  Pair at(int64_t r, int64_t c, int64_t ld) const { return {hi + r * ld + c, lo + r * ld + c}; }
};

int scale_copy(Pair in, int64_t rows, int64_t cols, int64_t ldi, float alpha, Pair out, int64_t ldo,
               cudaStream_t st) {
  const int blocks = (int)std::min<int64_t>(cdiv(rows * cols, 256), 148 * 16);
  scale_copy_kernel<<<blocks, 256, 0, st>>>(in.hi, in.lo, rows, cols, ldi, alpha, out.hi, out.lo, ldo);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

int64_t split_point(int64_t n) { return std::max<int64_t>((n / 2 / BASE) * BASE, BASE); }
int64_t round4(int64_t x) { return (x + 3) & ~int64_t(3); }

// Recursive in-place inverse of the n x n SPD block at A (leading dimension ld).
int inv_rec(Pair A, int64_t n, int64_t ld, Pair T1, Pair T2, unsigned* flags, cudaStream_t st) {
  if (n <= BASE) {
    static bool attr = false;
    if (!attr) {
      IC_CUDA(cudaFuncSetAttribute(gj_inverse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GJ_SMEM));
      attr = true;
    }
    gj_inverse_kernel<<<1, 512, GJ_SMEM, st>>>(A.hi, A.lo, (int)n, ld, flags);
    IC_CHECK_LAUNCH();
    return IC_OK;
  }
  const int64_t n1 = split_point(n);
  const int64_t n2 = n - n1;
  const int64_t ld2 = round4(n2);  // TMA needs 16-byte row strides
  Pair H11 = A, H12 = A.at(0, n1, ld), H21 = A.at(n1, 0, ld), H22 = A.at(n1, n1, ld);
  IC_TRY(inv_rec(H11, n1, ld, T1, T2, flags, st));  // H11 <- Ai
  // T1 [n2 x n1] = H21 * Ai^T   (Ct = B^T Ai)
  IC_TRY(gemm_tn(n2, n1, n1, 1.f, H21.hi, H21.lo, ld, H11.hi, H11.lo, ld, 0.f, nullptr, nullptr, n1, T1.hi,
                 T1.lo, n1, 3, st));
  // H22 <- S = H22 - H21 * T1^T
  IC_TRY(gemm_tn(n2, n2, n1, -1.f, H21.hi, H21.lo, ld, T1.hi, T1.lo, n1, 1.f, H22.hi, H22.lo, ld, H22.hi,
                 H22.lo, ld, 3, st));
  // H12 <- C = T1^T  [n1 x n2]
  IC_TRY(transpose(T1.hi, T1.lo, n2, n1, n1, 1.f, H12.hi, H12.lo, ld, st));
  IC_TRY(inv_rec(H22, n2, ld, T1, T2, flags, st));  // H22 <- Si
  // T2 [n1 x n2] = C * Si^T   (Z = C Si)
  IC_TRY(gemm_tn(n1, n2, n2, 1.f, H12.hi, H12.lo, ld, H22.hi, H22.lo, ld, 0.f, nullptr, nullptr, ld2, T2.hi,
                 T2.lo, ld2, 3, st));
  // H11 <- Ai + Z * C^T
  IC_TRY(gemm_tn(n1, n1, n2, 1.f, T2.hi, T2.lo, ld2, H12.hi, H12.lo, ld, 1.f, H11.hi, H11.lo, ld, H11.hi,
                 H11.lo, ld, 3, st));
  // H12 <- -Z ; H21 <- -Z^T
  IC_TRY(scale_copy(T2, n1, n2, ld2, -1.f, H12, ld, st));
  IC_TRY(transpose(T2.hi, T2.lo, n1, n2, ld2, -1.f, H21.hi, H21.lo, ld, st));
  return IC_OK;
}

}  // namespace

size_t spd_inverse_ws(int64_t n) {
  const int64_t n1 = split_point(n);
  const int64_t n2 = std::max<int64_t>(n - n1, 1);
  const size_t per = (size_t)n1 * (size_t)std::max<int64_t>(round4(n2), 4) * 4;
  return 4 * (per + 256) + 1024;
}

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
  if (ws_bytes < spd_inverse_ws(n)) return fail(IC_ERR_WORKSPACE, "spd_inverse: workspace too small");
  unsigned prev = 0;
  IC_TRY(read_and_clear_flags(&prev, st));
  if (damping >= 0.f) {
    damp_kernel<<<1, 1024, 0, st>>>(h_hi, h_lo, n, ldh, damping);
    IC_CHECK_LAUNCH();
  }
  const int64_t n1 = split_point(n);
  const int64_t n2 = std::max<int64_t>(n - n1, 1);
  Carver cv(ws, ws_bytes);
  const size_t per = (size_t)n1 * (size_t)std::max<int64_t>(round4(n2), 4);
  Pair T1{cv.take<float>(per), cv.take<float>(per)};
  Pair T2{cv.take<float>(per), cv.take<float>(per)};
  IC_TRY(inv_rec(Pair{h_hi, h_lo}, n, ldh, T1, T2, flags, st));
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
