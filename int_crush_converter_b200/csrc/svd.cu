// Pieces of the SVD-absorbed low-rank split (converter/svd.py:35-75, which
// calls torch.svd_lowrank: randomized range finder with power iterations, then
// an SVD of the small projected matrix).  The products run on the library's
// 3xTF32 GEMM (host side); the two small dense steps are here:
//   orth_kernel   -- orthonormal columns of X [m x q] (row-major, q <= 64) by
//                    classical Gram-Schmidt applied twice, one CTA; the QR
//                    step of the range finder;
//   jacobi_kernel -- eigenpairs of a symmetric q x q matrix (q <= 64) by cyclic
//                    Jacobi with all q/2 disjoint rotations of a round applied
//                    in parallel, one CTA in shared memory, eigenvalues sorted
//                    descending with their vectors; the small SVD via B B^T.
#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int QMAX = 64;

__device__ double block_sum(double v, double* red) {
  v = warp_sum_d(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

__global__ void __launch_bounds__(1024) orth_kernel(float* __restrict__ X, int64_t m, int q, int64_t ldx) {
  // classical Gram-Schmidt applied twice per column ("twice is enough"): the
  // projections of column j on the earlier columns come from one pass of
  // per-warp dot products (warp w takes columns w, w + 32, ...), then each
  // thread subtracts them from its rows in one sweep along the row
  __shared__ double red[32];
  __shared__ double dots[QMAX];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int j = 0; j < q; ++j) {
    for (int pass = 0; pass < 2; ++pass) {
      for (int i = warp; i < j; i += nw) {
        double d = 0.0;
        for (int64_t r = lane; r < m; r += 32) d += (double)X[r * ldx + i] * (double)X[r * ldx + j];
        d = warp_sum_d(d);
        if (lane == 0) dots[i] = d;
      }
      __syncthreads();
      for (int64_t r = threadIdx.x; r < m; r += blockDim.x) {
        const float* row = X + r * ldx;
        double x = (double)row[j];
        for (int i = 0; i < j; ++i) x -= dots[i] * (double)row[i];
        X[r * ldx + j] = (float)x;
      }
      __syncthreads();
    }
    double nn = 0.0;
    for (int64_t r = threadIdx.x; r < m; r += blockDim.x) nn += (double)X[r * ldx + j] * (double)X[r * ldx + j];
    nn = block_sum(nn, red);
    const double inv = nn > 0.0 ? 1.0 / sqrt(nn) : 0.0;
    for (int64_t r = threadIdx.x; r < m; r += blockDim.x) X[r * ldx + j] = (float)((double)X[r * ldx + j] * inv);
    __syncthreads();
  }
}

// A (q x q, row-major, symmetric) -> eigenvalues evals[q] (descending) and
// eigenvectors as the columns of V (q x q row-major).
__global__ void __launch_bounds__(1024) jacobi_kernel(const float* __restrict__ A, int q, int64_t lda,
                                                      float* __restrict__ evals, float* __restrict__ V,
                                                      int64_t ldv, int sweeps) {
  extern __shared__ double dyn[];
  double (*a)[QMAX + 1] = reinterpret_cast<double (*)[QMAX + 1]>(dyn);
  double (*v)[QMAX + 1] = reinterpret_cast<double (*)[QMAX + 1]>(dyn + QMAX * (QMAX + 1));
  __shared__ double cs[QMAX / 2], sn[QMAX / 2];
  __shared__ int pp[QMAX / 2], qq[QMAX / 2];
  __shared__ int order[QMAX];
  const int n = (q + 1) & ~1;  // even size (a zero row/column pads odd q)
  for (int idx = threadIdx.x; idx < n * n; idx += blockDim.x) {
    const int i = idx / n, j = idx % n;
    a[i][j] = (i < q && j < q) ? 0.5 * ((double)A[i * lda + j] + (double)A[j * lda + i]) : 0.0;
    v[i][j] = i == j ? 1.0 : 0.0;
  }
  __syncthreads();
  const int half = n / 2;
  for (int sw = 0; sw < sweeps; ++sw) {
    for (int round = 0; round < n - 1; ++round) {
      // round-robin pairing: position 0 fixed, the others rotate
      if ((int)threadIdx.x < half) {
        const int k = threadIdx.x;
        auto slot = [&](int s) { return s == 0 ? 0 : 1 + (s - 1 + round) % (n - 1); };
        int p = slot(k), r = slot(n - 1 - k);
        if (p > r) { const int t = p; p = r; r = t; }
        pp[k] = p;
        qq[k] = r;
        const double apq = a[p][r];
        double c = 1.0, s = 0.0;
        if (fabs(apq) > 1e-300) {
          const double theta = (a[r][r] - a[p][p]) / (2.0 * apq);
          const double t = (theta >= 0 ? 1.0 : -1.0) / (fabs(theta) + sqrt(theta * theta + 1.0));
          c = 1.0 / sqrt(t * t + 1.0);
          s = t * c;
        }
        cs[k] = c;
        sn[k] = s;
      }
      __syncthreads();
      // rows: a[p][:], a[r][:] <- rotation (J^T A)
      for (int idx = threadIdx.x; idx < half * n; idx += blockDim.x) {
        const int k = idx / n, col = idx % n;
        const int p = pp[k], r = qq[k];
        const double c = cs[k], s = sn[k];
        const double x = a[p][col], y = a[r][col];
        a[p][col] = c * x - s * y;
        a[r][col] = s * x + c * y;
      }
      __syncthreads();
      // columns: a[:][p], a[:][r] <- (J^T A) J ; V <- V J
      for (int idx = threadIdx.x; idx < half * n; idx += blockDim.x) {
        const int k = idx / n, row = idx % n;
        const int p = pp[k], r = qq[k];
        const double c = cs[k], s = sn[k];
        const double x = a[row][p], y = a[row][r];
        a[row][p] = c * x - s * y;
        a[row][r] = s * x + c * y;
        const double vx = v[row][p], vy = v[row][r];
        v[row][p] = c * vx - s * vy;
        v[row][r] = s * vx + c * vy;
      }
      __syncthreads();
    }
  }
  // sort by eigenvalue, descending (rank counting over the q real entries)
  if ((int)threadIdx.x < q) {
    const int i = threadIdx.x;
    int r = 0;
    for (int k = 0; k < q; ++k) r += (a[k][k] > a[i][i] || (a[k][k] == a[i][i] && k < i)) ? 1 : 0;
    order[r] = i;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < q * q; idx += blockDim.x) {
    const int row = idx / q, rk = idx % q;
    V[row * ldv + rk] = (float)v[row][order[rk]];
  }
  if ((int)threadIdx.x < q) evals[threadIdx.x] = (float)a[order[threadIdx.x]][order[threadIdx.x]];
}

}  // namespace
}  // namespace ic

using namespace ic;

extern "C" int ic_orthonormalize(float* X, int64_t m, int q, int64_t ldx, void* stream) {
  if (m <= 0 || q <= 0) return IC_OK;
  if (q > QMAX || q > m) return fail(IC_ERR_UNSUPPORTED, "orthonormalize: need 1 <= q <= min(m, %d)", QMAX);
  if (!X || ldx < q) return fail(IC_ERR_INVALID, "orthonormalize: bad arguments");
  orth_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(X, m, q, ldx);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

extern "C" int ic_sym_eig(const float* A, int q, int64_t lda, float* evals, float* V, int64_t ldv, void* stream) {
  if (q <= 0) return IC_OK;
  if (q > QMAX) return fail(IC_ERR_UNSUPPORTED, "sym_eig: q must be <= %d", QMAX);
  if (!A || !evals || !V || lda < q || ldv < q) return fail(IC_ERR_INVALID, "sym_eig: bad arguments");
  constexpr int SMEM = 2 * QMAX * (QMAX + 1) * 8;
  static std::atomic<unsigned long long> attr{0};
  IC_TRY(once_per_device(attr, [&]() -> int {
      IC_CUDA(cudaFuncSetAttribute(jacobi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
      return IC_OK;
    }));
  jacobi_kernel<<<1, 1024, SMEM, (cudaStream_t)stream>>>(A, q, lda, evals, V, ldv, 12);
  IC_CHECK_LAUNCH();
  return IC_OK;
}
