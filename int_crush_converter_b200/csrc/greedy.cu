// Greedy coordinate descent on the integer grid (converter/greedy.py:487-541).
//
// Per pass and per block of up to 128 columns:
//   cross[:, blk] = err * H[blk, :]^T          (tcgen05 GEMM, 3xTF32)
// then a block kernel walks the block's columns in order.  For column j the
// reference's cross term err @ H[j,:] - err_j H_jj is the GEMM value plus the
// exact rank-1 corrections delta_j' * H[j', j] of the block's columns j' < j
// already updated in this pass (no periodic recompute, no drift).  Candidates
// g in [qmin, qmax] are evaluated in ascending order with the reference's
// cost (e+(g-q)s)^2 H_jj + 2 (e+(g-q)s) cross; the first minimum wins.
#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int GROUP = 32;
constexpr int GB = 128;

struct GArgs {
  int8_t* Q;
  int64_t ldq;
  const float* S;
  int64_t lds;
  float* e_hi;
  float* e_lo;
  int64_t lde;
  const float* cross;
  const float* cross2;  // second K half of the cross terms (split product), or null
  int64_t ldx;
  const float* h_hi;
  const float* h_lo;
  int64_t ldh;
  int64_t M, j0;
  int bc;
  float qmin, qmax;
};

__global__ void __launch_bounds__(128) greedy_block_kernel(const GArgs a) {
  extern __shared__ float smem[];
  float* hs = smem;            // [bc][GB]
  float* ds = smem + GB * GB;  // [GB][32] deltas (column j, lane)
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int bc = a.bc, ng = (bc + GROUP - 1) / GROUP;
  const int64_t r = (int64_t)blockIdx.x * GROUP + lane;
  const bool rv = r < a.M;
  const int64_t rr = rv ? r : a.M - 1;
  // the block's H[j0 + j, j0 + k] (hi + lo) into shared memory; every
  // iteration's loads are independent, so they are unrolled to overlap their
  // latency (16-byte loads when the block is full and aligned)
  const bool v4 = bc == GB && ((a.ldh | a.j0) & 3) == 0 && (reinterpret_cast<uintptr_t>(a.h_hi) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(a.h_lo) & 15) == 0;
  if (v4) {
#pragma unroll 8
    for (int idx = threadIdx.x; idx < GB * GB / 4; idx += 128) {
      const int j = idx >> 5, k = (idx & 31) * 4;
      const int64_t o = (a.j0 + j) * a.ldh + a.j0 + k;
      const float4 h = *reinterpret_cast<const float4*>(a.h_hi + o);
      const float4 l = *reinterpret_cast<const float4*>(a.h_lo + o);
      *reinterpret_cast<float4*>(hs + j * GB + k) =
          make_float4(__fadd_rn(h.x, l.x), __fadd_rn(h.y, l.y), __fadd_rn(h.z, l.z), __fadd_rn(h.w, l.w));
    }
  } else {
#pragma unroll 8
    for (int idx = threadIdx.x; idx < bc * bc; idx += blockDim.x) {
      const int j = idx / bc, k = idx % bc;
      const int64_t o = (a.j0 + j) * a.ldh + a.j0 + k;
      hs[j * GB + k] = __fadd_rn(a.h_hi[o], a.h_lo[o]);
    }
  }
  const int cbase = g * GROUP;
  float cr[GROUP], er[GROUP], q[GROUP], s[GROUP];
#pragma unroll
  for (int c = 0; c < GROUP; ++c) {
    const bool ok = cbase + c < bc;
    const int64_t col = a.j0 + cbase + c;
    cr[c] = ok ? (a.cross2 ? __fadd_rn(a.cross[rr * a.ldx + cbase + c], a.cross2[rr * a.ldx + cbase + c])
                           : a.cross[rr * a.ldx + cbase + c])
               : 0.f;
    er[c] = ok ? __fadd_rn(a.e_hi[rr * a.lde + col], a.e_lo[rr * a.lde + col]) : 0.f;
    q[c] = ok ? (float)a.Q[rr * a.ldq + col] : 0.f;
    s[c] = ok ? a.S[rr * a.lds + col] : 0.f;
  }
  __syncthreads();
  for (int G = 0; G < ng; ++G) {
    if (g == G) {
#pragma unroll
      for (int c = 0; c < GROUP; ++c) {
        const int j = cbase + c;
        if (j < bc) {
          const float hjj = hs[j * GB + j];
          const float x = __fsub_rn(cr[c], __fmul_rn(er[c], hjj));
          float best = 0.f, bq = a.qmin;
          for (float gv = a.qmin; gv <= a.qmax; gv += 1.f) {
            const float ne = __fadd_rn(er[c], __fmul_rn(__fsub_rn(gv, q[c]), s[c]));
            const float cost = __fadd_rn(__fmul_rn(__fmul_rn(ne, ne), hjj), __fmul_rn(__fmul_rn(2.f, ne), x));
            if (gv == a.qmin || cost < best) {
              best = cost;
              bq = gv;
            }
          }
          const float delta = __fmul_rn(__fsub_rn(bq, q[c]), s[c]);
          q[c] = bq;
          er[c] = __fadd_rn(er[c], delta);
          ds[j * GROUP + lane] = delta;
#pragma unroll
          for (int c2 = c + 1; c2 < GROUP; ++c2) cr[c2] = __fadd_rn(cr[c2], __fmul_rn(delta, hs[j * GB + cbase + c2]));
        }
      }
    }
    __syncthreads();
    if (g > G) {
      const int jend = min(bc, (G + 1) * GROUP);
#pragma unroll 1
      for (int j = G * GROUP; j < jend; ++j) {
        const float d = ds[j * GROUP + lane];
        const float* hrow = hs + j * GB + cbase;
#pragma unroll
        for (int c = 0; c < GROUP; ++c) cr[c] = __fadd_rn(cr[c], __fmul_rn(d, hrow[c]));
      }
    }
  }
  if (!rv) return;
#pragma unroll
  for (int c = 0; c < GROUP; ++c) {
    if (cbase + c >= bc) continue;
    const int64_t col = a.j0 + cbase + c;
    a.Q[r * a.ldq + col] = (int8_t)q[c];
    const float h = to_tf32(er[c]);
    a.e_hi[r * a.lde + col] = h;
    a.e_lo[r * a.lde + col] = __fsub_rn(er[c], h);
  }
}

// err = Q * S - W as a TF32 hi/lo pair
__global__ void err_init_kernel(const float* __restrict__ W, int64_t ldw, const int8_t* __restrict__ Q, int64_t ldq,
                                const float* __restrict__ S, int64_t lds, int64_t M, int64_t N,
                                float* __restrict__ eh, float* __restrict__ el, int64_t lde) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / N, c = i % N;
    const float e = __fsub_rn(__fmul_rn((float)Q[r * ldq + c], S[r * lds + c]), W[r * ldw + c]);
    const float h = to_tf32(e);
    eh[r * lde + c] = h;
    el[r * lde + c] = __fsub_rn(e, h);
  }
}

constexpr size_t GSMEM = (size_t)GB * GB * 4 + (size_t)GB * GROUP * 4;

// ---------------------------------------------------------------------------
// Low-rank pass (converter/greedy.py:100-199, the kernel greedy_lowrank_triton
// launches per 64 columns, greedy.py:440-462): H ~ U_k diag(s_k) U_k^T + the
// exact diagonal.  Each thread owns one row: its projection err_lr = err U_k
// (k <= KMAX values) stays in registers for the whole pass; for every column
// j in order
//   cross = sum_i err_lr_i (s_i U[j,i]) - err_j H_jj
//   g in [qmin, qmax] ascending, cost = ne^2 H_jj + 2 ne cross with
//   ne = err_j + (g - q_j) max(s_rj, 1e-8); strict < against 1e30, so the
//   first minimum wins and q_j stays when no cost is below 1e30
//   err_j += (g - q_j) s;  err_lr_i += delta U[j,i]
// The rows s_i U[j,i] and U[j,i] of a 64-column block are staged in shared
// memory and read by every thread (broadcast).
constexpr int LR_COLS = 64;

struct LArgs {
  float* err;  // [M, N] Q * s - W, updated
  int64_t lde;
  int8_t* Q;
  int64_t ldq;
  const float* S;
  int64_t lds;
  const float* hdiag;  // [N]
  const float* U;      // [N, k] eigenvectors
  const float* SU;     // [N, k] s_i * U[j, i]
  int k;
  float* elr;  // [M, k] err U_k, updated
  int64_t M, N;
  float qmin, qmax;
};

template <int KMAX>
__global__ void __launch_bounds__(128) greedy_lowrank_kernel(const LArgs a) {
  __shared__ float su_s[LR_COLS][KMAX];
  __shared__ float u_s[LR_COLS][KMAX];
  __shared__ float h_s[LR_COLS];
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool rv = r < a.M;
  const int k = a.k;
  float e_lr[KMAX];
#pragma unroll
  for (int i = 0; i < KMAX; ++i) e_lr[i] = (rv && i < k) ? a.elr[r * k + i] : 0.f;
  for (int64_t j0 = 0; j0 < a.N; j0 += LR_COLS) {
    const int nc = (int)((a.N - j0) < LR_COLS ? (a.N - j0) : LR_COLS);
    __syncthreads();
    for (int idx = threadIdx.x; idx < nc * KMAX; idx += blockDim.x) {
      const int c = idx / KMAX, i = idx - c * KMAX;
      su_s[c][i] = i < k ? a.SU[(j0 + c) * k + i] : 0.f;
      u_s[c][i] = i < k ? a.U[(j0 + c) * k + i] : 0.f;
    }
    for (int c = threadIdx.x; c < nc; c += blockDim.x) h_s[c] = a.hdiag[j0 + c];
    __syncthreads();
    if (!rv) continue;
    for (int c = 0; c < nc; ++c) {
      const int64_t j = j0 + c;
      float cross = 0.f;
#pragma unroll
      for (int i = 0; i < KMAX; ++i)
        if (i < k) cross = __fmaf_rn(e_lr[i], su_s[c][i], cross);
      const float ej = a.err[r * a.lde + j];
      const float hjj = h_s[c];
      cross = __fsub_rn(cross, __fmul_rn(ej, hjj));
      const float sj = fmaxf(a.S[r * a.lds + j], 1e-8f);
      const float qo = (float)a.Q[r * a.ldq + j];
      float best = 1e30f, bq = qo;
      for (float g = a.qmin; g <= a.qmax; g += 1.f) {
        const float ne = __fadd_rn(ej, __fmul_rn(__fsub_rn(g, qo), sj));
        const float cost = __fadd_rn(__fmul_rn(__fmul_rn(ne, ne), hjj), __fmul_rn(__fmul_rn(2.f, ne), cross));
        if (cost < best) {
          best = cost;
          bq = g;
        }
      }
      bq = fminf(fmaxf(bq, a.qmin), a.qmax);
      const float d = __fmul_rn(__fsub_rn(bq, qo), sj);
      a.Q[r * a.ldq + j] = (int8_t)bq;
      a.err[r * a.lde + j] = __fadd_rn(ej, d);
#pragma unroll
      for (int i = 0; i < KMAX; ++i)
        if (i < k) e_lr[i] = __fmaf_rn(d, u_s[c][i], e_lr[i]);
    }
  }
  if (rv) {
#pragma unroll
    for (int i = 0; i < KMAX; ++i)
      if (i < k) a.elr[r * k + i] = e_lr[i];
  }
}

// The cross-term product of a block (M x 128 outputs, K = N) has one 128-row
// tile per 128 rows: at M = 8192 that is 64 CTAs on 148 SMs.  Its K range is
// split in two halves issued on the caller's stream and a side stream (event
// fork / join), so both halves run at once on twice the SMs; the block kernel
// adds the two partial sums (first half first).  IC_GREEDY_SPLIT=0 keeps one
// product.
bool split_on() {
  static const bool on = [] {
    const char* e = getenv("IC_GREEDY_SPLIT");
    return !(e && e[0] == '0');
  }();
  return on;
}
struct SideStream {
  cudaStream_t st = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
// one side stream and event pair per host thread and device
int side_stream(SideStream** out) {
  thread_local SideStream cache[64];
  int dev = 0;
  IC_CUDA(cudaGetDevice(&dev));
  SideStream& s = cache[dev & 63];
  if (!s.st) {
    IC_CUDA(cudaStreamCreateWithFlags(&s.st, cudaStreamNonBlocking));
    IC_CUDA(cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming));
    IC_CUDA(cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming));
  }
  *out = &s;
  return IC_OK;
}

}  // namespace
}  // namespace ic

using namespace ic;

extern "C" size_t ic_greedy_workspace_size(int64_t M, int64_t N) {
  const int64_t lde = (N + 3) & ~int64_t(3);
  return (size_t)M * lde * 4 * 2 + (size_t)M * GB * 4 * 2 + 4096;
}

extern "C" int ic_greedy_run(const float* W, int64_t ldw, int8_t* Q, int64_t ldq, const float* scale2d, int64_t lds,
                             const float* h_hi, const float* h_lo, int64_t ldh, int64_t M, int64_t N, int passes,
                             int qmin, int qmax, int gemm_passes, void* workspace, size_t workspace_bytes,
                             void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (M <= 0 || N <= 0 || passes <= 0) return IC_OK;
  if (M > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "greedy: too many rows");
  if (ldh % 4) return fail(IC_ERR_INVALID, "greedy: H leading dimension must be a multiple of 4");
  if (workspace_bytes < ic_greedy_workspace_size(M, N)) return fail(IC_ERR_WORKSPACE, "greedy: workspace too small");
  const int64_t lde = (N + 3) & ~int64_t(3);
  Carver cv(workspace, workspace_bytes);
  float* eh = cv.take<float>((size_t)M * lde);
  float* el = cv.take<float>((size_t)M * lde);
  float* cross = cv.take<float>((size_t)M * GB);
  float* cross2 = cv.take<float>((size_t)M * GB);
  const int64_t kh = (N / 2) & ~int64_t(31);
  const bool split = split_on() && kh >= 1024 && 2 * cdiv(M, 128) <= 160;
  SideStream* side = nullptr;
  if (split) IC_TRY(side_stream(&side));
  static std::atomic<unsigned long long> attr{0};
  IC_TRY(once_per_device(attr, [&]() -> int {
      IC_CUDA(cudaFuncSetAttribute(greedy_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GSMEM));
      return IC_OK;
    }));
  {
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(M * N, 256), 148 * 16));
    err_init_kernel<<<blocks, 256, 0, st>>>(W, ldw, Q, ldq, scale2d, lds, M, N, eh, el, lde);
    IC_CHECK_LAUNCH();
  }
  for (int p = 0; p < passes; ++p) {
    for (int64_t j0 = 0; j0 < N; j0 += GB) {
      const int bc = (int)std::min<int64_t>(GB, N - j0);
      if (split) {
        IC_CUDA(cudaEventRecord(side->fork, st));
        IC_CUDA(cudaStreamWaitEvent(side->st, side->fork, 0));
        IC_TRY(gemm_tn(M, bc, kh, 1.f, eh, el, lde, h_hi + j0 * ldh, h_lo + j0 * ldh, ldh, 0.f, nullptr, nullptr, GB,
                       cross, nullptr, GB, gemm_passes, st));
        IC_TRY(gemm_tn(M, bc, N - kh, 1.f, eh + kh, el + kh, lde, h_hi + j0 * ldh + kh, h_lo + j0 * ldh + kh, ldh,
                       0.f, nullptr, nullptr, GB, cross2, nullptr, GB, gemm_passes, side->st));
        IC_CUDA(cudaEventRecord(side->join, side->st));
        IC_CUDA(cudaStreamWaitEvent(st, side->join, 0));
      } else {
        IC_TRY(gemm_tn(M, bc, N, 1.f, eh, el, lde, h_hi + j0 * ldh, h_lo + j0 * ldh, ldh, 0.f, nullptr, nullptr, GB,
                       cross, nullptr, GB, gemm_passes, st));
      }
      GArgs a{Q, ldq, scale2d, lds, eh, el, lde, cross, split ? cross2 : nullptr, GB, h_hi, h_lo, ldh, M, j0, bc,
              (float)qmin, (float)qmax};
      greedy_block_kernel<<<(unsigned)cdiv(M, GROUP), 128, GSMEM, st>>>(a);
      IC_CHECK_LAUNCH();
    }
  }
  return IC_OK;
}

extern "C" int ic_greedy_lowrank_pass(float* err, int64_t lde, int8_t* Q, int64_t ldq, const float* scale2d,
                                      int64_t lds, const float* hdiag, const float* U, const float* SU, int k,
                                      float* err_lr, int64_t M, int64_t N, int qmin, int qmax, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (M <= 0 || N <= 0) return IC_OK;
  if (k < 1 || k > 64) return fail(IC_ERR_UNSUPPORTED, "greedy low-rank: rank must be in [1, 64], got %d", k);
  if (M > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "greedy: too many rows");
  if (!err || !Q || !scale2d || !hdiag || !U || !SU || !err_lr) return fail(IC_ERR_INVALID, "greedy: null operand");
  LArgs a{err, lde, Q, ldq, scale2d, lds, hdiag, U, SU, k, err_lr, M, N, (float)qmin, (float)qmax};
  const unsigned grid = (unsigned)cdiv(M, 128);
  if (k <= 8) greedy_lowrank_kernel<8><<<grid, 128, 0, st>>>(a);
  else if (k <= 16) greedy_lowrank_kernel<16><<<grid, 128, 0, st>>>(a);
  else if (k <= 32) greedy_lowrank_kernel<32><<<grid, 128, 0, st>>>(a);
  else greedy_lowrank_kernel<64><<<grid, 128, 0, st>>>(a);
  IC_CHECK_LAUNCH();
  return IC_OK;
}
