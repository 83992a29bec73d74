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
  for (int idx = threadIdx.x; idx < bc * bc; idx += blockDim.x) {
    const int j = idx / bc, k = idx % bc;
    const int64_t o = (a.j0 + j) * a.ldh + a.j0 + k;
    hs[j * GB + k] = __fadd_rn(a.h_hi[o], a.h_lo[o]);
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
