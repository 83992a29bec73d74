// ic_gptq_run_noalloc: the GPTQ column loop for callers that cannot allocate
// device memory -- for instance a host process whose device memory is wholly
// owned and capped by another allocator, or a latency-critical path where an
// allocation (and its possible implicit synchronisation) is not acceptable.
//
// The loop's scratch (the TF32 hi/lo error block of one super-block, plus the
// staging slice used when block_size % 4 != 0) lives in a fixed file-scope
// device array of IC_NOALLOC_SCRATCH_BYTES that every GPU loading this library
// holds until the process exits.  The library's 4-byte status word for the
// device is taken from the same kind of static storage if it does not exist
// yet.  The first call on a device resolves the arrays' device addresses
// (cudaGetSymbolAddress, with that device current); make that first call
// before any stream capture.  All calls share the one scratch array and it
// keeps the previous call's contents: nothing in it has to start at zero (the
// loop writes every scratch element before reading it), but calls that
// overlap on the GPU (different streams, or host threads on one device) race
// on it and must be serialised by the caller.
#include <mutex>

#include "common.cuh"
#include "internal.h"

static __device__ __align__(256) unsigned char g_noalloc_scratch[IC_NOALLOC_SCRATCH_BYTES];
static __device__ __align__(256) unsigned g_noalloc_flags;

namespace {
std::mutex g_mu;
void* g_scratch_addr[64] = {nullptr};

int setup_device(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return ic::fail(IC_ERR_CUDA, "gptq_run_noalloc: cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
    void* f = nullptr;
    e = cudaGetSymbolAddress(&f, g_noalloc_flags);
    if (e != cudaSuccess)
      return ic::fail(IC_ERR_CUDA, "gptq_run_noalloc: cudaGetSymbolAddress(flags) failed: %s", cudaGetErrorString(e));
    ic::register_device_flags(dev, static_cast<unsigned*>(f));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return IC_OK;
}
}  // namespace

extern "C" int ic_gptq_run_noalloc(float* W_work, int64_t ldw, const float* W0, int64_t ldw0, int64_t M, int64_t N,
                                   const float* hinv_hi, const float* hinv_lo, int64_t ldh, int block_size,
                                   int superblock, const float* scale, const float* zp, int qmin, int qmax,
                                   int8_t* codes, int64_t ldq, uint8_t* packed, int64_t ldp, double* row_sqerr,
                                   float* row_maxerr, int gemm_passes, void* stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ic::fail(IC_ERR_CUDA, "gptq_run_noalloc: no CUDA device: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return ic::fail(IC_ERR_UNSUPPORTED, "gptq_run_noalloc: device index %d", dev);
  if (M <= 0 || N <= 0)  // nothing to do: the same argument checks and result as ic_gptq_run, no scratch
    return ic_gptq_run(W_work, ldw, W0, ldw0, M, N, hinv_hi, hinv_lo, ldh, block_size, superblock, scale, zp,
                       qmin, qmax, codes, ldq, packed, ldp, row_sqerr, row_maxerr, gemm_passes, nullptr, 0, stream);
  const size_t need = ic_gptq_workspace_size(M, N, block_size, superblock);
  if (need > (size_t)IC_NOALLOC_SCRATCH_BYTES)
    return ic::fail(IC_ERR_UNSUPPORTED,
                    "gptq_run_noalloc: this shape needs %zu bytes of scratch but the built-in array holds %zu "
                    "(reduce rows or superblock, or use ic_gptq_run with a caller workspace)",
                    need, (size_t)IC_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  IC_TRY(setup_device(dev, &scratch));
  return ic_gptq_run(W_work, ldw, W0, ldw0, M, N, hinv_hi, hinv_lo, ldh, block_size, superblock, scale, zp, qmin,
                     qmax, codes, ldq, packed, ldp, row_sqerr, row_maxerr, gemm_passes, scratch,
                     (size_t)IC_NOALLOC_SCRATCH_BYTES, stream);
}
