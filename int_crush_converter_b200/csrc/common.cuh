// Shared helpers for the sm_100a kernels of libintcrush_b200.
//
// Error model: every entry point returns an ic_status (0 = ok).  Device-side
// failures that must not hang or fault the GPU (a wait that times out, a
// non-positive pivot, an out-of-range code) are recorded in a per-device
// status word that the host reads back; kernels never trap.
#pragma once
#include <atomic>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <algorithm>
#include <string>

#include "../../include/intcrush_b200.h"

namespace ic {

int fail(int code, const char* fmt, ...);

#define IC_CUDA(expr)                                                          \
  do {                                                                         \
    cudaError_t _e = (expr);                                                   \
    if (_e != cudaSuccess)                                                     \
      return ::ic::fail(IC_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,           \
                        cudaGetErrorString(_e), __FILE__, __LINE__);           \
  } while (0)

// Run `fn` (returning an IC_* status) once per device: kernel attributes such
// as the dynamic shared-memory opt-in are per device, so a process driving
// several GPUs must set them on each.
template <typename F>
inline int once_per_device(std::atomic<unsigned long long>& done, F&& fn) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(IC_ERR_CUDA, "cudaGetDevice failed");
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load() & bit) return IC_OK;
  const int r = fn();
  if (r != IC_OK) return r;
  done.fetch_or(bit);
  return IC_OK;
}

// |w| above this is corrupted data and zeroed before rotation in the fused
// per-layer calls (config.WEIGHT_OUTLIER_CLAMP, applied at pipeline.py:527-537)
constexpr float WEIGHT_OUTLIER_CLAMP = 1000.f;

void count_launch();
void add_launches(unsigned long long n);  // kernels a replayed CUDA graph runs
unsigned long long launches();

#define IC_CHECK_LAUNCH()                                                      \
  do {                                                                         \
    ::ic::count_launch();                                                      \
    cudaError_t _e = cudaGetLastError();                                       \
    if (_e != cudaSuccess)                                                     \
      return ::ic::fail(IC_ERR_CUDA, "kernel launch failed: %s (%s:%d)",       \
                        cudaGetErrorString(_e), __FILE__, __LINE__);           \
  } while (0)

#define IC_TRY(expr)                                                           \
  do {                                                                         \
    int _s = (expr);                                                           \
    if (_s != IC_OK) return _s;                                                \
  } while (0)

// ---- device-side status word -------------------------------------------------
enum : unsigned { DEV_TIMEOUT = 1u, DEV_NOT_PD = 2u, DEV_RANGE = 4u, DEV_BAD_SCALE = 8u };
unsigned* device_flags();  // per-device word, allocated once at first use

// Bounded wait on phase `parity` of a shared-memory mbarrier: true once the
// phase completed; false after `limit_ns` of globaltimer time, with
// DEV_TIMEOUT or-ed into *flags (if given).  Every mbarrier wait of the
// library goes through this, so no kernel can spin forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, unsigned* flags,
                                                  unsigned long long limit_ns) {
  unsigned long long t0 = 0;
  for (int spin = 0;; ++spin) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((spin & 255) == 0) {
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (spin == 0) {
        t0 = now;
      } else if (now - t0 > limit_ns) {
        if (flags) atomicOr(flags, DEV_TIMEOUT);
        return false;
      }
    }
  }
}

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---- reference rounding ---------------------------------------------------------
// _round_half_away_from_zero (converter/rounding.py:106-112):
//   where(x >= 0, floor(x + 0.5), ceil(x - 0.5)) with the fp32 add first.
__device__ __forceinline__ float rhaz(float x) {
  return x >= 0.f ? floorf(__fadd_rn(x, 0.5f)) : ceilf(__fsub_rn(x, 0.5f));
}
// torch.clamp semantics (NaN propagates)
__device__ __forceinline__ float clampf(float x, float lo, float hi) {
  return x != x ? x : fminf(fmaxf(x, lo), hi);
}
__device__ __forceinline__ float clamp_lo(float x, float lo) { return x != x ? x : fmaxf(x, lo); }

// Round-to-nearest TF32 (value stays a float with the low 13 mantissa bits 0).
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// Split x = hi + lo exactly: hi is TF32-representable (the tensor core consumes
// it without loss whether it truncates or rounds), lo = x - hi is the exact
// fp32 remainder (|lo| <= 2^-11 |x|, consumed at TF32 precision).
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = to_tf32(x);
  lo = __fsub_rn(x, hi);
}

template <typename T> __device__ __forceinline__ float load_as_f32(const T* p);
template <> __device__ __forceinline__ float load_as_f32<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float load_as_f32<__half>(const __half* p) { return __half2float(*p); }
template <> __device__ __forceinline__ float load_as_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

__device__ __forceinline__ double warp_sum_d(double v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// NaN-propagating max/min (torch.amax/amin propagate NaN)
__device__ __forceinline__ float nmax(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b);
}
__device__ __forceinline__ float nmin(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fminf(a, b);
}

}  // namespace ic
