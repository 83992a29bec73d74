// Library-wide plumbing: error strings, the per-device status word, version.
#include <stdarg.h>

#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace ic {

namespace {
thread_local std::string g_err;
std::mutex g_flag_mu;
unsigned* g_flags[64] = {nullptr};
std::atomic<unsigned long long> g_launches{0};
}  // namespace

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void add_launches(unsigned long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
unsigned long long launches() { return g_launches.load(); }

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

unsigned* device_flags() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_flag_mu);
  if (!g_flags[dev]) {
    unsigned* p = nullptr;
    if (cudaMalloc(&p, sizeof(unsigned)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(unsigned)) != cudaSuccess) return nullptr;
    g_flags[dev] = p;
  }
  return g_flags[dev];
}

// Lets a caller that must not allocate supply the status word of `dev` from
// its own storage; has no effect when the word already exists.
void register_device_flags(int dev, unsigned* p) {
  if (dev < 0 || dev >= 64 || !p) return;
  std::lock_guard<std::mutex> lk(g_flag_mu);
  if (!g_flags[dev]) g_flags[dev] = p;
}

int read_and_clear_flags(unsigned* out, cudaStream_t st) {
  unsigned* f = device_flags();
  if (!f) return fail(IC_ERR_CUDA, "device status word unavailable");
  unsigned h = 0;
  IC_CUDA(cudaMemcpyAsync(&h, f, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  IC_CUDA(cudaMemsetAsync(f, 0, sizeof(unsigned), st));
  IC_CUDA(cudaStreamSynchronize(st));
  *out = h;
  return IC_OK;
}

}  // namespace ic

extern "C" const char* ic_version(void) { return "libintcrush_b200 0.1.0 (sm_100a)"; }
extern "C" const char* ic_last_error(void) { return ic::g_err.c_str(); }

extern "C" int ic_device_check(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ic::fail(IC_ERR_CUDA, "no CUDA device: %s", cudaGetErrorString(e));
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return ic::fail(IC_ERR_UNSUPPORTED, "kernels are built for sm_100a; device is sm_%d%d", major, minor);
  return IC_OK;
}

extern "C" int ic_device_status(unsigned* flags_out, void* stream) {
  unsigned f = 0;
  int s = ic::read_and_clear_flags(&f, (cudaStream_t)stream);
  if (flags_out) *flags_out = f;
  return s;
}

extern "C" unsigned long long ic_launch_count(void) { return ic::g_launches.load(); }
