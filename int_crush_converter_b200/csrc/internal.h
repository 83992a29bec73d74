// Host-side functions shared between the translation units of the library.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ic {
// clamp > 0: weights with |w| > clamp are zeroed on load (the pipeline's
// outlier sanitize, pipeline.py:527-537); NaN passes through
int rotate_weights(const void* W, int dtype, int64_t M, int64_t N, int64_t ldw, int rot, float* out,
                   int64_t ldo, cudaStream_t st, float clamp = 0.f, const float* smooth = nullptr);
int rotate_hessian(const float* H, int64_t nbatch, int64_t n, int64_t ldh, int rot, float* out_hi,
                   float* out_lo, int64_t npad, int64_t ldo, cudaStream_t st,
                   const float* smooth = nullptr);
int split_tf32(const float* in, int64_t rows, int64_t cols, int64_t ldi, float* hi, float* lo,
               int64_t ldo, cudaStream_t st,
               const float* smooth = nullptr);
int gemm_tn(int64_t m, int64_t n, int64_t k, float alpha, const float* a_hi, const float* a_lo,
            int64_t lda, const float* b_hi, const float* b_lo, int64_t ldb, float beta,
            const float* c_hi, const float* c_lo, int64_t ldc, float* d_hi, float* d_lo,
            int64_t ldd, int passes, cudaStream_t st, int tri = 0);
// per-device set-up of the GEMM kernels (attributes, status word); call outside stream capture
int gemm_prepare();
int transpose(const float* in_hi, const float* in_lo, int64_t rows, int64_t cols, int64_t ldi,
              float alpha, float* out_hi, float* out_lo, int64_t ldo, cudaStream_t st);
// full = false: only the lower 128-tiles of H^-1 (diagonal tiles complete) are written
int spd_inverse(float* h_hi, float* h_lo, int64_t n, int64_t ldh, float damping, void* ws,
                size_t ws_bytes, cudaStream_t st, unsigned* status = nullptr, bool full = true);
size_t spd_inverse_ws(int64_t n);
int read_and_clear_flags(unsigned* out, cudaStream_t st);
void register_device_flags(int dev, unsigned* p);
int finalize_stats(const double* row_sqerr, const float* row_maxerr, int64_t M, double count,
                   double* stats, cudaStream_t st);

// workspace carving helper (256-byte aligned sub-allocations)
struct Carver {
  char* base;
  size_t cap, off = 0;
  Carver(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += count * sizeof(T);
    return p;
  }
  bool ok() const { return off <= cap; }
};
}  // namespace ic
