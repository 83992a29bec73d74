// D = beta*C + alpha * A * B^T on the 5th-generation tensor cores (sm_100a).
//
// One CTA computes a 128 x BN tile.  Warp roles (384 threads):
//   warp 0   : TMA producer (one thread) -- K-major fp32 tiles, 128B swizzle
//   warp 1   : MMA issuer (one thread)   -- tcgen05.mma.kind::tf32, M=128, N=BN, K=8
//   warp 2   : TMEM allocator
//   warps 4-11: epilogue -- two warps per TMEM lane quarter, 64 columns each:
//              tcgen05.ld 32x32b, chunk sums, beta*C + alpha*acc, store
// PASSES = 3 implements 3xTF32: operands arrive as hi/lo pairs (hi exactly
// TF32) and the accumulator receives hi*hi + hi*lo + lo*hi, giving close to
// fp32 accuracy (needed by the Hessian inverse and the GPTQ error feedback).
// Every mbarrier wait is bounded (globaltimer); on timeout the kernel records
// DEV_TIMEOUT in the device status word and finishes without waiting further.
// No TMA multicast is used anywhere: every CTA loads its own tiles.
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace ic {
namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements per 128-byte swizzle row
constexpr unsigned long long WAIT_LIMIT_NS = 4000000000ull;  // 4 s

struct GemmArgs {
  int m, n, k;
  float alpha, beta;
  const float* c_hi;
  const float* c_lo;
  long long ldc;
  float* d_hi;
  float* d_lo;
  long long ldd;
  unsigned* flags;
  int vec;  // C/D rows 16-byte aligned: vectorised epilogue
  int group;  // row-tiles per group of the tile order
  int chunk;  // k-tiles per TMEM accumulator chunk (3xTF32)
  int kofs;  // K index of column 0 of A/B in the full product (K-slab launches)
  int accum_in_place;  // D aliases C with beta == 1: a tile with K = 0 leaves D unchanged
  int lower_rows;      // > 0: enumerate only the lower tiles of the first lower_rows tile rows,
                       //      row by row from the top (square products with tri bit 0)
  int row_major;       // tile order row by row from the top (tri bit 1: longest K first)
  int tri;  // bit 0: only output tiles on/below the diagonal (n0 <= m0);
            // bit 1: A rows are zero left of their own index (upper triangular
            //        A), so the K loop starts at the tile's first row m0
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Bounded wait: returns false (and flags a timeout) instead of spinning forever.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned* flags) {
  return mbar_wait_bounded(bar, parity, flags, WAIT_LIMIT_NS);
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// UMMA shared-memory descriptor: K-major, 128B swizzle, 8-row core groups
// 1024 B apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;            // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO
  d |= (uint64_t)1 << 46;            // version
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

#define IC_TMEM_LD32(taddr, r)                                                                   \
  asm volatile(                                                                                  \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"   \
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"         \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),     \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),  \
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),           \
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),           \
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])            \
      : "r"(taddr))

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Grouped tile order: consecutive CTAs take `group` row-tiles times all
// column-tiles, column by column, so that a wave of CTAs reads a compact
// patch of A and B rows (and re-reads it from L2) instead of one A row-tile
// against every B tile.
constexpr int GROUP_M = 16;      // 128-row tiles per group (single-CTA kernel)
constexpr int PAIR_GROUP_M = 8;  // 256-row pair tiles per group
__device__ __forceinline__ void tile_of(int id, int mt, int nt, int group, int& tm, int& tn) {
  const int per = group * nt;
  const int g = id / per;
  const int first = g * group;
  const int gm = min(group, mt - first);
  const int local = id - g * per;
  tm = first + local % gm;
  tn = local / gm;
}

// Optional wait-time counters (build with -DIC_GEMM_PROFILE; off in the library)
#ifdef IC_GEMM_PROFILE
__device__ unsigned long long g_gemm_prof[8];
#define IC_PROF_T0() const long long _prof_t0 = clock64()
#define IC_PROF_ADD(i) atomicAdd(&g_gemm_prof[i], (unsigned long long)(clock64() - _prof_t0))
#else
#define IC_PROF_T0() \
  do {               \
  } while (0)
#define IC_PROF_ADD(i) \
  do {                 \
  } while (0)
#endif

constexpr int EPI_LD = 132;  // staged row stride in floats (float4 writes by row-per-lane are conflict-free)
constexpr int EPI_RB = 8;    // rows whose C loads are issued together

__device__ __forceinline__ float epi_value(const GemmArgs& a, float s, float c) {
  const float v = a.alpha * s;
  return fmaf(a.beta, c, v);
}

// D[row, n0 + lane*4 .. +3] for the warp's 32 rows, from the staged sums.
template <int BN, int ROWS>
__device__ __forceinline__ void epilogue_rows(const GemmArgs& a, const float* stage, int rbase, int n0, int lane) {
  static_assert(BN == 128, "one float4 per lane covers a 128-wide row");
  const int col = n0 + lane * 4;
  if (col >= a.n) return;
  const bool read_c = a.beta != 0.f && a.c_hi != nullptr;
  const bool full = a.vec && col + 4 <= a.n;
  for (int rr = 0; rr < ROWS; rr += EPI_RB) {
    float4 ch[EPI_RB], cl[EPI_RB];
#pragma unroll
    for (int i = 0; i < EPI_RB; ++i) {
      const int row = rbase + rr + i;
      ch[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      cl[i] = ch[i];
      if (read_c && full && row < a.m) {
        ch[i] = *reinterpret_cast<const float4*>(a.c_hi + (long long)row * a.ldc + col);
        if (a.c_lo) cl[i] = *reinterpret_cast<const float4*>(a.c_lo + (long long)row * a.ldc + col);
      }
    }
#pragma unroll
    for (int i = 0; i < EPI_RB; ++i) {
      const int row = rbase + rr + i;
      if (row >= a.m) break;
      const float4 sv = *reinterpret_cast<const float4*>(stage + (rr + i) * EPI_LD + lane * 4);
      const float sx[4] = {sv.x, sv.y, sv.z, sv.w};
      float* dh = a.d_hi + (long long)row * a.ldd + col;
      float* dl = a.d_lo ? a.d_lo + (long long)row * a.ldd + col : nullptr;
      if (full) {
        float v[4];
        if (read_c) {
          const float cx[4] = {ch[i].x + cl[i].x, ch[i].y + cl[i].y, ch[i].z + cl[i].z, ch[i].w + cl[i].w};
#pragma unroll
          for (int t = 0; t < 4; ++t) v[t] = epi_value(a, sx[t], cx[t]);
        } else {
#pragma unroll
          for (int t = 0; t < 4; ++t) v[t] = a.alpha * sx[t];
        }
        if (dl) {
          float4 h, l;
          split_tf32(v[0], h.x, l.x);
          split_tf32(v[1], h.y, l.y);
          split_tf32(v[2], h.z, l.z);
          split_tf32(v[3], h.w, l.w);
          *reinterpret_cast<float4*>(dh) = h;
          *reinterpret_cast<float4*>(dl) = l;
        } else {
          *reinterpret_cast<float4*>(dh) = make_float4(v[0], v[1], v[2], v[3]);
        }
      } else {
        for (int t = 0; t < 4 && col + t < a.n; ++t) {
          float x = a.alpha * sx[t];
          if (read_c) {
            float cv = a.c_hi[(long long)row * a.ldc + col + t];
            if (a.c_lo) cv += a.c_lo[(long long)row * a.ldc + col + t];
            x = fmaf(a.beta, cv, x);
          }
          if (dl) {
            float h, l;
            split_tf32(x, h, l);
            dh[t] = h;
            dl[t] = l;
          } else {
            dh[t] = x;
          }
        }
      }
    }
  }
}

// One epilogue warp (8 per CTA: two per TMEM lane quarter q = warp % 4, each
// owning 64 of the 128 accumulator columns).  It adds the chunk accumulators
// of its rows/columns in fp32 registers (round to nearest), releasing each
// chunk's accumulator with `release(b)`, then stages its sums in shared memory
// and, after its partner warp has staged the other half, writes 16 of the
// quarter's 32 rows of D.  Returns false if a wait timed out.
template <int NACC, bool CHUNKED, typename Release>
__device__ __forceinline__ void epilogue_warp(const GemmArgs& args, uint32_t tmem, unsigned char* smem, int warp,
                                              int lane, int nchunks, int chunk0, int m0, int n0,
                                              uint32_t accf0, Release release) {
  const int q = warp & 3, h = (warp - 4) >> 2;
  float sum[64];
#pragma unroll
  for (int j = 0; j < 64; ++j) sum[j] = 0.f;
  bool alive = true;
  for (int cl = 0; cl < nchunks; ++cl) {
    const int c = chunk0 + cl;  // global chunk index (accumulator ring slot and phase)
    const int b = c % NACC;
    if (!mbar_wait(accf0 + 8u * (uint32_t)b, (c / NACC) & 1, args.flags)) {
      alive = false;
      break;
    }
    asm volatile("tcgen05.fence::after_thread_sync;");
    uint32_t r0[32], r1[32];
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * 128 + h * 64);
    IC_TMEM_LD32(taddr, r0);
    IC_TMEM_LD32(taddr + 32, r1);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      sum[j] = __fadd_rn(sum[j], __uint_as_float(r0[j]));
      sum[32 + j] = __fadd_rn(sum[32 + j], __uint_as_float(r1[j]));
    }
    if (CHUNKED) {
      asm volatile("tcgen05.fence::before_thread_sync;");
      __syncwarp();
      if (lane == 0) release(b);
    }
  }
  // Stage through shared memory (the pipeline stages are idle once the last
  // accumulator has landed), then walk rows with the lanes along the row:
  // C/D accesses become row-contiguous, the C loads of several rows in flight.
  float* stage = reinterpret_cast<float*>(smem) + q * (32 * EPI_LD);
  if (alive) {
#pragma unroll
    for (int j4 = 0; j4 < 16; ++j4)
      *reinterpret_cast<float4*>(stage + lane * EPI_LD + h * 64 + j4 * 4) =
          make_float4(sum[j4 * 4], sum[j4 * 4 + 1], sum[j4 * 4 + 2], sum[j4 * 4 + 3]);
  }
  // both warps of the quarter (64 threads) meet on named barrier 1 + q
  asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
  if (alive) epilogue_rows<128, 16>(args, stage + h * 16 * EPI_LD, m0 + q * 32 + h * 16, n0, lane);
}

template <int BN, int PASSES>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * (PASSES == 3 ? 2 : 1);
  static constexpr int STAGES = 196608 / STAGE_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  // 3xTF32: K is accumulated in chunks of `chunk` k-tiles (default 4) into a ring of
  // TMEM accumulators; the epilogue adds the chunks in fp32 registers with
  // round-to-nearest.  The tensor core's own fp32 accumulation truncates, and
  // over a long K its bias adds up; chunking bounds that to chunk*32 terms.
  static constexpr bool CHUNKED = PASSES == 3;
  static constexpr int NACC = CHUNKED ? 4 : 1;  // ring of accumulators: the epilogue may lag NACC-1 chunks
  static constexpr int TMEM_COLS = NACC * BN;
  static_assert(4 * 32 * EPI_LD * 4 <= STAGES * STAGE_BYTES, "epilogue staging fits in the stages");
};

template <int BN, int PASSES>
__global__ void __launch_bounds__(384, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA_hi, const __grid_constant__ CUtensorMap tmA_lo,
                   const __grid_constant__ CUtensorMap tmB_hi, const __grid_constant__ CUtensorMap tmB_lo,
                   const GemmArgs args) {
  using C = Cfg<BN, PASSES>;
  constexpr int STAGES = C::STAGES;
  const int CH = C::CHUNKED ? args.chunk : (1 << 30);
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  // bars: full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], then the TMEM slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * C::NACC);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int mt = (args.m + BM - 1) / BM, nt = (args.n + BN - 1) / BN;
  const int ntiles = args.lower_rows > 0 ? args.lower_rows * (args.lower_rows + 1) / 2 : mt * nt;
  if (gridDim.x >= (unsigned)ntiles && (args.tri & 1) && args.lower_rows == 0 && !args.row_major) {
    // one tile per CTA and it is strictly upper: leave before any setup
    int tm, tn;
    tile_of(blockIdx.x, mt, nt, args.group, tm, tn);
    if (tn * BN > tm * BM) return;
  }

  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto accf_bar = [&](int b) { return smem_u32(bars + 2 * STAGES + b); };
  auto acce_bar = [&](int b) { return smem_u32(bars + 2 * STAGES + C::NACC + b); };
  auto a_hi = [&](int s) { return smem_u32(smem + s * C::STAGE_BYTES); };
  auto b_hi = [&](int s) { return smem_u32(smem + s * C::STAGE_BYTES + C::A_BYTES); };
  auto a_lo = [&](int s) { return smem_u32(smem + s * C::STAGE_BYTES + C::A_BYTES + C::B_BYTES); };
  auto b_lo = [&](int s) { return smem_u32(smem + s * C::STAGE_BYTES + 2 * C::A_BYTES + C::B_BYTES); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < C::NACC; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), 8);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;

  // Persistent over tiles: CTA b takes tiles b, b + grid, ...  The CTAs of a
  // wave start their tiles together and run at the same rate, so the A/B
  // panels a wave shares are re-read from L2 rather than DRAM.  Pipeline
  // stages and accumulators continue across tiles (global counters kt_g, ch_g).
  int kt_g = 0, ch_g = 0;
  bool ok = true;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    int tm, tn;
    if (args.lower_rows > 0) {
      // lower-triangle enumeration, row by row: rows near the top first, which
      // for a triangular A (tri bit 1) are the tiles with the longest K
      int r = (int)((sqrtf(8.f * (float)tile + 1.f) - 1.f) * 0.5f);
      while ((r + 1) * (r + 2) / 2 <= tile) ++r;
      while (r * (r + 1) / 2 > tile) --r;
      tm = r;
      tn = tile - r * (r + 1) / 2;
    } else if (args.row_major) {
      tm = tile / nt;
      tn = tile - tm * nt;
    } else {
      tile_of(tile, mt, nt, args.group, tm, tn);
    }
    const int m0 = tm * BM;
    const int n0 = tn * BN;
    if ((args.tri & 1) && n0 > m0) continue;  // strictly-upper tile of a symmetric/lower result
    const int kbase = (args.tri & 2) ? min(max(m0 - args.kofs, 0), args.k) : 0;
    const int ktiles = (args.k - kbase + BK - 1) / BK;
    const int nchunks = C::CHUNKED ? (ktiles + CH - 1) / CH : (ktiles > 0 ? 1 : 0);
    // a tile with nothing to add to D in place (a later K-slab of a triangular
    // product below its rows) keeps D as it is: no epilogue read/write
    if (ktiles == 0 && args.accum_in_place) continue;

    if (warp >= 4 && args.beta != 0.f && args.c_hi) {
      // warm L2 with this tile's C rows while the main loop runs
      const int row = m0 + (warp & 3) * 32 + lane;
      if (row < args.m) {
        for (int q = 2 * ((warp - 4) >> 2); q < 2 * ((warp - 4) >> 2) + 2; ++q) {
          const int col = n0 + q * 32;
          if (col >= args.n) break;
          prefetch_l2(args.c_hi + (long long)row * args.ldc + col);
          if (args.c_lo) prefetch_l2(args.c_lo + (long long)row * args.ldc + col);
        }
      }
    }
    if (warp == 0 && lane == 0 && ok) {
      // ---------------- TMA producer ----------------
      for (int kt = 0; kt < ktiles; ++kt) {
        const int g = kt_g + kt;
        const int s = g % STAGES;
        const uint32_t ph = (g / STAGES) & 1;
        bool ok_e = true;
        {
          IC_PROF_T0();
          if (g >= STAGES) ok_e = mbar_wait(empty_bar(s), ph ^ 1, args.flags);
          IC_PROF_ADD(2);
        }
        if (!ok_e) {
          ok = false;
          break;
        }
        mbar_expect_tx(full_bar(s), C::STAGE_BYTES);
        const int kx = kbase + kt * BK;
        tma_load_2d(a_hi(s), &tmA_hi, kx, m0, full_bar(s));
        tma_load_2d(b_hi(s), &tmB_hi, kx, n0, full_bar(s));
        if (PASSES == 3) {
          tma_load_2d(a_lo(s), &tmA_lo, kx, m0, full_bar(s));
          tma_load_2d(b_lo(s), &tmB_lo, kx, n0, full_bar(s));
        }
      }
    } else if (warp == 1 && lane == 0 && ok) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                 ((uint32_t)(BM >> 4) << 24);
#ifdef IC_GEMM_PROFILE
      const long long loop_t0 = clock64();
#endif
      for (int kt = 0; kt < ktiles && ok; ++kt) {
        const int chunk = ch_g + (C::CHUNKED ? kt / CH : 0);
        const int b = chunk % C::NACC;
        const bool first_in_chunk = C::CHUNKED ? (kt % CH == 0) : (kt == 0);
        {
          IC_PROF_T0();
          if (C::CHUNKED && first_in_chunk && chunk >= C::NACC &&
              !mbar_wait(acce_bar(b), ((chunk / C::NACC) & 1) ^ 1, args.flags))
            ok = false;
          IC_PROF_ADD(1);
        }
        if (!ok) break;
        const int g = kt_g + kt;
        const int s = g % STAGES;
        const uint32_t ph = (g / STAGES) & 1;
        {
          IC_PROF_T0();
          if (!mbar_wait(full_bar(s), ph, args.flags)) ok = false;
          IC_PROF_ADD(0);
        }
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t acc = tmem + (uint32_t)(b * BN);
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along K inside the swizzle row
          const uint64_t ah = sdesc(a_hi(s) + off), bh = sdesc(b_hi(s) + off);
          mma_tf32(acc, ah, bh, idesc, (first_in_chunk && kk == 0) ? 0u : 1u);
          if (PASSES == 3) {
            const uint64_t al = sdesc(a_lo(s) + off), bl = sdesc(b_lo(s) + off);
            mma_tf32(acc, ah, bl, idesc, 1u);
            mma_tf32(acc, al, bh, idesc, 1u);
          }
        }
        mma_commit(empty_bar(s));
        const bool last_in_chunk =
            C::CHUNKED ? (kt % CH == CH - 1 || kt == ktiles - 1) : (kt == ktiles - 1);
        if (last_in_chunk) mma_commit(accf_bar(b));
      }
#ifdef IC_GEMM_PROFILE
      atomicAdd(&g_gemm_prof[3], (unsigned long long)(clock64() - loop_t0));
      atomicAdd(&g_gemm_prof[5], 1ull);
#endif
    } else if (warp >= 4) {
      // ---------------- epilogue ----------------
      epilogue_warp<C::NACC, C::CHUNKED>(args, tmem, smem, warp, lane, nchunks, ch_g, m0, n0, accf_bar(0),
                                         [&](int b) {
                                           asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                                                            acce_bar(b))
                                                        : "memory");
                                         });
    }
    kt_g += ktiles;
    ch_g += nchunks;
    // the epilogue staged through the pipeline's shared memory: the next
    // tile's loads may only start once it is done
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
  }
  if (warp == 2) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2): a cluster of two CTAs on two SMs
// computes a 256 x 128 tile with one M=256 MMA stream issued by the leader
// (cluster rank 0).  Each CTA stages its own 128 rows of A and its own 64 rows
// of B (no multicast: every TMA load writes the issuing CTA's shared memory),
// so per SM the operand bytes per MMA drop by a quarter and four stages fit.
// Protocol:
//   full[s]   leader only; the leader arrives with expect_tx of both CTAs'
//             bytes, both CTAs' TMA loads complete_tx on it
//   empty[s]  in each CTA; the MMA commit arrives on both (multicast mask 3)
//   accf[b]   in each CTA; the MMA commit arrives on both
//   acce[b]   leader only, 16 arrivals (8 epilogue warps x 2 CTAs)
// Each CTA's epilogue reads its own TMEM (its 128 rows).  All waits are
// bounded; both CTAs always reach the closing cluster barrier.
struct PairCfg {
  static constexpr int A_BYTES = BM * BK * 4;       // 128 rows of A per CTA
  static constexpr int B_BYTES = 64 * BK * 4;       // 64 rows of B per CTA
  static constexpr int STAGE_BYTES = 2 * (A_BYTES + B_BYTES);
  static constexpr int STAGES = 196608 / STAGE_BYTES;  // 4
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  // k-tiles per accumulator chunk, as the single-CTA kernel's default (measured
  // on B200: triangular 16384 product 174.5 TF/s with 4, 171.7 with 2)
  static constexpr int CHUNK = 4;
  static constexpr int NACC = 4;           // ring of four 128-column accumulators
  static constexpr int TMEM_COLS = NACC * 128;
  static_assert(4 * 32 * EPI_LD * 4 <= STAGES * STAGE_BYTES, "epilogue staging fits in the stages");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory, completing on the leader's barrier
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* tm, int x, int y,
                                                 uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(leader_bar)
      : "memory");
}
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  const uint16_t mask = 3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

__global__ void __launch_bounds__(384, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA_hi, const __grid_constant__ CUtensorMap tmA_lo,
                     const __grid_constant__ CUtensorMap tmB_hi, const __grid_constant__ CUtensorMap tmB_lo,
                     const GemmArgs args) {
  using C = PairCfg;
  constexpr int STAGES = C::STAGES;
  constexpr int CH = C::CHUNK;
  constexpr int BN = 128;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * C::NACC);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  int pm, pn;
  tile_of(blockIdx.x >> 1, (args.m + 255) / 256, (args.n + BN - 1) / BN, PAIR_GROUP_M, pm, pn);
  const int mp = pm * 256;  // first row of the pair's tile
  const int m0 = mp + (int)rank * BM;
  const int n0 = pn * BN;
  // pair-uniform decisions (both CTAs run the same K loop)
  if ((args.tri & 1) && n0 > mp + BM) return;  // both halves strictly upper
  const int kbase = (args.tri & 2) ? min(max(mp - args.kofs, 0), args.k) : 0;
  const int ktiles = (args.k - kbase + BK - 1) / BK;
  const int nchunks = (ktiles + CH - 1) / CH;
  if (ktiles == 0 && args.accum_in_place) return;  // pair-uniform: D keeps its value

  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto accf_bar = [&](int b) { return smem_u32(bars + 2 * STAGES + b); };
  auto acce_bar = [&](int b) { return smem_u32(bars + 2 * STAGES + C::NACC + b); };
  auto a_hi = [&](int s) { return smem_u32(smem + s * C::STAGE_BYTES); };
  auto b_hi = [&](int s) { return smem_u32(smem + s * C::STAGE_BYTES + C::A_BYTES); };
  auto a_lo = [&](int s) { return smem_u32(smem + s * C::STAGE_BYTES + C::A_BYTES + C::B_BYTES); };
  auto b_lo = [&](int s) { return smem_u32(smem + s * C::STAGE_BYTES + 2 * C::A_BYTES + C::B_BYTES); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < C::NACC; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), 16);  // leader's copy is the one used: 8 epilogue warps x 2 CTAs
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  if (warp >= 4 && args.beta != 0.f && args.c_hi) {
    const int row = m0 + (warp & 3) * 32 + lane;
    if (row < args.m) {
      for (int q = 2 * ((warp - 4) >> 2); q < 2 * ((warp - 4) >> 2) + 2; ++q) {
        const int col = n0 + q * 32;
        if (col >= args.n) break;
        prefetch_l2(args.c_hi + (long long)row * args.ldc + col);
        if (args.c_lo) prefetch_l2(args.c_lo + (long long)row * args.ldc + col);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    for (int kt = 0; kt < ktiles; ++kt) {
      const int s = kt % STAGES;
      const uint32_t ph = (kt / STAGES) & 1;
      if (kt >= STAGES && !mbar_wait(empty_bar(s), ph ^ 1, args.flags)) break;
      if (leader) mbar_expect_tx(full_bar(s), 2 * C::STAGE_BYTES);
      const uint32_t fb = map_to_rank(full_bar(s), 0);
      const int kx = kbase + kt * BK;
      const int nb = n0 + (int)rank * 64;
      tma_load_2d_pair(a_hi(s), &tmA_hi, kx, m0, fb);
      tma_load_2d_pair(b_hi(s), &tmB_hi, kx, nb, fb);
      tma_load_2d_pair(a_lo(s), &tmA_lo, kx, m0, fb);
      tma_load_2d_pair(b_lo(s), &tmB_lo, kx, nb, fb);
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ---------------- MMA issuer (leader only) ----------------
    constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                               ((uint32_t)(256 >> 4) << 24);
    for (int kt = 0; kt < ktiles; ++kt) {
      const int chunk = kt / CH;
      const int b = chunk % C::NACC;
      const bool first_in_chunk = kt % CH == 0;
      if (first_in_chunk && chunk >= C::NACC && !mbar_wait(acce_bar(b), ((chunk / C::NACC) & 1) ^ 1, args.flags))
        break;
      const int s = kt % STAGES;
      const uint32_t ph = (kt / STAGES) & 1;
      if (!mbar_wait(full_bar(s), ph, args.flags)) break;
      asm volatile("tcgen05.fence::after_thread_sync;");
      const uint32_t acc = tmem + (uint32_t)(b * BN);
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint32_t off = kk * 32;
        const uint64_t ah = sdesc(a_hi(s) + off), bh = sdesc(b_hi(s) + off);
        const uint64_t al = sdesc(a_lo(s) + off), bl = sdesc(b_lo(s) + off);
        mma_tf32_pair(acc, ah, bh, idesc, (first_in_chunk && kk == 0) ? 0u : 1u);
        mma_tf32_pair(acc, ah, bl, idesc, 1u);
        mma_tf32_pair(acc, al, bh, idesc, 1u);
      }
      mma_commit_pair(empty_bar(s));
      if (kt % CH == CH - 1 || kt == ktiles - 1) mma_commit_pair(accf_bar(b));
    }
  } else if (warp >= 4) {
    // ---------------- epilogue (both CTAs, own rows) ----------------
    epilogue_warp<C::NACC, true>(args, tmem, smem, warp, lane, nchunks, 0, m0, n0, accf_bar(0), [&](int b) {
      remote_arrive(map_to_rank(acce_bar(b), 0));
    });
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers or read its operands
  if (warp == 2) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  // looked up once, thread-safely (layers may be issued from several host threads)
  static const EncodeTiledFn fn = [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return EncodeTiledFn(nullptr);
  }();
  return fn;
}

int make_map(CUtensorMap* tm, const float* base, int64_t rows, int64_t k, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(IC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(IC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%lld k=%lld ld=%lld", (int)r,
                (long long)rows, (long long)k, (long long)ld);
  return IC_OK;
}

// dynamic shared memory opt-in, once per device (function attributes are per device)
template <int BN, int PASSES>
int prepare() {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  IC_CUDA(cudaGetDevice(&dev));
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load() & bit) return IC_OK;
  IC_CUDA(cudaFuncSetAttribute(gemm_tn_kernel<BN, PASSES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Cfg<BN, PASSES>::SMEM));
  done.fetch_or(bit);
  return IC_OK;
}

// CTAs of a GEMM launch.  Default: one per tile.  IC_GEMM_CTAS=c makes the
// kernel persistent with at most c CTAs.  Measured on B200 inside the
// multi-stream layer pipeline, persistence lost 3-6%: resident CTAs hold SMs the
// other streams' latency-bound kernels need, and the DRAM traffic of a 16384^3
// product did not drop (167 GB either way).
int persistent_ctas(int* out) {
  static const int cap = [] {
    const char* e = getenv("IC_GEMM_CTAS");
    return (e && atoi(e) > 0) ? atoi(e) : INT32_MAX;
  }();
  *out = cap;
  return IC_OK;
}

template <int BN, int PASSES>
int launch(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh, const CUtensorMap& bl,
           const GemmArgs& a, cudaStream_t st) {
  using C = Cfg<BN, PASSES>;
  IC_TRY((prepare<BN, PASSES>()));
  const int64_t tiles = a.lower_rows > 0 ? (int64_t)a.lower_rows * (a.lower_rows + 1) / 2
                                         : cdiv(a.n, BN) * cdiv(a.m, BM);
  if (tiles > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "gemm: too many tiles");
  if (tiles == 0) return IC_OK;
  int ctas = 0;
  IC_TRY(persistent_ctas(&ctas));
  gemm_tn_kernel<BN, PASSES><<<(unsigned)std::min<int64_t>(tiles, ctas), 384, C::SMEM, st>>>(ah, al, bh, bl, a);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

int prepare_pair() {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  IC_CUDA(cudaGetDevice(&dev));
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load() & bit) return IC_OK;
  IC_CUDA(cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg::SMEM));
  done.fetch_or(bit);
  return IC_OK;
}

int launch_pair(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh, const CUtensorMap& bl,
                const GemmArgs& a, cudaStream_t st) {
  IC_TRY(prepare_pair());
  cudaLaunchConfig_t cfg{};
  const int64_t ctas = 2 * cdiv(a.n, 128) * cdiv(a.m, 256);
  if (ctas > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "gemm: too many tiles");
  cfg.gridDim = dim3((unsigned)ctas, 1, 1);
  cfg.blockDim = dim3(384, 1, 1);
  cfg.dynamicSmemBytes = PairCfg::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;  // the CTA pair lies along the cluster's x
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  IC_CUDA(cudaLaunchKernelEx(&cfg, gemm_pair_kernel, ah, al, bh, bl, a));
  IC_CHECK_LAUNCH();
  return IC_OK;
}

// CTA pairs for every 3xTF32 product with more than one 128-row tile, opt-in
// with IC_GEMM_PAIR=1: measured on B200 they lose on the many small products of
// the inverse's recursion.
bool pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("IC_GEMM_PAIR");
    return e && e[0] == '1';
  }();
  return on;
}
// CTA pairs for 3xTF32 products of at least this many output elements (m * n;
// IC_GEMM_PAIR_MIN overrides, 0 = never).  Measured on B200: the triangular
// 16384 product runs 166 vs 161 TF/s on pairs, and the benchmark gains ~0.8%
// with pairs from 8192 x 8192 up (3694-3699 vs 3658-3673 Mparams/s).
int64_t pair_min_elems() {
  static const int64_t v = [] {
    const char* e = getenv("IC_GEMM_PAIR_MIN");
    if (!e) return (int64_t)1 << 26;
    return atoll(e) > 0 ? (int64_t)atoll(e) : INT64_MAX;
  }();
  return v;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int gemm_prepare() {
  IC_TRY((prepare<128, 3>()));
  IC_TRY((prepare<128, 1>()));
  IC_TRY(prepare_pair());
  return device_flags() ? IC_OK : fail(IC_ERR_CUDA, "device status word unavailable");
}

namespace {
// Tile-order group height and accumulator chunk length (IC_GEMM_GROUP,
// IC_GEMM_CHUNK override the defaults for tuning).  Measured on B200: chunks of
// 4 k-tiles (128 K) were 2-4% faster in the bench than 2 and keep the inverse
// within 8x LAPACK's error; 8 exceeded that bound.  Group heights 8 and 16
// tie; 32 is slower at 16384^3.
int tune_group() {
  static const int v = [] {
    const char* e = getenv("IC_GEMM_GROUP");
    return (e && atoi(e) > 0) ? atoi(e) : GROUP_M;
  }();
  return v;
}
int tune_chunk() {
  static const int v = [] {
    const char* e = getenv("IC_GEMM_CHUNK");
    return (e && atoi(e) > 0) ? atoi(e) : 4;
  }();
  return v;
}

// Tile orders for triangular products, opt-in with IC_GEMM_TRI_ORDER=1: only
// the lower tiles, row by row, longest K first.  Measured on B200 it balances
// the 4096 triangular product better (129 vs 119 TF/s) but loses the grouped
// order's L2 reuse at 16384 (154 vs 161 TF/s) and 2% of the benchmark, so the
// grouped order over all tiles stays the default.
bool tile_order_on() {
  static const bool on = [] {
    const char* e = getenv("IC_GEMM_TRI_ORDER");
    return e && e[0] == '1';
  }();
  return on;
}

int gemm_once(int64_t m, int64_t n, int64_t k, float alpha, const float* a_hi, const float* a_lo,
              int64_t lda, const float* b_hi, const float* b_lo, int64_t ldb, float beta,
              const float* c_hi, const float* c_lo, int64_t ldc, float* d_hi, float* d_lo,
              int64_t ldd, int passes, cudaStream_t st, int tri, int kofs) {
  if (m <= 0 || n <= 0) return IC_OK;
  if (passes != 1 && passes != 3) return fail(IC_ERR_INVALID, "gemm: passes must be 1 or 3");
  if (passes == 3 && (!a_lo || !b_lo)) return fail(IC_ERR_INVALID, "gemm: 3xTF32 needs lo parts");
  if (!a_hi || !b_hi || !d_hi) return fail(IC_ERR_INVALID, "gemm: null operand");
  if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return fail(IC_ERR_UNSUPPORTED, "gemm: size");
  if ((lda | ldb) & 3) return fail(IC_ERR_INVALID, "gemm: A/B leading dimensions must be multiples of 4");
  if (!aligned16(a_hi) || !aligned16(b_hi) || (passes == 3 && (!aligned16(a_lo) || !aligned16(b_lo))))
    return fail(IC_ERR_INVALID, "gemm: A/B operands must be 16-byte aligned");
  const bool vec = !((ldc | ldd) & 3) && aligned16(d_hi) && (!c_hi || aligned16(c_hi)) &&
                   (!c_lo || aligned16(c_lo)) && (!d_lo || aligned16(d_lo));
  unsigned* flags = device_flags();
  if (!flags) return fail(IC_ERR_CUDA, "device status word unavailable");
  const int in_place = beta == 1.f && c_hi == d_hi && c_lo == d_lo && ldc == ldd;
  const int64_t mt = cdiv(m, BM);
  int lower_rows = 0;
  if ((tri & 1) && m == n && tile_order_on()) {
    lower_rows = (int)mt;
    // accumulating a K-slab of a triangular A in place: tile rows starting at
    // or below the slab's end get nothing from it and are not launched
    if ((tri & 2) && in_place) lower_rows = (int)std::min<int64_t>(mt, cdiv(kofs + (k > 0 ? k : 0), BM));
  }
  const int row_major = (tri & 2) && lower_rows == 0 && tile_order_on();
  GemmArgs a{(int)m, (int)n, (int)(k > 0 ? k : 0), alpha, beta, c_hi, c_lo, (long long)ldc,
             d_hi, d_lo, (long long)ldd, flags, vec ? 1 : 0, tune_group(), tune_chunk(), kofs, in_place,
             lower_rows, row_major, tri};
  const int64_t kk = k > 0 ? k : 1;
  CUtensorMap ah, al, bh, bl;
  if (passes == 3 && m > BM && (pair_enabled() || m * n >= pair_min_elems())) {
    IC_TRY(make_map(&ah, a_hi, m, kk, lda, BM));
    IC_TRY(make_map(&bh, b_hi, n, kk, ldb, 64));
    IC_TRY(make_map(&al, a_lo, m, kk, lda, BM));
    IC_TRY(make_map(&bl, b_lo, n, kk, ldb, 64));
    return launch_pair(ah, al, bh, bl, a, st);
  }
  if (passes == 3) {
    IC_TRY(make_map(&ah, a_hi, m, kk, lda, BM));
    IC_TRY(make_map(&bh, b_hi, n, kk, ldb, 128));
    IC_TRY(make_map(&al, a_lo, m, kk, lda, BM));
    IC_TRY(make_map(&bl, b_lo, n, kk, ldb, 128));
    return launch<128, 3>(ah, al, bh, bl, a, st);
  }
  IC_TRY(make_map(&ah, a_hi, m, kk, lda, BM));
  IC_TRY(make_map(&bh, b_hi, n, kk, ldb, 128));
  return launch<128, 1>(ah, ah, bh, bh, a, st);
}

// K per launch for large products.  A 128-row operand panel of a long-K
// product (128 x K x 8 bytes as a hi/lo pair: 16.8 MB at K = 16384) is too
// large for the CTAs sharing it to find it in L2, so a 16384^3 product read
// 167 GB from DRAM (38x its operands) on B200.  Split into K-slabs of this
// width, each accumulating into D (the running sum is exact fp32, the same one
// rounding per slab as the kernel's chunk sums).
// IC_GEMM_SLAB=0 turns the split off.  Measured on B200 with fp32 running
// sums between slabs: slabs of 8192 run the isolated triangular 16384 product
// 1% faster (173.3 vs 171.7 TF/s) and unsplit 8192 products 10% faster, but
// the benchmark, with four streams sharing L2, 0.5% slower (3685 vs 3704);
// 2048 is slower everywhere (160.2 TF/s at 16384).
int slab_k() {
  static const int v = [] {
    const char* e = getenv("IC_GEMM_SLAB");
    return e ? atoi(e) : 4096;
  }();
  return v;
}
}  // namespace

int gemm_tn(int64_t m, int64_t n, int64_t k, float alpha, const float* a_hi, const float* a_lo,
            int64_t lda, const float* b_hi, const float* b_lo, int64_t ldb, float beta,
            const float* c_hi, const float* c_lo, int64_t ldc, float* d_hi, float* d_lo,
            int64_t ldd, int passes, cudaStream_t st, int tri) {
  const int64_t sk = slab_k();
  if (passes != 3 || sk <= 0 || sk % BK || k < 2 * sk || m * n < (int64_t(1) << 26))
    return gemm_once(m, n, k, alpha, a_hi, a_lo, lda, b_hi, b_lo, ldb, beta, c_hi, c_lo, ldc, d_hi, d_lo, ldd,
                     passes, st, tri, 0);
  // Between slabs the running sum is held as plain fp32 in D's hi part (the
  // exact value a hi/lo pair would hold, half the bytes to read and write);
  // the last slab reads it and writes D as the pair.
  for (int64_t k0 = 0; k0 < k; k0 += sk) {
    const int64_t kw = std::min(sk, k - k0);
    const bool first = k0 == 0, last = k0 + kw >= k;
    IC_TRY(gemm_once(m, n, kw, alpha, a_hi + k0, a_lo + k0, lda, b_hi + k0, b_lo + k0, ldb, first ? beta : 1.f,
                     first ? c_hi : d_hi, first ? c_lo : nullptr, first ? ldc : ldd, d_hi, last ? d_lo : nullptr,
                     ldd, passes, st, tri, (int)k0));
  }
  return IC_OK;
}

}  // namespace ic

extern "C" int ic_gemm_tn(int64_t m, int64_t n, int64_t k, float alpha, const float* a_hi,
                          const float* a_lo, int64_t lda, const float* b_hi, const float* b_lo,
                          int64_t ldb, float beta, const float* c_hi, const float* c_lo, int64_t ldc,
                          float* d_hi, float* d_lo, int64_t ldd, int passes, void* stream) {
  return ic::gemm_tn(m, n, k, alpha, a_hi, a_lo, lda, b_hi, b_lo, ldb, beta, c_hi, c_lo, ldc, d_hi, d_lo,
                     ldd, passes, static_cast<cudaStream_t>(stream));
}

namespace ic {
namespace {
// One thread waits on an mbarrier that nothing arrives on: the library's
// bounded wait must give up after limit_ns, record DEV_TIMEOUT and return.
__global__ void wait_selftest_kernel(unsigned* flags, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  mbar_init(b, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  mbar_wait_bounded(b, 0, flags, limit_ns);
}
}  // namespace
}  // namespace ic

extern "C" int ic_selftest_bounded_wait(unsigned long long limit_ns, void* stream) {
  if (limit_ns < 100000ull || limit_ns > 2000000000ull)
    return ic::fail(IC_ERR_INVALID, "selftest wait limit must be in [0.1 ms, 2 s]");
  unsigned* flags = ic::device_flags();
  if (!flags) return ic::fail(IC_ERR_CUDA, "device status word unavailable");
  ic::wait_selftest_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(flags, limit_ns);
  IC_CHECK_LAUNCH();
  return IC_OK;
}

extern "C" int ic_gemm_tn_tri(int64_t m, int64_t n, int64_t k, float alpha, const float* a_hi,
                              const float* a_lo, int64_t lda, const float* b_hi, const float* b_lo,
                              int64_t ldb, float beta, const float* c_hi, const float* c_lo, int64_t ldc,
                              float* d_hi, float* d_lo, int64_t ldd, int tri, void* stream) {
  if (tri < 0 || tri > 3) return ic::fail(IC_ERR_INVALID, "gemm: tri must be in [0,3]");
  return ic::gemm_tn(m, n, k, alpha, a_hi, a_lo, lda, b_hi, b_lo, ldb, beta, c_hi, c_lo, ldc, d_hi, d_lo,
                     ldd, 3, static_cast<cudaStream_t>(stream), tri);
}
