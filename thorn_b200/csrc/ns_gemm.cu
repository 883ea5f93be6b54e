// Newton-Schulz GEMMs on the 5th-generation tensor cores (sm_100a).
//
// One persistent kernel serves every product of the NS iteration:
//   D = alpha * A @ op(B) + beta * C          (fp32 accumulate in TMEM)
//   D2 = D + diag2 * I                         (optional second output)
// A is K-major ([M, K] row-major) or MN-major ([K, M], the Gram product of a
// tall input kept in its original orientation).  B is either K-major ([N, K],
// used for X X^T) or MN-major ([K, N], used for every other product).  With
// `sym` the output is known to be symmetric up to rounding, and only tiles that
// touch the lower triangle are computed.  The output is split into 128 x 128
// blocks: a block on the diagonal is stored exactly as computed, a block below
// it is stored and mirrored into the block above, so off-diagonal blocks are
// exactly symmetric.  (The reference's Triton kernel, thorn.py:53-139, does the
// same with its autotuned BLOCK_SIZE_M: diagonal tiles as computed, the other
// triangle mirrored.  For a matrix of at most 128 rows the output is the plain
// product.)  With `trans_out`, D is stored transposed (the tall-matrix final
// product).
//
// Roles per CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: fills a ring of shared-memory stages
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (128 x BN x 16)
//   warps 2..5  epilogue: tcgen05.ld -> alpha/beta/diag -> global stores
// Two TMEM accumulators (2 x BN columns) let the epilogue of one tile overlap
// the MMAs of the next.  Every mbarrier wait is bounded by a wall-clock limit;
// a timeout sets *err, raises a CTA-wide abort flag and lets all roles exit
// through the normal teardown (TMEM is always freed).
#include <cuda.h>
#include <math.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <vector>

#include "common.cuh"

namespace thorn {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 16-bit = one 128-byte swizzle row
constexpr int kThreadsG = 192;
// Default limit of every mbarrier wait (thorn_set_wait_limit_ns changes it).
constexpr uint64_t kTimeoutNs = 10ull * 1000 * 1000 * 1000;

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmem = kStages * kStageBytes + kBarBytes + 1024;
};

struct Params {
  CUtensorMap tmA;
  CUtensorMap tmB;
  // staged epilogue (2-CTA kernel, `tma_epi`): 32 x 32 blocks, 64-byte swizzle
  CUtensorMap tmC;   // C operand, [batch or 1][M][N]
  CUtensorMap tmD;   // D, [batch][M][N], or [batch][N][M] with trans_out
  CUtensorMap tmD2;  // D2, [batch][M][N]
  const void* C;
  void* D;
  void* D2;
  int64_t c_bs, c_ld, d_bs, d_ld, d2_bs, d2_ld;
  int M, N, K, batch;
  float alpha, beta, diag2;
  int sym, trans_out, c_vec, d_vec, tma_epi, c_bcast, l2hint;
  int tiles_m, tiles_n, tiles_per_mat, total_tiles, num_kb;
  int col_major;  // 2-CTA kernel, full tiles: tile index runs down the columns (tm fastest)
  int* err;
  uint64_t wait_limit_ns;  // limit of every mbarrier wait before the CTA gives up
  int test_stall;          // failure test: producers issue no loads, so the MMA warp's wait runs out
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Abort path only: TMA loads and MMAs that this CTA issued before its roles gave
// up may still be in flight.  They complete within microseconds, so every thread
// lets 1 ms of global time pass before the CTA's final synchronisation, TMEM
// release and exit.
constexpr uint64_t kSettleNs = 1000ull * 1000;
__device__ __forceinline__ void abort_settle(volatile int* abort) {
  if (!*abort) return;
  const uint64_t t0 = global_ns();
  while (global_ns() - t0 < kSettleNs) {
  }
}
// Bounded wait on the phase with parity `parity`.  Returns false after `limit_ns`
// or when another role of this CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* err,
                                          uint64_t limit_ns) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (abort && *abort) return false;
      if (global_ns() - t0 > limit_ns) {
        if (err) atomicExch(err, 1);
        if (abort) *abort = 1;
        return false;
      }
    }
  }
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tm, uint32_t bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// TMA bulk store of a shared-memory block (bulk async-group of the issuing thread).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tm, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// all but the newest N bulk groups of this thread have finished reading shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Programmatic dependent launch: let the next grid on the stream be scheduled
// now (its CTAs take SMs as this grid's CTAs exit), and wait until the previous
// grid has completed and its memory is visible.  Without a programmatic launch
// both are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm100 layout: version 1).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: kind::f16, fp32 accumulate; A/B K-major (0) or MN-major (1).
__host__ __device__ constexpr uint32_t idesc_f16(int bn, bool bf16, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

template <int BN>
__device__ __forceinline__ void decode_tile(const Params& p, int t, int& b, int& tm, int& tn) {
  b = t / p.tiles_per_mat;
  int l = t - b * p.tiles_per_mat;
  if (!p.sym) {
    tm = l / p.tiles_n;
    tn = l - tm * p.tiles_n;
    return;
  }
  tm = 0;
  for (;;) {
    int cnt = min(p.tiles_n, (tm * BM + BM - 1) / BN + 1);
    if (l < cnt || tm + 1 >= p.tiles_m) {
      tn = l;
      return;
    }
    l -= cnt;
    ++tm;
  }
}

// Epilogue of one 32-column chunk of a thread's accumulator row: alpha/beta/C,
// one rounding, optional second output D + diag2 I, and plain, transposed or
// mirrored (symmetric) stores with bounds checks.  The 32 columns of a chunk and
// the 32 rows of a warp each lie in one 128-block; with `sym` the caller passes
// only chunks whose block is not right of the rows' block.
template <class T>
__device__ __forceinline__ void epilogue_chunk(const Params& p, float* v, int row, bool row_ok, int col0,
                                               T* D, T* D2, const T* Cb) {
  const bool full = row_ok && col0 + 32 <= p.N;
  if (Cb != nullptr) {
    float cv[32];
    if (full && p.c_vec) {
      load_n(Cb + (int64_t)row * p.c_ld + col0, cv, 8, true);
      load_n(Cb + (int64_t)row * p.c_ld + col0 + 8, cv + 8, 8, true);
      load_n(Cb + (int64_t)row * p.c_ld + col0 + 16, cv + 16, 8, true);
      load_n(Cb + (int64_t)row * p.c_ld + col0 + 24, cv + 24, 8, true);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        cv[j] = (row_ok && col0 + j < p.N) ? to_f(Cb[(int64_t)row * p.c_ld + col0 + j]) : 0.f;
    }
    // alpha acc and beta C each rounded, then their sum: the roundings of torch's
    // alpha / beta scaling, in a fixed order (no contraction into an fma)
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(__fmul_rn(p.alpha, v[j]), __fmul_rn(p.beta, cv[j]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(p.alpha, v[j]);
  }
  // round once to the output type
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = rnd<T>(v[j]);

  for (int out = 0; out < (D2 ? 2 : 1); ++out) {
    T* O = out == 0 ? D : D2;
    const int64_t ld = out == 0 ? p.d_ld : p.d2_ld;
    float w[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = (out == 1 && row == col0 + j) ? rnd<T>(v[j] + p.diag2) : v[j];
    if (p.trans_out) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row_ok && col0 + j < p.N) O[(int64_t)(col0 + j) * ld + row] = from_f<T>(w[j]);
      continue;
    }
    if (full && p.d_vec) {
      T* dst = O + (int64_t)row * ld + col0;
      store_n(dst, w, 8, true);
      store_n(dst + 8, w + 8, 8, true);
      store_n(dst + 16, w + 16, 8, true);
      store_n(dst + 24, w + 24, 8, true);
    } else if (row_ok) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) O[(int64_t)row * ld + col0 + j] = from_f<T>(w[j]);
    }
    if (p.sym && (col0 >> 7) < (row >> 7)) {
      // a chunk of an off-diagonal block: mirror it; lanes hold consecutive rows -> coalesced
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row_ok && col0 + j < p.N) O[(int64_t)(col0 + j) * ld + row] = from_f<T>(w[j]);
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int BN, bool A_MN, bool B_MN, class T>
__global__ void __launch_bounds__(kThreadsG, 1) ns_gemm_kernel(const __grid_constant__ Params p) {
  using C_ = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C_::kStages * C_::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + C_::kStages * C_::kBBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + C_::kStages;
  uint64_t* tfull = bars + 2 * C_::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C_::kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 4 * 32);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"((uint32_t)C_::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // set-up above overlaps the previous grid's tail; global memory only after it has finished
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0 && !p.test_stall) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < p.total_tiles && !*abort_flag; t += gridDim.x) {
        int b, tm, tn;
        decode_tile<BN>(p, t, b, tm, tn);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.err, p.wait_limit_ns)) break;
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_expect_tx(fb, C_::kStageBytes);
          if (!A_MN) {
            tma_load_3d(smem_u32(sA + stage * C_::kABytes), &p.tmA, fb, kb * BK, tm * BM, b);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_3d(smem_u32(sA + stage * C_::kABytes + c * (64 * BK * 2)), &p.tmA, fb, tm * BM + c * 64,
                          kb * BK, b);
          }
          if (!B_MN) {
            tma_load_3d(smem_u32(sB + stage * C_::kBBytes), &p.tmB, fb, kb * BK, tn * BN, b);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(smem_u32(sB + stage * C_::kBBytes + c * (64 * BK * 2)), &p.tmB, fb, tn * BN + c * 64,
                          kb * BK, b);
          }
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer -----------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BN, sizeof(T) == 2 && !std::is_same<T, __half>::value, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = blockIdx.x; t < p.total_tiles && !*abort_flag; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1u, abort_flag, p.err, p.wait_limit_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, p.err, p.wait_limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C_::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * C_::kBBytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc(a0 + kk * 2048, 64 * BK * 2, 1024) : sdesc(a0 + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc(b0 + kk * 2048, 64 * BK * 2, 1024) : sdesc(b0 + kk * 32, 16, 1024);
            umma(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&empty[stage]));
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&tfull[acc]));
      }
    }
  } else {
    // ------------------------------ epilogue -------------------------------
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int rloc = q * 32 + lane;
    const T* Cp = reinterpret_cast<const T*>(p.C);
    T* Dp = reinterpret_cast<T*>(p.D);
    T* D2p = reinterpret_cast<T*>(p.D2);
    int it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, p.err, p.wait_limit_ns)) break;
      tc_fence_after();
      int b, tm, tn;
      decode_tile<BN>(p, t, b, tm, tn);
      const int row = tm * BM + rloc;
      const bool row_ok = row < p.M;
      const int row_blk = (tm * BM + q * 32) >> 7;  // the 128-block of this warp's rows
      T* D = Dp + (int64_t)b * p.d_bs;
      T* D2 = D2p ? D2p + (int64_t)b * p.d2_bs : nullptr;
      const T* Cb = Cp ? Cp + (int64_t)b * p.c_bs : nullptr;
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        const int col0 = tn * BN + ch * 32;
        if (col0 >= p.N) break;
        if (p.sym && (col0 >> 7) > row_blk) continue;  // a block above the diagonal: the mirror writes it
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + ch * 32), v);
        epilogue_chunk(p, v, row, row_ok, col0, D, D2, Cb);
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&tempty[acc]));
    }
  }

  abort_settle(abort_flag);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"((uint32_t)C_::kTmemCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// 2-CTA variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2.  Each CTA loads its own 128 rows of A and its own
// 128 rows (columns of the tile) of B; the MMA of the leader CTA (cluster rank
// 0) reads both CTAs' shared memory and accumulates rows 0-127 in the leader's
// TMEM and rows 128-255 in the peer's.  Per SM this halves the B operand bytes
// that TMA moves for the same tensor-core work.
//   full[s]   leader only: both CTAs' TMA loads complete on it (leader expects
//             all 64 KB); the peer reaches it through its cluster address
//   empty[s]  both CTAs: the leader's MMA commits to each CTA's copy
//   tfull[a]  both CTAs: the leader commits to each CTA's copy
//   tempty[a] leader only: 256 arrivals, the peer's epilogue arrives remotely
// ---------------------------------------------------------------------------
constexpr int BM2 = 256;  // rows of a cluster tile (128 per CTA)
constexpr int kStages2 = 6;
constexpr int kHalfBytes = 128 * BK * 2;  // 16 KB: one CTA's A (or B) slab per stage
// Staged epilogue: per epilogue warp two buffer pairs, each a 32 x 32 block of
// the output (2 KB, also the landing place of the C block) and its transpose.
constexpr int kEpiBlock = 32 * 32 * 2;
constexpr int kEpiWarpBytes = 4 * kEpiBlock;
constexpr int kEpiBytes = 4 * kEpiWarpBytes;
constexpr int kSmem2 = kStages2 * 2 * kHalfBytes + kEpiBytes + 256 + 1024;
static_assert(kSmem2 <= 232448, "2-CTA kernel exceeds 227 KB of shared memory");

// Byte offset of element (r, c) in a 32 x 32 block of 16-bit values stored in
// the layout of a CU_TENSOR_MAP_SWIZZLE_64B box: 64-byte rows whose four
// 16-byte chunks are permuted by chunk ^= (r / 2) % 4.  Rows written this way
// (one row per lane) and columns (one element per lane) are both free of bank
// conflicts.
__device__ __forceinline__ uint32_t sw64_off(int r, int c) {
  return (uint32_t)(r * 64 + ((((c >> 3) ^ (r >> 1)) & 3) << 4) + ((c & 7) << 1));
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* tm, uint32_t bar_cluster, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// The same loads and stores with an L2 cache policy (2-CTA kernel, `l2hint`):
// operand tiles are re-read by other clusters and should stay (evict_last),
// output blocks are not re-read by this kernel (evict_first).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_load_3d_pair_hint(uint32_t dst, const CUtensorMap* tm, uint32_t bar_cluster, int x,
                                                      int y, int z, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.cta_group::2.L2::cache_hint "
      "[%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_store_3d_hint(const CUtensorMap* tm, uint32_t src, int x, int y, int z,
                                                  uint64_t pol) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4}], [%1], %5;" ::
                   "l"(reinterpret_cast<uint64_t>(tm)),
               "r"(src), "r"(x), "r"(y), "r"(z), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

__host__ __device__ constexpr uint32_t idesc_f16_m256(bool bf16, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(BM2 >> 4) << 24);
}

__device__ __forceinline__ void decode_tile2(const Params& p, int t, int& b, int& tm, int& tn) {
  b = t / p.tiles_per_mat;
  int l = t - b * p.tiles_per_mat;
  if (!p.sym) {
    if (p.col_major) {
      tn = l / p.tiles_m;
      tm = l - tn * p.tiles_m;
    } else {
      tm = l / p.tiles_n;
      tn = l - tm * p.tiles_n;
    }
    return;
  }
  tm = 0;
  for (;;) {
    const int cnt = min(p.tiles_n, tm + 1);  // square 256 x 256 tiles on or below the diagonal
    if (l < cnt || tm + 1 >= p.tiles_m) {
      tn = l;
      return;
    }
    l -= cnt;
    ++tm;
  }
}

// Number of 32-column blocks of tile t that the epilogue warp with rows
// [row_base, row_base + 32) of the tile stores (a prefix of the tile's 8).
__device__ __forceinline__ int warp_blocks(const Params& p, int t, int row_base, int& b, int& tm, int& tn) {
  decode_tile2(p, t, b, tm, tn);
  const int row0 = tm * BM2 + row_base;
  if (row0 >= p.M) return 0;
  int nv = min(8, (p.N - tn * 256 + 31) >> 5);
  if (p.sym) nv = min(nv, (((row0 | 127) - tn * 256) >> 5) + 1);  // blocks up to the end of the rows' 128-block
  return max(nv, 0);
}

// Position (t2, ch2) of the block after (t, ch) in the warp's processing order.
__device__ __forceinline__ bool next_block(const Params& p, int t, int ch, int nv, int step, int row_base, int& t2,
                                           int& ch2, int& b2, int& tm2, int& tn2) {
  if (ch + 1 < nv) {
    t2 = t;
    ch2 = ch + 1;
    decode_tile2(p, t, b2, tm2, tn2);
    return true;
  }
  for (t2 = t + step; t2 < p.total_tiles; t2 += step) {
    if (warp_blocks(p, t2, row_base, b2, tm2, tn2) > 0) {
      ch2 = 0;
      return true;
    }
  }
  return false;
}

template <bool A_MN, bool B_MN, class T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsG, 1)
    ns_gemm2_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages2 * kHalfBytes;
  uint8_t* sEpi = sB + kStages2 * kHalfBytes;  // 1024-byte aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + kEpiBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages2;
  uint64_t* tfull = bars + 2 * kStages2;
  uint64_t* tempty = tfull + 2;
  uint64_t* cbar = tempty + 2;  // [4 epilogue warps][2 buffers]: C block landed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(cbar + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 2 * 4 * 32);
    }
    for (int i = 0; i < 8; ++i) mbar_init(smem_u32(&cbar[i]), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs are initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // set-up above overlaps the previous grid's tail; global memory only after it has finished
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ------------------------------ producer (both CTAs) -------------------
    if (lane == 0 && !p.test_stall) {
      int stage = 0;
      uint32_t phase = 0;
      const int row_off = (int)rank * 128;
      const uint64_t pol_keep = l2_policy_evict_last();
      auto load = [&](uint32_t dst, const CUtensorMap* tm, uint32_t bar, int x, int y, int z) {
        if (p.l2hint) tma_load_3d_pair_hint(dst, tm, bar, x, y, z, pol_keep);
        else tma_load_3d_pair(dst, tm, bar, x, y, z);
      };
      for (int t = cid; t < p.total_tiles && !*abort_flag; t += nclusters) {
        int b, tm, tn;
        decode_tile2(p, t, b, tm, tn);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.err, p.wait_limit_ns)) break;
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_expect_tx(smem_u32(&full[stage]), 4 * kHalfBytes);
          const uint32_t a_dst = smem_u32(sA + stage * kHalfBytes);
          const uint32_t b_dst = smem_u32(sB + stage * kHalfBytes);
          if (!A_MN) {
            load(a_dst, &p.tmA, fb, kb * BK, tm * BM2 + row_off, b);
          } else {
            load(a_dst, &p.tmA, fb, tm * BM2 + row_off, kb * BK, b);
            load(a_dst + 64 * BK * 2, &p.tmA, fb, tm * BM2 + row_off + 64, kb * BK, b);
          }
          if (!B_MN) {
            load(b_dst, &p.tmB, fb, kb * BK, tn * 256 + row_off, b);
          } else {
            load(b_dst, &p.tmB, fb, tn * 256 + row_off, kb * BK, b);
            load(b_dst + 64 * BK * 2, &p.tmB, fb, tn * 256 + row_off + 64, kb * BK, b);
          }
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (leader) --------------------
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16_m256(sizeof(T) == 2 && !std::is_same<T, __half>::value, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = cid; t < p.total_tiles && !*abort_flag; t += nclusters, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1u, abort_flag, p.err, p.wait_limit_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 256);
        bool ok = true;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, p.err, p.wait_limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * kHalfBytes);
          const uint32_t b0 = smem_u32(sB + stage * kHalfBytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc(a0 + kk * 2048, 64 * BK * 2, 1024) : sdesc(a0 + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc(b0 + kk * 2048, 64 * BK * 2, 1024) : sdesc(b0 + kk * 32, 16, 1024);
            umma_pair(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 0));
          umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 0));
        umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
      }
    }
  } else if (p.tma_epi) {
    // ------------------------------ staged epilogue (both CTAs) ------------
    // Warp q stores rows [row0, row0 + 32) of each tile, 32 columns at a time:
    // TMEM -> registers -> alpha/beta/C, one rounding -> a swizzled 2 KB block
    // (and its transpose when the block is mirrored or the output transposed)
    // -> TMA bulk stores.  Blocks alternate between two buffer pairs; C blocks
    // are TMA-loaded one block ahead into the buffer the next block uses.
    const int q = warp & 3;
    const int row_base = (int)rank * 128 + q * 32;
    uint8_t* gE = sEpi + q * kEpiWarpBytes;
    const uint32_t sE = smem_u32(gE);
    const uint32_t cb0 = smem_u32(&cbar[2 * q]);
    const bool has_c = p.C != nullptr;
    const bool has_d2 = p.D2 != nullptr;
    const uint64_t pol_out = l2_policy_evict_first();
    auto store = [&](const CUtensorMap* tm, uint32_t src, int x, int y, int z) {
      if (p.l2hint) tma_store_3d_hint(tm, src, x, y, z, pol_out);
      else tma_store_3d(tm, src, x, y, z);
    };
    bool c_inflight = false;  // a C load was issued and not yet waited for
    int c_buf = 0;
    uint32_t c_par = 0;
    auto load_c = [&](int n_blk, int b2, int tm2, int tn2, int ch2) {
      const int k2 = n_blk & 1;
      if (lane == 0) {
        bulk_wait_read<1>();  // stores of block n_blk - 2 no longer read buffer k2
        mbar_expect_tx(cb0 + 8 * k2, kEpiBlock);
        tma_load_3d(sE + k2 * 2 * kEpiBlock, &p.tmC, cb0 + 8 * k2, tn2 * 256 + ch2 * 32, tm2 * BM2 + row_base,
                    p.c_bcast ? 0 : b2);
      }
      c_inflight = true;
      c_buf = k2;
      c_par = (uint32_t)(n_blk >> 1) & 1u;
    };
    if (has_c) {
      int b2, tm2, tn2;
      for (int t0 = cid; t0 < p.total_tiles; t0 += nclusters)
        if (warp_blocks(p, t0, row_base, b2, tm2, tn2) > 0) {
          load_c(0, b2, tm2, tn2, 0);
          break;
        }
    }
    int n = 0;  // blocks handled by this warp so far
    int it = 0;
    bool aborted = false;
    for (int t = cid; t < p.total_tiles && !aborted; t += nclusters, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
      // warp-uniform outcome: the .sync.aligned TMEM loads and __syncwarp below need all lanes
      if (!__all_sync(0xffffffffu,
                      mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, p.err, p.wait_limit_ns)))
        break;
      tc_fence_after();
      int b, tm, tn;
      const int nv = warp_blocks(p, t, row_base, b, tm, tn);
      const int row0 = tm * BM2 + row_base;
      if (nv == 0) {
        tc_fence_before();
        mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
        continue;
      }
#pragma unroll 1
      for (int ch = 0; ch < nv; ++ch, ++n) {
        const int col0 = tn * 256 + ch * 32;
        const int k = n & 1;
        uint8_t* gM = gE + k * 2 * kEpiBlock;
        uint8_t* gT = gM + kEpiBlock;
        const uint32_t sM = sE + k * 2 * kEpiBlock;
        const uint32_t sT = sM + kEpiBlock;
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 256 + ch * 32), v);
        if (ch == nv - 1) {  // accumulator fully read: hand it back to the MMA warp
          tc_fence_before();
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
        }
        if (has_c) {
          if (!__all_sync(0xffffffffu,
                          mbar_wait(cb0 + 8 * k, (uint32_t)(n >> 1) & 1u, abort_flag, p.err, p.wait_limit_ns))) {
            aborted = true;
            break;
          }
          c_inflight = false;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 r = *reinterpret_cast<const uint4*>(gM + sw64_off(lane, 8 * c));
            const T* h = reinterpret_cast<const T*>(&r);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              v[8 * c + i] = __fadd_rn(__fmul_rn(p.alpha, v[8 * c + i]), __fmul_rn(p.beta, to_f(h[i])));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(p.alpha, v[j]);
          if (lane == 0) bulk_wait_read<1>();  // stores of block n - 2 no longer read buffer k
        }
        __syncwarp();
        const bool diag = row0 == col0;                             // holds the matrix diagonal (D2 patch)
        const bool mirror = p.sym && (row0 >> 7) > (col0 >> 7);  // an off-diagonal 128-block
        if (!p.trans_out) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 r;
            T* h = reinterpret_cast<T*>(&r);
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = from_f<T>(v[8 * c + i]);
            *reinterpret_cast<uint4*>(gM + sw64_off(lane, 8 * c)) = r;
          }
        }
        if (mirror || p.trans_out) {
#pragma unroll
          for (int j = 0; j < 32; ++j) *reinterpret_cast<T*>(gT + sw64_off(j, lane)) = from_f<T>(v[j]);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (!p.trans_out) store(&p.tmD, sM, col0, row0, b);
          if (mirror || p.trans_out) store(&p.tmD, sT, row0, col0, b);
          if (has_d2 && !diag) {
            store(&p.tmD2, sM, col0, row0, b);
            if (mirror) store(&p.tmD2, sT, row0, col0, b);
          }
          bulk_commit();
        }
        if (has_d2 && diag) {
          // D2 = D + diag2 I: patch the block's diagonal once D's store has read it
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
          float dv = 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j == lane) dv = v[j];
          *reinterpret_cast<T*>(gM + sw64_off(lane, lane)) = from_f<T>(rnd<T>(dv) + p.diag2);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            store(&p.tmD2, sM, col0, row0, b);
            bulk_commit();
          }
        }
        if (has_c) {
          int t2, ch2, b2, tm2, tn2;
          if (next_block(p, t, ch, nv, nclusters, row_base, t2, ch2, b2, tm2, tn2)) load_c(n + 1, b2, tm2, tn2, ch2);
        }
      }
    }
    if (lane == 0) bulk_wait_all<0>();
    // a C block still in flight (abort path) must land before the CTA exits
    if (c_inflight) mbar_wait(cb0 + 8 * c_buf, c_par, nullptr, p.err, p.wait_limit_ns);
  } else {
    // ------------------------------ epilogue (both CTAs) -------------------
    const int q = warp & 3;
    const int rloc = (int)rank * 128 + q * 32 + lane;
    const T* Cp = reinterpret_cast<const T*>(p.C);
    T* Dp = reinterpret_cast<T*>(p.D);
    T* D2p = reinterpret_cast<T*>(p.D2);
    int it = 0;
    for (int t = cid; t < p.total_tiles; t += nclusters, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, p.err, p.wait_limit_ns)) break;
      tc_fence_after();
      int b, tm, tn;
      decode_tile2(p, t, b, tm, tn);
      const int row = tm * BM2 + rloc;
      const bool row_ok = row < p.M;
      const int row_blk = (tm * BM2 + (int)rank * 128 + q * 32) >> 7;  // the 128-block of this warp's rows
      T* D = Dp + (int64_t)b * p.d_bs;
      T* D2 = D2p ? D2p + (int64_t)b * p.d2_bs : nullptr;
      const T* Cb = Cp ? Cp + (int64_t)b * p.c_bs : nullptr;
#pragma unroll 1
      for (int ch = 0; ch < 256 / 32; ++ch) {
        const int col0 = tn * 256 + ch * 32;
        if (col0 >= p.N) break;
        if (p.sym && (col0 >> 7) > row_blk) continue;  // a block above the diagonal: the mirror writes it
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 256 + ch * 32), v);
        epilogue_chunk(p, v, row, row_ok, col0, D, D2, Cb);
      }
      tc_fence_before();
      mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
    }
  }

  abort_settle(abort_flag);
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512u) : "memory");
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    else
      cudaGetLastError();
  });
  return fn;
}

struct DevInfo {
  int sms = 0;
  int major = 0;
};
static DevInfo dev_info() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static std::vector<DevInfo> cache;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1);
  if (cache[dev].sms == 0) {
    cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].major, cudaDevAttrComputeCapabilityMajor, dev);
  }
  return cache[dev];
}

// 3-D tiled tensor map over [batch][rows][inner] with 128-byte swizzle.
static int make_map(CUtensorMap* m, const void* base, int dtype, int64_t inner, int64_t rows, int64_t batch,
                    int64_t ld, int64_t bs, int box_inner, int box_rows,
                    CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return THORN_ERR_UNSUPPORTED;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)batch};
  int64_t bstride = bs > 0 ? bs : ld * rows;
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(bstride * 2)};
  cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dtype == THORN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? THORN_OK : THORN_ERR_ARG;
}

}  // namespace gemm

// One GEMM of the NS iteration (all pointers device, 16-bit elements).
struct GemmOp {
  const void* A = nullptr;
  int64_t a_ld = 0, a_bs = 0;
  bool a_mn = false;
  const void* B = nullptr;
  int64_t b_ld = 0, b_bs = 0;
  bool b_mn = false;
  const void* C = nullptr;
  int64_t c_ld = 0, c_bs = 0;
  void* D = nullptr;
  int64_t d_ld = 0, d_bs = 0;
  void* D2 = nullptr;
  int64_t d2_ld = 0, d2_bs = 0;
  int M = 0, N = 0, K = 0, batch = 1;
  float alpha = 1.f, beta = 0.f, diag2 = 0.f;
  bool sym = false, trans_out = false;
};

// Algorithmic work of the GEMMs issued so far (for roofline reporting).
static std::atomic<uint64_t> g_flops_dense{0}, g_flops_exec{0};

// Programmatic dependent launch of the NS GEMMs (1) or plain stream order (0, default).
static std::atomic<int> g_gemm_pdl{0};
// L2 cache policies on the 2-CTA kernel's operand loads and output stores (1) or none (0, default).
static std::atomic<int> g_l2_hints{0};
// Limit of every mbarrier wait in the NS GEMMs, and the failure-test switch (producers issue no loads).
static std::atomic<uint64_t> g_wait_limit_ns{gemm::kTimeoutNs};
static std::atomic<int> g_test_stall{0};

template <int BN, bool AMN, bool BMN, class T>
static int launch_gemm(gemm::Params& prm, int grid, cudaStream_t st) {
  using C_ = gemm::Cfg<BN>;
  static std::once_flag attr_once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(attr_once[dev & 63], []() {
    cudaFuncSetAttribute(gemm::ns_gemm_kernel<BN, AMN, BMN, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         C_::kSmem);
  });
  if (g_gemm_pdl.load() != 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(gemm::kThreadsG, 1, 1);
    cfg.dynamicSmemBytes = C_::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, gemm::ns_gemm_kernel<BN, AMN, BMN, T>, prm);
  } else {
    gemm::ns_gemm_kernel<BN, AMN, BMN, T><<<grid, gemm::kThreadsG, C_::kSmem, st>>>(prm);
  }
  count_launch();
  return check_launch();
}

template <bool AMN, bool BMN, class T>
static int launch_gemm2(gemm::Params& prm, int64_t total, int sms, cudaStream_t st) {
  static std::once_flag attr_once[64];
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(attr_once[dev & 63], [sms, dev]() {
    auto k = gemm::ns_gemm2_kernel<AMN, BMN, T>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm::kSmem2);
    // persistent grid: as many CTA pairs as can be resident at once
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    cfg.blockDim = dim3(gemm::kThreadsG, 1, 1);
    cfg.dynamicSmemBytes = gemm::kSmem2;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sms / 2;
    }
    max_clusters[dev & 63] = n;
  });
  const int clusters = (int)min64(total, (int64_t)std::max(1, max_clusters[dev & 63]));
  if (g_gemm_pdl.load() != 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(gemm::kThreadsG, 1, 1);
    cfg.dynamicSmemBytes = gemm::kSmem2;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, gemm::ns_gemm2_kernel<AMN, BMN, T>, prm);
  } else {
    gemm::ns_gemm2_kernel<AMN, BMN, T><<<2 * clusters, gemm::kThreadsG, gemm::kSmem2, st>>>(prm);
  }
  count_launch();
  return check_launch();
}

template <class T>
static int launch_any2(const GemmOp& op, gemm::Params& prm, int64_t total, int sms, cudaStream_t st) {
  if (op.a_mn) return op.b_mn ? launch_gemm2<true, true, T>(prm, total, sms, st)
                              : launch_gemm2<true, false, T>(prm, total, sms, st);
  if (op.b_mn) return launch_gemm2<false, true, T>(prm, total, sms, st);
  return launch_gemm2<false, false, T>(prm, total, sms, st);
}

static std::atomic<int> g_pair_tiles{1};
static std::atomic<int> g_staged_epilogue{1};

template <class T>
static int launch_any(const GemmOp& op, int BN, gemm::Params& prm, int grid, cudaStream_t st) {
  // every operand layout: A and B each K-major or MN-major
  if (BN == 256) {
    if (op.a_mn) return op.b_mn ? launch_gemm<256, true, true, T>(prm, grid, st)
                                : launch_gemm<256, true, false, T>(prm, grid, st);
    if (op.b_mn) return launch_gemm<256, false, true, T>(prm, grid, st);
    return launch_gemm<256, false, false, T>(prm, grid, st);
  }
  if (op.a_mn) return op.b_mn ? launch_gemm<128, true, true, T>(prm, grid, st)
                              : launch_gemm<128, true, false, T>(prm, grid, st);
  if (op.b_mn) return launch_gemm<128, false, true, T>(prm, grid, st);
  return launch_gemm<128, false, false, T>(prm, grid, st);
}

int run_gemm(const GemmOp& op, int dtype, int* err, cudaStream_t st) {
  using namespace gemm;
  if (op.M <= 0 || op.N <= 0 || op.K <= 0 || op.batch <= 0) return THORN_OK;
  if (!op.A || !op.B || !op.D) return THORN_ERR_ARG;
  if (dtype != THORN_F16 && dtype != THORN_BF16) return THORN_ERR_ARG;
  if (op.sym && op.M != op.N) return THORN_ERR_ARG;
  // TMA: 16-byte aligned bases and strides
  if (!aligned16(op.A) || !aligned16(op.B) || (op.a_ld % 8) || (op.b_ld % 8) || (op.a_bs % 8) || (op.b_bs % 8))
    return THORN_ERR_ALIGN;
  DevInfo di = dev_info();
  if (di.major != 10) return THORN_ERR_UNSUPPORTED;
  Params prm;
  memset(&prm, 0, sizeof(prm));
  // 2-CTA 256 x 256 cluster tiles when both output dimensions fill them
  const bool pair = g_pair_tiles.load() != 0 && op.M >= 256 && op.N >= 256 && di.sms >= 2;
  const int BN = pair ? 256 : ((op.N > 128) ? 256 : 128);
  const int BMt = pair ? BM2 : BM;
  const int a_box_rows = 128;  // rows of A one CTA loads per stage (half of a pair tile)
  const int b_box_rows = pair ? 128 : BN;
  int rc = op.a_mn ? make_map(&prm.tmA, op.A, dtype, op.M, op.K, op.batch, op.a_ld, op.a_bs, 64, BK)
                   : make_map(&prm.tmA, op.A, dtype, op.K, op.M, op.batch, op.a_ld, op.a_bs, BK, a_box_rows);
  if (rc) return rc;
  if (op.b_mn) rc = make_map(&prm.tmB, op.B, dtype, op.N, op.K, op.batch, op.b_ld, op.b_bs, 64, BK);
  else rc = make_map(&prm.tmB, op.B, dtype, op.K, op.N, op.batch, op.b_ld, op.b_bs, BK, b_box_rows);
  if (rc) return rc;
  prm.C = op.C;
  prm.D = op.D;
  prm.D2 = op.D2;
  prm.c_bs = op.c_bs;
  prm.c_ld = op.c_ld;
  prm.d_bs = op.d_bs;
  prm.d_ld = op.d_ld;
  prm.d2_bs = op.d2_bs;
  prm.d2_ld = op.d2_ld;
  prm.M = op.M;
  prm.N = op.N;
  prm.K = op.K;
  prm.batch = op.batch;
  prm.alpha = op.alpha;
  prm.beta = op.beta;
  prm.diag2 = op.diag2;
  prm.sym = op.sym;
  prm.trans_out = op.trans_out;
  prm.c_vec = op.C && aligned16(op.C) && (op.c_ld % 8) == 0 && (op.c_bs % 8) == 0;
  prm.d_vec = aligned16(op.D) && (op.d_ld % 8) == 0 && (op.d_bs % 8) == 0 &&
              (!op.D2 || (aligned16(op.D2) && (op.d2_ld % 8) == 0 && (op.d2_bs % 8) == 0));
  // staged epilogue (2-CTA tiles): TMA maps of C, D, D2 with 32 x 32 boxes
  const bool c_al = !op.C || (aligned16(op.C) && (op.c_ld % 8) == 0 && (op.c_bs % 8) == 0);
  prm.tma_epi = pair && g_staged_epilogue.load() != 0 && prm.d_vec && c_al && !(op.D2 && op.trans_out);
  if (prm.tma_epi) {
    const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_64B;
    rc = op.trans_out ? make_map(&prm.tmD, op.D, dtype, op.M, op.N, op.batch, op.d_ld, op.d_bs, 32, 32, sw)
                      : make_map(&prm.tmD, op.D, dtype, op.N, op.M, op.batch, op.d_ld, op.d_bs, 32, 32, sw);
    if (rc) return rc;
    if (op.D2) {
      rc = make_map(&prm.tmD2, op.D2, dtype, op.N, op.M, op.batch, op.d2_ld, op.d2_bs, 32, 32, sw);
      if (rc) return rc;
    }
    if (op.C) {
      prm.c_bcast = op.c_bs == 0;
      rc = make_map(&prm.tmC, op.C, dtype, op.N, op.M, prm.c_bcast ? 1 : op.batch, op.c_ld,
                    prm.c_bcast ? op.c_ld * op.M : op.c_bs, 32, 32, sw);
      if (rc) return rc;
    }
  }
  prm.l2hint = pair && g_l2_hints.load() != 0;
  prm.tiles_m = (op.M + BMt - 1) / BMt;
  prm.tiles_n = (op.N + BN - 1) / BN;
  // A wide output (the m x n products of Gram NS: 16 x 56 cluster tiles at 4096 x 14336)
  // walked row by row has every wave of clusters read all of B's panels (the whole
  // 117 MB n-side operand) while A's few panels sit idle in L2.  Down the columns a wave
  // reads all of the small m-side operand (32 MB) and ~5 panels of B, which stay in L2.
  prm.col_major = (pair && !op.sym && prm.tiles_n > prm.tiles_m) ? 1 : 0;
  if (op.sym) {
    int cnt = 0;
    for (int tm = 0; tm < prm.tiles_m; ++tm)
      cnt += pair ? std::min(prm.tiles_n, tm + 1) : std::min(prm.tiles_n, (tm * BM + BM - 1) / BN + 1);
    prm.tiles_per_mat = cnt;
  } else {
    prm.tiles_per_mat = prm.tiles_m * prm.tiles_n;
  }
  const int64_t total = (int64_t)prm.tiles_per_mat * op.batch;
  if (total > (int64_t)INT32_MAX) return THORN_ERR_ARG;
  prm.total_tiles = (int)total;
  prm.num_kb = (op.K + BK - 1) / BK;
  prm.err = err;
  prm.wait_limit_ns = g_wait_limit_ns.load();
  prm.test_stall = g_test_stall.load();
  const int grid = (int)min64(total, (int64_t)di.sms);
  const double dense = 2.0 * op.M * (double)op.N * op.K * op.batch;
  const double exec = 2.0 * BMt * (double)BN * (prm.num_kb * (double)BK) * total;
  g_flops_dense.fetch_add((uint64_t)dense);
  g_flops_exec.fetch_add((uint64_t)exec);
  if (pair)
    return dtype == THORN_BF16 ? launch_any2<__nv_bfloat16>(op, prm, total, di.sms, st)
                               : launch_any2<__half>(op, prm, total, di.sms, st);
  return dtype == THORN_BF16 ? launch_any<__nv_bfloat16>(op, BN, prm, grid, st)
                             : launch_any<__half>(op, BN, prm, grid, st);
}

// ---------------------------------------------------------------------------
// Newton-Schulz of small matrices, one CTA per matrix (min dim <= 128, max dim
// <= 512): X and every m x m iterate stay in shared memory for all iterations,
// accumulators in TMEM, so a batch of small matrices (conv kernels, heads) is
// one launch instead of one launch per product.  Same recurrences, operand
// orders and roundings as the GEMM sequence of thorn_ns_batched; a matrix of at
// most 128 rows is one 128-block, so every product is the plain product.
//
// Shared-memory layout of every operand: row-major, split into 64-column chunks
// of 128 rows x 128 bytes (16 KB) in the 128-byte swizzle of the tensor maps
// (16-byte unit u of row r stored at unit u ^ (r % 8)).  One layout serves as a
// K-major operand (rows = M or N, K along the row) and as an MN-major one (rows
// = K), so no operand is ever copied or transposed.  Rows and columns beyond
// the matrix are zero.
// ---------------------------------------------------------------------------
namespace nss {

constexpr int kThreads = 128;  // thread t owns TMEM lane t = output row t
constexpr int kChunk = 128 * 128;  // bytes of one 64-column chunk
constexpr int kMaxIters = 16;
constexpr int kMaxN = 512;  // largest max(rows, cols)

struct Params {
  const void* x;  // [batch][rows][ld_in], the NS input in the matrix's own orientation
  void* out;      // [batch][rows][cols]
  int64_t ld_in;
  int batch, rows, cols;
  int m, n;  // min / max dim
  int tall, gram;
  int iters;
  uint32_t restart_mask;  // bit i: Gram restart before iteration i
  float coef[3 * kMaxIters];
  int* err;
  uint64_t wait_limit_ns;
  int test_stall;  // failure test: no MMA is issued, so the first completion wait runs out
};

__host__ __device__ constexpr int round_up(int x, int a) { return (x + a - 1) / a * a; }

// Shared memory of one CTA: X (n padded to 64-column chunks) + three m x m
// buffers (two 64-column chunks each) + barrier words.
__host__ __device__ inline int smem_bytes(int n) { return (round_up(n, 64) / 64 + 6) * kChunk + 1024 + 64; }

__device__ __forceinline__ uint32_t off(int r, int c) {
  return (uint32_t)((c >> 6) * kChunk + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + ((c & 7) << 1));
}

// tcgen05 descriptors of one operand buffer for K step kk (16 elements)
__device__ __forceinline__ uint64_t desc_k(uint32_t base, int kk, int row0) {  // K-major: rows = M or N
  return gemm::sdesc(base + (kk >> 2) * kChunk + (kk & 3) * 32 + row0 * 128, 16, 1024);
}
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int kk, int col0) {  // MN-major: rows = K
  return gemm::sdesc(base + (col0 >> 6) * kChunk + kk * 2048, kChunk, 1024);
}

// D[128 x N] (TMEM columns [0, N)) = A[128 x K] @ B[K x N]; issued by one thread.
// A: K-major (A[i][k] at row i) or MN-major (A[i][k] at row k: the transpose of
// the buffer).  B: K-major (B[k][j] at row j: the transpose of the buffer, for
// X X^T) or MN-major (B[k][j] at row k).
__device__ __forceinline__ void mma(uint32_t tmem, uint32_t a, bool a_mn, uint32_t b, bool b_mn, int K, int N,
                                    bool bf16) {
  for (int n0 = 0; n0 < N; n0 += 256) {
    const int nn = min(256, N - n0);
    const uint32_t idesc = gemm::idesc_f16(nn, bf16, a_mn, b_mn);
    for (int kk = 0; kk < K / 16; ++kk) {
      const uint64_t ad = a_mn ? desc_mn(a, kk, 0) : desc_k(a, kk, 0);
      const uint64_t bd = b_mn ? desc_mn(b, kk, n0) : desc_k(b, kk, n0);
      gemm::umma(tmem + (uint32_t)n0, ad, bd, idesc, kk != 0 ? 1u : 0u);
    }
  }
}

template <class T>
__device__ __forceinline__ void load8(const uint8_t* buf, int r, int c, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(buf + off(r, c));
  unpack2(u.x, v[0], v[1], (T*)nullptr);
  unpack2(u.y, v[2], v[3], (T*)nullptr);
  unpack2(u.z, v[4], v[5], (T*)nullptr);
  unpack2(u.w, v[6], v[7], (T*)nullptr);
}
template <class T>
__device__ __forceinline__ void store8(uint8_t* buf, int r, int c, const float* v) {
  uint4 u;
  u.x = pack2(v[0], v[1], (T*)nullptr);
  u.y = pack2(v[2], v[3], (T*)nullptr);
  u.z = pack2(v[4], v[5], (T*)nullptr);
  u.w = pack2(v[6], v[7], (T*)nullptr);
  *reinterpret_cast<uint4*>(buf + off(r, c)) = u;
}

// Epilogue of one product for this thread's row: D = alpha acc + beta C (C in
// shared memory, may be the destination itself: each thread reads and writes
// only its own row), one rounding; optional second output D2 = D + diag2 I.
// Columns >= nv and rows >= mv are written as zero.  dst == nullptr: the final
// product, stored to global memory in the caller's orientation.
template <class T>
__device__ __forceinline__ void epilogue(uint32_t tmem_row, int row, int N, int nv, int mv, float alpha, float beta,
                                         const uint8_t* C, uint8_t* dst, uint8_t* dst2, float diag2, const Params& p,
                                         T* gout) {
  for (int c0 = 0; c0 < N; c0 += 32) {
    float v[32];
    gemm::tmem_ld32(tmem_row + (uint32_t)c0, v);
    if (C != nullptr) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float cv[8];
        load8<T>(C, row, c0 + 8 * q, cv);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[8 * q + j] = __fadd_rn(__fmul_rn(alpha, v[8 * q + j]), __fmul_rn(beta, cv[j]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(alpha, v[j]);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (row < mv && c0 + j < nv) ? rnd<T>(v[j]) : 0.f;
    if (gout != nullptr) {
      if (row < mv) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (c0 + j >= nv) break;
          // wide: out[row][col]; tall: the result is the transpose, out[col][row]
          if (p.tall) gout[(int64_t)(c0 + j) * p.cols + row] = from_f<T>(v[j]);
          else gout[(int64_t)row * p.cols + c0 + j] = from_f<T>(v[j]);
        }
      }
      continue;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) store8<T>(dst, row, c0 + 8 * q, v + 8 * q);
    if (dst2 != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row == c0 + j && row < mv) v[j] = rnd<T>(v[j] + diag2);
#pragma unroll
      for (int q = 0; q < 4; ++q) store8<T>(dst2, row, c0 + 8 * q, v + 8 * q);
    }
  }
}

template <class T>
__global__ void __launch_bounds__(kThreads, 1) ns_small_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int n_pad = round_up(p.n, 64);
  uint8_t* X = smem;
  uint8_t* B0 = X + (n_pad / 64) * kChunk;  // Gram: R; square: A = X X^T
  uint8_t* B1 = B0 + 2 * kChunk;            // Gram: Z; square: B = c A A + b A
  uint8_t* B2 = B1 + 2 * kChunk;            // Gram: Q
  uint64_t* bar = reinterpret_cast<uint64_t*>(B2 + 2 * kChunk);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int b = blockIdx.x;
  const bool bf16 = !std::is_same<T, __half>::value;
  const int m = p.m, n = p.n;
  // K extents in 16-element MMA steps; N extents in whole 64-column chunks
  const int Km = round_up(m, 16), Nm = round_up(m, 64), Kn = round_up(n, 16), Nn = round_up(n, 64);
  const uint32_t tcols = Nn > 256 ? 512u : (Nn > 128 ? 256u : (Nn > 64 ? 128u : 64u));

  if (tid == 0) {
    gemm::mbar_init(gemm::smem_u32(bar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     gemm::smem_u32(tmem_holder)),
                 "r"(tcols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // X (wide orientation, m x n) from global memory, zero beyond the matrix
  {
    const T* xg = reinterpret_cast<const T*>(p.x) + (int64_t)b * p.rows * p.ld_in;
    const int units = 128 * (n_pad / 8);  // 16-byte units of X
    for (int u = tid; u < units; u += kThreads) {
      const int r = u / (n_pad / 8), c = (u % (n_pad / 8)) * 8;
      if (!p.tall && r < m && c + 8 <= n) {  // 8 whole elements of a row: one 16-byte load
        *reinterpret_cast<uint4*>(X + off(r, c)) = *reinterpret_cast<const uint4*>(xg + (int64_t)r * p.ld_in + c);
        continue;
      }
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // X[r][c + j] = x[r][c + j] (wide) or x[c + j][r] (tall)
        const bool in = r < m && c + j < n;
        v[j] = in ? to_f(p.tall ? xg[(int64_t)(c + j) * p.ld_in + r] : xg[(int64_t)r * p.ld_in + c + j]) : 0.f;
      }
      store8<T>(X, r, c, v);
    }
    // the m x m buffers start at zero (their padding must stay zero)
    for (int u = tid; u < 6 * kChunk / 16; u += kThreads) reinterpret_cast<uint4*>(B0)[u] = make_uint4(0, 0, 0, 0);
  }
  gemm::tc_fence_before();
  __syncthreads();
  gemm::tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t tmem_row = tmem + ((uint32_t)(warp * 32) << 16);
  const uint32_t sX = gemm::smem_u32(X), s0 = gemm::smem_u32(B0), s1 = gemm::smem_u32(B1), s2 = gemm::smem_u32(B2);
  uint32_t phase = 0;
  bool ok = true;
  T* gout = reinterpret_cast<T*>(p.out) + (int64_t)b * p.rows * p.cols;

  // one product: operands ready in shared memory -> MMAs -> wait -> epilogue
  auto product = [&](uint32_t a, bool a_mn, uint32_t bb, bool b_mn, int K, int N, int nv, float alpha, float beta,
                     const uint8_t* C, uint8_t* dst, uint8_t* dst2, float diag2, T* g) {
    if (!ok) return;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes -> tensor core
    gemm::tc_fence_before();
    __syncthreads();
    gemm::tc_fence_after();
    if (tid == 0 && !p.test_stall) {
      mma(tmem, a, a_mn, bb, b_mn, K, N, bf16);
      gemm::umma_commit(gemm::smem_u32(bar));
    }
    // every thread takes the same branch: the TMEM loads and barriers below need the whole CTA
    ok = __syncthreads_and(gemm::mbar_wait(gemm::smem_u32(bar), phase, nullptr, p.err, p.wait_limit_ns) ? 1 : 0);
    if (!ok) return;
    phase ^= 1u;
    gemm::tc_fence_after();
    epilogue<T>(tmem_row, tid, N, nv, m, alpha, beta, C, dst, dst2, diag2, p, g);
    gemm::tc_fence_before();
  };

  if (p.gram) {
    uint8_t *R = B0, *Z = B1, *Q = B2;
    const uint32_t sR = s0, sZ = s1, sQ = s2;
    product(sX, false, sX, false, Kn, Nm, m, 1.f, 0.f, nullptr, R, nullptr, 0.f, nullptr);  // R = X X^T
    for (int i = 0; i < p.iters && ok; ++i) {
      const float a = p.coef[3 * i], bc = p.coef[3 * i + 1], c = p.coef[3 * i + 2];
      const bool rs = (p.restart_mask >> i) & 1u;
      if (rs && i != 0) {
        product(sQ, false, sX, true, Km, Nn, n, 1.f, 0.f, nullptr, X, nullptr, 0.f, nullptr);  // X = Q X
        product(sX, false, sX, false, Kn, Nm, m, 1.f, 0.f, nullptr, R, nullptr, 0.f, nullptr);  // R = X X^T
      }
      if (i != 0 && !rs) {
        product(sR, false, sR, true, Km, Nm, m, c, bc, R, Z, nullptr, 0.f, nullptr);  // Z = c R R + b R
        product(sQ, false, sZ, true, Km, Nm, m, 1.f, a, Q, Q, nullptr, 0.f, nullptr);  // Q = Q Z + a Q
      } else {
        product(sR, false, sR, true, Km, Nm, m, c, bc, R, Z, Q, a, nullptr);  // Z = c R R + b R; Q = Z + a I
      }
      if (i < p.iters - 1 && !((p.restart_mask >> (i + 1)) & 1u)) {
        product(sR, false, sZ, true, Km, Nm, m, 1.f, a, R, R, nullptr, 0.f, nullptr);  // RZ = R Z + a R
        product(sZ, false, sR, true, Km, Nm, m, 1.f, a, R, R, nullptr, 0.f, nullptr);  // R = Z RZ + a RZ
      }
    }
    // out = Q X; a tall input gets X^T Q (thorn.py:653) = (Q^T X)^T
    product(sQ, p.tall != 0, sX, true, Km, Nn, n, 1.f, 0.f, nullptr, nullptr, nullptr, 0.f, gout);
  } else {
    uint8_t *A = B0, *Bm = B1;
    const uint32_t sA = s0, sB = s1;
    for (int i = 0; i < p.iters && ok; ++i) {
      const float a = p.coef[3 * i], bc = p.coef[3 * i + 1], c = p.coef[3 * i + 2];
      const bool last = i == p.iters - 1;
      product(sX, false, sX, false, Km, Nm, m, 1.f, 0.f, nullptr, A, nullptr, 0.f, nullptr);  // A = X X^T
      product(sA, false, sA, true, Km, Nm, m, c, bc, A, Bm, nullptr, 0.f, nullptr);          // B = c A A + b A
      product(sB, false, sX, true, Km, Nm, m, 1.f, a, X, last ? nullptr : X, nullptr, 0.f,
              last ? gout : nullptr);  // X = a X + B X
    }
  }
  if (!ok) {  // a wait ran out: let an MMA still in flight land before the TMEM is released
    const uint64_t t0 = gemm::global_ns();
    while (gemm::global_ns() - t0 < gemm::kSettleNs) {
    }
  }
  gemm::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    gemm::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
  }
}

}  // namespace nss

static std::atomic<int> g_ns_small{1};

// Dense-equivalent FLOPs of the reference's GEMMs for one matrix (roofline counters).
static double dense_ns_flops(int64_t m, int64_t n, int iters, bool) {
  const double M = (double)m, N = (double)n;
  if (m == n) return iters * (4.0 * M * M * N + 2.0 * M * M * M);
  return 28.0 * M * M * M + 8.0 * M * M * N;
}

// The small-matrix kernel for one thorn_ns_batched call, or THORN_ERR_UNSUPPORTED
// when the shape or settings do not fit it (the caller then runs the GEMM sequence).
int run_ns_small(const void* x, void* out, int64_t batch, int64_t rows, int64_t cols, int dtype,
                 const double* coeffs, int iters, const int32_t* restarts, int n_restarts, int* err,
                 cudaStream_t st) {
  const int64_t m = std::min(rows, cols), n = std::max(rows, cols);
  if (g_ns_small.load() == 0 || m > 128 || n > nss::kMaxN || iters < 1 || iters > nss::kMaxIters ||
      batch > INT32_MAX)
    return THORN_ERR_UNSUPPORTED;
  gemm::DevInfo di = gemm::dev_info();
  if (di.major != 10) return THORN_ERR_UNSUPPORTED;
  nss::Params p;
  memset(&p, 0, sizeof(p));
  p.x = x;
  p.out = out;
  p.ld_in = thorn_ns_ld(cols);
  p.batch = (int)batch;
  p.rows = (int)rows;
  p.cols = (int)cols;
  p.m = (int)m;
  p.n = (int)n;
  p.tall = rows > cols;
  p.gram = m != n;
  p.iters = iters;
  for (int k = 0; k < n_restarts; ++k)
    if (restarts[k] >= 0 && restarts[k] < nss::kMaxIters) p.restart_mask |= 1u << restarts[k];
  for (int i = 0; i < 3 * iters; ++i) p.coef[i] = (float)coeffs[i];
  p.err = err;
  p.wait_limit_ns = g_wait_limit_ns.load();
  p.test_stall = g_test_stall.load();
  const int smem = nss::smem_bytes((int)n);
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], []() {
    cudaFuncSetAttribute(nss::ns_small_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         nss::smem_bytes(nss::kMaxN));
    cudaFuncSetAttribute(nss::ns_small_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         nss::smem_bytes(nss::kMaxN));
  });
  if (dtype == THORN_BF16)
    nss::ns_small_kernel<__nv_bfloat16><<<(unsigned)batch, nss::kThreads, smem, st>>>(p);
  else
    nss::ns_small_kernel<__half><<<(unsigned)batch, nss::kThreads, smem, st>>>(p);
  count_launch();
  const double d = dense_ns_flops(m, n, iters, n_restarts > 0) * (double)batch;
  g_flops_dense.fetch_add((uint64_t)d);
  g_flops_exec.fetch_add((uint64_t)d);
  return check_launch();
}

}  // namespace thorn

using namespace thorn;

// ===========================================================================
// Newton-Schulz sequencer (thorn.py:626-662)
// ===========================================================================
namespace {
struct NsLayout {
  int64_t m, n, ldm, ldn;
  bool gram;
  int64_t xs, ms;  // bytes of one [batch, m, ldn] / [batch, m, ldm] buffer (256-aligned)
  int64_t total;
};
// Buffer sizes of one NS call.  Every product is overflow-checked: a size that
// does not fit in int64 leaves total = -1 (the callers reject it).
NsLayout ns_layout(int64_t batch, int64_t rows, int64_t cols) {
  NsLayout L;
  L.m = std::min(rows, cols);
  L.n = std::max(rows, cols);
  L.gram = L.m != L.n;
  L.ldm = L.ldn = L.xs = L.ms = 0;
  L.total = -1;
  if (L.n > (INT64_MAX >> 4)) return L;  // the padded leading dimensions would overflow
  L.ldm = thorn_ns_ld(L.m);
  L.ldn = thorn_ns_ld(L.n);
  auto bytes = [&](int64_t ld, int64_t* out) {
    int64_t v = 0;
    if (__builtin_mul_overflow(batch, L.m, &v) || __builtin_mul_overflow(v, ld, &v) ||
        __builtin_mul_overflow(v, (int64_t)2, &v) || v > INT64_MAX - 255)
      return false;
    *out = (v + 255) / 256 * 256;
    return true;
  };
  if (!bytes(L.ldn, &L.xs) || !bytes(L.ldm, &L.ms)) return L;
  int64_t a = 0, b = 0;
  if (L.gram) {
    if (__builtin_mul_overflow(L.xs, (int64_t)2, &a) || __builtin_mul_overflow(L.ms, (int64_t)5, &b) ||
        __builtin_add_overflow(a, b, &L.total))
      L.total = -1;
  } else if (__builtin_mul_overflow(L.ms, (int64_t)4, &L.total)) {
    L.total = -1;
  }
  return L;
}
}  // namespace

extern "C" int64_t thorn_ns_workspace_bytes(int64_t batch, int64_t rows, int64_t cols) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  return ns_layout(batch, rows, cols).total;
}

extern "C" int thorn_ns_batched(const void* x, void* out, void* workspace, int64_t workspace_bytes, int64_t batch,
                                int64_t rows, int64_t cols, int ns_dtype, const double* coeffs, int iters,
                                const int32_t* restarts, int n_restarts, int* err_flag, void* stream) {
  if (batch < 0 || rows < 0 || cols < 0 || iters < 0 || n_restarts < 0) return THORN_ERR_ARG;
  if (batch == 0 || rows == 0 || cols == 0) return THORN_OK;
  if (!x || !out || !workspace || (iters > 0 && !coeffs) || (n_restarts > 0 && !restarts)) return THORN_ERR_ARG;
  if (ns_dtype != THORN_F16 && ns_dtype != THORN_BF16) return THORN_ERR_ARG;
  if (batch > INT32_MAX || rows > INT32_MAX || cols > INT32_MAX) return THORN_ERR_ARG;
  const NsLayout L = ns_layout(batch, rows, cols);
  if (L.total < 0 || workspace_bytes < L.total) return THORN_ERR_ARG;
  if (!aligned16(x) || !aligned16(workspace)) return THORN_ERR_ALIGN;
  cudaStream_t st = (cudaStream_t)stream;
  // small matrices: the whole iteration in one launch, operands resident in shared memory
  if (iters > 0) {
    const int rs = run_ns_small(x, out, batch, rows, cols, ns_dtype, coeffs, iters, restarts, n_restarts, err_flag, st);
    if (rs != THORN_ERR_UNSUPPORTED) return rs;
  }
  const bool tall = rows > cols;
  const int m = (int)L.m, n = (int)L.n, B = (int)batch;
  const int64_t ldm = L.ldm, ldn = L.ldn;
  auto in_restarts = [&](int i) {
    for (int k = 0; k < n_restarts; ++k)
      if (restarts[k] == i) return true;
    return false;
  };
  uint8_t* ws = (uint8_t*)workspace;
  int rc = THORN_OK;
  // product A @ Bm of two m x m matrices.  Bm is read MN-major: the symmetric
  // outputs are exactly symmetric only off their diagonal 128-blocks, so Bm and
  // Bm^T may differ there and the product must be the reference's A @ Bm.
  auto mm = [&](const void* A, const void* Bm, const void* C, void* D, void* D2, float alpha, float beta,
                float diag2) {
    GemmOp op;
    op.A = A; op.a_ld = ldm; op.a_bs = m * ldm;
    op.B = Bm; op.b_ld = ldm; op.b_bs = m * ldm; op.b_mn = true;
    op.C = C; op.c_ld = ldm; op.c_bs = m * ldm;
    op.D = D; op.d_ld = ldm; op.d_bs = m * ldm;
    op.D2 = D2; op.d2_ld = ldm; op.d2_bs = m * ldm;
    op.M = m; op.N = m; op.K = m; op.batch = B;
    op.alpha = alpha; op.beta = beta; op.diag2 = diag2; op.sym = true;
    return run_gemm(op, ns_dtype, err_flag, st);
  };
  // Gram matrix X X^T of a [m, n] matrix with leading dim ld
  auto gramm = [&](const void* X, int64_t ld, int K, void* D) {
    GemmOp op;
    op.A = X; op.a_ld = ld; op.a_bs = m * ld;
    op.B = X; op.b_ld = ld; op.b_bs = m * ld; op.b_mn = false;
    op.D = D; op.d_ld = ldm; op.d_bs = m * ldm;
    op.M = m; op.N = m; op.K = K; op.batch = B;
    op.sym = true;
    return run_gemm(op, ns_dtype, err_flag, st);
  };
  // Q @ X with X [m, N] (MN-major second operand), optional C = X.  With q_t
  // the first operand is Q^T (Q read MN-major): the tall final product
  // X^T @ Q = (Q^T @ X)^T of thorn.py:653, stored transposed.
  auto qx = [&](const void* Q, const void* X, int64_t ldx, int N, const void* C, float beta, void* D, int64_t d_ld,
                int64_t d_bs, bool trans, bool q_t) {
    GemmOp op;
    op.A = Q; op.a_ld = ldm; op.a_bs = m * ldm; op.a_mn = q_t;
    op.B = X; op.b_ld = ldx; op.b_bs = m * ldx; op.b_mn = true;
    op.C = C; op.c_ld = ldx; op.c_bs = m * ldx;
    op.D = D; op.d_ld = d_ld; op.d_bs = d_bs;
    op.M = m; op.N = N; op.K = m; op.batch = B;
    op.beta = beta; op.trans_out = trans;
    return run_gemm(op, ns_dtype, err_flag, st);
  };
  // The same two products for a tall input kept in its original orientation:
  // u is [n, m] (ld ldm) and X = u^T.  X X^T = u^T u reads u MN-major for both
  // operands; Q @ X = Q u^T reads u as a K-major second operand.
  auto gramm_tall = [&](const void* U, void* D) {
    GemmOp op;
    op.A = U; op.a_ld = ldm; op.a_bs = n * ldm; op.a_mn = true;
    op.B = U; op.b_ld = ldm; op.b_bs = n * ldm; op.b_mn = true;
    op.D = D; op.d_ld = ldm; op.d_bs = m * ldm;
    op.M = m; op.N = m; op.K = n; op.batch = B;
    op.sym = true;
    return run_gemm(op, ns_dtype, err_flag, st);
  };
  auto qx_tall = [&](const void* Q, const void* U, void* D, int64_t d_ld, int64_t d_bs, bool trans, bool q_t) {
    GemmOp op;
    op.A = Q; op.a_ld = ldm; op.a_bs = m * ldm; op.a_mn = q_t;
    op.B = U; op.b_ld = ldm; op.b_bs = n * ldm; op.b_mn = false;
    op.D = D; op.d_ld = d_ld; op.d_bs = d_bs;
    op.M = m; op.N = n; op.K = m; op.batch = B;
    op.trans_out = trans;
    return run_gemm(op, ns_dtype, err_flag, st);
  };
#define NS_TRY(expr)          \
  do {                        \
    rc = (expr);              \
    if (rc) return rc;        \
  } while (0)

  if (L.gram) {
    void* Xb[2] = {ws, ws + L.xs};
    uint8_t* mbase = ws + 2 * L.xs;
    void* R = mbase;
    void* Z = mbase + L.ms;
    void* Qb[2] = {mbase + 2 * L.ms, mbase + 3 * L.ms};
    void* RZ = mbase + 4 * L.ms;
    const void* X = x;
    bool x_is_input_tall = tall;  // X is still the caller's tall input (original orientation)
    int xi = 0, qi = 0;
    NS_TRY(tall ? gramm_tall(X, R) : gramm(X, ldn, n, R));
    for (int i = 0; i < iters; ++i) {
      const float a = (float)coeffs[3 * i], b = (float)coeffs[3 * i + 1], c = (float)coeffs[3 * i + 2];
      const bool rs = in_restarts(i);
      if (rs && i != 0) {
        if (x_is_input_tall) NS_TRY(qx_tall(Qb[qi], X, Xb[xi], ldn, m * ldn, false, false));
        else NS_TRY(qx(Qb[qi], X, ldn, n, nullptr, 0.f, Xb[xi], ldn, m * ldn, false, false));
        X = Xb[xi];
        x_is_input_tall = false;
        xi ^= 1;
        NS_TRY(gramm(X, ldn, n, R));
      }
      if (i != 0 && !rs) {
        NS_TRY(mm(R, R, R, Z, nullptr, c, b, 0.f));                   // Z = c R R + b R
        NS_TRY(mm(Qb[qi], Z, Qb[qi], Qb[qi ^ 1], nullptr, 1.f, a, 0.f));  // Q = Q Z + a Q
        qi ^= 1;
      } else {
        NS_TRY(mm(R, R, R, Z, Qb[qi], c, b, a));  // Z = c R R + b R ; Q = Z + a I
      }
      if (i < iters - 1 && !in_restarts(i + 1)) {
        NS_TRY(mm(R, Z, R, RZ, nullptr, 1.f, a, 0.f));   // RZ = R Z + a R
        NS_TRY(mm(Z, RZ, RZ, R, nullptr, 1.f, a, 0.f));  // R = Z RZ + a RZ
      }
    }
    if (iters == 0) return THORN_ERR_ARG;
    // out = Q @ X; for tall inputs X^T @ Q (thorn.py:653) = (Q^T @ X)^T, stored transposed
    if (x_is_input_tall) NS_TRY(qx_tall(Qb[qi], X, out, (int64_t)m, (int64_t)m * n, true, true));
    else
      NS_TRY(qx(Qb[qi], X, ldn, n, nullptr, 0.f, out, tall ? (int64_t)m : (int64_t)n, (int64_t)m * n, tall, tall));
  } else {
    void* Xb[2] = {ws, ws + L.ms};
    void* A = ws + 2 * L.ms;
    void* Bm = ws + 3 * L.ms;
    const void* X = x;
    int xi = 0;
    if (iters == 0) return THORN_ERR_ARG;
    for (int i = 0; i < iters; ++i) {
      const float a = (float)coeffs[3 * i], b = (float)coeffs[3 * i + 1], c = (float)coeffs[3 * i + 2];
      NS_TRY(gramm(X, ldm, m, A));                         // A = X X^T
      NS_TRY(mm(A, A, A, Bm, nullptr, c, b, 0.f));         // B = c A A + b A
      const bool last = i == iters - 1;
      void* D = last ? out : Xb[xi];
      NS_TRY(qx(Bm, X, ldm, m, X, a, D, last ? (int64_t)m : ldm, last ? (int64_t)m * m : m * ldm, false,
                false));  // X = a X + B X
      X = D;
      xi ^= 1;
    }
  }
#undef NS_TRY
  return THORN_OK;
}

extern "C" int thorn_sym_addmm(const void* A, const void* B, const void* C, void* O, int64_t batch, int64_t M,
                               int64_t K, int c_batched, float alpha, float beta, int dtype, int* err_flag,
                               void* stream) {
  if (batch < 0 || M < 0 || K < 0) return THORN_ERR_ARG;
  if (batch == 0 || M == 0) return THORN_OK;
  if (batch > INT32_MAX || M > INT32_MAX || K > INT32_MAX) return THORN_ERR_ARG;
  if ((M % 8) || (K % 8)) return THORN_ERR_ALIGN;
  GemmOp op;
  op.A = A; op.a_ld = K; op.a_bs = M * K;
  op.B = B; op.b_ld = M; op.b_bs = K * M; op.b_mn = true;
  op.C = C; op.c_ld = M; op.c_bs = c_batched ? M * M : 0;
  op.D = O; op.d_ld = M; op.d_bs = M * M;
  op.M = (int)M; op.N = (int)M; op.K = (int)K; op.batch = (int)batch;
  op.alpha = alpha; op.beta = C ? beta : 0.f; op.sym = true;
  if (K == 0) return THORN_ERR_ARG;
  return run_gemm(op, dtype, err_flag, (cudaStream_t)stream);
}

extern "C" int thorn_set_gemm_pair(int enable) { return g_pair_tiles.exchange(enable ? 1 : 0); }

extern "C" int thorn_set_gemm_staged_epilogue(int enable) { return g_staged_epilogue.exchange(enable ? 1 : 0); }

extern "C" int thorn_set_gemm_pdl(int enable) { return g_gemm_pdl.exchange(enable ? 1 : 0); }

extern "C" int thorn_set_gemm_l2_hints(int enable) { return g_l2_hints.exchange(enable ? 1 : 0); }

extern "C" uint64_t thorn_set_wait_limit_ns(uint64_t limit_ns) {
  if (limit_ns == 0) limit_ns = gemm::kTimeoutNs;
  return g_wait_limit_ns.exchange(limit_ns);
}

extern "C" int thorn_set_gemm_test_stall(int enable) { return g_test_stall.exchange(enable ? 1 : 0); }

extern "C" int thorn_set_ns_small(int enable) { return g_ns_small.exchange(enable ? 1 : 0); }

// Dense-equivalent and executed tensor-core FLOPs issued so far (for roofline reports).
extern "C" void thorn_gemm_flops(double* dense, double* executed) {
  if (dense) *dense = (double)g_flops_dense.load();
  if (executed) *executed = (double)g_flops_exec.load();
}

// ===========================================================================
// Newton-Schulz without any device allocation
// ===========================================================================
// Some callers cannot hand this library a workspace: a custom call inside a
// host framework (an XLA/JAX FFI handler, for instance) receives only its
// operands and no allocator, and code that must not allocate after start-up
// cannot call cudaMalloc (it synchronises the device and can fail under memory
// pressure).  For them the NS workspace lives in this fixed device array.  It
// is part of the module image: every GPU on which the library's kernels are
// loaded holds it until the process exits.
static __device__ __align__(256) unsigned char g_ns_static_workspace[THORN_NS_STATIC_WORKSPACE_BYTES];

namespace {
// Device address of g_ns_static_workspace on the current device.  The symbol's
// name in host code is only a host-side stand-in; the address is looked up once
// per device (with that device current) and cached.
int static_workspace(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return THORN_ERR_CUDA;
  }
  static std::mutex mu;
  static void* addr[64] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_ns_static_workspace);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return THORN_ERR_CUDA;
    }
    addr[dev] = p;
  }
  *out = addr[dev];
  return THORN_OK;
}
}  // namespace

extern "C" int thorn_ns_batched_static(const void* x, void* out, int64_t batch, int64_t rows, int64_t cols,
                                       int ns_dtype, const double* coeffs, int iters, const int32_t* restarts,
                                       int n_restarts, int* err_flag, void* stream) {
  if (batch < 0 || rows < 0 || cols < 0) return THORN_ERR_ARG;
  if (batch == 0 || rows == 0 || cols == 0) return THORN_OK;
  const int64_t need = thorn_ns_workspace_bytes(batch, rows, cols);
  if (need < 0 || need > (int64_t)THORN_NS_STATIC_WORKSPACE_BYTES) return THORN_ERR_TOO_LARGE;
  void* ws = nullptr;
  const int rc = static_workspace(&ws);
  if (rc) return rc;
  return thorn_ns_batched(x, out, ws, (int64_t)THORN_NS_STATIC_WORKSPACE_BYTES, batch, rows, cols, ns_dtype, coeffs,
                          iters, restarts, n_restarts, err_flag, stream);
}
