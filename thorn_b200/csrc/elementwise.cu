// HBM-bound kernels of the THORN step: multi-tensor (R)Adam(-atan2)W, the
// orthogonalized group's momentum / NS-input / per-neuron-norm / apply passes
// and the magnitude-direction decoupling helpers.
//
// Every kernel here reads each operand once with 16-byte vector accesses and
// writes each result once.  Tensors of one call are packed into a by-value
// kernel parameter (pointer table + block prefix) so one launch covers many
// parameters; blocks find their tensor with a short scan of the prefix.
#include <atomic>
#include <mutex>
#include <math.h>
#include <type_traits>
#include <vector>

#include "common.cuh"

namespace thorn {

static std::atomic<uint64_t> g_launches{0};
static std::atomic<int> g_last_cuda_error{0};

void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int check_launch() {
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) {
    g_last_cuda_error.store((int)e);
    cudaGetLastError();
    return THORN_ERR_CUDA;
  }
  return THORN_OK;
}

// ---------------------------------------------------------------------------
// multi-tensor packing
// ---------------------------------------------------------------------------
constexpr int kThreads = 256;
constexpr int kMaxT = 24;
constexpr int64_t kMaxGrid = 1ll << 30;

template <class E>
struct Pack {
  E t[kMaxT];
  int64_t start[kMaxT + 1];
  int vec[kMaxT];
  int n;
};

template <class E>
__device__ __forceinline__ int find_tensor(const Pack<E>& pk, int64_t bid) {
  int i = 0;
  while (i + 1 < pk.n && bid >= pk.start[i + 1]) ++i;
  return i;
}

// Build packs of up to kMaxT tensors and launch `launch(pack, nblocks)` for each.
template <class E, class Blocks, class Vec, class Launch>
static int launch_packed(const E* ts, int n, Blocks blocks_of, Vec vec_of, Launch launch) {
  Pack<E> pk;
  pk.n = 0;
  int64_t total = 0;
  auto flush = [&]() -> int {
    if (pk.n == 0) return THORN_OK;
    launch(pk, total);
    count_launch();
    int st = check_launch();
    pk.n = 0;
    total = 0;
    return st;
  };
  for (int i = 0; i < n; ++i) {
    int64_t nb = blocks_of(ts[i]);
    if (nb <= 0) continue;
    if (pk.n == kMaxT || total + nb > kMaxGrid) {
      int st = flush();
      if (st) return st;
    }
    pk.t[pk.n] = ts[i];
    pk.vec[pk.n] = vec_of(ts[i]) ? 1 : 0;
    pk.start[pk.n] = total;
    total += nb;
    pk.n++;
    pk.start[pk.n] = total;
  }
  return flush();
}

static inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Bring the 128-byte line holding p into L2 ahead of its load.  The momentum
// pass issues it for the row two iterations ahead (16 rows further down the
// tile): each thread then has more DRAM requests in flight than its registers
// hold (0.5 ms less per Llama-3-8B step).  One lane per 128-byte line issues it.
// The same prefetch in the NS input, apply and finalize passes measured no gain.
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// 2-D tiling used by the matrix kernels: a tile is kTR rows x 256 columns of
// one sub-matrix; each warp owns kTR/8 rows and each lane 8 consecutive columns.
constexpr int kTR = 64;
constexpr int kTC = 256;

struct Tile {
  int64_t b, r0, c0;
};
__device__ __forceinline__ Tile tile_of(int64_t local, int64_t rows, int64_t cols) {
  const int64_t tr = (rows + kTR - 1) / kTR, tc = (cols + kTC - 1) / kTC;
  Tile t;
  t.b = local / (tr * tc);
  int64_t rem = local - t.b * tr * tc;
  t.r0 = (rem / tc) * kTR;
  t.c0 = (rem % tc) * kTC;
  return t;
}
static inline int64_t tiles_of(int64_t batch, int64_t rows, int64_t cols) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  return batch * cdiv(rows, kTR) * cdiv(cols, kTC);
}

// ===========================================================================
// (R)Adam(-atan2)W  (thorn.py:147-185, 838-888)
// ===========================================================================
constexpr int kAdamChunk = kThreads * 8 * 4;  // elements per block

struct AdamScalars {
  float w1, beta2, w2, wd, eps;  // w1 = 1 - beta1, w2 = 1 - beta2 (formed in double)
};
struct AdamArgs {
  Pack<thorn_adam_tensor> pk;
  AdamScalars s;
};

template <class P, class S>
__global__ void __launch_bounds__(kThreads) adam_kernel(const __grid_constant__ AdamArgs a) {
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_adam_tensor& e = a.pk.t[ti];
  const bool vec = a.pk.vec[ti];
  const int64_t base = (int64_t(blockIdx.x) - a.pk.start[ti]) * kAdamChunk;
  const float w1 = a.s.w1, w2 = a.s.w2;
  const P* g = (const P*)e.g;
  S* M = (S*)e.m;
  S* V = (S*)e.v;
  P* p = (P*)e.p;
#pragma unroll 1
  for (int it = 0; it < 4; ++it) {
    const int64_t i0 = base + int64_t(it) * (kThreads * 8) + threadIdx.x * 8;
    if (i0 >= e.numel) break;
    const int n = (int)min64(8, e.numel - i0);
    float gv[8], mv[8], vv[8];
    load_n(g + i0, gv, n, vec);
    load_n(M + i0, mv, n, vec);
    load_n(V + i0, vv, n, vec);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      mv[k] = mv[k] + (gv[k] - mv[k]) * w1;
      vv[k] = vv[k] * a.s.beta2 + (gv[k] * gv[k]) * w2;
    }
    store_n(M + i0, mv, n, vec);
    store_n(V + i0, vv, n, vec);
    if (p != nullptr) {
      float pv[8];
      load_n(p + i0, pv, n, vec);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float u;
        if (e.degenerate) u = mv[k];
        else if (a.s.eps == 0.f) u = atan2f(mv[k] * e.bc1, sqrtf(vv[k] * e.bc2));
        else u = (mv[k] * e.bc1) / (sqrtf(vv[k] * e.bc2) + a.s.eps);
        if (a.s.wd > 0.f && u * pv[k] >= 0.f) u = u + a.s.wd * pv[k];
        pv[k] = pv[k] - e.lr * u;
      }
      store_n(p + i0, pv, n, vec);
    }
  }
}

// ===========================================================================
// deterministic segment reductions
// ===========================================================================
// True (in every thread) for the block that arrives last on `cnt` out of
// `total` blocks.  Partials written before the call by any thread of any
// block are visible to the last block afterwards.  The last block resets the
// counter, so scratch buffers stay reusable.
__device__ __forceinline__ bool last_block(unsigned* cnt, unsigned total) {
  __shared__ int is_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = atomicAdd(cnt, 1u);
    is_last = (old == total - 1) ? 1 : 0;
    if (is_last) *cnt = 0u;
  }
  __syncthreads();
  const bool last = is_last != 0;
  if (last) __threadfence();
  return last;
}

// Fixed-order block sum of n partials (strided per thread, then a fixed tree).
// The partials are zeroed after they are read, so a scratch buffer is all
// zero again once its kernel finishes and any later call may reuse it.
__device__ __forceinline__ float ordered_sum(float* x, int64_t n, float* red) {
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    s += __ldcg(x + i);
    x[i] = 0.f;
  }
  return block_sum(s, red);
}

// Scratch of the momentum pass: counters first, then partial sums.
struct PreLayout {
  int64_t tr, tc, T;
  int64_t pn, ps, pr, pc;  // float offsets: [b][tile], [b][tile], [b][ct][r], [b][rt][c]
  int64_t bytes;
};
__host__ __device__ inline PreLayout pre_layout(int64_t B, int64_t R, int64_t C, bool md) {
  PreLayout L;
  L.tr = (R + kTR - 1) / kTR;
  L.tc = (C + kTC - 1) / kTC;
  L.T = B * L.tr * L.tc;
  L.pn = 0;
  L.ps = L.pn + (L.T + 3) / 4 * 4;
  L.pr = L.ps + (md ? (L.T + 3) / 4 * 4 : 0);
  L.pc = L.pr + (md ? (B * L.tc * R + 3) / 4 * 4 : 0);
  const int64_t nf = L.pc + (md ? B * L.tr * C : 0);
  L.bytes = nf * 4;
  return L;
}

// Scratch of a per-sub-matrix sum over 2-D tiles (post / sumsq): B counters,
// padded to 16 bytes, then B x tiles fp64 partials.
__host__ __device__ inline int64_t tiles_per_mat(int64_t R, int64_t C) {
  return ((R + kTR - 1) / kTR) * ((C + kTC - 1) / kTC);
}
__host__ __device__ inline int64_t sq_pf(int64_t B) { return (B + 3) / 4 * 4; }  // 4-byte words of counters
__host__ __device__ inline int64_t sq_bytes(int64_t B, int64_t R, int64_t C) {
  return sq_pf(B) * 4 + B * tiles_per_mat(R, C) * 8;
}

// Fixed-order fp64 block sum of n partials (each zeroed after it is read).
__device__ __forceinline__ double ordered_sum_d(double* x, int64_t n, double* red) {
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    s += __ldcg(x + i);
    x[i] = 0.0;
  }
  return block_sum_d(s, red);
}

// Sum of squares of a sub-matrix (the decouple_md renorm, thorn.py:1414-1416,
// 1716-1717): per-tile fp64 partials, then the last tile block of each
// sub-matrix writes the fixed-order fp64 sum rounded once to fp32.  The
// reference sums in fp32; fp64 keeps the sum within one rounding of the exact
// value, which the renorm's scale factor (and with it the whole parameter)
// carries straight into the update.
__device__ __forceinline__ void tile_sum_to(float* out, void* scratch, const Tile& t, int64_t B, int64_t R,
                                            int64_t C, double v, double* red) {
  unsigned* cnt = (unsigned*)scratch;
  double* part = reinterpret_cast<double*>((char*)scratch + sq_pf(B) * 4);
  const int64_t tpm = tiles_per_mat(R, C);
  const int64_t lt = (t.r0 / kTR) * ((C + kTC - 1) / kTC) + t.c0 / kTC;
  const double tot = block_sum_d(v, red);
  if (threadIdx.x == 0) part[t.b * tpm + lt] = tot;
  if (last_block(cnt + t.b, (unsigned)tpm)) {
    const double s = ordered_sum_d(part + t.b * tpm, tpm, red);
    if (threadIdx.x == 0) out[t.b] = (float)s;
  }
}

// ===========================================================================
// momentum + Nesterov (+ MD direction recovery)  (thorn.py:1376-1381, 890-908)
// ===========================================================================
// 8 consecutive fp32 values (two 16-byte loads when aligned), zero past n
__device__ __forceinline__ void load8f(const float* p, float* v, int n, bool vec) {
  if (vec && n == 8) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    return;
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = k < n ? p[k] : 0.f;
}

// u = g + beta1 * m rounded to the NS input type U for 8 elements, evaluated
// identically by the momentum pass (for the norm) and by the NS-input pass (for X).
template <class U>
__device__ __forceinline__ void nesterov_u8(const float* g, const float* m, float b1, float* u) {
#pragma unroll
  for (int k = 0; k < 8; ++k) u[k] = __fmaf_rn(b1, m[k], g[k]);
  rnd8<U>(u);
}
struct PreArgs {
  Pack<thorn_ortho_pre_tensor> pk;
  float beta1;
  int write_grad;
};

// PACKED: every tensor of the launch is a 16-bit parameter with decouple_md and
// rows of whole 16-byte chunks (the host sorts tensors into such launches), so
// the direction recovery runs as packed products only.
template <class P, class S, class U, bool MD, bool PACKED = false>
__global__ void __launch_bounds__(kThreads) ortho_pre_kernel(const __grid_constant__ PreArgs a) {
  __shared__ float red[32];
  __shared__ float colacc[MD ? 8 : 1][MD ? kTC : 1];
  constexpr bool kHalfP = !std::is_same<P, float>::value;
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_ortho_pre_tensor& e = a.pk.t[ti];
  const bool vec = a.pk.vec[ti];
  const int64_t local = int64_t(blockIdx.x) - a.pk.start[ti];
  const Tile t = tile_of(local, e.rows, e.cols);
  const PreLayout L = pre_layout(e.batch, e.rows, e.cols, MD);
  const int64_t rt = t.r0 / kTR, ct = t.c0 / kTC;
  float* sf = (float*)e.scratch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = t.c0 + lane * 8;
  const int nc = (int)max64(0, min64(8, e.cols - c));
  const float b1 = a.beta1;
  const bool scalar_gain = MD && e.scalar_gain;
  const bool momentum = e.m != nullptr;
  float sq = 0.f;
  float csum[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) csum[k] = 0.f;
  float csp[8];
  if (MD && !scalar_gain) load8f(e.col_sp + t.b * e.cols + c, csp, nc, vec);
  // 16-bit parameters in whole 16-byte chunks: the direction recovery as packed
  // products (mul2), which round exactly like the fp32 products + roundings of
  // the general path below
  static_assert(!PACKED || (MD && kHalfP), "the packed kernel serves 16-bit parameters with decouple_md");
  const bool packed = PACKED && nc == 8;
  uint32_t cs2[4] = {0u, 0u, 0u, 0u};
  if constexpr (PACKED) {
    if (packed && !scalar_gain) {
#pragma unroll
      for (int q = 0; q < 4; ++q) cs2[q] = pack2(csp[2 * q], csp[2 * q + 1], (P*)nullptr);
    }
  }
  float rsum_scalar = 0.f;
  for (int rr = warp; rr < kTR; rr += 8) {
    const int64_t r = t.r0 + rr;
    if (r >= e.rows) break;
    if (rr + 16 < kTR && r + 16 < e.rows && nc > 0) {  // this warp's row two iterations ahead
      const int64_t offp = (t.b * e.rows + r + 16) * e.cols + c;
      if (momentum && (lane & (16 / sizeof(S) - 1)) == 0) prefetch_l2((const S*)e.m + offp);
      if ((lane & (16 / sizeof(P) - 1)) == 0) {
        prefetch_l2((const P*)e.g + offp);
        if (MD) prefetch_l2((const P*)e.p + offp);
      }
    }
    float rs = 0.f;
    if (nc > 0) {
      const int64_t off = (t.b * e.rows + r) * e.cols + c;
      float gv[8], mv[8];
      if (momentum) load_n((const S*)e.m + off, mv, nc, vec);
      if constexpr (PACKED) {
        if (packed) {
          const uint4 g4 = *reinterpret_cast<const uint4*>((const P*)e.g + off);
          const uint4 p4 = *reinterpret_cast<const uint4*>((const P*)e.p + off);
          const float rsp = scalar_gain ? e.row_sp[0] : e.row_sp[t.b * e.rows + r];
          const uint32_t rs2 = pack2(rsp, rsp, (P*)nullptr);
          const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w}, pw[4] = {p4.x, p4.y, p4.z, p4.w};
          uint32_t pvo[4], geo[4];
          float part = 0.f;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t gain2 = scalar_gain ? rs2 : mul2<P>(rs2, cs2[q]);  // gain = rs cs
            float p0, p1, d0, d1;
            unpack2(pw[q], p0, p1, (P*)nullptr);
            unpack2(gain2, d0, d1, (P*)nullptr);
            // fast division (<= 2 fp32 ulp) before the rounding to the param dtype
            pvo[q] = pack2(__fdividef(p0, d0), __fdividef(p1, d1), (P*)nullptr);  // p /= gain
            const uint32_t pg2 = mul2<P>(pvo[q], gw[q]);                           // p_g = p g
            if (scalar_gain) {
              float a0, a1;
              unpack2(pg2, a0, a1, (P*)nullptr);
              part = __fadd_rn(__fadd_rn(part, a0), a1);
            } else {
              float c0, c1, r0, r1;
              unpack2(mul2<P>(pg2, cs2[q]), c0, c1, (P*)nullptr);  // p_g * col gain (row-gain gradient)
              unpack2(mul2<P>(pg2, rs2), r0, r1, (P*)nullptr);     // p_g * row gain (column-gain gradient)
              part = __fadd_rn(__fadd_rn(part, c0), c1);
              csum[2 * q] = __fadd_rn(csum[2 * q], r0);
              csum[2 * q + 1] = __fadd_rn(csum[2 * q + 1], r1);
            }
            geo[q] = mul2<P>(gw[q], gain2);  // g *= gain
            unpack2(geo[q], gv[2 * q], gv[2 * q + 1], (P*)nullptr);
          }
          rs = part;
          *reinterpret_cast<uint4*>((P*)e.p + off) = make_uint4(pvo[0], pvo[1], pvo[2], pvo[3]);
          if (a.write_grad) *reinterpret_cast<uint4*>((P*)e.g + off) = make_uint4(geo[0], geo[1], geo[2], geo[3]);
        }
      }
      if constexpr (!PACKED) {
        load_n((const P*)e.g + off, gv, nc, vec);
        if (MD) {
          // every step below rounds 8 values to the param dtype at once (packed
          // conversions); lanes k >= nc hold padding and are neither summed nor stored
          float pv[8], gain[8], pg[8];
          load_n((const P*)e.p + off, pv, nc, vec);
          const float rsp = scalar_gain ? e.row_sp[0] : e.row_sp[t.b * e.rows + r];
#pragma unroll
          for (int k = 0; k < 8; ++k) gain[k] = scalar_gain ? rsp : __fmul_rn(rsp, csp[k]);
          if (!scalar_gain) rnd8<P>(gain);
          // fast division (<= 2 fp32 ulp) before the rounding to the param dtype
#pragma unroll
          for (int k = 0; k < 8; ++k) pv[k] = __fdividef(pv[k], gain[k]);
          rnd8<P>(pv);
#pragma unroll
          for (int k = 0; k < 8; ++k) pg[k] = __fmul_rn(pv[k], gv[k]);
          rnd8<P>(pg);
          float part = 0.f;
          if (scalar_gain) {
#pragma unroll
            for (int k = 0; k < 8; ++k)
              if (k < nc) part = __fadd_rn(part, pg[k]);
          } else {
            float pc[8], pr[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              pc[k] = __fmul_rn(pg[k], csp[k]);
              pr[k] = __fmul_rn(pg[k], rsp);
            }
            rnd8<P>(pc);
            rnd8<P>(pr);
#pragma unroll
            for (int k = 0; k < 8; ++k)
              if (k < nc) {
                part = __fadd_rn(part, pc[k]);
                csum[k] = __fadd_rn(csum[k], pr[k]);
              }
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) gv[k] = __fmul_rn(gv[k], gain[k]);
          rnd8<P>(gv);
          rs = part;
          store_n((P*)e.p + off, pv, nc, vec);
          if (a.write_grad) store_n((P*)e.g + off, gv, nc, vec);
        }
      }
      if (momentum) {
        float u[8];
        // m = m * beta1 + g as two rounded torch ops (thorn.py:1376-1381): no fma
#pragma unroll
        for (int k = 0; k < 8; ++k) mv[k] = __fmul_rn(mv[k], b1);
        rnd8<S>(mv);
#pragma unroll
        for (int k = 0; k < 8; ++k) mv[k] = __fadd_rn(mv[k], gv[k]);
        rnd8<S>(mv);
        nesterov_u8<U>(gv, mv, b1, u);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k < nc) sq = __fmaf_rn(u[k], u[k], sq);
        store_n((S*)e.m + off, mv, nc, vec);
      }
    }
    if (MD) {
      rs = warp_sum(rs);
      if (scalar_gain) rsum_scalar += rs;
      else if (lane == 0) sf[L.pr + (t.b * L.tc + ct) * e.rows + r] = rs;
    }
  }
  const int64_t gt = (t.b * L.tr + rt) * L.tc + ct;  // tile index within the tensor
  if (momentum) {
    const float tot = block_sum(sq, red);
    if (threadIdx.x == 0) sf[L.pn + gt] = tot;
  }
  if (MD) {
    if (scalar_gain) {
      const float s2 = block_sum(lane == 0 ? rsum_scalar : 0.f, red);
      if (threadIdx.x == 0) sf[L.ps + gt] = s2;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) colacc[warp][lane * 8 + k] = csum[k];
      __syncthreads();
      const int cc = threadIdx.x;  // one column per thread (kTC == kThreads)
      if (t.c0 + cc < e.cols) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) s += colacc[w][cc];
        sf[L.pc + (t.b * L.tr + rt) * e.cols + t.c0 + cc] = s;
      }
    }
  }
}

// Fixed-order sums of the momentum pass's partials (no atomics in the pass
// itself).  Blocks per tensor and batch: one for the sum of squares (and a
// scalar gain), ceil(rows/256) for row-gain sums, ceil(cols/256) for
// column-gain sums.  Every partial read is zeroed again.
struct PreRedArgs {
  Pack<thorn_ortho_pre_tensor> pk;
  int md;
};
__host__ __device__ inline int64_t pre_red_blocks(int64_t B, int64_t R, int64_t C, bool split) {
  return B * (1 + (split ? (R + 255) / 256 + (C + 255) / 256 : 0));
}

// Sequential sum of x[0], x[stride], ..., x[(n-1)*stride] (each zeroed after it
// is read), with eight loads in flight per thread.
__device__ __forceinline__ float strided_sum(float* x, int64_t stride, int64_t n) {
  float s = 0.f;
  int64_t i = 0;
  for (; i + 8 <= n; i += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldcg(x + (i + j) * stride);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x[(i + j) * stride] = 0.f;
      s += v[j];
    }
  }
  for (; i < n; ++i) {
    s += __ldcg(x + i * stride);
    x[i * stride] = 0.f;
  }
  return s;
}

__global__ void __launch_bounds__(kThreads) pre_reduce_kernel(const __grid_constant__ PreRedArgs a) {
  __shared__ float red[32];
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_ortho_pre_tensor& e = a.pk.t[ti];
  const bool md = a.md != 0;
  const bool split = md && !e.scalar_gain;
  const PreLayout L = pre_layout(e.batch, e.rows, e.cols, md);
  float* sf = (float*)e.scratch;
  const int64_t per_b = pre_red_blocks(1, e.rows, e.cols, split);
  const int64_t local = int64_t(blockIdx.x) - a.pk.start[ti];
  const int64_t b = local / per_b;
  int64_t k = local - b * per_b;
  const int64_t tpm = L.tr * L.tc;
  if (k == 0) {
    if (e.m != nullptr) {
      const float s = ordered_sum(sf + L.pn + b * tpm, tpm, red);
      if (threadIdx.x == 0) e.normsq[b] = s;
    }
    if (md && !split && b == 0) {  // a scalar gain sums over the whole tensor
      const float s = ordered_sum(sf + L.ps, L.T, red);
      if (threadIdx.x == 0) e.row_gsum[0] = s;
    }
    return;
  }
  k -= 1;
  const int64_t nrb = (e.rows + 255) / 256;
  if (k < nrb) {
    const int64_t r = k * 256 + threadIdx.x;
    if (r < e.rows) e.row_gsum[b * e.rows + r] = strided_sum(sf + L.pr + b * L.tc * e.rows + r, e.rows, L.tc);
    return;
  }
  k -= nrb;
  const int64_t cc = k * 256 + threadIdx.x;
  if (cc < e.cols) e.col_gsum[b * e.cols + cc] = strided_sum(sf + L.pc + b * L.tr * e.cols + cc, e.cols, L.tr);
}

// ===========================================================================
// NS input: normalise + cast (+ transpose tall sub-matrices)  (thorn.py:629-635)
// ===========================================================================
struct CastArgs {
  Pack<thorn_ns_cast_tensor> pk;
  float beta1;
};


template <class P, class S, class U, class X>
__global__ void __launch_bounds__(kThreads) ns_cast_kernel(const __grid_constant__ CastArgs a) {
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_ns_cast_tensor& e = a.pk.t[ti];
  const bool vec = a.pk.vec[ti];
  const Tile t = tile_of(int64_t(blockIdx.x) - a.pk.start[ti], e.rows, e.cols);
  const float d = sqrtf(e.normsq[t.b]) + 1e-8f;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = t.c0 + lane * 8;
  const int nc = (int)max64(0, min64(8, e.cols - c));
  if (nc == 0) return;
  const int64_t ld = ns_ld(e.cols);
  const P* G = (const P*)e.g;
  const S* M = (const S*)e.m;
  // u / (||u|| + 1e-8) as an IEEE division, like the reference (thorn.py:633),
  // then one rounding to the 16-bit NS type
  const bool md = e.md != 0;
  const bool split = md && !e.scalar_gain;
  float csp[8];
  if (split) load8f(e.col_sp + t.b * e.cols + c, csp, nc, vec);
  for (int rr = warp; rr < kTR; rr += 8) {
    const int64_t r = t.r0 + rr;
    if (r >= e.rows) break;
    const int64_t off = (t.b * e.rows + r) * e.cols + c;
    float gv[8], mv[8], v[8];
    load_n(G + off, gv, nc, vec);
    load_n(M + off, mv, nc, vec);
    const float rsp = md ? (split ? e.row_sp[t.b * e.rows + r] : e.row_sp[0]) : 1.f;
    if (md) {  // the gradient times its magnitude gain, as the momentum pass formed it
      float gain[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) gain[k] = split ? __fmul_rn(rsp, csp[k]) : rsp;
      if (split) rnd8<P>(gain);
#pragma unroll
      for (int k = 0; k < 8; ++k) gv[k] = __fmul_rn(gv[k], gain[k]);
      rnd8<P>(gv);
    }
    nesterov_u8<U>(gv, mv, a.beta1, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __fdiv_rn(v[k], d);
    store_n((X*)e.x + (t.b * e.rows + r) * ld + c, v, nc, vec);
  }
}

// ===========================================================================
// per-neuron norm statistics (thorn.py:205-253)
// ===========================================================================
struct PnnArgs {
  Pack<thorn_pnn_tensor> pk;
  float eps;
};
constexpr int kPnnRowsPerBlock = 8;
__host__ __device__ inline int64_t pnn_pf(int64_t B) { return (B + 3) / 4 * 4; }

template <class U, class P>
__global__ void __launch_bounds__(kThreads) pnn_stats_kernel(const __grid_constant__ PnnArgs a) {
  __shared__ float red[32];
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_pnn_tensor& e = a.pk.t[ti];
  const bool vec = a.pk.vec[ti];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nrb = (e.rows + kPnnRowsPerBlock - 1) / kPnnRowsPerBlock;  // row blocks per matrix
  const int64_t local = int64_t(blockIdx.x) - a.pk.start[ti];
  const int64_t b = local / nrb, rb = local - b * nrb;
  const int64_t r = rb * kPnnRowsPerBlock + warp;
  unsigned* cnt = (unsigned*)e.scratch;
  float* rsq = (float*)e.scratch + pnn_pf(e.batch);  // [batch*rows] sumsq_r
  float* rss = rsq + e.batch * e.rows;                 // [batch*rows] s_r^2 sumsq_r
  if (r < e.rows) {
    const U* row = (const U*)e.U + (b * e.rows + r) * e.cols;
    float s = 0.f;
    for (int64_t c = lane * 8; c < e.cols; c += 256) {
      const int n = (int)min64(8, e.cols - c);
      float v[8];
      load_n(row + c, v, n, vec);
      rnd8<P>(v);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < n) s += v[k] * v[k];
    }
    s = warp_sum(s);
    if (lane == 0) {
      const float inv_n = 1.f / (float)e.cols;
      const float sc = rsqrtf(fmaxf(s * inv_n, a.eps));
      e.row_scale[b * e.rows + r] = sc;
      rsq[b * e.rows + r] = s;
      rss[b * e.rows + r] = sc * sc * s;
    }
  }
  if (last_block(cnt + b, (unsigned)nrb)) {
    const float s0 = ordered_sum(rsq + b * e.rows, e.rows, red);
    const float s1 = ordered_sum(rss + b * e.rows, e.rows, red);
    if (threadIdx.x == 0) {
      e.mat_stats[2 * b] = s0;
      e.mat_stats[2 * b + 1] = s1;
    }
    if (e.fold) {
      const float gscale = sqrtf(s0) / fmaxf(sqrtf(s1), a.eps);
      for (int64_t i = threadIdx.x; i < e.rows; i += blockDim.x) {
        float* q = e.row_scale + b * e.rows + i;
        *q = __ldcg(q) * gscale;
      }
    }
  }
}

// ===========================================================================
// apply: pnn scaling + cautious weight decay + update  (thorn.py:187-203, 255-280)
// ===========================================================================
struct PostArgs {
  Pack<thorn_ortho_post_tensor> pk;
  float wd, eps;
};

template <class U, class P>
__global__ void __launch_bounds__(kThreads) ortho_post_kernel(const __grid_constant__ PostArgs a) {
  __shared__ double red[32];
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_ortho_post_tensor& e = a.pk.t[ti];
  const bool vec = a.pk.vec[ti];
  const Tile t = tile_of(int64_t(blockIdx.x) - a.pk.start[ti], e.rows, e.cols);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = t.c0 + lane * 8;
  const int nc = (int)max64(0, min64(8, e.cols - c));
  float gscale = 1.f;
  if (e.mat_stats != nullptr) {
    gscale = sqrtf(e.mat_stats[2 * t.b]) / fmaxf(sqrtf(e.mat_stats[2 * t.b + 1]), a.eps);
  }
  double sq = 0.0;
  for (int rr = warp; rr < kTR; rr += 8) {
    const int64_t r = t.r0 + rr;
    if (r >= e.rows || nc == 0) break;
    const int64_t off = (t.b * e.rows + r) * e.cols + c;
    float scale = 1.f;
    if (e.row_scale != nullptr) scale = e.row_scale[t.b * e.rows + r] * gscale;
    float uv[8], pv[8];
    load_n((const U*)e.U + off, uv, nc, vec);
    load_n((const P*)e.p + off, pv, nc, vec);
    if (e.round_u) rnd8<P>(uv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float u = uv[k];
      if (e.row_scale != nullptr) u = u * scale;
      if (a.wd > 0.f && u * pv[k] >= 0.f) u = u + a.wd * pv[k];
      pv[k] = pv[k] - e.lr * u;
    }
    rnd8<P>(pv);
    if (e.p_normsq != nullptr) {
      // eight squares in fp32 (each exact for a 16-bit parameter), their sum into fp64
      float s8 = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < nc) s8 = __fmaf_rn(pv[k], pv[k], s8);
      sq += (double)s8;
    }
    store_n((P*)e.p + off, pv, nc, vec);
  }
  if (e.p_normsq != nullptr) tile_sum_to(e.p_normsq, e.scratch, t, e.batch, e.rows, e.cols, sq, red);
}

// ===========================================================================
// MD helpers (thorn.py:910-977, 1414-1421)
// ===========================================================================
struct MdPrepArgs {
  Pack<thorn_md_prep_tensor> pk;
};
struct MdGradArgs {
  Pack<thorn_md_grad_tensor> pk;
};

template <class P>
__global__ void __launch_bounds__(kThreads) md_prep_kernel(const __grid_constant__ MdPrepArgs a) {
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_md_prep_tensor& e = a.pk.t[ti];
  const int64_t i = (int64_t(blockIdx.x) - a.pk.start[ti]) * kThreads + threadIdx.x;
  if (i >= e.n) return;
  const float x = to_f(((const P*)e.gain)[i]);
  const float s = x > 20.f ? x : log1pf(expf(x));  // F.softplus(beta=1, threshold=20)
  e.sp[i] = rnd<P>(s);
  if (e.sig) e.sig[i] = rnd<P>(1.f / (1.f + expf(-x)));
}

template <class P>
__global__ void __launch_bounds__(kThreads) md_gain_grad_kernel(const __grid_constant__ MdGradArgs a) {
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_md_grad_tensor& e = a.pk.t[ti];
  const int64_t i = (int64_t(blockIdx.x) - a.pk.start[ti]) * kThreads + threadIdx.x;
  if (i >= e.n) return;
  ((P*)e.grad)[i] = from_f<P>(rnd<P>(e.gsum[i]) * e.sig[i]);
}

struct FinalArgs {
  Pack<thorn_md_final_tensor> pk;
};

template <class P>
__global__ void __launch_bounds__(kThreads) md_finalize_kernel(const __grid_constant__ FinalArgs a) {
  constexpr bool kHalfP = !std::is_same<P, float>::value;
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_md_final_tensor& e = a.pk.t[ti];
  const bool vec = a.pk.vec[ti];
  const Tile t = tile_of(int64_t(blockIdx.x) - a.pk.start[ti], e.rows, e.cols);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = t.c0 + lane * 8;
  const int nc = (int)max64(0, min64(8, e.cols - c));
  if (nc == 0) return;
  float f = 1.f;
  const bool renorm = e.normsq != nullptr;
  if (renorm) {
    float nrm = rnd<P>(sqrtf(e.normsq[t.b]));
    float tgt = e.target[t.b * e.target_stride];
    f = rnd<P>(tgt / rnd<P>(nrm + 1e-8f));
  }
  const bool split = !e.scalar_gain;
  float csp[8];
  if (split) load8f(e.col_sp + t.b * e.cols + c, csp, nc, vec);
  if constexpr (kHalfP) {
    if (vec && nc == 8) {
      // every factor (renorm scale, row gain, column gain) is a value of P, so each
      // multiply-and-round is one packed product
      const uint32_t f2 = pack2(f, f, (P*)nullptr);
      uint32_t cs2[4] = {0u, 0u, 0u, 0u};
      if (split) {
#pragma unroll
        for (int q = 0; q < 4; ++q) cs2[q] = pack2(csp[2 * q], csp[2 * q + 1], (P*)nullptr);
      }
      for (int rr = warp; rr < kTR; rr += 8) {
        const int64_t r = t.r0 + rr;
        if (r >= e.rows) break;
        P* pp = (P*)e.p + (t.b * e.rows + r) * e.cols + c;
        const uint4 p4 = *reinterpret_cast<const uint4*>(pp);
        const float rsp = split ? e.row_sp[t.b * e.rows + r] : e.row_sp[0];
        const uint32_t rs2 = pack2(rsp, rsp, (P*)nullptr);
        uint32_t w[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (renorm) w[q] = mul2<P>(w[q], f2);
          w[q] = mul2<P>(w[q], rs2);
          if (split) w[q] = mul2<P>(w[q], cs2[q]);
        }
        *reinterpret_cast<uint4*>(pp) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      return;
    }
  }
  for (int rr = warp; rr < kTR; rr += 8) {
    const int64_t r = t.r0 + rr;
    if (r >= e.rows) break;
    const int64_t off = (t.b * e.rows + r) * e.cols + c;
    float pv[8];
    load_n((const P*)e.p + off, pv, nc, vec);
    const float rsp = split ? e.row_sp[t.b * e.rows + r] : e.row_sp[0];
    if (renorm) {
#pragma unroll
      for (int k = 0; k < 8; ++k) pv[k] = __fmul_rn(pv[k], f);
      rnd8<P>(pv);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) pv[k] = __fmul_rn(pv[k], rsp);
    rnd8<P>(pv);
    if (split) {
#pragma unroll
      for (int k = 0; k < 8; ++k) pv[k] = __fmul_rn(pv[k], csp[k]);
      rnd8<P>(pv);
    }
    store_n((P*)e.p + off, pv, nc, vec);
  }
}

struct SumsqArgs {
  Pack<thorn_sumsq_tensor> pk;
};

template <class T>
__global__ void __launch_bounds__(kThreads) sumsq_kernel(const __grid_constant__ SumsqArgs a) {
  __shared__ double red[32];
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_sumsq_tensor& e = a.pk.t[ti];
  const bool vec = a.pk.vec[ti];
  const Tile t = tile_of(int64_t(blockIdx.x) - a.pk.start[ti], e.rows, e.cols);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = t.c0 + lane * 8;
  const int nc = (int)max64(0, min64(8, e.cols - c));
  double sq = 0.0;
  for (int rr = warp; rr < kTR; rr += 8) {
    const int64_t r = t.r0 + rr;
    if (r >= e.rows || nc == 0) break;
    float v[8];
    load_n((const T*)e.x + (t.b * e.rows + r) * e.cols + c, v, nc, vec);
    float s8 = 0.f;  // eight squares in fp32, their sum into fp64
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k < nc) s8 = __fmaf_rn(v[k], v[k], s8);
    sq += (double)s8;
  }
  tile_sum_to(e.out, e.scratch, t, e.batch, e.rows, e.cols, sq, red);
}

// ===========================================================================
// Magma statistics  (thorn.py:806-829, with the direction recovery of 896-905)
// ===========================================================================
// Scratch: one counter (padded to 16 bytes), then 3 fp64 partials per tile.
__host__ __device__ inline int64_t magma_bytes(int64_t B, int64_t R, int64_t C) {
  return 16 + 3 * B * tiles_per_mat(R, C) * 8;
}

struct MagmaArgs {
  Pack<thorn_magma_tensor> pk;
};

// softplus(beta=1, threshold=20) rounded to the gain dtype, as F.softplus
template <class G>
__device__ __forceinline__ float softplus_g(const G* gain, int64_t i) {
  const float x = to_f(gain[i]);
  return rnd<G>(x > 20.f ? x : log1pf(expf(x)));
}

// Each tile block sums g'*m, g'^2 and m^2 of its 64 x 256 tile (fp32 sums of eight
// products, accumulated in fp64) and stores three partials; the last block of the
// tensor adds all partials in tile order and writes the three fp64 totals.
template <class G, class M>
__global__ void __launch_bounds__(kThreads) magma_stats_kernel(const __grid_constant__ MagmaArgs a) {
  __shared__ double red[32];
  const int ti = find_tensor(a.pk, blockIdx.x);
  const thorn_magma_tensor& e = a.pk.t[ti];
  const bool vec = a.pk.vec[ti];
  const int64_t lt = int64_t(blockIdx.x) - a.pk.start[ti];
  const Tile t = tile_of(lt, e.rows, e.cols);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = t.c0 + lane * 8;
  const int nc = (int)max64(0, min64(8, e.cols - c));
  const G* rg = (const G*)e.row_gain;
  const G* cg = (const G*)e.col_gain;
  float csp[8];  // softplus of this lane's column gains (split gain), or the scalar gain in csp[0]
#pragma unroll
  for (int k = 0; k < 8; ++k) csp[k] = 1.f;
  if (rg != nullptr) {
    if (e.scalar_gain) {
      csp[0] = softplus_g(rg, 0);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < nc) csp[k] = softplus_g(cg, t.b * e.cols + c + k);
    }
  }
  double dot = 0.0, gg = 0.0, mm = 0.0;
  for (int rr = warp; rr < kTR; rr += 8) {
    const int64_t r = t.r0 + rr;
    if (r >= e.rows || nc == 0) break;
    const int64_t off = (t.b * e.rows + r) * e.cols + c;
    float g[8], m[8];
    load_n((const G*)e.g + off, g, nc, vec);
    load_n((const M*)e.m + off, m, nc, vec);
    if (rg != nullptr) {
      if (e.scalar_gain) {
#pragma unroll
        for (int k = 0; k < 8; ++k) g[k] = rnd<G>(__fmul_rn(g[k], csp[0]));
      } else {
        const float rsp = softplus_g(rg, t.b * e.rows + r);
#pragma unroll
        for (int k = 0; k < 8; ++k) g[k] = rnd<G>(__fmul_rn(g[k], rnd<G>(__fmul_rn(rsp, csp[k]))));
      }
    }
    float d8 = 0.f, g8 = 0.f, m8 = 0.f;  // zero past nc: load_n fills 0
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      d8 = __fmaf_rn(g[k], m[k], d8);
      g8 = __fmaf_rn(g[k], g[k], g8);
      m8 = __fmaf_rn(m[k], m[k], m8);
    }
    dot += (double)d8;
    gg += (double)g8;
    mm += (double)m8;
  }
  unsigned* cnt = (unsigned*)e.scratch;
  double* part = reinterpret_cast<double*>((char*)e.scratch + 16);
  const int64_t T = a.pk.start[ti + 1] - a.pk.start[ti];
  const double sd = block_sum_d(dot, red);
  const double sg = block_sum_d(gg, red);
  const double sm = block_sum_d(mm, red);
  if (threadIdx.x == 0) {
    part[lt] = sd;
    part[T + lt] = sg;
    part[2 * T + lt] = sm;
  }
  if (last_block(cnt, (unsigned)T)) {
    const double td = ordered_sum_d(part, T, red);
    const double tg = ordered_sum_d(part + T, T, red);
    const double tm = ordered_sum_d(part + 2 * T, T, red);
    if (threadIdx.x == 0) {
      e.out[0] = td;
      e.out[1] = tg;
      e.out[2] = tm;
    }
  }
}

// ---------------------------------------------------------------------------
// dispatch helpers
// ---------------------------------------------------------------------------
template <class F>
static int dispatch1(int dt, F f) {
  switch (dt) {
    case THORN_F32: f((float*)nullptr); return THORN_OK;
    case THORN_BF16: f((__nv_bfloat16*)nullptr); return THORN_OK;
    case THORN_F16: f((__half*)nullptr); return THORN_OK;
  }
  return THORN_ERR_ARG;
}
template <class F>
static int dispatch2(int a, int b, F f) {
  int st = THORN_OK;
  int r = dispatch1(a, [&](auto* pa) {
    int r2 = dispatch1(b, [&](auto* pb) { f(pa, pb); });
    if (r2) st = r2;
  });
  return r ? r : st;
}
static bool valid_dt(int d) { return d == THORN_F32 || d == THORN_BF16 || d == THORN_F16; }
static size_t dt_size(int d) { return d == THORN_F32 ? 4 : 2; }
static float dt_eps(int d) {
  return d == THORN_F32 ? 1.1920928955078125e-07f : (d == THORN_BF16 ? 0.0078125f : 0.0009765625f);
}

}  // namespace thorn

using namespace thorn;

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" int thorn_abi_version(void) { return 1; }

extern "C" int64_t thorn_ns_ld(int64_t n) { return ns_ld(n); }

extern "C" const char* thorn_status_string(int s) {
  switch (s) {
    case THORN_OK: return "ok";
    case THORN_ERR_ARG: return "invalid argument";
    case THORN_ERR_ALIGN: return "misaligned pointer or leading dimension";
    case THORN_ERR_CUDA: return "CUDA error";
    case THORN_ERR_UNSUPPORTED: return "unsupported device or configuration";
    case THORN_ERR_TOO_LARGE: return "problem needs more than the 64 MiB static NS workspace";
  }
  return "unknown status";
}

extern "C" uint64_t thorn_launch_count(void) { return g_launches.load(); }
extern "C" int thorn_last_cuda_error(void) { return g_last_cuda_error.load(); }

extern "C" int thorn_adamw_multi(const thorn_adam_tensor* ts, int n, int p_dtype, int s_dtype, double beta1,
                                 double beta2, float weight_decay, float eps, void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(p_dtype) || !valid_dt(s_dtype)) return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i)
    if (ts[i].numel < 0 || (ts[i].numel > 0 && (!ts[i].g || !ts[i].m || !ts[i].v))) return THORN_ERR_ARG;
  AdamScalars sc{(float)(1.0 - beta1), (float)beta2, (float)(1.0 - beta2), weight_decay, eps};
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  int d = dispatch2(p_dtype, s_dtype, [&](auto* pp, auto* ps) {
    using P = std::remove_pointer_t<decltype(pp)>;
    using S = std::remove_pointer_t<decltype(ps)>;
    rc = launch_packed(
        ts, n, [](const thorn_adam_tensor& e) { return cdiv(e.numel, kAdamChunk); },
        [](const thorn_adam_tensor& e) {
          return aligned16(e.g) && aligned16(e.m) && aligned16(e.v) && (e.p == nullptr || aligned16(e.p));
        },
        [&](const Pack<thorn_adam_tensor>& pk, int64_t nb) {
          AdamArgs a;
          a.pk = pk;
          a.s = sc;
          adam_kernel<P, S><<<(unsigned)nb, kThreads, 0, st>>>(a);
        });
  });
  return d ? d : rc;
}

extern "C" int thorn_ortho_pre_multi(const thorn_ortho_pre_tensor* ts, int n, int p_dtype, int s_dtype,
                                     int u_dtype, float beta1, int md, int write_grad, void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(p_dtype) || !valid_dt(s_dtype) || !valid_dt(u_dtype))
    return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i) {
    const auto& e = ts[i];
    if (e.batch < 0 || e.rows < 0 || e.cols < 0) return THORN_ERR_ARG;
    if (e.batch * e.rows * e.cols > 0 && (!e.g || (e.m && !e.normsq) || (!e.m && !md) || (md && !e.p) || !e.scratch))
      return THORN_ERR_ARG;
    if (e.batch * e.rows * e.cols > 0 && md &&
        (!e.row_gsum || !e.row_sp || (!e.scalar_gain && (!e.col_sp || !e.col_gsum))))
      return THORN_ERR_ARG;
  }
  PreArgs base;
  base.beta1 = beta1;
  base.write_grad = write_grad;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  auto blocks = [](const thorn_ortho_pre_tensor& e) { return tiles_of(e.batch, e.rows, e.cols); };
  auto vec = [](const thorn_ortho_pre_tensor& e) {
    return (e.cols % 8) == 0 && (e.p == nullptr || aligned16(e.p)) && aligned16(e.g) &&
           (e.m == nullptr || aligned16(e.m));
  };
  int d = dispatch2(p_dtype, s_dtype, [&](auto* pp, auto* ps) {
    using P = std::remove_pointer_t<decltype(pp)>;
    using S = std::remove_pointer_t<decltype(ps)>;
    int d2 = dispatch1(u_dtype, [&](auto* pu) {
      using U = std::remove_pointer_t<decltype(pu)>;
      bool split_done = false;
      if constexpr (!std::is_same<P, float>::value) {
        if (md) {
          // tensors whose rows are whole 16-byte chunks take the packed kernel, the rest the general one
          std::vector<thorn_ortho_pre_tensor> whole, rest;
          for (int i = 0; i < n; ++i) (vec(ts[i]) ? whole : rest).push_back(ts[i]);
          rc = launch_packed(whole.data(), (int)whole.size(), blocks, vec,
                             [&](const Pack<thorn_ortho_pre_tensor>& pk, int64_t nb) {
                               PreArgs a = base;
                               a.pk = pk;
                               ortho_pre_kernel<P, S, U, true, true><<<(unsigned)nb, kThreads, 0, st>>>(a);
                             });
          if (rc == THORN_OK)
            rc = launch_packed(rest.data(), (int)rest.size(), blocks, vec,
                               [&](const Pack<thorn_ortho_pre_tensor>& pk, int64_t nb) {
                                 PreArgs a = base;
                                 a.pk = pk;
                                 ortho_pre_kernel<P, S, U, true><<<(unsigned)nb, kThreads, 0, st>>>(a);
                               });
          split_done = true;
        }
      }
      if (!split_done)
        rc = launch_packed(ts, n, blocks, vec, [&](const Pack<thorn_ortho_pre_tensor>& pk, int64_t nb) {
          PreArgs a = base;
          a.pk = pk;
          if (md) ortho_pre_kernel<P, S, U, true><<<(unsigned)nb, kThreads, 0, st>>>(a);
          else ortho_pre_kernel<P, S, U, false><<<(unsigned)nb, kThreads, 0, st>>>(a);
        });
      if (rc == THORN_OK) {
        rc = launch_packed(
            ts, n,
            [md](const thorn_ortho_pre_tensor& e) -> int64_t {
              if (e.batch <= 0 || e.rows <= 0 || e.cols <= 0) return 0;
              return pre_red_blocks(e.batch, e.rows, e.cols, md && !e.scalar_gain);
            },
            [](const thorn_ortho_pre_tensor&) { return false; },
            [&](const Pack<thorn_ortho_pre_tensor>& pk, int64_t nb) {
              PreRedArgs a;
              a.pk = pk;
              a.md = md;
              pre_reduce_kernel<<<(unsigned)nb, kThreads, 0, st>>>(a);
            });
      }
    });
    if (d2) rc = d2;
  });
  return d ? d : rc;
}

extern "C" int thorn_ns_cast_multi(const thorn_ns_cast_tensor* ts, int n, int p_dtype, int s_dtype, int u_dtype,
                                   int ns_dtype, float beta1, void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(p_dtype) || !valid_dt(s_dtype) || !valid_dt(u_dtype) ||
      (ns_dtype != THORN_F16 && ns_dtype != THORN_BF16))
    return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i) {
    const auto& e = ts[i];
    if (e.batch < 0 || e.rows < 0 || e.cols < 0) return THORN_ERR_ARG;
    if (e.batch * e.rows * e.cols > 0 && (!e.g || !e.m || !e.x || !e.normsq)) return THORN_ERR_ARG;
    if (e.batch * e.rows * e.cols > 0 && e.md && (!e.row_sp || (!e.scalar_gain && !e.col_sp))) return THORN_ERR_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  auto blocks = [](const thorn_ns_cast_tensor& e) { return tiles_of(e.batch, e.rows, e.cols); };
  auto vec = [](const thorn_ns_cast_tensor& e) {
    return (e.cols % 8) == 0 && aligned16(e.g) && aligned16(e.m) && aligned16(e.x);
  };
  int d = dispatch2(p_dtype, s_dtype, [&](auto* pp, auto* ps) {
    using P = std::remove_pointer_t<decltype(pp)>;
    using S = std::remove_pointer_t<decltype(ps)>;
    int d2 = dispatch2(u_dtype, ns_dtype, [&](auto* pu, auto* px) {
      using U = std::remove_pointer_t<decltype(pu)>;
      using X = std::remove_pointer_t<decltype(px)>;
      if constexpr (std::is_same<X, float>::value) {
        rc = THORN_ERR_ARG;
      } else {
        rc = launch_packed(ts, n, blocks, vec, [&](const Pack<thorn_ns_cast_tensor>& pk, int64_t nb) {
          CastArgs a;
          a.pk = pk;
          a.beta1 = beta1;
          ns_cast_kernel<P, S, U, X><<<(unsigned)nb, kThreads, 0, st>>>(a);
        });
      }
    });
    if (d2) rc = d2;
  });
  return d ? d : rc;
}

extern "C" int thorn_pnn_stats_multi(const thorn_pnn_tensor* ts, int n, int u_dtype, int p_dtype, void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(u_dtype) || !valid_dt(p_dtype)) return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i)
    if (ts[i].batch * ts[i].rows * ts[i].cols > 0 && (!ts[i].U || !ts[i].row_scale || !ts[i].mat_stats || !ts[i].scratch))
      return THORN_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  const float eps = dt_eps(p_dtype);
  auto blocks = [](const thorn_pnn_tensor& e) -> int64_t {
    if (e.batch <= 0 || e.rows <= 0 || e.cols <= 0) return 0;
    return e.batch * cdiv(e.rows, kPnnRowsPerBlock);
  };
  auto vec = [](const thorn_pnn_tensor& e) { return (e.cols % 8) == 0 && aligned16(e.U); };
  int d = dispatch2(u_dtype, p_dtype, [&](auto* pu, auto* pp) {
    using U = std::remove_pointer_t<decltype(pu)>;
    using P = std::remove_pointer_t<decltype(pp)>;
    rc = launch_packed(ts, n, blocks, vec, [&](const Pack<thorn_pnn_tensor>& pk, int64_t nb) {
      PnnArgs a;
      a.pk = pk;
      a.eps = eps;
      pnn_stats_kernel<U, P><<<(unsigned)nb, kThreads, 0, st>>>(a);
    });
  });
  return d ? d : rc;
}

extern "C" int thorn_ortho_post_multi(const thorn_ortho_post_tensor* ts, int n, int u_dtype, int p_dtype,
                                      float weight_decay, void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(u_dtype) || !valid_dt(p_dtype)) return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i)
    if (ts[i].batch * ts[i].rows * ts[i].cols > 0 && (!ts[i].U || !ts[i].p || (ts[i].p_normsq && !ts[i].scratch)))
      return THORN_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  const float eps = dt_eps(p_dtype);
  auto blocks = [](const thorn_ortho_post_tensor& e) { return tiles_of(e.batch, e.rows, e.cols); };
  auto vec = [](const thorn_ortho_post_tensor& e) { return (e.cols % 8) == 0 && aligned16(e.U) && aligned16(e.p); };
  int d = dispatch2(u_dtype, p_dtype, [&](auto* pu, auto* pp) {
    using U = std::remove_pointer_t<decltype(pu)>;
    using P = std::remove_pointer_t<decltype(pp)>;
    rc = launch_packed(ts, n, blocks, vec, [&](const Pack<thorn_ortho_post_tensor>& pk, int64_t nb) {
      PostArgs a;
      a.pk = pk;
      a.wd = weight_decay;
      a.eps = eps;
      ortho_post_kernel<U, P><<<(unsigned)nb, kThreads, 0, st>>>(a);
    });
  });
  return d ? d : rc;
}

extern "C" int thorn_md_prep_multi(const thorn_md_prep_tensor* ts, int n, int p_dtype, void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(p_dtype)) return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i)
    if (ts[i].n < 0 || (ts[i].n > 0 && (!ts[i].gain || !ts[i].sp))) return THORN_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  int d = dispatch1(p_dtype, [&](auto* pp) {
    using P = std::remove_pointer_t<decltype(pp)>;
    rc = launch_packed(
        ts, n, [](const thorn_md_prep_tensor& e) { return cdiv(e.n, kThreads); },
        [](const thorn_md_prep_tensor&) { return false; },
        [&](const Pack<thorn_md_prep_tensor>& pk, int64_t nb) {
          MdPrepArgs a;
          a.pk = pk;
          md_prep_kernel<P><<<(unsigned)nb, kThreads, 0, st>>>(a);
        });
  });
  return d ? d : rc;
}

extern "C" int thorn_md_gain_grad_multi(const thorn_md_grad_tensor* ts, int n, int p_dtype, void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(p_dtype)) return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i)
    if (ts[i].n < 0 || (ts[i].n > 0 && (!ts[i].gsum || !ts[i].sig || !ts[i].grad))) return THORN_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  int d = dispatch1(p_dtype, [&](auto* pp) {
    using P = std::remove_pointer_t<decltype(pp)>;
    rc = launch_packed(
        ts, n, [](const thorn_md_grad_tensor& e) { return cdiv(e.n, kThreads); },
        [](const thorn_md_grad_tensor&) { return false; },
        [&](const Pack<thorn_md_grad_tensor>& pk, int64_t nb) {
          MdGradArgs a;
          a.pk = pk;
          md_gain_grad_kernel<P><<<(unsigned)nb, kThreads, 0, st>>>(a);
        });
  });
  return d ? d : rc;
}

extern "C" int thorn_md_finalize_multi(const thorn_md_final_tensor* ts, int n, int p_dtype, void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(p_dtype)) return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i) {
    const auto& e = ts[i];
    if (e.batch * e.rows * e.cols == 0) continue;  // an empty shard: nothing to check or launch
    if (!e.p) return THORN_ERR_ARG;
    if (e.normsq && !e.target) return THORN_ERR_ARG;
    if (!e.row_sp || (!e.scalar_gain && !e.col_sp)) return THORN_ERR_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  auto blocks = [](const thorn_md_final_tensor& e) { return tiles_of(e.batch, e.rows, e.cols); };
  auto vec = [](const thorn_md_final_tensor& e) { return (e.cols % 8) == 0 && aligned16(e.p); };
  int d = dispatch1(p_dtype, [&](auto* pp) {
    using P = std::remove_pointer_t<decltype(pp)>;
    rc = launch_packed(ts, n, blocks, vec, [&](const Pack<thorn_md_final_tensor>& pk, int64_t nb) {
      FinalArgs a;
      a.pk = pk;
      md_finalize_kernel<P><<<(unsigned)nb, kThreads, 0, st>>>(a);
    });
  });
  return d ? d : rc;
}

extern "C" int64_t thorn_sumsq_scratch_bytes(int64_t batch, int64_t rows, int64_t cols) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  return sq_bytes(batch, rows, cols);
}

extern "C" int64_t thorn_ortho_pre_scratch_bytes(int64_t batch, int64_t rows, int64_t cols, int md) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  return pre_layout(batch, rows, cols, md != 0).bytes;
}

extern "C" int64_t thorn_pnn_scratch_bytes(int64_t batch, int64_t rows) {
  if (batch <= 0 || rows <= 0) return 0;
  return (pnn_pf(batch) + 2 * batch * rows) * 4;
}

extern "C" int thorn_sumsq_multi(const thorn_sumsq_tensor* ts, int n, int dtype, void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(dtype)) return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i) {
    const auto& e = ts[i];
    if (e.batch < 0 || e.rows < 0 || e.cols < 0) return THORN_ERR_ARG;
    if (e.batch * e.rows * e.cols > 0 && (!e.x || !e.out || !e.scratch)) return THORN_ERR_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  auto blocks = [](const thorn_sumsq_tensor& e) { return tiles_of(e.batch, e.rows, e.cols); };
  auto vec = [](const thorn_sumsq_tensor& e) { return (e.cols % 8) == 0 && aligned16(e.x); };
  int d = dispatch1(dtype, [&](auto* px) {
    using T = std::remove_pointer_t<decltype(px)>;
    rc = launch_packed(ts, n, blocks, vec, [&](const Pack<thorn_sumsq_tensor>& pk, int64_t nb) {
      SumsqArgs a;
      a.pk = pk;
      sumsq_kernel<T><<<(unsigned)nb, kThreads, 0, st>>>(a);
    });
  });
  (void)dt_size;
  return d ? d : rc;
}

extern "C" int64_t thorn_magma_scratch_bytes(int64_t batch, int64_t rows, int64_t cols) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  return magma_bytes(batch, rows, cols);
}

extern "C" int thorn_magma_stats_multi(const thorn_magma_tensor* ts, int n, int g_dtype, int m_dtype,
                                       void* stream) {
  if (n < 0 || (n > 0 && ts == nullptr) || !valid_dt(g_dtype) || !valid_dt(m_dtype)) return THORN_ERR_ARG;
  for (int i = 0; i < n; ++i) {
    const auto& e = ts[i];
    if (e.batch < 0 || e.rows < 0 || e.cols < 0) return THORN_ERR_ARG;
    if (e.batch * e.rows * e.cols == 0) continue;
    if (!e.g || !e.m || !e.out || !e.scratch) return THORN_ERR_ARG;
    if (e.row_gain && !e.scalar_gain && !e.col_gain) return THORN_ERR_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int rc = THORN_OK;
  auto blocks = [](const thorn_magma_tensor& e) { return tiles_of(e.batch, e.rows, e.cols); };
  auto vec = [](const thorn_magma_tensor& e) { return (e.cols % 8) == 0 && aligned16(e.g) && aligned16(e.m); };
  int d = dispatch2(g_dtype, m_dtype, [&](auto* pg, auto* pm) {
    using G = std::remove_pointer_t<decltype(pg)>;
    using M = std::remove_pointer_t<decltype(pm)>;
    rc = launch_packed(ts, n, blocks, vec, [&](const Pack<thorn_magma_tensor>& pk, int64_t nb) {
      MagmaArgs a;
      a.pk = pk;
      magma_stats_kernel<G, M><<<(unsigned)nb, kThreads, 0, st>>>(a);
    });
  });
  return d ? d : rc;
}
