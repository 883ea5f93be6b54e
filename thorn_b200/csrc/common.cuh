// Shared device/host helpers for the THORN sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <type_traits>
#include <stdint.h>

#include "thorn_b200.h"

namespace thorn {

// ---------------------------------------------------------------------------
// dtype handling: every kernel computes in fp32 and rounds once on store,
// which is how the reference's Triton kernels and torch's CUDA ops behave.
// ---------------------------------------------------------------------------
template <int DT> struct dtype_of;
template <> struct dtype_of<THORN_F32> { using T = float; };
template <> struct dtype_of<THORN_BF16> { using T = __nv_bfloat16; };
template <> struct dtype_of<THORN_F16> { using T = __half; };

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }

template <class T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// leading dimension of NS operands: rows padded to 8 elements (16 bytes) for TMA
__host__ __device__ __forceinline__ int64_t ns_ld(int64_t n) { return (n + 7) / 8 * 8; }

// value after a round trip through storage type T
template <class T> __device__ __forceinline__ float rnd(float x) { return to_f(from_f<T>(x)); }

// 8 consecutive elements <-> fp32 registers (16B-aligned vector path)
template <class T> struct Vec8;
template <> struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float* v) {
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
};
// Two fp32 values -> one packed pair of 16-bit values, one conversion
// instruction (cvt.rn.bf16x2.f32 / cvt.rn.f16x2.f32), round-to-nearest-even
// per element exactly like the scalar conversions.
__device__ __forceinline__ uint32_t pack2(float lo, float hi, __nv_bfloat16*) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi, __half*) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ void unpack2(uint32_t u, float& lo, float& hi, __nv_bfloat16*) {
  lo = __uint_as_float(u << 16);
  hi = __uint_as_float(u & 0xFFFF0000u);
}
__device__ __forceinline__ void unpack2(uint32_t u, float& lo, float& hi, __half*) {
  const __half2 h = *reinterpret_cast<const __half2*>(&u);
  const float2 f = __half22float2(h);
  lo = f.x;
  hi = f.y;
}

// Round 8 fp32 values to T and back (T = float: no-op), two per instruction.
template <class T>
__device__ __forceinline__ void rnd8(float* v) {
  if constexpr (!std::is_same<T, float>::value) {
#pragma unroll
    for (int i = 0; i < 8; i += 2) unpack2(pack2(v[i], v[i + 1], (T*)nullptr), v[i], v[i + 1], (T*)nullptr);
  }
}

// Packed 16-bit products.  The fp32 product of two bf16 (or two fp16) values is
// exact, so one packed multiply with round-to-nearest-even gives, per element,
// exactly the fp32 product rounded once to T: an fp32 multiply and a rounding
// to T in one instruction for two elements.
template <class T> struct Pair2;
template <> struct Pair2<__nv_bfloat16> { using V = __nv_bfloat162; };
template <> struct Pair2<__half> { using V = __half2; };
template <class T>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
  using V = typename Pair2<T>::V;
  const V r = __hmul2(*reinterpret_cast<const V*>(&a), *reinterpret_cast<const V*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}

template <class H> struct Vec8Half {
  static __device__ __forceinline__ void load(const H* p, float* v) {
    const uint4 r = *reinterpret_cast<const uint4*>(p);
    unpack2(r.x, v[0], v[1], (H*)nullptr);
    unpack2(r.y, v[2], v[3], (H*)nullptr);
    unpack2(r.z, v[4], v[5], (H*)nullptr);
    unpack2(r.w, v[6], v[7], (H*)nullptr);
  }
  static __device__ __forceinline__ void store(H* p, const float* v) {
    uint4 r;
    r.x = pack2(v[0], v[1], (H*)nullptr);
    r.y = pack2(v[2], v[3], (H*)nullptr);
    r.z = pack2(v[4], v[5], (H*)nullptr);
    r.w = pack2(v[6], v[7], (H*)nullptr);
    *reinterpret_cast<uint4*>(p) = r;
  }
};
template <> struct Vec8<__nv_bfloat16> : Vec8Half<__nv_bfloat16> {};
template <> struct Vec8<__half> : Vec8Half<__half> {};

// Load/store n<=8 elements starting at p (scalar path for ragged edges).
template <class T>
__device__ __forceinline__ void load_n(const T* p, float* v, int n, bool vec) {
  if (vec && n == 8) { Vec8<T>::load(p, v); return; }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = i < n ? to_f(p[i]) : 0.f;
}
template <class T>
__device__ __forceinline__ void store_n(T* p, const float* v, int n, bool vec) {
  if (vec && n == 8) { Vec8<T>::store(p, v); return; }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < n) p[i] = from_f<T>(v[i]);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Block-wide sum; every thread gets the result.  blockDim.x multiple of 32, <= 1024.
__device__ __forceinline__ float block_sum(float x, float* red /* >= 32 floats */) {
  x = warp_sum(x);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = x;
  __syncthreads();
  float t = (l < nw) ? red[l] : 0.f;
  t = warp_sum(t);
  return t;
}

__device__ __forceinline__ double warp_sum_d(double x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Block-wide fp64 sum; every thread gets the result.  blockDim.x multiple of 32, <= 1024.
__device__ __forceinline__ double block_sum_d(double x, double* red /* >= 32 doubles */) {
  x = warp_sum_d(x);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = x;
  __syncthreads();
  double t = (l < nw) ? red[l] : 0.0;
  t = warp_sum_d(t);
  return t;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
void count_launch(int n = 1);
int check_launch();  // cudaPeekAtLastError -> status

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace thorn
