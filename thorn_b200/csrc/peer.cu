// Peer-memory exchange of the sharded path over NVLink / NVSwitch.
//
// Every rank owns one device arena (cudaMalloc) that the other ranks of its
// shard group map with CUDA IPC.  The NS-input pass then writes each row slab
// straight into the owner's arena with ordinary stores (the gather is fused
// into that kernel), result rows go back by copy-engine peer copies (no SMs
// taken from the Newton-Schulz GEMMs), and the ranks order these transfers
// with flags in the arenas: a sender releases a per-sender 64-bit slot at
// system scope once its stores or copies are done, and the receiver waits
// (bounded) until every slot holds the current step's value.  Slot values only
// grow from step to step, so they never need resetting.
#include <stdint.h>
#include <string.h>

#include "common.cuh"

namespace thorn {
namespace {

constexpr int kMaxPeers = 64;

struct SignalArgs {
  uint64_t* slot[kMaxPeers];
  int n;
  uint64_t value;
};

// One thread per destination: everything this stream wrote before (earlier
// kernels' peer stores, copies) is made visible at system scope, then the
// slot is released.
__global__ void peer_signal_kernel(const __grid_constant__ SignalArgs a) {
  const int i = threadIdx.x;
  if (i >= a.n) return;
  asm volatile("fence.sc.sys;" ::: "memory");
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a.slot[i]), "l"(a.value) : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One thread per slot: acquire-poll until the slot reaches `value`.  A wait
// that exceeds limit_ns sets *err (3) and returns, so a lost peer ends in an
// error status the host reads, never in a hung GPU.
__global__ void peer_wait_kernel(const uint64_t* slots, int n, uint64_t value, uint64_t limit_ns, int* err) {
  const int i = threadIdx.x;
  if (i >= n) return;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(slots + i) : "memory");
    if (v >= value) return;
    if (globaltimer_ns() - t0 > limit_ns) {
      if (err != nullptr) atomicExch(err, 3);
      return;
    }
    __nanosleep(200);
  }
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return THORN_OK;
  cudaGetLastError();
  return THORN_ERR_CUDA;
}

}  // namespace
}  // namespace thorn

using namespace thorn;

extern "C" int thorn_peer_alloc(int64_t bytes, void** out) {
  if (bytes <= 0 || out == nullptr) return THORN_ERR_ARG;
  *out = nullptr;
  void* p = nullptr;
  int rc = cuda_status(cudaMalloc(&p, (size_t)bytes));
  if (rc) return rc;
  rc = cuda_status(cudaMemset(p, 0, (size_t)bytes));
  if (rc) {
    cudaFree(p);
    return rc;
  }
  *out = p;
  return THORN_OK;
}

extern "C" int thorn_peer_free(void* p) { return p == nullptr ? THORN_OK : cuda_status(cudaFree(p)); }

extern "C" int thorn_ipc_handle(const void* p, void* handle) {
  if (p == nullptr || handle == nullptr) return THORN_ERR_ARG;
  cudaIpcMemHandle_t h;
  const int rc = cuda_status(cudaIpcGetMemHandle(&h, const_cast<void*>(p)));
  if (rc) return rc;
  static_assert(sizeof(h) == THORN_IPC_HANDLE_BYTES, "CUDA IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return THORN_OK;
}

extern "C" int thorn_ipc_open(const void* handle, void** out) {
  if (handle == nullptr || out == nullptr) return THORN_ERR_ARG;
  *out = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int thorn_ipc_close(void* p) { return p == nullptr ? THORN_OK : cuda_status(cudaIpcCloseMemHandle(p)); }

extern "C" int thorn_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes < 0 || (bytes > 0 && (dst == nullptr || src == nullptr))) return THORN_ERR_ARG;
  if (bytes == 0) return THORN_OK;
  return cuda_status(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, (cudaStream_t)stream));
}

extern "C" int thorn_peer_signal(uint64_t* const* slots, int n, uint64_t value, void* stream) {
  if (n < 0 || n > kMaxPeers || (n > 0 && slots == nullptr)) return THORN_ERR_ARG;
  if (n == 0) return THORN_OK;
  SignalArgs a;
  a.n = n;
  a.value = value;
  for (int i = 0; i < n; ++i) {
    if (slots[i] == nullptr || (reinterpret_cast<uintptr_t>(slots[i]) & 7u)) return THORN_ERR_ARG;
    a.slot[i] = slots[i];
  }
  peer_signal_kernel<<<1, 32 * ((n + 31) / 32), 0, (cudaStream_t)stream>>>(a);
  count_launch();
  return check_launch();
}

extern "C" int thorn_peer_wait(const uint64_t* slots, int n, uint64_t value, uint64_t limit_ns, int* err_flag,
                               void* stream) {
  if (n < 0 || n > kMaxPeers || (n > 0 && slots == nullptr) || (reinterpret_cast<uintptr_t>(slots) & 7u))
    return THORN_ERR_ARG;
  if (n == 0) return THORN_OK;
  peer_wait_kernel<<<1, 32 * ((n + 31) / 32), 0, (cudaStream_t)stream>>>(slots, n, value, limit_ns, err_flag);
  count_launch();
  return check_launch();
}
