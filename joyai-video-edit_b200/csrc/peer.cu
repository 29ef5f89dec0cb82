// Copy-engine all-gather of the chunk's K/V blocks between the ranks of one node.
//
// The sequence-parallel block gathers every rank's K/V rows of the current chunk
// before the attention over them (the all-gather at the attention boundary of
// deploy/xvideo/models/dit/dit.py:154-189, 498).  Run as an NCCL kernel it takes SMs
// and issue slots from the attention over the cache rows that it overlaps, and
// slows down beside it.  Here the bytes move on the copy engines instead: each rank
// maps the other ranks' K/V buffers (CUDA IPC, peer access over NVLink) and pulls
// their blocks with one cudaMemcpyAsync per (peer, tensor), on one stream per peer;
// no SM touches the data.
//
// Ordering between ranks uses two flag words per (rank, peer) in IPC-mapped device
// memory, written by tiny kernels with system-scope release stores and read with
// acquire loads:
//   ready[r] on rank q = the last step whose block rank r has written (q may pull it)
//   done[r]  on rank q = the last step in which rank r finished pulling q's block
//                        (q may overwrite its block for the next step)
// Every wait is bounded (2 s of wall time, then the device fault counter is raised
// and the kernel returns), so a rank that never arrives ends in a recorded fault
// instead of a hung GPU.
#include <string.h>

#include "pipeline.cuh"

namespace jo {
namespace {

constexpr int kMaxPeers = 16;

struct PeerFlags {
  unsigned long long* p[kMaxPeers];  // flag word of this rank on rank q (null: skip)
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Thread q stores `value` into rank q's copy of this rank's flag word.  The stores
// follow (stream order) the kernels whose writes they publish; the fence makes those
// writes visible system-wide before any flag is.
__global__ void peer_signal_kernel(const PeerFlags f, int world, unsigned long long value) {
  const int q = threadIdx.x;
  __threadfence_system();
  if (q < world && f.p[q] != nullptr) st_release_sys(f.p[q], value);
}

// Thread q waits (bounded) until flags[q] >= value, for every q != skip.
__global__ void peer_wait_kernel(const unsigned long long* flags, int world, int skip, unsigned long long value,
                                 unsigned int* fault) {
  const int q = threadIdx.x;
  if (q >= world || q == skip) return;
  if (ld_acquire_sys(flags + q) >= value) return;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys(flags + q) < value) {
    if (globaltimer() - t0 > kWaitNs) {
      atomicAdd(fault, 1u);
      return;
    }
    __nanosleep(256);
  }
}

}  // namespace
}  // namespace jo

using namespace jo;

extern "C" {

int jo_ipc_alloc(int64_t bytes, void** ptr) {
  const char* op = "ipc_alloc";
  if (!ptr) return fail(JO_ERR_INVALID, "%s: null output", op);
  *ptr = nullptr;
  if (bytes <= 0) return fail(JO_ERR_SHAPE, "%s: bad size %lld", op, (long long)bytes);
  void* p = nullptr;
  if (cudaError_t e = cudaMalloc(&p, (size_t)bytes)) {
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "%s: cudaMalloc(%lld) failed: %s", op, (long long)bytes, cudaGetErrorString(e));
  }
  if (cudaError_t e = cudaMemset(p, 0, (size_t)bytes)) {
    cudaGetLastError();
    cudaFree(p);
    return fail(JO_ERR_CUDA, "%s: cudaMemset failed: %s", op, cudaGetErrorString(e));
  }
  *ptr = p;
  return JO_OK;
}

int jo_ipc_free(void* ptr) {
  if (!ptr) return JO_OK;
  if (cudaError_t e = cudaFree(ptr)) {
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "ipc_free: cudaFree failed: %s", cudaGetErrorString(e));
  }
  return JO_OK;
}

int jo_ipc_handle(const void* ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == JO_IPC_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle) return fail(JO_ERR_INVALID, "ipc_handle: null operand");
  cudaIpcMemHandle_t h;
  if (cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr))) {
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "ipc_handle: cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  return JO_OK;
}

int jo_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(JO_ERR_INVALID, "ipc_open: null operand");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess)) {
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "ipc_open: cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return JO_OK;
}

int jo_ipc_close(void* ptr) {
  if (!ptr) return JO_OK;
  if (cudaError_t e = cudaIpcCloseMemHandle(ptr)) {
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "ipc_close: cudaIpcCloseMemHandle failed: %s", cudaGetErrorString(e));
  }
  return JO_OK;
}

int jo_peer_signal(void* const* peer_flags, int world, uint64_t value, void* stream) {
  const char* op = "peer_signal";
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (world < 1 || world > kMaxPeers) return fail(JO_ERR_SHAPE, "%s: world %d not in [1, %d]", op, world, kMaxPeers);
  if (!peer_flags) return fail(JO_ERR_INVALID, "%s: null flag table", op);
  PeerFlags f{};
  for (int q = 0; q < world; ++q) {
    if (peer_flags[q] && (reinterpret_cast<uintptr_t>(peer_flags[q]) & 7u))
      return fail(JO_ERR_ALIGN, "%s: flag words must be 8-byte aligned", op);
    f.p[q] = reinterpret_cast<unsigned long long*>(peer_flags[q]);
  }
  peer_signal_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(f, world, (unsigned long long)value);
  if (cudaError_t e = cudaGetLastError()) return launch_failed(e, op);
  return after_launch("peer_signal_kernel");
}

int jo_peer_wait(const uint64_t* flags, int world, int skip, uint64_t value, void* stream) {
  const char* op = "peer_wait";
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (world < 1 || world > kMaxPeers) return fail(JO_ERR_SHAPE, "%s: world %d not in [1, %d]", op, world, kMaxPeers);
  if (!flags || (reinterpret_cast<uintptr_t>(flags) & 7u)) return fail(JO_ERR_ALIGN, "%s: bad flag array", op);
  peer_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(reinterpret_cast<const unsigned long long*>(flags), world,
                                                       skip, (unsigned long long)value, di->fault);
  if (cudaError_t e = cudaGetLastError()) return launch_failed(e, op);
  return after_launch("peer_wait_kernel");
}

int jo_peer_copy(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes < 0) return fail(JO_ERR_SHAPE, "peer_copy: bad size");
  if (bytes == 0) return JO_OK;
  if (!dst || !src) return fail(JO_ERR_INVALID, "peer_copy: null operand");
  if (cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream)) {
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "peer_copy: cudaMemcpyAsync failed: %s", cudaGetErrorString(e));
  }
  return JO_OK;
}

}  // extern "C"
