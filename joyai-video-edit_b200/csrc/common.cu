// Host-side plumbing shared by every entry point: error strings, per-device
// facts, launch accounting.
#include <cuda.h>  // driver types for the context-id entry points (resolved at run time)

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

// Bounded-wait expiries of this library's kernels on each device (one copy
// per device context); kernels receive its address, jo_device_fault_count
// reads and clears it.
__device__ unsigned int g_jo_faults = 0;

namespace {
thread_local char g_last_error[512] = "";
std::atomic<uint64_t> g_launches{0};

constexpr int kMaxDevices = 64;
jo::DeviceInfo g_info[kMaxDevices];
std::once_flag g_info_once[kMaxDevices];
int g_info_status[kMaxDevices];
jo::SymbolCache g_fault_cache;

// Unique id of the calling thread's current context (0 when unknown), through the
// driver entry points cuCtxGetCurrent / cuCtxGetId resolved once via the runtime.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_current = nullptr;
CtxGetIdFn g_ctx_id = nullptr;
std::once_flag g_drv_once;
uint64_t context_id() {
  std::call_once(g_drv_once, [] {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", (void**)&g_ctx_current, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      g_ctx_current = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", (void**)&g_ctx_id, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      g_ctx_id = nullptr;
    cudaGetLastError();
  });
  if (!g_ctx_current || !g_ctx_id) return 0;
  CUcontext c = nullptr;
  if (g_ctx_current(&c) != CUDA_SUCCESS || c == nullptr) return 0;
  unsigned long long id = 0;
  if (g_ctx_id(c, &id) != CUDA_SUCCESS) return 0;
  return (uint64_t)id + 1;  // never 0
}
std::mutex g_symbol_mu;
}  // namespace

namespace jo {

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int launch_failed(cudaError_t e, const char* what) {
  cudaGetLastError();
  return fail(JO_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
}

int after_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(JO_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return JO_OK;
}

int device_info(const DeviceInfo** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(JO_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(JO_ERR_CUDA, "device index %d out of range", dev);
  std::call_once(g_info_once[dev], [dev]() {
    DeviceInfo& d = g_info[dev];
    d.ordinal = dev;
    cudaError_t r = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (r == cudaSuccess) r = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    if (r == cudaSuccess) r = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (r == cudaSuccess)
      r = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    g_info_status[dev] = (r == cudaSuccess) ? JO_OK : JO_ERR_CUDA;
  });
  if (g_info_status[dev] != JO_OK) return fail(JO_ERR_CUDA, "device %d: attribute query failed", dev);
  DeviceInfo& d = g_info[dev];
  if (d.major != 10 || d.minor != 0)
    return fail(JO_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", dev,
                d.major, d.minor);
  // the fault counter's address in the device's current context (looked up again
  // if the context was re-created)
  void* fault = nullptr;
  if (int s = symbol_address(g_fault_cache, &g_jo_faults, dev, nullptr, &fault, "fault counter")) return s;
  d.fault = static_cast<unsigned int*>(fault);
  *out = &d;
  return JO_OK;
}

int symbol_address(SymbolCache& cache, const void* symbol, int dev, cudaStream_t stream, void** out,
                   const char* what) {
  if (dev < 0 || dev >= kMaxDevices) return fail(JO_ERR_CUDA, "%s: device index %d out of range", what, dev);
  const uint64_t ctx = context_id();
  if (ctx != 0 && cache.ctx[dev].load(std::memory_order_acquire) == ctx) {
    *out = cache.addr[dev].load(std::memory_order_relaxed);
    return JO_OK;
  }
  if (stream != nullptr) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) cudaGetLastError();
    if (cs != cudaStreamCaptureStatusNone)
      return fail(JO_ERR_INVALID,
                  "%s: the first call on device %d (in its current context) must come before any stream "
                  "capture: it looks up the device address of a static array",
                  what, dev);
  }
  std::lock_guard<std::mutex> lock(g_symbol_mu);
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, symbol);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "%s: cudaGetSymbolAddress failed on device %d: %s", what, dev, cudaGetErrorString(e));
  }
  cache.addr[dev].store(p, std::memory_order_relaxed);
  cache.ctx[dev].store(context_id(), std::memory_order_release);  // 0 (unknown) keeps looking up every call
  *out = p;
  return JO_OK;
}

int reserve_smem(const void* kernel, int bytes, std::atomic<uint64_t>& done, const DeviceInfo* di,
                 const char* what) {
  const uint64_t bit = 1ull << di->ordinal;
  if (done.load(std::memory_order_acquire) & bit) return JO_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "%s: cannot reserve %d bytes of shared memory: %s", what, bytes, cudaGetErrorString(e));
  }
  done.fetch_or(bit, std::memory_order_acq_rel);
  return JO_OK;
}

int prefer_max_carveout(const void* kernel, std::atomic<uint64_t>& done, const DeviceInfo* di, const char* what) {
  const uint64_t bit = 1ull << di->ordinal;
  if (done.load(std::memory_order_acquire) & bit) return JO_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                             (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "%s: cannot set the shared-memory carveout: %s", what, cudaGetErrorString(e));
  }
  done.fetch_or(bit, std::memory_order_acq_rel);
  return JO_OK;
}

int occupancy(const void* kernel, int threads, size_t smem) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    return 1;
  }
  return n > 0 ? n : 1;
}

}  // namespace jo

extern "C" {

int jo_abi_version(void) { return 1; }

const char* jo_status_name(int status) {
  switch (status) {
    case JO_OK: return "JO_OK";
    case JO_ERR_INVALID: return "JO_ERR_INVALID";
    case JO_ERR_SHAPE: return "JO_ERR_SHAPE";
    case JO_ERR_ALIGN: return "JO_ERR_ALIGN";
    case JO_ERR_DTYPE: return "JO_ERR_DTYPE";
    case JO_ERR_CUDA: return "JO_ERR_CUDA";
    case JO_ERR_UNSUPPORTED: return "JO_ERR_UNSUPPORTED";
    default: return "JO_ERR_UNKNOWN";
  }
}

const char* jo_last_error(void) { return g_last_error; }

uint64_t jo_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int jo_device_fault_count(uint32_t* count) {
  if (!count) return jo::fail(JO_ERR_INVALID, "device_fault_count: null pointer");
  const jo::DeviceInfo* di;
  if (int s = jo::device_info(&di)) return s;
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaMemcpy(&v, di->fault, sizeof(v), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(di->fault, &zero, sizeof(zero), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return jo::fail(JO_ERR_CUDA, "device_fault_count: %s", cudaGetErrorString(e));
  *count = v;
  return JO_OK;
}

}  // extern "C"
