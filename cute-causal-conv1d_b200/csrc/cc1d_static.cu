// cc1d_bwd_launch_static: the backward launcher for callers that cannot allocate device
// memory.
//
// The regular backward (cc1d_bwd_launch) needs a scratch workspace from its caller.
// Some callers have no way to provide one: plugin hosts that hand a kernel only its
// input and output buffers, inference servers that run with a fixed device-memory
// budget and forbid allocations once serving starts, and code that must launch without
// touching the device allocator (an allocation can synchronise the device or fragment a
// pool).  For them this entry point takes its scratch from one array that lives in the
// library itself, so the call allocates nothing.
//
// The array is a file-scope __device__ variable of kStaticScratchBytes bytes: every GPU
// on which the library is used holds it until the process exits.  Host code cannot use
// the variable's name as a device address, so the address is looked up once per device
// with cudaGetSymbolAddress (on the first call on that device, which should therefore
// happen before any stream capture) and passed to the kernels like a caller workspace.
// The looked-up address is kept for the life of the process, so the entry point must not
// be used across a device reset (cudaDeviceReset), which can move the array.
// All calls share the array: two calls that overlap on the GPU (different streams, or
// the same array used from several threads without ordering) race on it.
#include <cstdio>
#include <mutex>

#include "cc1d_launch.h"

namespace {

constexpr int64_t kStaticScratchBytes = CC1D_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};

thread_local char g_msg[320];

// Device address of the scratch array on the current device (looked up once).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

cc1d_status cc1d_bwd_launch_static(const cc1d_bwd_params* params, void* stream) {
  if (!params) return cc1d_bwd_launch(params, stream);  // reports the NULL params
  const int64_t need = cc1d_bwd_workspace_bytes(params);
  if (need < 0) return cc1d_bwd_launch(params, stream);  // reports the argument error
  if (need > kStaticScratchBytes) {
    std::snprintf(g_msg, sizeof(g_msg),
                  "cc1d_bwd_launch_static: this problem needs %lld bytes of scratch, more than the %lld "
                  "bytes of the library's static array; use cc1d_bwd_launch with a caller workspace",
                  (long long)need, (long long)kStaticScratchBytes);
    cc1d::set_last_error(g_msg);
    return CC1D_ERR_VALUE;
  }
  void* scratch = nullptr;
  const cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess) {
    std::snprintf(g_msg, sizeof(g_msg), "cc1d_bwd_launch_static: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    cc1d::set_last_error(g_msg);
    return CC1D_ERR_CUDA;
  }
  cc1d_bwd_params p = *params;
  p.workspace = scratch;
  p.workspace_bytes = kStaticScratchBytes;
  return cc1d_bwd_launch(&p, stream);
}

}  // extern "C"
