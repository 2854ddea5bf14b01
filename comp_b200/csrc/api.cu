// C-ABI plumbing: version, per-thread last error, launch counter, device facts, CUDA IPC helpers.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "b2q_internal.h"

namespace b2q {

static thread_local char t_err[512] = "";
static std::atomic<long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

int after_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B2Q_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return B2Q_OK;
}

static std::mutex g_dev_mu;
static DeviceInfo g_dev[64];

int device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(B2Q_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(B2Q_ECUDA, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_dev[dev].sms == 0) {
    DeviceInfo d;
    e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return fail(B2Q_ECUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    g_dev[dev] = d;
  }
  *out = g_dev[dev];
  return B2Q_OK;
}

}  // namespace b2q

extern "C" {

const char* b2q_version(void) { return "comp_b200 0.1.0 sm_100a"; }

int b2q_last_error(char* buf, size_t len) {
  const size_t n = strlen(b2q::t_err);
  if (buf && len) {
    const size_t c = n < len - 1 ? n : len - 1;
    memcpy(buf, b2q::t_err, c);
    buf[c] = '\0';
  }
  return (int)n;
}

long long b2q_launch_count(void) { return b2q::g_launches.load(std::memory_order_relaxed); }

// cuMemGetAddressRange through the runtime's driver entry-point lookup (no link-time dependency on libcuda).
typedef int (*MemGetAddressRangeFn)(unsigned long long* base, size_t* size, unsigned long long ptr);

int b2q_ipc_get_handle(void* dev_ptr, void* handle_out64, uint64_t* offset_out) {
  if (!dev_ptr || !handle_out64 || !offset_out) return b2q::fail(B2Q_EINVAL, "b2q_ipc_get_handle: null pointer");
  static MemGetAddressRangeFn range_fn = nullptr;
  if (!range_fn) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return b2q::fail(B2Q_ECUDA, "b2q_ipc_get_handle: cuMemGetAddressRange not available");
    range_fn = reinterpret_cast<MemGetAddressRangeFn>(fn);
  }
  unsigned long long base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<unsigned long long>(dev_ptr)) != 0)
    return b2q::fail(B2Q_ECUDA, "b2q_ipc_get_handle: cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return b2q::fail(B2Q_ECUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  memcpy(handle_out64, &h, 64);
  *offset_out = reinterpret_cast<unsigned long long>(dev_ptr) - base;
  return B2Q_OK;
}

int b2q_ipc_open_handle(const void* handle64, void** dev_ptr_out) {
  if (!handle64 || !dev_ptr_out) return b2q::fail(B2Q_EINVAL, "b2q_ipc_open_handle: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return b2q::fail(B2Q_ECUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return B2Q_OK;
}

int b2q_ipc_close_handle(void* dev_ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return b2q::fail(B2Q_ECUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return B2Q_OK;
}

}  // extern "C"
