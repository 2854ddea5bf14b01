// Fused quantize + GEMV with the activations and the output in pinned host memory.
//
// A decode loop that keeps its activations on the host (a CPU-side sampler, an FFI caller whose tensors live in host
// memory) pays for two memcpys per layer around the GEMV: the host-to-device copy of x, which also ends the
// programmatic overlap with the previous layer (a kernel after a memcpy waits for the memcpy), and the device-to-host
// copy of Y. Here both transfers are made by kernels through the host buffers' device mappings instead:
//   * a copy kernel reads x over PCIe into a device staging area. It loads its share of x before griddepcontrol.wait,
//     so the PCIe reads overlap the previous kernel's tail, and lets the GEMV launch at once, so the GEMV's weight
//     stream starts while x is still arriving (the GEMV reads x only after its own griddepcontrol.wait);
//   * the fused GEMV (exactly b2q_quant_gemv_ws, same schedule, same bytes) stores Y straight into the host buffer;
//     each output value crosses PCIe once, spread over the kernel's run.
// The host pointers are checked with cudaPointerGetAttributes before anything is launched: memory that is not
// page-locked and mapped for the current device is refused (B2Q_EINVAL), so no kernel ever receives a host address
// the GPU cannot reach.
#include <algorithm>

#include "b2q_internal.h"

namespace b2q {

constexpr int kCopyThreads = 256;
constexpr int kCopyVec = 4;  // float4 loads held per thread across the dependency wait

// x [M][ldx] f32 (16-byte aligned rows, read through the host mapping) -> stage [M][K] f32 (device).
__global__ void __launch_bounds__(kCopyThreads) pinned_x_copy_kernel(const float4* __restrict__ x, int64_t ldx4,
                                                                      float4* __restrict__ stage, int64_t K4,
                                                                      int64_t total4) {
  // The GEMV may launch at once: it touches only its (immutable) weights before its own griddepcontrol.wait, which
  // returns only after this grid has completed -- and this grid completes only after the wait below.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t stride = (int64_t)gridDim.x * kCopyThreads;
  const int64_t i0 = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x;
  float4 v[kCopyVec];
#pragma unroll
  for (int u = 0; u < kCopyVec; ++u) {
    const int64_t i = i0 + u * stride;
    if (i < total4) {
      const int64_t m = i / K4, c = i - m * K4;
      v[u] = x[m * ldx4 + c];
    }
  }
  // the previous kernel on the stream may still read the staging area (a call that reused this workspace)
  asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
  for (int u = 0; u < kCopyVec; ++u) {
    const int64_t i = i0 + u * stride;
    if (i < total4) stage[i] = v[u];
  }
  for (int64_t i = i0 + kCopyVec * stride; i < total4; i += stride) {  // rows beyond what the grid holds at once
    const int64_t m = i / K4, c = i - m * K4;
    stage[i] = x[m * ldx4 + c];
  }
}

// Y = 0 through the host mapping (K == 0: every sum is empty).
__global__ void __launch_bounds__(kCopyThreads) pinned_zero_kernel(float* __restrict__ y, int64_t total) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int64_t i = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; i < total; i += (int64_t)gridDim.x * kCopyThreads)
    y[i] = 0.f;
}

static size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// Device address of a page-locked host buffer for the current device, or an error if it has none.
static int mapped(const char* who, const char* what, const void* host, void** dev) {
  cudaPointerAttributes at{};
  cudaError_t e = cudaPointerGetAttributes(&at, host);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(B2Q_EINVAL, "%s: %s is not a CUDA-visible pointer: %s", who, what, cudaGetErrorString(e));
  }
  if (at.type != cudaMemoryTypeHost || at.devicePointer == nullptr)
    return fail(B2Q_EINVAL,
                "%s: %s must be page-locked host memory mapped for this device (cudaHostAlloc, cudaHostRegister "
                "with cudaHostRegisterMapped, torch pin_memory)",
                who, what);
  *dev = at.devicePointer;
  return B2Q_OK;
}

}  // namespace b2q

extern "C" size_t b2q_pinned_workspace_size(int fmt, int64_t N, int64_t K, int64_t M) {
  if (fmt < 0 || fmt > 4 || N <= 0 || K <= 0 || M <= 0) return 0;
  return b2q::align256((size_t)M * (size_t)K * sizeof(float)) + b2q_workspace_size(fmt, N, K, M);
}

extern "C" int b2q_quant_gemv_pinned(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x_host,
                                     int64_t ldx, float* y_host, int64_t N, int64_t K, int64_t M, void* workspace,
                                     size_t workspace_bytes, b2q_stream_t stream) {
  using namespace b2q;
  static const char* who = "b2q_quant_gemv_pinned";
  if (fmt < 0 || fmt > 4)
    return fail(B2Q_EINVAL, "%s: fmt %d is not Q4_0 (0), TQ2_0 (1), Q8_0 (2), IQ4_NL (3) or Q4_K (4)", who, fmt);
  if (N < 0 || K < 0 || M < 0) return fail(B2Q_EINVAL, "%s: negative size", who);
  if (N == 0 || M == 0) return B2Q_OK;  // empty output: nothing is touched
  void* y_dev = nullptr;
  int rc = mapped(who, "y", y_host, &y_dev);
  if (rc) return rc;
  DeviceInfo di;
  rc = device_info(&di);
  if (rc) return rc;
  if (K == 0) {  // empty sums: Y = 0, written by a kernel (nothing else is touched)
    if (!aligned(y_dev, 4)) return fail(B2Q_EALIGN, "%s: y must be 4-byte aligned", who);
    const int64_t total = M * N;
    const int grid = (int)std::min<int64_t>((total + kCopyThreads - 1) / kCopyThreads, (int64_t)di.sms * 4);
    cudaError_t le = launch_maybe_pdl(pinned_zero_kernel, dim3(grid), dim3(kCopyThreads), 0, (cudaStream_t)stream,
                                      reinterpret_cast<float*>(y_dev), total);
    if (le != cudaSuccess) {
      cudaGetLastError();
      return fail(B2Q_ECUDA, "%s: launch failed: %s", who, cudaGetErrorString(le));
    }
    return after_launch(who);
  }
  void* x_dev = nullptr;
  rc = mapped(who, "x", x_host, &x_dev);
  if (rc) return rc;
  if (ldx < K || (ldx % 4) || !aligned(x_dev, 16))
    return fail(B2Q_EALIGN, "%s: x must be 16-byte aligned with ldx >= K and a multiple of 4", who);
  const size_t xbytes = align256((size_t)M * (size_t)K * sizeof(float));
  const size_t need = b2q_pinned_workspace_size(fmt, N, K, M);
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < need)
    return fail(B2Q_EINVAL, "%s: workspace must be 256-byte aligned device memory of at least %zu bytes (got %zu)",
                who, need, workspace ? workspace_bytes : (size_t)0);
  const size_t gemv_ws = need - xbytes;
  float* stage = reinterpret_cast<float*>(workspace);
  void* gws = gemv_ws ? reinterpret_cast<uint8_t*>(workspace) + xbytes : nullptr;
  // the GEMV's argument checks run before anything is launched
  rc = check_quant_gemv_args(who, fmt, wq, ldwq, ws, stage, reinterpret_cast<float*>(y_dev), N, K, M);
  if (rc) return rc;
  const int64_t K4 = K / 4, total4 = M * K4;
  const int64_t want = (total4 + (int64_t)kCopyThreads * kCopyVec - 1) / ((int64_t)kCopyThreads * kCopyVec);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)di.sms * 8));
  cudaError_t le = launch_maybe_pdl(pinned_x_copy_kernel, dim3(grid), dim3(kCopyThreads), 0, (cudaStream_t)stream,
                                    reinterpret_cast<const float4*>(x_dev), ldx / 4, reinterpret_cast<float4*>(stage),
                                    K4, total4);
  if (le != cudaSuccess) {
    cudaGetLastError();
    return fail(B2Q_ECUDA, "%s: copy launch failed: %s", who, cudaGetErrorString(le));
  }
  rc = after_launch(who);
  if (rc) return rc;
  return b2q_quant_gemv_ws(fmt, wq, ldwq, ws, stage, K, nullptr, nullptr, reinterpret_cast<float*>(y_dev), N, K, M,
                           gws, gemv_ws, stream);
}

extern "C" int b2q_host_device_pointer(const void* host, void** dev) {
  using namespace b2q;
  if (!dev) return fail(B2Q_EINVAL, "b2q_host_device_pointer: null output");
  *dev = nullptr;
  return mapped("b2q_host_device_pointer", "the buffer", host, dev);
}

extern "C" int b2q_stage_pinned(const float* x_host, int64_t ldx, float* stage, int64_t M, int64_t K,
                                b2q_stream_t stream) {
  using namespace b2q;
  static const char* who = "b2q_stage_pinned";
  if (M < 0 || K < 0) return fail(B2Q_EINVAL, "%s: negative size", who);
  if (M == 0 || K == 0) return B2Q_OK;
  void* x_dev = nullptr;
  int rc = mapped(who, "x", x_host, &x_dev);
  if (rc) return rc;
  if (K % 4 || ldx < K || (ldx % 4) || !aligned(x_dev, 16))
    return fail(B2Q_EALIGN, "%s: x must be 16-byte aligned, K and ldx multiples of 4, ldx >= K", who);
  if (!stage || !aligned(stage, 16)) return fail(B2Q_EALIGN, "%s: stage must be 16-byte aligned device memory", who);
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, stage) != cudaSuccess || at.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return fail(B2Q_EINVAL, "%s: stage must be device memory", who);
  }
  DeviceInfo di;
  rc = device_info(&di);
  if (rc) return rc;
  const int64_t K4 = K / 4, total4 = M * K4;
  const int64_t want = (total4 + (int64_t)kCopyThreads * kCopyVec - 1) / ((int64_t)kCopyThreads * kCopyVec);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)di.sms * 8));
  cudaError_t le = launch_maybe_pdl(pinned_x_copy_kernel, dim3(grid), dim3(kCopyThreads), 0, (cudaStream_t)stream,
                                    reinterpret_cast<const float4*>(x_dev), ldx / 4, reinterpret_cast<float4*>(stage),
                                    K4, total4);
  if (le != cudaSuccess) {
    cudaGetLastError();
    return fail(B2Q_ECUDA, "%s: launch failed: %s", who, cudaGetErrorString(le));
  }
  return after_launch(who);
}
