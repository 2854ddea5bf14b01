// Host-side internals shared by the .cu translation units: error reporting, launch accounting, device facts.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>

#include "../../include/comp_b200.h"

namespace b2q {

// Records a printf-style message as the calling thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);

// Checks the CUDA launch status of the kernel just enqueued and counts it.
int after_launch(const char* what);

// Per-device facts, cached after the first query (thread-safe).
struct DeviceInfo {
  int sms = 0;
  int max_smem_optin = 0;  // bytes of dynamic shared memory one CTA may opt into
};
int device_info(DeviceInfo* out);

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Whether kernels launch with programmatic dependent launch (b2q_set_pipeline; on by default).
bool pdl_enabled();

// Launches `kernel` on `stream`, with the programmatic-stream-serialization attribute when PDL is enabled.
template <typename... KArgs, typename... Args>
cudaError_t launch_maybe_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// The argument checks of the fused quantize + GEMV entry points (f32 activations x [M][K], row stride K), without a
// launch (gemv.cu).
int check_quant_gemv_args(const char* who, int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x,
                          const float* y, int64_t N, int64_t K, int64_t M);

// Fused quantize + split-K GEMV with exactly `splits` K splits, partial sums in `workspace` (gemv.cu).
int quant_gemv_forced_split(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                            float* y, int64_t N, int64_t K, int64_t M, int splits, float* workspace,
                            size_t workspace_bytes, cudaStream_t stream);

}  // namespace b2q
