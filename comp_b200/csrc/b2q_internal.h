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

// Fused quantize + split-K GEMV with exactly `splits` K splits, partial sums in `workspace` (gemv.cu).
int quant_gemv_forced_split(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                            float* y, int64_t N, int64_t K, int64_t M, int splits, float* workspace,
                            size_t workspace_bytes, cudaStream_t stream);

}  // namespace b2q
