// Split-K GEMV for callers that cannot allocate device memory.
//
// Some callers of this library cannot hand it a scratch buffer: an inference engine that reserves all of a GPU's
// memory when it starts and gives out no further buffers, or a caller that reaches the library through a plain C
// FFI (Go, Java, Rust) and has no device allocator of its own. b2q_quant_gemv_ws needs a caller-allocated workspace
// for its split-K partial sums; this entry point runs the same schedule with the partial sums in a fixed array
// inside the library, so the caller passes only inputs and outputs and nothing is allocated.
//
// The array is a file-scope __device__ variable: every GPU that loads the library holds it (kStaticScratchBytes)
// until the process exits. Host code cannot use the array's name as a device address, so its address is taken once
// per device with cudaGetSymbolAddress (on the first call made with that device current) and passed to the kernels.
// The address is kept per device ordinal for the life of the process: a cudaDeviceReset (or another teardown of the
// device's primary context) may reload the module elsewhere, after which this entry point must not be called again.
#include <mutex>

#include "b2q_internal.h"

namespace b2q {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB per GPU: splits * M * N partial f32 sums

static __device__ __align__(256) float g_static_scratch[kStaticScratchBytes / sizeof(float)];

static std::mutex g_scratch_mu;
static void* g_scratch_addr[64];  // device address of g_static_scratch, per device ordinal (set once)

static int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(B2Q_ECUDA, "b2q_quant_gemv_splitk_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(B2Q_ECUDA, "b2q_quant_gemv_splitk_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return fail(B2Q_ECUDA, "b2q_quant_gemv_splitk_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return B2Q_OK;
}

}  // namespace b2q

extern "C" size_t b2q_noalloc_scratch_bytes(void) { return b2q::kStaticScratchBytes; }

extern "C" int b2q_quant_gemv_splitk_noalloc(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws,
                                             const float* x, int64_t ldx, float* y, int64_t N, int64_t K, int64_t M,
                                             int splits, b2q_stream_t stream) {
  using namespace b2q;
  if (fmt < 0 || fmt > 4)
    return fail(B2Q_EINVAL,
                "b2q_quant_gemv_splitk_noalloc: fmt %d is not Q4_0 (0), TQ2_0 (1), Q8_0 (2), IQ4_NL (3) or Q4_K (4)", fmt);
  if (splits >= 2 && N > 0 && M > 0 && (size_t)splits * (size_t)M * (size_t)N * sizeof(float) > kStaticScratchBytes)
    return fail(B2Q_ERANGE,
                "b2q_quant_gemv_splitk_noalloc: %d splits x M=%lld x N=%lld partial sums exceed the %zu-byte "
                "built-in scratch; use b2q_quant_gemv_ws with a workspace of b2q_workspace_size bytes instead",
                splits, (long long)M, (long long)N, kStaticScratchBytes);
  void* scratch = nullptr;
  int rc = static_scratch(&scratch);
  if (rc) return rc;
  return quant_gemv_forced_split(fmt, wq, ldwq, ws, x, ldx, y, N, K, M, splits, reinterpret_cast<float*>(scratch),
                                 kStaticScratchBytes, (cudaStream_t)stream);
}
