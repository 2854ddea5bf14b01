// Instantiations of the TMA-ring GEMV kernels (see gemv_kernels.cuh), and the device error word they write.
#include "gemv_kernels.cuh"

namespace b2q {

template <int FMT, bool XREG>
static KernelFn pick(int R, int MC) {
  if (MC == 1) {
    if (R == 16) return XREG ? gemv_ring_kernel<FMT, 16, 1, true> : nullptr;
    switch (R) {
      case 1: return gemv_ring_kernel<FMT, 1, 1, XREG>;
      case 2: return gemv_ring_kernel<FMT, 2, 1, XREG>;
      case 4: return gemv_ring_kernel<FMT, 4, 1, XREG>;
      default: return gemv_ring_kernel<FMT, 8, 1, XREG>;
    }
  }
  if (MC == 2 && XREG) {  // two columns, each thread's chunks of both in registers
    switch (R) {
      case 1: return gemv_ring_kernel<FMT, 1, 2, true>;
      case 2: return gemv_ring_kernel<FMT, 2, 2, true>;
      case 4: return gemv_ring_kernel<FMT, 4, 2, true>;
      default: return gemv_ring_kernel<FMT, 8, 2, true>;
    }
  }
  if (MC == 4 && XREG) {  // three or four columns, each thread's chunks of all in registers
    switch (R) {
      case 1: return gemv_ring_kernel<FMT, 1, 4, true>;
      case 2: return gemv_ring_kernel<FMT, 2, 4, true>;
      case 4: return gemv_ring_kernel<FMT, 4, 4, true>;
      default: return gemv_ring_kernel<FMT, 8, 4, true>;
    }
  }
  switch (R) {
    case 1: return gemv_ring_kernel<FMT, 1, 4, false>;
    case 2: return gemv_ring_kernel<FMT, 2, 4, false>;
    case 4: return gemv_ring_kernel<FMT, 4, 4, false>;
    default: return gemv_ring_kernel<FMT, 8, 4, false>;
  }
}

KernelFn ring_kernel_for(int fmt, int R, int MC, bool xreg) {
  if (fmt == 0) return xreg ? pick<0, true>(R, MC) : pick<0, false>(R, MC);
  if (fmt == 2) return xreg ? pick<2, true>(R, MC) : pick<2, false>(R, MC);
  if (fmt == 3) return xreg ? pick<3, true>(R, MC) : pick<3, false>(R, MC);
  if (fmt == 4) return xreg ? pick<4, true>(R, MC) : pick<4, false>(R, MC);
  return xreg ? pick<1, true>(R, MC) : pick<1, false>(R, MC);
}

}  // namespace b2q

extern "C" int b2q_device_error(int* code, int clear) {
  using namespace b2q;
  if (!code) return fail(B2Q_EINVAL, "b2q_device_error: null pointer");
  cudaError_t e = cudaMemcpyFromSymbol(code, g_device_error, sizeof(int));
  if (e != cudaSuccess) return fail(B2Q_ECUDA, "b2q_device_error: %s", cudaGetErrorString(e));
  if (clear && *code) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return fail(B2Q_ECUDA, "b2q_device_error: %s", cudaGetErrorString(e));
  }
  return B2Q_OK;
}
