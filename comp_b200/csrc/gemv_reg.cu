// Instantiations of the register-streaming GEMV kernels (see gemv_kernels.cuh).
#include "gemv_kernels.cuh"

namespace b2q {

template <int FMT, bool BYTES, bool XREG>
static KernelFn pick(int R, int MC) {
  if (MC == 1) {
    switch (R) {
      case 1: return gemv_reg_kernel<FMT, 1, 1, BYTES, XREG>;
      case 2: return gemv_reg_kernel<FMT, 2, 1, BYTES, XREG>;
      case 4: return gemv_reg_kernel<FMT, 4, 1, BYTES, XREG>;
      default: return gemv_reg_kernel<FMT, 8, 1, BYTES, XREG>;
    }
  }
  switch (R) {
    case 1: return gemv_reg_kernel<FMT, 1, 4, BYTES, false>;
    case 2: return gemv_reg_kernel<FMT, 2, 4, BYTES, false>;
    case 4: return gemv_reg_kernel<FMT, 4, 4, BYTES, false>;
    default: return gemv_reg_kernel<FMT, 8, 4, BYTES, false>;
  }
}

KernelFn reg_kernel_for(int fmt, bool bytes, int R, int MC, bool xreg) {
  if (MC != 1) xreg = false;
  if (fmt == 4) return nullptr;  // Q4_K runs on the TMA ring only
  if (fmt == 0) {
    if (bytes) return xreg ? pick<0, true, true>(R, MC) : pick<0, true, false>(R, MC);
    return xreg ? pick<0, false, true>(R, MC) : pick<0, false, false>(R, MC);
  }
  if (fmt == 2) {
    if (bytes) return xreg ? pick<2, true, true>(R, MC) : pick<2, true, false>(R, MC);
    return xreg ? pick<2, false, true>(R, MC) : pick<2, false, false>(R, MC);
  }
  if (fmt == 3) {
    if (bytes) return xreg ? pick<3, true, true>(R, MC) : pick<3, true, false>(R, MC);
    return xreg ? pick<3, false, true>(R, MC) : pick<3, false, false>(R, MC);
  }
  if (bytes) return xreg ? pick<1, true, true>(R, MC) : pick<1, true, false>(R, MC);
  return xreg ? pick<1, false, true>(R, MC) : pick<1, false, false>(R, MC);
}

}  // namespace b2q
