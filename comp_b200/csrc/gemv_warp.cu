// Instantiations of the warp-rows GEMV kernel (one activation column): Q4_0, TQ2_0, Q8_0 and IQ4_NL, R = 1, 2, 4
// rows per group.
#include "gemv_kernels.cuh"

namespace b2q {

KernelFn warp_kernel_for(int fmt, int R) {
  if (fmt == 0) {
    switch (R) {
      case 1: return gemv_warp_kernel<0, 1>;
      case 2: return gemv_warp_kernel<0, 2>;
      case 4: return gemv_warp_kernel<0, 4>;
    }
  } else if (fmt == 2) {
    switch (R) {
      case 1: return gemv_warp_kernel<2, 1>;
      case 2: return gemv_warp_kernel<2, 2>;
      case 4: return gemv_warp_kernel<2, 4>;
    }
  } else if (fmt == 3) {
    switch (R) {
      case 1: return gemv_warp_kernel<3, 1>;
      case 2: return gemv_warp_kernel<3, 2>;
      case 4: return gemv_warp_kernel<3, 4>;
    }
  } else if (fmt == 1) {
    switch (R) {
      case 1: return gemv_warp_kernel<1, 1>;
      case 2: return gemv_warp_kernel<1, 2>;
      case 4: return gemv_warp_kernel<1, 4>;
    }
  }
  return nullptr;
}

}  // namespace b2q
