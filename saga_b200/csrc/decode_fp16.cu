// Instantiations of the fused decode kernel for fp16 (one translation unit
// per dtype keeps the builds parallel).
#include "decode_kernel.cuh"

namespace saga {

const void* pick_decode_kernel_fp16(int D, int mode, bool tc, bool mask) {
  if (tc) return mask ? pick_d_mode<__half, true, true>(D, mode) : pick_d_mode<__half, true, false>(D, mode);
  return mask ? pick_d_mode<__half, false, true>(D, mode) : pick_d_mode<__half, false, false>(D, mode);
}

}  // namespace saga
