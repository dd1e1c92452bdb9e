// Instantiations of the fused decode kernel for fp32 (one translation unit
// per dtype keeps the builds parallel).
#include "decode_kernel.cuh"

namespace saga {

const void* pick_decode_kernel_fp32(int D, int mode, bool tc, bool mask, bool shard, bool paged) {
  if (shard) return nullptr;  // sequence sharding runs on the tensor-core path only
  if (paged)
    return mask ? pick_d_mode<float, false, true, false, true>(D, mode) : pick_d_mode<float, false, false, false, true>(D, mode);
  return mask ? pick_d_mode<float, false, true, false>(D, mode) : pick_d_mode<float, false, false, false>(D, mode);
}

}  // namespace saga
