// Instantiations of the fused decode kernel for fp16 (one translation unit
// per dtype keeps the builds parallel).
#include "decode_kernel.cuh"

namespace saga {

const void* pick_decode_kernel_fp16(int D, int mode, bool tc, bool mask, bool shard, bool paged) {
  if (paged) {  // paged caches (not with sharding)
    if (shard) return nullptr;
    if (tc) return mask ? pick_d_mode<__half, true, true, false, true>(D, mode) : pick_d_mode<__half, true, false, false, true>(D, mode);
    return mask ? pick_d_mode<__half, false, true, false, true>(D, mode) : pick_d_mode<__half, false, false, false, true>(D, mode);
  }
  if (shard) {
    if (!tc) return nullptr;
    return mask ? pick_d_mode<__half, true, true, true>(D, mode) : pick_d_mode<__half, true, false, true>(D, mode);
  }
  if (tc) return mask ? pick_d_mode<__half, true, true, false>(D, mode) : pick_d_mode<__half, true, false, false>(D, mode);
  return mask ? pick_d_mode<__half, false, true, false>(D, mode) : pick_d_mode<__half, false, false, false>(D, mode);
}

}  // namespace saga
