// Instantiations of the fused decode kernel for bf16 (one translation unit
// per dtype keeps the builds parallel).
#include "decode_kernel.cuh"

namespace saga {

const void* pick_decode_kernel_bf16(int D, int mode, bool tc, bool mask, bool shard, bool paged) {
  if (paged) {  // paged caches (not with sharding)
    if (shard) return nullptr;
    if (tc) return mask ? pick_d_mode<__nv_bfloat16, true, true, false, true>(D, mode) : pick_d_mode<__nv_bfloat16, true, false, false, true>(D, mode);
    return mask ? pick_d_mode<__nv_bfloat16, false, true, false, true>(D, mode) : pick_d_mode<__nv_bfloat16, false, false, false, true>(D, mode);
  }
  if (shard) {
    if (!tc) return nullptr;
    return mask ? pick_d_mode<__nv_bfloat16, true, true, true>(D, mode) : pick_d_mode<__nv_bfloat16, true, false, true>(D, mode);
  }
  if (tc) return mask ? pick_d_mode<__nv_bfloat16, true, true, false>(D, mode) : pick_d_mode<__nv_bfloat16, true, false, false>(D, mode);
  return mask ? pick_d_mode<__nv_bfloat16, false, true, false>(D, mode) : pick_d_mode<__nv_bfloat16, false, false, false>(D, mode);
}

}  // namespace saga
