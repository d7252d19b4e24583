// pd_decode_mma_f16.cu -- tensor-core decode kernel instantiations for __half K/V: head dims
// 64, 128 and 256, q-head chunks of 1, 2, 4 or 8 (per-warp stages, swizzled pool maps).
#include "pd_decode_kernel.cuh"

namespace pd {

#define PD_MMA_ROW(D) \
  {launch_decode<__half, D, 1, false, true>, launch_decode<__half, D, 2, false, true>, \
   launch_decode<__half, D, 4, false, true>, launch_decode<__half, D, 8, false, true>}

static const DecodeLaunchFn kMmaTable[3][4] = {PD_MMA_ROW(64), PD_MMA_ROW(128), PD_MMA_ROW(256)};
#undef PD_MMA_ROW

DecodeLaunchFn decode_launcher_mma_f16(int d_index, int gt_index) {
  if (d_index < 3 || d_index >= 6 || gt_index < 0 || gt_index >= 4) return nullptr;
  return kMmaTable[d_index - 3][gt_index];
}

}  // namespace pd
