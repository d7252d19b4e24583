// pd_decode_f16.cu -- decode kernel instantiations for __half K/V (one file per dtype so the
// build compiles them in parallel). Head dims 8..256, q-head chunks of 1, 2, 4 or 8.
#include "pd_decode_kernel.cuh"

namespace pd {

#define PD_ROW(D) \
  {launch_decode<__half, D, 1>, launch_decode<__half, D, 2>, launch_decode<__half, D, 4>, \
   launch_decode<__half, D, 8>}

static const DecodeLaunchFn kTable[6][4] = {PD_ROW(8),  PD_ROW(16),  PD_ROW(32),
                                            PD_ROW(64), PD_ROW(128), PD_ROW(256)};
#undef PD_ROW

// (8 q heads per item never take the shared-stage kernel: see geometry() in pd_api.cu.)
#define PD_CTA_ROW(D) \
  {launch_decode<__half, D, 1, true>, launch_decode<__half, D, 2, true>, launch_decode<__half, D, 4, true>, nullptr}

static const DecodeLaunchFn kCtaTable[3][4] = {PD_CTA_ROW(64), PD_CTA_ROW(128), PD_CTA_ROW(256)};
#undef PD_CTA_ROW

DecodeLaunchFn decode_launcher_cta_f16(int d_index, int gt_index) {
  if (d_index < 3 || d_index >= 6 || gt_index < 0 || gt_index >= 4) return nullptr;
  return kCtaTable[d_index - 3][gt_index];
}

DecodeLaunchFn decode_launcher_f16(int d_index, int gt_index) {
  if (d_index < 0 || d_index >= 6 || gt_index < 0 || gt_index >= 4) return nullptr;
  return kTable[d_index][gt_index];
}

}  // namespace pd
