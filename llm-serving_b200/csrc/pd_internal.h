// pd_internal.h -- host-side declarations shared by the translation units of the library.
#pragma once

#include "pd_common.cuh"

namespace pd {

DecodeLaunchFn decode_launcher_f32(int d_index, int gt_index);
DecodeLaunchFn decode_launcher_f16(int d_index, int gt_index);
DecodeLaunchFn decode_launcher_bf16(int d_index, int gt_index);
// Shared-stage (CTA) decode kernels: head_dim 64..256 (d_index 3..5), bf16 / fp16.
DecodeLaunchFn decode_launcher_cta_f16(int d_index, int gt_index);
DecodeLaunchFn decode_launcher_cta_bf16(int d_index, int gt_index);
// Tensor-core decode kernels (per-warp stages, 128-byte-swizzled pool maps): head_dim 64..256
// (d_index 3..5), bf16 / fp16.
DecodeLaunchFn decode_launcher_mma_f16(int d_index, int gt_index);
DecodeLaunchFn decode_launcher_mma_bf16(int d_index, int gt_index);

// Append: copies K and V rows into their pool slots. src/dst dtype codes as PD_F32/F16/BF16.
cudaError_t launch_append(const AppendParams& p, int src_dtype, int dst_dtype, bool vec16,
                          cudaStream_t stream);

// Chunked prefill attention over the paged pool (bf16/fp16, head_dim 64/128/256, group 1/2/4/8).
bool prefill_supported(int dtype, int head_dim, int group);
int prefill_tile_tokens(int head_dim);  // key tokens per tile (TMA boxes are at most this long)
size_t prefill_smem_bytes(int head_dim);
cudaError_t launch_prefill(const PrefillParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, int dtype,
                           int head_dim, int group, int max_seqlen_q, int batch, int n_kv_head,
                           cudaStream_t stream);

// The same prefill on the tcgen05 tensor cores (TMEM accumulators); its pool maps have
// one-piece boxes of at most prefill_tc_tile_tokens() tokens.
int prefill_tc_tile_tokens(int head_dim);
cudaError_t launch_prefill_tc(const PrefillParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, int dtype,
                              int head_dim, int group, int max_seqlen_q, int batch, int n_kv_head,
                              cudaStream_t stream);

// Log-sum-exp merge of n_parts (m, l, acc) triples into the normalised output.
cudaError_t launch_merge(const MergeParams& p, int dtype, cudaStream_t stream);

}  // namespace pd
