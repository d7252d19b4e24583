// pd_append.cu -- paged-KV append (decode write and prefill write) for sm_100a.
//
// Replaces the two index_copy_ launches of PagedPool.write_slots (model/paged.py:236-239)
// with one launch that moves K and V together. Token i of the source goes to flat pool row
// `slot` = block_id * block_size + offset, i.e. block slot / bs, position slot % bs of the
// (n_blocks, block_size, n_kv_head, head_dim) pool. The slot comes either from a slot-id
// vector (write_slots) or, for the decode step, straight from the int32 block table and the
// int64 position of the row (PagedKV._refresh_slots, model/paged.py:499-501, done in the
// kernel). Same-dtype copies are bit copies; a dtype change rounds to nearest even, which is
// what torch's Tensor.to does. A slot or block id outside the pool is skipped and recorded
// in the device error word (the reference's index_copy_ would raise a device assert).
// Optionally the K rows get their rotary embedding on the way in (the rotation the model
// applies just before the write, model/layers.py apply_rotary_emb_partial).
#include "pd_internal.h"

namespace pd {

namespace {

template <typename S, typename Dt, int V>
struct Mover;

// V == 8: eight consecutive head_dim elements per thread, 16-byte aligned rows.
template <typename S, typename Dt>
struct Mover<S, Dt, 8> {
  __device__ __forceinline__ static void move(Dt* dst, const S* src) {
    float f[8];
    if constexpr (sizeof(S) == 4) {
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(src + 4);
      f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
      f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
      const uint4 r = *reinterpret_cast<const uint4*>(src);
      if constexpr (std::is_same<S, Dt>::value) {
        *reinterpret_cast<uint4*>(dst) = r;  // bit copy
        return;
      }
      Elem<S>::unpack(r, f);
    }
    if constexpr (std::is_same<S, Dt>::value && sizeof(S) == 4) {
      *reinterpret_cast<float4*>(dst) = make_float4(f[0], f[1], f[2], f[3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(f[4], f[5], f[6], f[7]);
    } else if constexpr (sizeof(Dt) == 4) {
      *reinterpret_cast<float4*>(dst) = make_float4(f[0], f[1], f[2], f[3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(f[4], f[5], f[6], f[7]);
    } else {
      *reinterpret_cast<uint4*>(dst) = Elem<Dt>::pack(f);
    }
  }
};

template <typename S, typename Dt>
struct Mover<S, Dt, 1> {
  __device__ __forceinline__ static void move(Dt* dst, const S* src) {
    if constexpr (std::is_same<S, Dt>::value) {
      *dst = *src;
    } else {
      *dst = Elem<Dt>::from_float(Elem<S>::to_float(*src));
    }
  }
};

template <typename S, typename Dt, int V>
__global__ void __launch_bounds__(256) pd_append_kernel(const AppendParams p) {
  const int per_row = p.head_dim / V;
  const int64_t per_token = int64_t(p.n_kv_head) * per_row;
  const int64_t total = p.n_tokens * per_token;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / per_token;
    const int rem = int(i - t * per_token);
    const int h = rem / per_row;
    const int d = (rem - h * per_row) * V;
    int64_t blk, off;
    if (p.use_table) {
      const int64_t pos = p.pos[t];
      const int64_t page = pos >= 0 ? pos / p.block_size : -1;
      if (page < 0 || page >= p.max_blocks) {
        if (rem == 0) atomicOr(p.err, DEVERR_APPEND_RANGE);
        continue;
      }
      blk = p.table[t * p.bt_stride + page];
      off = pos - page * p.block_size;
    } else {
      const int64_t slot = p.slot_i64 ? reinterpret_cast<const int64_t*>(p.slots)[t]
                                      : int64_t(reinterpret_cast<const int32_t*>(p.slots)[t]);
      if (slot < 0) {
        if (rem == 0) atomicOr(p.err, DEVERR_APPEND_RANGE);
        continue;
      }
      blk = slot / p.block_size;
      off = slot - blk * p.block_size;
    }
    if (blk < 0 || blk >= p.n_blocks) {
      if (rem == 0) atomicOr(p.err, DEVERR_APPEND_RANGE);
      continue;
    }
    const S* krow = reinterpret_cast<const S*>(p.k) + t * p.k_s0 + h * p.k_s1;
    const S* vs = reinterpret_cast<const S*>(p.v) + t * p.v_s0 + h * p.v_s1 + d;
    Dt* kd = reinterpret_cast<Dt*>(p.k_pool) + blk * p.kp_sb + off * p.kp_sn + h * p.kp_sh + d;
    Dt* vd = reinterpret_cast<Dt*>(p.v_pool) + blk * p.vp_sb + off * p.vp_sn + h * p.vp_sh + d;
    if constexpr (std::is_same<S, Dt>::value) {
      if (p.rope_cos != nullptr) {  // K rotated first (same dtype throughout, checked on the host)
        const S* cs = reinterpret_cast<const S*>(p.rope_cos) + t * p.rope_stride;
        const S* sn = reinterpret_cast<const S*>(p.rope_sin) + t * p.rope_stride;
#pragma unroll
        for (int j = 0; j < V; ++j) kd[j] = rope_elem(krow, cs, sn, d + j, p.rope_dim);
      } else {
        Mover<S, Dt, V>::move(kd, krow + d);
      }
    } else {
      Mover<S, Dt, V>::move(kd, krow + d);
    }
    Mover<S, Dt, V>::move(vd, vs);
  }
}

template <typename S, typename Dt>
cudaError_t launch_typed(const AppendParams& p, bool vec, cudaStream_t stream) {
  const int v = vec ? 8 : 1;
  const int64_t total = p.n_tokens * p.n_kv_head * (p.head_dim / v);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (vec)
    pd_append_kernel<S, Dt, 8><<<unsigned(blocks), threads, 0, stream>>>(p);
  else
    pd_append_kernel<S, Dt, 1><<<unsigned(blocks), threads, 0, stream>>>(p);
  return cudaGetLastError();
}

template <typename S>
cudaError_t launch_dst(const AppendParams& p, int dst, bool vec, cudaStream_t stream) {
  switch (dst) {
    case 0: return launch_typed<S, float>(p, vec, stream);
    case 1: return launch_typed<S, __half>(p, vec, stream);
    case 2: return launch_typed<S, __nv_bfloat16>(p, vec, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_append(const AppendParams& p, int src_dtype, int dst_dtype, bool vec16,
                          cudaStream_t stream) {
  switch (src_dtype) {
    case 0: return launch_dst<float>(p, dst_dtype, vec16, stream);
    case 1: return launch_dst<__half>(p, dst_dtype, vec16, stream);
    case 2: return launch_dst<__nv_bfloat16>(p, dst_dtype, vec16, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace pd
