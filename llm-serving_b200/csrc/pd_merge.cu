// pd_merge.cu -- log-sum-exp merge of split-KV partials (sm_100a).
//
// Input: n_parts triples (m, l, acc) per (row, q head), fp32: part i's m and l are
// (B, H) at m + i * ml_stride (resp. l), its acc (B, H, D) at acc + i * acc_stride. m is the max of the log2-scaled scores of
// the part (-inf when the part saw no token), l = sum exp2(s - m), acc = sum exp2(s - m) v.
// Output: out[b, h] = sum_p 2^(m_p - M) acc_p / max(sum_p 2^(m_p - M) l_p, 1), M = max_p m_p,
// i.e. the reference's acc / max(l, 1) (model/triton_decode.py:639) over the union of the
// parts; a row whose parts are all empty decodes to zeros. One warp per (row, head), lanes
// over head_dim in float4 steps; the partials are a few hundred KB, so this is launch-bound.
#include "pd_internal.h"

namespace pd {

namespace {

template <typename T>
__global__ void __launch_bounds__(256) pd_merge_kernel(const MergeParams p) {
  const int warps = blockDim.x >> 5;
  const int64_t pair = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t pairs = int64_t(p.batch) * p.n_head;
  if (pair >= pairs) return;
  float M = -INFINITY;
  for (int i = lane; i < p.n_parts; i += 32) M = fmaxf(M, p.m[i * p.ml_stride + pair]);
  for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL_MASK, M, o));
  const int64_t b = pair / p.n_head;
  const int64_t h = pair - b * p.n_head;
  T* out = reinterpret_cast<T*>(p.out) + b * p.o_sb + h * p.o_sh;
  if (M == -INFINITY) {
    for (int d = lane; d < p.head_dim; d += 32) out[d] = Elem<T>::from_float(0.f);
    return;
  }
  float L = 0.f;
  for (int i = lane; i < p.n_parts; i += 32) {
    const float mi = p.m[i * p.ml_stride + pair];
    L += p.l[i * p.ml_stride + pair] * exp2f(mi - M);
  }
  for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(FULL_MASK, L, o);
  const float inv = 1.f / fmaxf(L, 1.f);
  for (int d = lane * 4; d < p.head_dim; d += 128) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < p.n_parts; ++i) {
      const float f = exp2f(p.m[i * p.ml_stride + pair] - M);
      const float4 x = *reinterpret_cast<const float4*>(p.acc + i * p.acc_stride + pair * p.head_dim + d);
      a.x = fmaf(f, x.x, a.x);
      a.y = fmaf(f, x.y, a.y);
      a.z = fmaf(f, x.z, a.z);
      a.w = fmaf(f, x.w, a.w);
    }
    out[d + 0] = Elem<T>::from_float(a.x * inv);
    out[d + 1] = Elem<T>::from_float(a.y * inv);
    out[d + 2] = Elem<T>::from_float(a.z * inv);
    out[d + 3] = Elem<T>::from_float(a.w * inv);
  }
}

}  // namespace

cudaError_t launch_merge(const MergeParams& p, int dtype, cudaStream_t stream) {
  const int64_t pairs = int64_t(p.batch) * p.n_head;
  if (pairs == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = (pairs + 7) / 8;
  switch (dtype) {
    case 0: pd_merge_kernel<float><<<unsigned(blocks), threads, 0, stream>>>(p); break;
    case 1: pd_merge_kernel<__half><<<unsigned(blocks), threads, 0, stream>>>(p); break;
    case 2: pd_merge_kernel<__nv_bfloat16><<<unsigned(blocks), threads, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace pd
