// pd_common.cuh -- device helpers shared by the paged-decode kernels (sm_100a).
//
// PTX wrappers for mbarrier / TMA (cp.async.bulk.tensor), element conversions and the
// parameter blocks the host launchers fill. Nothing here allocates or synchronises.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pd {

constexpr unsigned FULL_MASK = 0xffffffffu;

// Device error word bits (mirrors PD_DEVERR_* in include/paged_decode.h).
constexpr unsigned DEVERR_WAIT_TIMEOUT = 1u;
constexpr unsigned DEVERR_APPEND_RANGE = 2u;

// A bounded wait on an mbarrier or an arrival counter gives up after this many nanoseconds of
// %globaltimer (the launch's `wait_ns`, which pd_set_wait_limit can shorten to exercise the
// error path). The drain of copies still in flight after such a failure, and a warp's exit
// bookkeeping, always use the fixed limits below, so that a CTA never retires with a copy in
// flight and the workspace epoch always advances.
constexpr unsigned long long WAIT_LIMIT_NS = 1000000000ull;      // 1 s (default wait_ns, exit)
constexpr unsigned long long DRAIN_LIMIT_NS = 100000000ull;      // 0.1 s per stage

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x >> 1); }

// ------------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Limits below this are test limits (pd_set_wait_limit): every wait under such a limit gives
// up at once, whether or not its phase is complete, so a test can run the error path
// deterministically (the drains after it use DRAIN_LIMIT_NS and always finish).
constexpr unsigned long long TEST_LIMIT_NS = 1000ull;

// Warp-collective bounded wait: returns true once every lane has observed the phase with
// the given parity complete, false (uniformly) once `limit_ns` has elapsed.
__device__ __forceinline__ bool warp_wait_phase(uint32_t bar, uint32_t parity,
                                                unsigned long long limit_ns) {
  if (limit_ns < TEST_LIMIT_NS) return false;
  bool done = mbar_try_wait(bar, parity);
  if (__all_sync(FULL_MASK, done)) return true;
  unsigned long long start = global_timer_ns();
  for (unsigned iter = 1;; ++iter) {
    if (!done) done = mbar_try_wait(bar, parity);
    if (__all_sync(FULL_MASK, done)) return true;
    if ((iter & 63u) == 0) {
      unsigned long long now = __shfl_sync(FULL_MASK, global_timer_ns(), 0);
      unsigned long long t0 = __shfl_sync(FULL_MASK, start, 0);
      if (now - t0 > limit_ns) return false;
    }
  }
}

// 4-D tiled TMA load into shared memory, completing `bytes` on the mbarrier.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 5-D tiled TMA load (the 128-byte-swizzled pool map of the tensor-core decode path).
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// L2 policy for data read once: its lines are the first evicted, so a stream of K/V that is
// larger than L2 does not push out what the launch still needs there (split partials, the
// block table, q).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// tma_load_4d / tma_load_5d with an L2 cache policy (from createpolicy).
__device__ __forceinline__ void tma_load_4d_hint(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                 int c0, int c1, int c2, int c3, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d_hint(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                 int c0, int c1, int c2, int c3, int c4, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "l"(pol)
      : "memory");
}

// ---- warp-level tensor-core fragments (mma.sync / ldmatrix / movmatrix) ----------------
// Fragment layouts (g = lane / 4, c = lane % 4), 16-bit elements packed in pairs, the lower
// column in the low half:
//   A 16x16 (row-major): a0 (row g, k 2c..2c+1), a1 (row g+8, ..), a2 (row g, k 2c+8..),
//                        a3 (row g+8, k 2c+8..); A 16x8: a0, a1.
//   B 16x8 (k x n):      b0 (k 2c..2c+1, n g), b1 (k 2c+8.., n g); B 8x8: b0.
//   C/D 16x8 fp32:       c0, c1 (row g, cols 2c, 2c+1), c2, c3 (row g+8, same cols).
// ldmatrix: lane l gives the shared address of row l % 8 of matrix l / 8; register i holds
// matrix i in the A/B layout above (transposed with .trans). The smem reads are volatile so
// that they stay after the barrier waits that publish the bytes.

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Transpose of an 8x8 16-bit matrix held one pair per lane (row g, cols 2c..2c+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
struct Mma;

template <>
struct Mma<__nv_bfloat16> {
  // d += A (16x16) * B (16x8), fp32 accumulation.
  __device__ __forceinline__ static void m16n8k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                  uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  // d += A (16x8) * B (8x8).
  __device__ __forceinline__ static void m16n8k8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
  }
};

template <>
struct Mma<__half> {
  __device__ __forceinline__ static void m16n8k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                  uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static void m16n8k8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
  }
};

// Programmatic dependent launch. griddep_wait blocks until the grid this launch depends on
// (the previous kernel in the stream, when the launch allowed overlapping it) has completed
// and its memory is visible; without such a dependency it returns at once.
// griddep_launch_dependents lets the next kernel of the stream start launching.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Atomic add at GPU scope with acquire-release semantics: it releases this thread's earlier
// writes (and those that its warp ordered before it with __syncwarp) and, when its answer says
// that every other piece has arrived, acquires theirs; after a __syncwarp the whole warp may
// read them.
__device__ __forceinline__ unsigned long long atom_add_acq_rel_gpu(unsigned long long* p,
                                                                   unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.add.acq_rel.gpu.global.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}

// Atomic add at GPU scope with release semantics: this thread's earlier writes (and those of
// threads synchronised with it, e.g. by __syncwarp) are visible before the add is.
__device__ __forceinline__ unsigned long long atom_add_release_gpu(unsigned long long* p,
                                                                   unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.add.release.gpu.global.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}

// Prefetches one 128-byte line into L2.
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

// Orders this thread's generic-proxy shared-memory writes before later async-proxy (TMA)
// accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------ element conversion
// A "chunk" is 16 bytes of one row: 8 bf16/fp16 or 4 fp32 elements.

template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static constexpr int PER_CHUNK = 4;
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    f[0] = __uint_as_float(r.x);
    f[1] = __uint_as_float(r.y);
    f[2] = __uint_as_float(r.z);
    f[3] = __uint_as_float(r.w);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
  __device__ __forceinline__ static void unpack_pairs(const uint4& r, float2* f) {
    f[0] = make_float2(__uint_as_float(r.x), __uint_as_float(r.y));
    f[1] = make_float2(__uint_as_float(r.z), __uint_as_float(r.w));
  }
  __device__ __forceinline__ static float to_float(float x) { return x; }
  __device__ __forceinline__ static float from_float(float x) { return x; }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int PER_CHUNK = 8;
  // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 pattern.
  __device__ __forceinline__ static void unpack2(uint32_t w, float* f) {
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xffff0000u);
  }
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    unpack2(r.x, f + 0);
    unpack2(r.y, f + 2);
    unpack2(r.z, f + 4);
    unpack2(r.w, f + 6);
  }
  __device__ __forceinline__ static float2 pair(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  __device__ __forceinline__ static void unpack_pairs(const uint4& r, float2* f) {
    f[0] = pair(r.x);
    f[1] = pair(r.y);
    f[2] = pair(r.z);
    f[3] = pair(r.w);
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // round to nearest even
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
  __device__ __forceinline__ static float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_float(float x) {
    return __float2bfloat16_rn(x);
  }
};

template <>
struct Elem<__half> {
  static constexpr int PER_CHUNK = 8;
  __device__ __forceinline__ static void unpack2(uint32_t w, float* f) {
    float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w));
    f[0] = v.x;
    f[1] = v.y;
  }
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    unpack2(r.x, f + 0);
    unpack2(r.y, f + 2);
    unpack2(r.z, f + 4);
    unpack2(r.w, f + 6);
  }
  __device__ __forceinline__ static void unpack_pairs(const uint4& r, float2* f) {
    f[0] = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
    f[1] = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    f[2] = __half22float2(*reinterpret_cast<const __half2*>(&r.z));
    f[3] = __half22float2(*reinterpret_cast<const __half2*>(&r.w));
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
  __device__ __forceinline__ static float to_float(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_float(float x) { return __float2half_rn(x); }
};

// ------------------------------------------------------------------ rotary embedding

// Element e of a head row x after GPT-NeoX rotary embedding over its first rot_dim elements
// (pairs (i, i + rot_dim / 2); elements past rot_dim pass through), with the rounding of
// torch's elementwise ops in the row's dtype (model/layers.py apply_rotary_emb_partial):
//   out[i]        = r(r(x1 * cos) - r(x2 * sin))
//   out[i + half] = r(r(x1 * sin) + r(x2 * cos))
// where r() rounds to T. Every operation is an explicitly rounded fp32 op, never contracted
// into an FMA, so every thread that computes an element gets the same bits.
template <typename T>
__device__ __forceinline__ T rope_elem(const T* x, const T* cos, const T* sin, int e, int rot_dim) {
  using E = Elem<T>;
  if (e >= rot_dim) return x[e];
  const int half = rot_dim >> 1;
  const int i = e < half ? e : e - half;
  const float x1 = E::to_float(x[i]), x2 = E::to_float(x[i + half]);
  const float c = E::to_float(cos[i]), s = E::to_float(sin[i]);
  if (e < half) {
    const float a = E::to_float(E::from_float(__fmul_rn(x1, c)));
    const float b = E::to_float(E::from_float(__fmul_rn(x2, s)));
    return E::from_float(__fsub_rn(a, b));
  }
  const float a = E::to_float(E::from_float(__fmul_rn(x1, s)));
  const float b = E::to_float(E::from_float(__fmul_rn(x2, c)));
  return E::from_float(__fadd_rn(a, b));
}

// The 16-byte chunk of the rotated row x that starts at element e0. Kept out of line: the
// decode kernel calls it only for the appended row of a tile, and inlining it into the
// streaming loop costs registers there.
template <typename T>
__device__ __noinline__ uint4 rope_chunk(const T* x, const T* cos, const T* sin, int e0, int rot_dim) {
  constexpr int N = 16 / int(sizeof(T));
  union {
    T v[N];
    uint4 u;
  } out;
#pragma unroll
  for (int j = 0; j < N; ++j) out.v[j] = rope_elem(x, cos, sin, e0 + j, rot_dim);
  return out.u;
}

// ------------------------------------------------------------------ parameter blocks

// Everything the decode kernel reads besides the two TMA descriptors. Element strides.
struct DecodeParams {
  const void* q;
  int64_t q_sb, q_sh;
  void* out;  // mode 0: (B, H, D) in the input dtype
  int64_t o_sb, o_sh;
  float* part_m;    // mode 1: (B, H)
  float* part_l;    // mode 1: (B, H)
  float* part_acc;  // mode 1: (B, H, D)
  const int32_t* table;
  int64_t bt_stride;
  const int32_t* seqlen;
  unsigned long long* counters;  // (B * H_kv * n_gchunks) arrival counters: (epoch << 32) | count
  float* ws_ml;     // (workers * 2, 2 * GT) partial m | l
  float* ws_acc;    // (workers * 2, GT * D) partial accumulators
  unsigned* err;    // device error word
  int32_t max_blocks;
  int32_t capacity;  // max_blocks * block_size (seqlen clamp)
  int32_t batch;
  int32_t n_head;
  int32_t n_kv_head;
  int32_t group;      // n_head / n_kv_head
  int32_t n_gchunks;  // group / GT
  int32_t block_size;
  int32_t log2_bs;
  int32_t box_tokens;  // tokens per TMA box = min(TILE, block_size)
  int32_t log2_box;
  int32_t mode;        // 0: normalised output, 1: (m, l, acc) partials
  int32_t stages;      // pipeline depth per warp
  int32_t min_tiles;   // minimum tiles per active warp (unit split)
  int32_t row_cost;    // column split: extra virtual columns charged to every row start
  int32_t smem_arrays_off;
  int32_t smem_stage_off;
  float scale_log2;
  // Launch id ("epoch") bookkeeping in the workspace header. Each launch reads its epoch
  // from *epoch_word; the last of its warps to leave (counted on *exit_counter, tagged like
  // the item counters) stores epoch + 1 there, so consecutive launches on one workspace --
  // replays of a captured CUDA graph included -- never share an epoch.
  unsigned* epoch_word;
  unsigned long long* exit_counter;
  uint32_t tag_salt;  // even; mixed into the counters' tags (counter_tag in pd_decode_kernel.cuh)
  // Step cache of the work split (nullptr: off). One STEP_REC_BYTES record per physical warp
  // (blockIdx.x * warps + warp), written by a launch that computed its split and read by later
  // launches whose lengths hash to the same key (the layers of one decode step): see
  // StepRecord in pd_decode_kernel.cuh.
  unsigned char* step_rec;
  unsigned long long step_salt;  // the plan's geometry and launch shape, mixed into the key
  int32_t step_table;  // 1: the block table never changes, so cached table windows are valid
  unsigned long long wait_ns;  // limit of mbarrier and arrival-counter waits
  // Fused append (append != 0): before the decode reads them, row b's new K and V rows
  // (app_k/app_v, same dtype as the pool, 16-byte aligned) are stored at logical position
  // app_pos[b] of the row, i.e. pool block table[b, pos / bs], slot pos % bs, and the tile
  // that covers that position takes the two rows from the source instead of from its TMA
  // copy. Precondition: no other row of the launch reads an appended slot.
  int32_t append;
  const void* app_k;
  const void* app_v;
  int64_t app_k_sb, app_k_sh, app_v_sb, app_v_sh;
  const int64_t* app_pos;
  void* pool_k;
  void* pool_v;
  int64_t pk_sb, pk_sn, pk_sh;  // pool element strides: block, token, head
  int64_t pv_sb, pv_sn, pv_sh;
  int64_t n_blocks;
  // Rotary embedding of the appended K rows (rope_cos == nullptr: none). Row b uses
  // rope_cos/rope_sin + b * rope_stride (rope_dim / 2 entries each, the pool dtype).
  const void* rope_cos;
  const void* rope_sin;
  int64_t rope_stride;
  int32_t rope_dim;
};

struct AppendParams {
  void* k_pool;
  void* v_pool;
  int64_t kp_sb, kp_sn, kp_sh;
  int64_t vp_sb, vp_sn, vp_sh;
  int64_t n_blocks;
  const void* slots;  // slot-id variant (int32 or int64)
  const int32_t* table;
  int64_t bt_stride;
  const int64_t* pos;
  const void* k;
  const void* v;
  int64_t k_s0, k_s1, v_s0, v_s1;
  unsigned* err;
  int64_t n_tokens;
  int32_t max_blocks;
  int32_t block_size;
  int32_t n_kv_head;
  int32_t head_dim;
  int32_t use_table;  // 1: slot from block table + pos, 0: from slots
  int32_t slot_i64;
  // Rotary embedding of the K rows before they are stored (rope_cos == nullptr: none);
  // source, pool and tables share one dtype. Token t uses rope_cos/rope_sin + t * rope_stride.
  const void* rope_cos;
  const void* rope_sin;
  int64_t rope_stride;
  int32_t rope_dim;
};

// Chunked prefill over the paged pool (pd_prefill.cu). Element strides.
struct PrefillParams {
  const void* q;        // (total_q, H, D)
  int64_t q_st, q_sh;
  void* out;            // (total_q, H, D)
  int64_t o_st, o_sh;
  const int32_t* cu_q;      // (B + 1) query-token offsets
  const int32_t* seqlen_k;  // (B) keys per row, the chunk included
  const int32_t* table;
  int64_t bt_stride;
  int32_t max_blocks;
  int32_t capacity;     // max_blocks * block_size
  int32_t block_size;
  int32_t box_tokens;   // min(block_size, 64)
  float scale_log2;
  unsigned* err;
  unsigned long long wait_ns;  // limit of the stage waits
  // tcgen05 kernel only: 1 when the pool maps are grouped (one copy per box of box_tokens
  // tokens and every 128-byte piece, landing as 8-token groups of all pieces), 0 when each copy
  // is one piece of box_tokens rows.
  int32_t grouped;
  // Filled by the tcgen05 launcher (its grid is 1-D: query tile, kv head, row).
  int32_t batch;
  int32_t n_kv_head;
  int32_t q_tiles;
};

struct MergeParams {
  const float* m;
  const float* l;
  const float* acc;
  void* out;
  int64_t o_sb, o_sh;
  int64_t ml_stride;   // elements between parts of m (and of l)
  int64_t acc_stride;  // elements between parts of acc
  int32_t n_parts;
  int32_t batch;
  int32_t n_head;
  int32_t head_dim;
};

// Host-side launcher signatures (one instantiation per dtype / head_dim / group tile).
// pdl: launch with programmatic stream serialisation (may overlap the previous kernel).
typedef cudaError_t (*DecodeLaunchFn)(const DecodeParams&, const CUtensorMap&, const CUtensorMap&,
                                      dim3, dim3, size_t, cudaStream_t, bool pdl);

}  // namespace pd
