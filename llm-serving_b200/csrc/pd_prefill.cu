// pd_prefill.cu -- block-table-aware chunked-prefill attention for sm_100a (bf16 / fp16 pools,
// head_dim 64, 128 or 256, 1, 2, 4 or 8 q heads per kv head).
//
// What it computes: for every row b, its new query tokens q[cu_q[b] .. cu_q[b+1]) (the chunk,
// Sq = cu_q[b+1] - cu_q[b] tokens) attend causally to the row's Lk = seqlen_k[b] tokens in the
// paged pool, the chunk's own K/V included (already appended): query token i sits at absolute
// position Lk - Sq + i and sees keys 0 .. Lk - Sq + i. This is the causal convention of
// flash-attn's varlen kernel with a block table (the reference's prefill, flash_attn 2.8.3
// varlen with causal=True, bottom-right aligned), with softmax(q k^T * scale) in fp32 and fp32
// P.V. A chunk of one token is exactly the paged decode.
//
// How (B200): one CTA of 4 warps per (64 query rows, kv head, row); rows are (token, q head)
// pairs of one kv head's group, token-major, so the group's q heads share every K/V tile.
//  * K/V tiles of 64 tokens (32 at head_dim 256) stream through 2 shared-memory stages by TMA from the pool's
//    128-byte-swizzled 5-D map (one box per block part), completing on mbarriers; thread 0
//    refills a stage once every warp has consumed it.
//  * Each warp owns 16 rows: S = Q K^T (m16n8k16, Q fragments held in registers from a
//    swizzled shared tile), fp32 online softmax per row in log2 units, then O += P V with P as
//    hi + lo 16-bit operands taken straight from the S accumulators (no shared-memory trip),
//    so the product carries P to about 2^-17 and matches fp32 P.V.
//  * Key tiles past the CTA's last query position are never loaded; the causal mask and the
//    row end are applied per element. V rows past the row end are zeroed in shared memory
//    before use, so stale bytes never reach the accumulators.
//  * Every wait is bounded (1 s of %globaltimer); on expiry the CTA records
//    DEVERR_WAIT_TIMEOUT and returns after draining its copies.
#include "paged_decode.h"
#include "pd_common.cuh"
#include "pd_internal.h"

namespace pd {

namespace {

constexpr int PF_ROWS = 64;    // query rows per CTA
constexpr int PF_WARPS = 4;

template <typename T, int D, int G>
struct PrefillCfg {
  static_assert(D == 64 || D == 128 || D == 256, "prefill: head_dim 64, 128 or 256");
  static constexpr int KT = D == 256 ? 32 : 64;   // tokens per K/V tile (two CTAs per SM fit)
  static constexpr int NT = KT / 8;               // 8-token n-tiles of S
  static constexpr int KK = KT / 16;              // 16-token k-steps of P.V
  // Q fragments stay in registers up to head_dim 128; at 256 the O accumulators need the
  // room, and each k-step's fragment is re-read from the shared Q tile per key tile.
  static constexpr bool HOLD_Q = D <= 128;
  static constexpr int ROW_BYTES = D * 2;
  static constexpr int KS = D / 16;               // q.K k-steps
  static constexpr int DN = D / 8;                // 8-wide head_dim tiles of O
  static constexpr int TILE_BYTES = KT * ROW_BYTES;  // K (or V) bytes of one tile
  static constexpr int Q_BYTES = PF_ROWS * ROW_BYTES;
  static constexpr int TQ = PF_ROWS / G;          // query tokens per CTA
};

// Byte offset of 16-byte unit u of row r in a swizzled tile whose 128-byte pieces are
// `piece_rows` rows apart: piece-major, rows of 128 bytes, unit XOR (row % 8).
__device__ __forceinline__ uint32_t swz(int r, int u, int piece_rows) {
  return uint32_t((u >> 3) * piece_rows * 128 + r * 128 + (((u & 7) ^ (r & 7)) << 4));
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(PF_WARPS * 32, 1)
    pd_prefill_kernel(const __grid_constant__ PrefillParams p, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap) {
  using C = PrefillCfg<T, D, G>;
  using E = Elem<T>;
  using X = Mma<T>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int b = blockIdx.y;
  const int h = blockIdx.z;
  const int q_begin = __ldg(p.cu_q + b);
  const int sq = __ldg(p.cu_q + b + 1) - q_begin;
  int lk = __ldg(p.seqlen_k + b);
  lk = lk < 0 ? 0 : (lk > p.capacity ? p.capacity : lk);
  const int tok0 = blockIdx.x * C::TQ;  // first query token of this CTA
  if (sq <= 0 || tok0 >= sq) return;
  const int ntok = sq - tok0 < C::TQ ? sq - tok0 : C::TQ;
  const int ctx = lk - sq;  // keys before the chunk (may be negative: bad input, masked below)
  // keys this CTA needs: 0 .. ctx + tok0 + ntok - 1
  int kend = ctx + tok0 + ntok;
  if (kend > lk) kend = lk;
  if (kend < 0) kend = 0;
  const int ntiles = (kend + C::KT - 1) / C::KT;

  // shared memory: [2 full barriers | pad | Q tile | 2 stages of (K tile, V tile)], 1 KB aligned
  const uint32_t base = smem_addr(smem_raw);
  unsigned char* smem = smem_raw + (((base + 1023u) & ~1023u) - base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  unsigned char* qs = smem + 1024;
  unsigned char* stages = qs + C::Q_BYTES;
  const uint32_t qs_addr = smem_addr(qs);
  const uint32_t st_addr = smem_addr(stages);

  if (tid == 0) {
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
    mbar_init(smem_addr(bars + 0), 1);
    mbar_init(smem_addr(bars + 1), 1);
    fence_barrier_init();
  }
  __syncthreads();

  const int bs = p.block_size;
  const int bt = p.box_tokens;  // tokens per TMA box (min(bs, 64))
  const int npages = (lk + bs - 1) / bs;
  auto issue = [&](int kt, int st) {  // thread 0 only
    const int t0 = kt * C::KT;
    const int covered = kend - t0 < C::KT ? kend - t0 : C::KT;  // >= 1
    const int boxes = (covered + bt - 1) / bt;
    const uint32_t bar = smem_addr(bars + st);
    const uint32_t kdst = st_addr + uint32_t(st) * 2u * C::TILE_BYTES;
    const uint32_t vdst = kdst + C::TILE_BYTES;
    const uint32_t box_bytes = uint32_t(bt) * C::ROW_BYTES;
    mbar_arrive_expect_tx(bar, 2u * uint32_t(boxes) * box_bytes);
    for (int j = 0; j < boxes; ++j) {
      const int tok = t0 + j * bt;
      const int page = tok / bs;
      const int off = tok - page * bs;
      const int blk = page < npages && page < p.max_blocks ? __ldg(p.table + int64_t(b) * p.bt_stride + page) : 0;
      tma_load_5d(kdst + j * box_bytes, &kmap, bar, 0, off, h, 0, blk);
      tma_load_5d(vdst + j * box_bytes, &vmap, bar, 0, off, h, 0, blk);
    }
  };
  if (tid == 0) {
    if (ntiles > 0) issue(0, 0);
    if (ntiles > 1) issue(1, 1);
  }

  // Q tile -> swizzled shared memory (rows past the chunk are zero)
  const T* qg = reinterpret_cast<const T*>(p.q);
  for (int i = tid; i < PF_ROWS * (D / 8); i += blockDim.x) {
    const int r = i / (D / 8), u = i - r * (D / 8);
    const int tok = tok0 + r / G;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r / G < ntok)
      v = __ldg(reinterpret_cast<const uint4*>(qg + int64_t(q_begin + tok) * p.q_st +
                                               int64_t(h * G + r % G) * p.q_sh + u * 8));
    *reinterpret_cast<uint4*>(qs + swz(r, u, PF_ROWS)) = v;
  }
  __syncthreads();
  const uint32_t qrow_addr = qs_addr;  // lane's A-fragment row: warp * 16 + (lane & 15)
  const int qr = warp * 16 + (lane & 15);
  uint32_t qa[C::HOLD_Q ? C::KS : 1][4];
  if constexpr (C::HOLD_Q) {
#pragma unroll
    for (int ks = 0; ks < C::KS; ++ks) ldsm_x4(qrow_addr + swz(qr, 2 * ks + (lane >> 4), PF_ROWS), qa[ks]);
  }

  // this thread's rows (g and g + 8 of the warp) and their last visible key
  int row_last[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = warp * 16 + g + 8 * hr;
    const int i = r / G;
    row_last[hr] = i < ntok ? ctx + tok0 + i : kend - 1;  // padding rows: any finite row
  }
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[C::DN][4];
#pragma unroll
  for (int dn = 0; dn < C::DN; ++dn) o[dn][0] = o[dn][1] = o[dn][2] = o[dn][3] = 0.f;

  bool failed = false;
  for (int kt = 0; kt < ntiles; ++kt) {
    const int st = kt & 1;
    if (!warp_wait_phase(smem_addr(bars + st), uint32_t((kt >> 1) & 1), p.wait_ns)) {
      failed = true;
    }
    if (__syncthreads_or(failed)) {
      if (warp == 0) {  // the whole warp: the bounded wait is a warp-collective
        if (lane == 0) atomicOr(p.err, DEVERR_WAIT_TIMEOUT);
        for (int k2 = kt; k2 < ntiles && k2 < kt + 2; ++k2)  // copies possibly in flight
          warp_wait_phase(smem_addr(bars + (k2 & 1)), uint32_t((k2 >> 1) & 1), DRAIN_LIMIT_NS);
      }
      return;
    }
    const int t0 = kt * C::KT;
    const uint32_t kaddr = st_addr + uint32_t(st) * 2u * C::TILE_BYTES;
    const uint32_t vaddr = kaddr + C::TILE_BYTES;
    const int valid = kend - t0 < C::KT ? kend - t0 : C::KT;
    if (valid < C::KT) {  // zero V rows past the row end (stale or pool bytes)
      unsigned char* vs = stages + size_t(st) * 2 * C::TILE_BYTES + C::TILE_BYTES;
      for (int i = tid; i < (C::KT - valid) * (D / 8); i += blockDim.x) {
        const int t = valid + i / (D / 8), u = i % (D / 8);
        const int box = t / bt, tb = t - box * bt;
        *reinterpret_cast<uint4*>(vs + box * bt * C::ROW_BYTES + swz(tb, u, bt)) = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncthreads();
    }
    // token t of the tile: box t / bt, row t % bt of that box
    auto krow = [&](int t) -> uint32_t { return uint32_t((t / bt) * bt * C::ROW_BYTES); };

    // ---- S = Q K^T over the tile's 8-token n-tiles
    float s[C::NT][4];
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    if constexpr (C::HOLD_Q) {
#pragma unroll
      for (int nt = 0; nt < C::NT; ++nt) {
        const int t = nt * 8 + (lane & 7);
        const uint32_t rb = kaddr + krow(t);
        const int tb = t % bt;
#pragma unroll
        for (int ks = 0; ks < C::KS; ks += 2) {
          uint32_t kb[4];
          ldsm_x4(rb + swz(tb, 2 * ks + (lane >> 3), bt), kb);
          X::m16n8k16(s[nt], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[0], kb[1]);
          X::m16n8k16(s[nt], qa[ks + 1][0], qa[ks + 1][1], qa[ks + 1][2], qa[ks + 1][3], kb[2], kb[3]);
        }
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < C::KS; ks += 2) {
        uint32_t q0[4], q1[4];
        ldsm_x4(qrow_addr + swz(qr, 2 * ks + (lane >> 4), PF_ROWS), q0);
        ldsm_x4(qrow_addr + swz(qr, 2 * ks + 2 + (lane >> 4), PF_ROWS), q1);
#pragma unroll
        for (int nt = 0; nt < C::NT; ++nt) {
          const int t = nt * 8 + (lane & 7);
          uint32_t kb[4];
          ldsm_x4(kaddr + krow(t) + swz(t % bt, 2 * ks + (lane >> 3), bt), kb);
          X::m16n8k16(s[nt], q0[0], q0[1], q0[2], q0[3], kb[0], kb[1]);
          X::m16n8k16(s[nt], q1[0], q1[1], q1[2], q1[3], kb[2], kb[3]);
        }
      }
    }
    // ---- mask, online softmax (rows g and g + 8 of the warp)
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hr = e >> 1;
        const int key = t0 + nt * 8 + 2 * c + (e & 1);
        const float x = s[nt][e] * p.scale_log2;
        s[nt][e] = key <= row_last[hr] ? x : -INFINITY;
        tmax[hr] = fmaxf(tmax[hr], s[nt][e]);
      }
    }
    float alpha[2], m_use[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      tmax[hr] = fmaxf(tmax[hr], __shfl_xor_sync(FULL_MASK, tmax[hr], 1));
      tmax[hr] = fmaxf(tmax[hr], __shfl_xor_sync(FULL_MASK, tmax[hr], 2));
      const float mn = fmaxf(m_run[hr], tmax[hr]);
      m_use[hr] = mn == -INFINITY ? 0.f : mn;  // a row with no visible key in this tile yet
      alpha[hr] = exp2f(m_run[hr] - m_use[hr]);
      m_run[hr] = mn;
      l_run[hr] *= alpha[hr];
    }
#pragma unroll
    for (int dn = 0; dn < C::DN; ++dn) {
      o[dn][0] *= alpha[0];
      o[dn][1] *= alpha[0];
      o[dn][2] *= alpha[1];
      o[dn][3] *= alpha[1];
    }
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[nt][e] = exp2f(s[nt][e] - m_use[e >> 1]);
        l_run[e >> 1] += s[nt][e];
      }
    }
    // ---- O += P V: A = P from the S accumulators (hi + lo), B = V^T fragments by ldmatrix.trans
#pragma unroll
    for (int kk = 0; kk < C::KK; ++kk) {
      uint32_t ah[4], al[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float* src = s[2 * kk + (q >> 1)] + 2 * (q & 1);
        ah[q] = E::pack2(src[0], src[1]);
        float hf[2];
        E::unpack2(ah[q], hf);
        al[q] = E::pack2(src[0] - hf[0], src[1] - hf[1]);
      }
      const int t = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
      const uint32_t rb = vaddr + krow(t);
      const int tb = t % bt;
#pragma unroll
      for (int dp = 0; dp < C::DN; dp += 2) {
        uint32_t vb[4];
        ldsm_x4_trans(rb + swz(tb, dp + (lane >> 4), bt), vb);
        X::m16n8k16(o[dp], ah[0], ah[1], ah[2], ah[3], vb[0], vb[1]);
        X::m16n8k16(o[dp + 1], ah[0], ah[1], ah[2], ah[3], vb[2], vb[3]);
        X::m16n8k16(o[dp], al[0], al[1], al[2], al[3], vb[0], vb[1]);
        X::m16n8k16(o[dp + 1], al[0], al[1], al[2], al[3], vb[2], vb[3]);
      }
    }
    __syncthreads();  // every warp has read stage st
    if (tid == 0 && kt + 2 < ntiles) {
      fence_proxy_async_smem();  // the zeroed V rows are generic-proxy writes
      issue(kt + 2, st);
    }
  }

  // ---- normalise and store: lane holds rows g / g + 8, columns dn * 8 + 2c, +1
  T* og = reinterpret_cast<T*>(p.out);
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = l_run[hr];
    l += __shfl_xor_sync(FULL_MASK, l, 1);
    l += __shfl_xor_sync(FULL_MASK, l, 2);
    const float inv = 1.f / fmaxf(l, 1.f);
    const int r = warp * 16 + g + 8 * hr;
    const int i = r / G;
    if (i >= ntok) continue;
    T* dst = og + int64_t(q_begin + tok0 + i) * p.o_st + int64_t(h * G + r % G) * p.o_sh + 2 * c;
#pragma unroll
    for (int dn = 0; dn < C::DN; ++dn)
      *reinterpret_cast<uint32_t*>(dst + dn * 8) = E::pack2(o[dn][2 * hr] * inv, o[dn][2 * hr + 1] * inv);
  }
}

template <typename T, int D, int G>
cudaError_t launch_prefill_t(const PrefillParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                             int max_seqlen_q, int batch, int n_kv_head, cudaStream_t stream) {
  using C = PrefillCfg<T, D, G>;
  auto fn = pd_prefill_kernel<T, D, G>;
  const size_t smem = prefill_smem_bytes(D);
  static int attr_smem[64] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 64 && attr_smem[dev] < int(smem)) {
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    attr_smem[dev] = int(smem);
  }
  const dim3 grid((max_seqlen_q + C::TQ - 1) / C::TQ, batch, n_kv_head);
  fn<<<grid, PF_WARPS * 32, smem, stream>>>(p, kmap, vmap);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_prefill_g(const PrefillParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                             int group, int max_seqlen_q, int batch, int n_kv_head, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_prefill_t<T, D, 1>(p, kmap, vmap, max_seqlen_q, batch, n_kv_head, stream);
    case 2: return launch_prefill_t<T, D, 2>(p, kmap, vmap, max_seqlen_q, batch, n_kv_head, stream);
    case 4: return launch_prefill_t<T, D, 4>(p, kmap, vmap, max_seqlen_q, batch, n_kv_head, stream);
    case 8: return launch_prefill_t<T, D, 8>(p, kmap, vmap, max_seqlen_q, batch, n_kv_head, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

size_t prefill_smem_bytes(int head_dim) {
  // barriers (1 KB with the alignment slack), the Q tile, 2 stages of K + V tiles, and 1 KB
  // of run-time re-alignment slack
  return 1024 + size_t(PF_ROWS) * head_dim * 2 + 2 * 2 * size_t(prefill_tile_tokens(head_dim)) * head_dim * 2 +
         1024;
}

int prefill_tile_tokens(int head_dim) { return head_dim == 256 ? 32 : 64; }

bool prefill_supported(int dtype, int head_dim, int group) {
  return (dtype == PD_BF16 || dtype == PD_F16) && (head_dim == 64 || head_dim == 128 || head_dim == 256) &&
         (group == 1 || group == 2 || group == 4 || group == 8);
}

cudaError_t launch_prefill(const PrefillParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, int dtype,
                           int head_dim, int group, int max_seqlen_q, int batch, int n_kv_head,
                           cudaStream_t stream) {
  if (dtype == PD_BF16) {
    if (head_dim == 64)
      return launch_prefill_g<__nv_bfloat16, 64>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
    if (head_dim == 256)
      return launch_prefill_g<__nv_bfloat16, 256>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
    return launch_prefill_g<__nv_bfloat16, 128>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
  }
  if (head_dim == 64)
    return launch_prefill_g<__half, 64>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
  if (head_dim == 256)
    return launch_prefill_g<__half, 256>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
  return launch_prefill_g<__half, 128>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
}

}  // namespace pd
