// pd_decode_mma.cuh -- tensor-core consumer of the paged decode kernel (bf16 / fp16 pools,
// head_dim 64..256).
//
// Same arithmetic as the CUDA-core consumer (model/triton_decode.py:595-636 of the
// reference: fp32 scores, fp32 online softmax in log2 units, fp32 P.V), issued as warp-level
// tensor-core instructions instead of packed FMAs and shuffles. The per-tile instruction
// count drops from O(TILE * GT * D / 32) to a few dozen, which is what bounds the kernel when
// a worker carries several q heads of a wide head (Qwen3.5: D = 256, 4 q heads per kv head).
//
// Per tile of TILE tokens of one kv head, the warp computes
//   S^T = K q^T     (M = tokens, N = 8 q-head columns, K = head_dim): m16n8k16, fp32 accum.
//   O^T += V^T P^T  (M = head_dim, N = 8 q-head columns, K = tokens).
// q heads past GT are zero columns. Tiles of 8 tokens (head_dim 256) use the upper half of
// the 16-row A operand as zeros for S^T and m16n8k8 for P.V.
// The probabilities enter the P.V product as two 16-bit operands, P = hi + lo with
// hi = round(P) and lo = round(P - hi): the product then carries P to 2^-17 relative (bf16)
// and matches fp32 P.V within fp32 accumulation error. The S^T accumulator layout (token
// rows, head columns) becomes the B operand of P.V by one movmatrix transpose per 8 tokens.
//
// Shared-memory layout of a stage (K, then V): the pool's TMA map splits a row into 128-byte
// pieces with the 128-byte swizzle, box (64 elements, box_tokens, 1 head, D / 64 pieces):
// smem row R = piece * box_tokens + token holds 128 bytes whose 16-byte unit u sits at unit
// u ^ (R % 8). Eight consecutive tokens of one piece therefore hit eight distinct bank
// groups, and every ldmatrix is conflict-free. Boxes (box_tokens >= 8) start 1 KB aligned.
#pragma once

#include "pd_common.cuh"

namespace pd {

template <typename T, int D, int GT>
struct MmaCfg {
  static_assert(sizeof(T) == 2, "tensor-core decode needs 16-bit K/V");
  static_assert(D == 64 || D == 128 || D == 256, "tensor-core decode: head_dim 64, 128 or 256");
  static_assert(GT >= 1 && GT <= 8, "at most 8 q heads per worker item");
  static constexpr int ROW_BYTES = D * 2;
  static constexpr int PIECES = D / 64;              // 128-byte pieces of a row
  static constexpr int TILE = 4096 / ROW_BYTES;      // tokens per stage: 32, 16, 8
  static constexpr bool HALF = TILE == 8;            // S^T uses 8 of the 16 A rows
  static constexpr int MT = HALF ? 1 : TILE / 16;    // 16-token tiles (S^T rows, P.V k-steps)
  static constexpr int KS = D / 16;                  // q.K k-steps
  static constexpr int DM = D / 16;                  // head_dim tiles of O^T
  static constexpr int R = HALF ? 2 : MT * 4;        // scores held per lane
  static constexpr int CH = KS >= 4 * MT ? 4 / MT : 1;  // independent S^T accumulator chains
};

// One warp's tensor-core consumer state. Score j of a lane (g = lane / 4, c = lane % 4) is
// token (j / 4) * 16 + ((j / 2) % 2) * 8 + g of the tile, q-head column 2c + (j % 2).
template <typename T, int D, int GT>
struct MmaWorker {
  using M = MmaCfg<T, D, GT>;
  using E = Elem<T>;
  using X = Mma<T>;

  int lane, g, c;
  uint32_t k_row[M::MT];  // byte offset of this lane's ldmatrix row in a K tile, per 16-token tile
  uint32_t v_row[M::MT];  // same for the transposed V reads
  uint32_t kx[4], vx[4];  // swizzled 16-byte unit offsets of this lane, per (k-step % 4)
  uint32_t piece_stride;  // bytes between the 128-byte pieces of one token (box_tokens * 128)
  uint32_t box_bytes;     // bytes of one TMA box (box_tokens tokens)
  int log2_box;

  uint32_t qb[M::KS][2];  // q^T as B fragments (zero columns past GT)
  float o[M::DM][4];      // O^T accumulators: (d = dm * 16 + g [+ 8], q head 2c [+ 1])
  float m_run[2], l_run[2];  // per q-head column 2c + e; l is this lane's partial sum

  __device__ __forceinline__ uint32_t row_off(int t) const {
    return uint32_t(t >> log2_box) * box_bytes + uint32_t(t & ((1 << log2_box) - 1)) * 128u;
  }

  __device__ __forceinline__ void init(int lane_, int box_tokens, int log2_box_) {
    lane = lane_;
    g = lane >> 2;
    c = lane & 3;
    log2_box = log2_box_;
    piece_stride = uint32_t(box_tokens) * 128u;
    box_bytes = uint32_t(box_tokens) * uint32_t(M::ROW_BYTES);
    const int r8 = lane & 7;
    if constexpr (M::HALF) {
      k_row[0] = row_off(r8);
      v_row[0] = k_row[0];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        kx[k] = uint32_t(((2 * (k & 2) + (lane >> 3)) ^ r8) << 4);  // k-step pair at 2 * (k & 2)
        vx[k] = kx[k];
      }
    } else {
#pragma unroll
      for (int mt = 0; mt < M::MT; ++mt) {
        k_row[mt] = row_off(mt * 16 + r8 + 8 * ((lane >> 3) & 1));
        v_row[mt] = row_off(mt * 16 + r8 + 8 * (lane >> 4));
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        kx[k] = uint32_t(((2 * k + (lane >> 4)) ^ r8) << 4);
        vx[k] = uint32_t(((2 * k + ((lane >> 3) & 1)) ^ r8) << 4);
      }
    }
  }

  // Opens an item: q rows hq0 .. hq0 + GT - 1 of qrow (head stride q_sh) as B fragments.
  __device__ __forceinline__ void start(const T* qrow, int64_t q_sh, int hq0) {
    const bool live = g < GT;
    const T* qh = qrow + int64_t(hq0 + (live ? g : 0)) * q_sh + 2 * c;
#pragma unroll
    for (int ks = 0; ks < M::KS; ++ks) {
      qb[ks][0] = live ? __ldg(reinterpret_cast<const unsigned int*>(qh + ks * 16)) : 0u;
      qb[ks][1] = live ? __ldg(reinterpret_cast<const unsigned int*>(qh + ks * 16 + 8)) : 0u;
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      m_run[e] = -INFINITY;
      l_run[e] = 0.f;
    }
#pragma unroll
    for (int dm = 0; dm < M::DM; ++dm) o[dm][0] = o[dm][1] = o[dm][2] = o[dm][3] = 0.f;
  }

  // Scores of the K tile at shared address kbase, scaled to log2 units; tokens at or past
  // valid_rows get -inf.
  __device__ __forceinline__ void scores(uint32_t kbase, int valid_rows, float scale_log2,
                                         float (&sc)[M::R]) const {
    float acc[M::MT][M::CH][4];
#pragma unroll
    for (int mt = 0; mt < M::MT; ++mt)
#pragma unroll
      for (int ch = 0; ch < M::CH; ++ch) acc[mt][ch][0] = acc[mt][ch][1] = acc[mt][ch][2] = acc[mt][ch][3] = 0.f;
    if constexpr (M::HALF) {
#pragma unroll
      for (int ks = 0; ks < M::KS; ks += 2) {
        uint32_t a[4];
        ldsm_x4(kbase + k_row[0] + uint32_t(ks >> 2) * piece_stride + kx[ks & 3], a);
        X::m16n8k16(acc[0][ks % M::CH], a[0], 0u, a[1], 0u, qb[ks][0], qb[ks][1]);
        X::m16n8k16(acc[0][(ks + 1) % M::CH], a[2], 0u, a[3], 0u, qb[ks + 1][0], qb[ks + 1][1]);
      }
    } else {
#pragma unroll
      for (int mt = 0; mt < M::MT; ++mt) {
#pragma unroll
        for (int ks = 0; ks < M::KS; ++ks) {
          uint32_t a[4];
          ldsm_x4(kbase + k_row[mt] + uint32_t(ks >> 2) * piece_stride + kx[ks & 3], a);
          X::m16n8k16(acc[mt][ks % M::CH], a[0], a[1], a[2], a[3], qb[ks][0], qb[ks][1]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < M::R; ++j) {
      const int mt = j >> 2, i = j & 3;
      float s = acc[mt][0][i];
#pragma unroll
      for (int ch = 1; ch < M::CH; ++ch) s += acc[mt][ch][i];
      const int tok = mt * 16 + ((j >> 1) & 1) * 8 + g;
      sc[j] = tok < valid_rows ? s * scale_log2 : -INFINITY;
    }
  }

  // Online-softmax max update (only when some score of the tile exceeds the running max).
  __device__ __forceinline__ void max_update(const float (&sc)[M::R]) {
    bool exceeds = false;
#pragma unroll
    for (int j = 0; j < M::R; ++j) exceeds |= sc[j] > m_run[j & 1];
    if (__builtin_expect(__any_sync(FULL_MASK, exceeds), 0)) {
      float t[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < M::R; ++j) t[j & 1] = fmaxf(t[j & 1], sc[j]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        t[0] = fmaxf(t[0], __shfl_xor_sync(FULL_MASK, t[0], off));
        t[1] = fmaxf(t[1], __shfl_xor_sync(FULL_MASK, t[1], off));
      }
      float alpha[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float mn = fmaxf(m_run[e], t[e]);  // finite: the tile has a live row
        alpha[e] = exp2f(m_run[e] - mn);
        m_run[e] = mn;
        l_run[e] *= alpha[e];
      }
#pragma unroll
      for (int dm = 0; dm < M::DM; ++dm) {
        o[dm][0] *= alpha[0];
        o[dm][1] *= alpha[1];
        o[dm][2] *= alpha[0];
        o[dm][3] *= alpha[1];
      }
    }
  }

  // P = exp2(s - m) as hi + lo 16-bit pairs, transposed into B fragments (tokens 8 * h .. +7).
  __device__ __forceinline__ static void p_operand(float p0, float p1, uint32_t& bh, uint32_t& bl) {
    const uint32_t hi = E::pack2(p0, p1);
    float hf[2];
    E::unpack2(hi, hf);
    const uint32_t lo = E::pack2(p0 - hf[0], p1 - hf[1]);
    bh = movmatrix_trans(hi);
    bl = movmatrix_trans(lo);
  }

  // Keeps the 16-bit halves of V pairs whose token (t, t + 1) is below valid_rows.
  __device__ __forceinline__ static uint32_t pair_mask(int t, int valid_rows) {
    return (t < valid_rows ? 0x0000ffffu : 0u) | (t + 1 < valid_rows ? 0xffff0000u : 0u);
  }

  // Probabilities of the tile and O^T += V^T P^T from the V tile at shared address vbase.
  // Tokens at or past valid_rows have P = 0 and their V is masked to zero (stale bytes, even
  // NaN patterns, never reach the accumulators).
  __device__ __forceinline__ void pv(uint32_t vbase, const float (&sc)[M::R], int valid_rows, bool full) {
    float pr[M::R];
#pragma unroll
    for (int j = 0; j < M::R; ++j) {
      pr[j] = exp2f(sc[j] - m_run[j & 1]);
      l_run[j & 1] += pr[j];
    }
    if constexpr (M::HALF) {
      uint32_t bh, bl;
      p_operand(pr[0], pr[1], bh, bl);
      const uint32_t mk = full ? 0xffffffffu : pair_mask(2 * c, valid_rows);
#pragma unroll
      for (int dm = 0; dm < M::DM; dm += 2) {
        uint32_t a[4];
        ldsm_x4_trans(vbase + v_row[0] + uint32_t(dm >> 2) * piece_stride + vx[dm & 3], a);
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] &= mk;
        X::m16n8k8(o[dm], a[0], a[1], bh);
        X::m16n8k8(o[dm + 1], a[2], a[3], bh);
        X::m16n8k8(o[dm], a[0], a[1], bl);
        X::m16n8k8(o[dm + 1], a[2], a[3], bl);
      }
    } else {
#pragma unroll
      for (int kp = 0; kp < M::MT; ++kp) {
        uint32_t bh0, bl0, bh1, bl1;
        p_operand(pr[kp * 4 + 0], pr[kp * 4 + 1], bh0, bl0);
        p_operand(pr[kp * 4 + 2], pr[kp * 4 + 3], bh1, bl1);
        const uint32_t mk0 = full ? 0xffffffffu : pair_mask(kp * 16 + 2 * c, valid_rows);
        const uint32_t mk1 = full ? 0xffffffffu : pair_mask(kp * 16 + 8 + 2 * c, valid_rows);
#pragma unroll
        for (int dm = 0; dm < M::DM; ++dm) {
          uint32_t a[4];
          ldsm_x4_trans(vbase + v_row[kp] + uint32_t(dm >> 2) * piece_stride + vx[dm & 3], a);
          a[0] &= mk0;
          a[1] &= mk0;
          a[2] &= mk1;
          a[3] &= mk1;
          X::m16n8k16(o[dm], a[0], a[1], a[2], a[3], bh0, bh1);
          X::m16n8k16(o[dm], a[0], a[1], a[2], a[3], bl0, bl1);
        }
      }
    }
  }

  // Normaliser of q-head columns 2c, 2c + 1 summed over the warp's lanes (every lane).
  __device__ __forceinline__ void total_l(float (&l_tot)[2]) const {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float x = l_run[e];
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) x += __shfl_xor_sync(FULL_MASK, x, off);
      l_tot[e] = x;
    }
  }

  // Normalised output of the item's GT heads: out_h0 points at head hq0, head stride o_sh.
  // Each (d, head) pair is transposed to (head, d) pairs so that a lane stores 4 bytes of one
  // head row.
  __device__ __forceinline__ void store_out(T* out_h0, int64_t o_sh, const float (&l_tot)[2]) const {
    const float inv0 = 1.f / fmaxf(l_tot[0], 1.f);
    const float inv1 = 1.f / fmaxf(l_tot[1], 1.f);
    T* dst = out_h0 + int64_t(g < GT ? g : 0) * o_sh + 2 * c;
#pragma unroll
    for (int dm = 0; dm < M::DM; ++dm) {
      const uint32_t y0 = movmatrix_trans(E::pack2(o[dm][0] * inv0, o[dm][1] * inv1));
      const uint32_t y1 = movmatrix_trans(E::pack2(o[dm][2] * inv0, o[dm][3] * inv1));
      if (g < GT) {
        *reinterpret_cast<unsigned int*>(dst + dm * 16) = y0;
        *reinterpret_cast<unsigned int*>(dst + dm * 16 + 8) = y1;
      }
    }
  }

  // Unnormalised fp32 accumulators of the item's GT heads, head-major rows of D floats.
  __device__ __forceinline__ void store_acc(float* dst) const {
#pragma unroll
    for (int dm = 0; dm < M::DM; ++dm) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int h = 2 * c + (i & 1);
        if (h < GT) dst[h * D + dm * 16 + g + 8 * (i >> 1)] = o[dm][i];
      }
    }
  }

  // (m, l) of the item's heads into m_dst[h], l_dst[h] (lanes 0..3 hold columns 2c, 2c + 1).
  __device__ __forceinline__ void store_ml(float* m_dst, float* l_dst, const float (&l_tot)[2]) const {
    if (g == 0) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (2 * c + e < GT) {
          m_dst[2 * c + e] = m_run[e];
          l_dst[2 * c + e] = l_tot[e];
        }
      }
    }
  }

  // Shared-memory address of 16-byte unit u (0 .. D / 8 - 1) of token t's row in a tile.
  __device__ __forceinline__ uint32_t unit_addr(uint32_t base, int t, int u) const {
    return base + row_off(t) + uint32_t(u >> 3) * piece_stride + uint32_t(((u & 7) ^ (t & 7)) << 4);
  }
};

}  // namespace pd
