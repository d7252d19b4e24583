/*
 * pd_oracle.c -- CPU restatement of the reference's paged-decode path. TEST INFRASTRUCTURE.
 *
 * This file is the checker, never the product: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load it. The shipped path is the sm_100a
 * library in llm-serving_b200/; it has no CPU fallback and never calls into this file.
 *
 * Every function restates one reference function (paths relative to the reference root):
 *   oracle_paged_decode    tests/reference/paged.py:225-274  reference_paged_decode
 *                          (per row: gather the row's tokens through the block table, fp32
 *                          scores * scale, fp32 softmax, probs @ V, cast to the q dtype;
 *                          a zero-length row is zero)
 *   oracle_decode_partials same maths, emitting the split-KV triple (m, l, acc) in the
 *                          log2 domain of model/triton_decode.py:576-639 over a token range
 *   oracle_lse_merge       the merge of such triples: acc / max(l, 1) over their union
 *   oracle_append_slots    model/paged.py:188-239 write_slots (index_copy_ of K/V rows into
 *                          flat slots, dtype cast with round-to-nearest-even)
 *   oracle_append_table    tests/reference/paged.py:93-124 write_token_reference (row's
 *                          token at block_table[pos / bs], offset pos % bs)
 *   oracle_gather_pool     tests/reference/paged.py:40-90 gather_pool (dense zero-padded
 *                          (B, H_kv, lpad, D) copy of the rows' logical K/V)
 *   oracle_seat_decode     model/attention/hand_baddbmm.py:80-126 decode with the additive
 *                          bias of model/slab.py:302-328 / hand_baddbmm.py:129-149 (bf16
 *                          rounding after q*scale, after the scores, after the softmax and of
 *                          the output, as torch does for bf16 tensors)
 *
 * Element storage: dtype 0 = fp32, 1 = fp16, 2 = bf16 (raw 16-bit patterns). Rows are
 * parallelised with OpenMP; `threads` <= 0 uses the OpenMP default.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ element conversion */

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t f32_to_bf16(float f) { /* round to nearest even; NaN stays NaN */
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40u);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else { /* subnormal: renormalise */
      int e = -1;
      do {
        e++;
        man <<= 1;
      } while ((man & 0x400u) == 0);
      man &= 0x3ffu;
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (man << 13);
  } else {
    u = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t f32_to_f16(float f) { /* round to nearest even */
  uint32_t u;
  memcpy(&u, &f, 4);
  uint32_t sign = (u >> 16) & 0x8000u;
  int32_t exp = (int32_t)((u >> 23) & 0xffu);
  uint32_t man = u & 0x7fffffu;
  if (exp == 255) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
  int32_t e = exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t half = 1u << (shift - 1);
    uint32_t rest = man & ((1u << shift) - 1u);
    uint32_t out = man >> shift;
    if (rest > half || (rest == half && (out & 1u))) out++;
    return (uint16_t)(sign | out);
  }
  uint32_t out = ((uint32_t)e << 10) | (man >> 13);
  uint32_t rest = man & 0x1fffu;
  if (rest > 0x1000u || (rest == 0x1000u && (out & 1u))) out++;
  return (uint16_t)(sign | out);
}

static float load_elem(const void* base, int64_t i, int dtype) {
  switch (dtype) {
    case 0: return ((const float*)base)[i];
    case 1: return f16_to_f32(((const uint16_t*)base)[i]);
    default: return bf16_to_f32(((const uint16_t*)base)[i]);
  }
}

static void store_elem(void* base, int64_t i, int dtype, float x) {
  switch (dtype) {
    case 0: ((float*)base)[i] = x; break;
    case 1: ((uint16_t*)base)[i] = f32_to_f16(x); break;
    default: ((uint16_t*)base)[i] = f32_to_bf16(x); break;
  }
}

static float round_to(float x, int dtype) {
  if (dtype == 1) return f16_to_f32(f32_to_f16(x));
  if (dtype == 2) return bf16_to_f32(f32_to_bf16(x));
  return x;
}

static void set_threads(int threads) {
  if (threads > 0) omp_set_num_threads(threads);
}

/* Pool element (block, token, head, d) with element strides of dims 0..2 and unit d. */
static inline int64_t pool_index(const int64_t* s, int64_t blk, int64_t tok, int64_t h, int64_t d) {
  return blk * s[0] + tok * s[1] + h * s[2] + d;
}

/* ------------------------------------------------------------------ decode (fp32 oracle) */

/*
 * q (B, H, D) contiguous; pools with element strides ks/vs; table (B, max_blocks) int32 row
 * stride bt_stride; seqlen (B,) int32; out_f32 (B, H, D) receives the fp32 result before
 * the final cast; out (B, H, D) in `dtype` receives the cast (either may be NULL).
 * Returns 0, or -1 for a seqlen outside [0, max_blocks * bs] or a block id outside the pool.
 */
__attribute__((target_clones("avx2", "default")))
int oracle_paged_decode(const void* q, const void* k, const void* v, const int64_t* ks,
                        const int64_t* vs, int64_t n_blocks, int bs, const int32_t* table,
                        int64_t bt_stride, int max_blocks, const int32_t* seqlen, int B, int H,
                        int H_kv, int D, int dtype, float scale, float* out_f32, void* out,
                        int threads) {
  const int G = H / H_kv;
  int bad = 0;
  set_threads(threads);
#pragma omp parallel for schedule(dynamic, 1) reduction(| : bad)
  for (int64_t bh = 0; bh < (int64_t)B * H_kv; ++bh) {
    const int b = (int)(bh / H_kv), hk = (int)(bh % H_kv);
    const int n = seqlen[b];
    if (n < 0 || (int64_t)n > (int64_t)max_blocks * bs) {
      bad = 1;
      continue;
    }
    float* kf = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * D);
    float* vf = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * D);
    float* sc = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    float* qf = (float*)malloc(sizeof(float) * (size_t)D);
    float* ctx = (float*)malloc(sizeof(float) * (size_t)D);
    for (int t = 0; t < n && !bad; ++t) {
      const int32_t blk = table[(int64_t)b * bt_stride + t / bs];
      if (blk < 0 || blk >= n_blocks) {
        bad = 1;
        break;
      }
      for (int d = 0; d < D; ++d) {
        kf[(int64_t)t * D + d] = load_elem(k, pool_index(ks, blk, t % bs, hk, d), dtype);
        vf[(int64_t)t * D + d] = load_elem(v, pool_index(vs, blk, t % bs, hk, d), dtype);
      }
    }
    for (int g = 0; g < G && !bad; ++g) {
      const int h = hk * G + g;
      const int64_t orow = ((int64_t)b * H + h) * D;
      if (n == 0) {
        for (int d = 0; d < D; ++d) {
          if (out_f32) out_f32[orow + d] = 0.f;
          if (out) store_elem(out, orow + d, dtype, 0.f);
        }
        continue;
      }
      for (int d = 0; d < D; ++d) qf[d] = load_elem(q, orow + d, dtype);
      float mx = -INFINITY;
      for (int t = 0; t < n; ++t) {
        float s = 0.f;
#pragma omp simd reduction(+ : s)
        for (int d = 0; d < D; ++d) s += qf[d] * kf[(int64_t)t * D + d];
        s *= scale;
        sc[t] = s;
        if (s > mx) mx = s;
      }
      float sum = 0.f;
      for (int t = 0; t < n; ++t) {
        sc[t] = expf(sc[t] - mx);
        sum += sc[t];
      }
      for (int t = 0; t < n; ++t) sc[t] /= sum;
      for (int d = 0; d < D; ++d) ctx[d] = 0.f;
      for (int t = 0; t < n; ++t) {
        const float p = sc[t];
        const float* vr = vf + (int64_t)t * D;
#pragma omp simd
        for (int d = 0; d < D; ++d) ctx[d] += p * vr[d];
      }
      for (int d = 0; d < D; ++d) {
        if (out_f32) out_f32[orow + d] = ctx[d];
        if (out) store_elem(out, orow + d, dtype, ctx[d]);
      }
    }
    free(kf);
    free(vf);
    free(sc);
    free(qf);
    free(ctx);
  }
  return bad ? -1 : 0;
}

/*
 * Split-KV triple over logical tokens [tok_begin[b], tok_end[b]) of each row (clamped to
 * [0, seqlen[b]]): m = max of s2 = (q.k) * scale_log2, l = sum exp2(s2 - m),
 * acc = sum exp2(s2 - m) v. An empty range gives (-inf, 0, 0). Outputs fp32 (B, H) and
 * (B, H, D). This is the algebra of the online softmax in model/triton_decode.py:596-639.
 */
__attribute__((target_clones("avx2", "default")))
int oracle_decode_partials(const void* q, const void* k, const void* v, const int64_t* ks,
                           const int64_t* vs, int64_t n_blocks, int bs, const int32_t* table,
                           int64_t bt_stride, const int32_t* seqlen, const int32_t* tok_begin,
                           const int32_t* tok_end, int B, int H, int H_kv, int D, int dtype,
                           float scale_log2, float* m_out, float* l_out, float* acc_out,
                           int threads) {
  const int G = H / H_kv;
  int bad = 0;
  set_threads(threads);
#pragma omp parallel for schedule(dynamic, 1) reduction(| : bad)
  for (int64_t bh = 0; bh < (int64_t)B * H; ++bh) {
    const int b = (int)(bh / H), h = (int)(bh % H), hk = h / G;
    int t0 = tok_begin ? tok_begin[b] : 0;
    int t1 = tok_end ? tok_end[b] : seqlen[b];
    if (t0 < 0) t0 = 0;
    if (t1 > seqlen[b]) t1 = seqlen[b];
    float* acc = acc_out + bh * D;
    for (int d = 0; d < D; ++d) acc[d] = 0.f;
    if (t1 <= t0) {
      m_out[bh] = -INFINITY;
      l_out[bh] = 0.f;
      continue;
    }
    float* qf = (float*)malloc(sizeof(float) * (size_t)D);
    float* sc = (float*)malloc(sizeof(float) * (size_t)(t1 - t0));
    for (int d = 0; d < D; ++d) qf[d] = load_elem(q, bh * D + d, dtype);
    float mx = -INFINITY;
    for (int t = t0; t < t1; ++t) {
      const int32_t blk = table[(int64_t)b * bt_stride + t / bs];
      if (blk < 0 || blk >= n_blocks) {
        bad = 1;
        break;
      }
      float s = 0.f;
      for (int d = 0; d < D; ++d) s += qf[d] * load_elem(k, pool_index(ks, blk, t % bs, hk, d), dtype);
      s *= scale_log2;
      sc[t - t0] = s;
      if (s > mx) mx = s;
    }
    if (!bad) {
      float l = 0.f;
      for (int t = t0; t < t1; ++t) {
        const int32_t blk = table[(int64_t)b * bt_stride + t / bs];
        const float p = exp2f(sc[t - t0] - mx);
        l += p;
        for (int d = 0; d < D; ++d) acc[d] += p * load_elem(v, pool_index(vs, blk, t % bs, hk, d), dtype);
      }
      m_out[bh] = mx;
      l_out[bh] = l;
    }
    free(qf);
    free(sc);
  }
  return bad ? -1 : 0;
}

/* Merge n_parts triples stacked on a leading axis into out (B, H, D) in `dtype`. */
void oracle_lse_merge(const float* m, const float* l, const float* acc, int n_parts, int B, int H,
                      int D, int dtype, float* out_f32, void* out) {
  const int64_t pairs = (int64_t)B * H;
  for (int64_t bh = 0; bh < pairs; ++bh) {
    float M = -INFINITY;
    for (int p = 0; p < n_parts; ++p)
      if (m[p * pairs + bh] > M) M = m[p * pairs + bh];
    float L = 0.f;
    for (int p = 0; p < n_parts; ++p)
      if (M != -INFINITY) L += l[p * pairs + bh] * exp2f(m[p * pairs + bh] - M);
    const float inv = 1.f / (L > 1.f ? L : 1.f);
    for (int d = 0; d < D; ++d) {
      float a = 0.f;
      if (M != -INFINITY)
        for (int p = 0; p < n_parts; ++p) a += exp2f(m[p * pairs + bh] - M) * acc[(p * pairs + bh) * D + d];
      const float r = M == -INFINITY ? 0.f : a * inv;
      if (out_f32) out_f32[bh * D + d] = r;
      if (out) store_elem(out, bh * D + d, dtype, r);
    }
  }
}

/* ------------------------------------------------------------------ append (bit-exact) */

static void copy_row(void* dst, int64_t dst_off, int dst_dtype, const void* src, int64_t src_off,
                     int src_dtype, int D) {
  if (dst_dtype == src_dtype) {
    const size_t es = dst_dtype == 0 ? 4 : 2;
    memcpy((char*)dst + dst_off * es, (const char*)src + src_off * es, es * (size_t)D);
    return;
  }
  for (int d = 0; d < D; ++d) store_elem(dst, dst_off + d, dst_dtype, load_elem(src, src_off + d, src_dtype));
}

/*
 * Token i of k/v (rows with element strides src_s[0], src_s[1]; unit d) into flat slot
 * slots[i] of the pools. Returns the number of tokens skipped because their slot was
 * outside the pool (the reference's index_copy_ raises there).
 */
int64_t oracle_append_slots(void* kp, void* vp, const int64_t* kps, const int64_t* vps, int64_t n_blocks,
                            int bs, int pool_dtype, const int64_t* slots, const void* k,
                            const int64_t* k_s, const void* v, const int64_t* v_s, int src_dtype,
                            int64_t n_tokens, int H_kv, int D) {
  int64_t skipped = 0;
  for (int64_t i = 0; i < n_tokens; ++i) {
    const int64_t slot = slots[i];
    if (slot < 0 || slot >= n_blocks * bs) {
      skipped++;
      continue;
    }
    const int64_t blk = slot / bs, off = slot % bs;
    for (int h = 0; h < H_kv; ++h) {
      copy_row(kp, pool_index(kps, blk, off, h, 0), pool_dtype, k, i * k_s[0] + h * k_s[1], src_dtype, D);
      copy_row(vp, pool_index(vps, blk, off, h, 0), pool_dtype, v, i * v_s[0] + h * v_s[1], src_dtype, D);
    }
  }
  return skipped;
}

/* Row b's token to block table[b, pos[b] / bs], offset pos[b] % bs. Returns rows skipped. */
int64_t oracle_append_table(void* kp, void* vp, const int64_t* kps, const int64_t* vps, int64_t n_blocks,
                            int bs, int pool_dtype, const int32_t* table, int64_t bt_stride,
                            int max_blocks, const int64_t* pos, const void* k, const int64_t* k_s,
                            const void* v, const int64_t* v_s, int src_dtype, int B, int H_kv, int D) {
  int64_t skipped = 0;
  for (int b = 0; b < B; ++b) {
    const int64_t p = pos[b];
    if (p < 0 || p / bs >= max_blocks) {
      skipped++;
      continue;
    }
    const int64_t blk = table[(int64_t)b * bt_stride + p / bs];
    if (blk < 0 || blk >= n_blocks) {
      skipped++;
      continue;
    }
    for (int h = 0; h < H_kv; ++h) {
      copy_row(kp, pool_index(kps, blk, p % bs, h, 0), pool_dtype, k, (int64_t)b * k_s[0] + h * k_s[1], src_dtype, D);
      copy_row(vp, pool_index(vps, blk, p % bs, h, 0), pool_dtype, v, (int64_t)b * v_s[0] + h * v_s[1], src_dtype, D);
    }
  }
  return skipped;
}

/* ------------------------------------------------------------------ seat / gather path */

/*
 * Dense (B, H_kv, lpad, D) copies of each row's first lengths[b] logical tokens (zeros past
 * the length), in the pool dtype. Returns -1 if a length exceeds lpad or the table.
 */
int oracle_gather_pool(const void* k, const void* v, const int64_t* ks, const int64_t* vs, int64_t n_blocks,
                       int bs, const int32_t* table, int64_t bt_stride, int max_blocks,
                       const int32_t* lengths, int B, int H_kv, int D, int dtype, int lpad, void* out_k,
                       void* out_v, int threads) {
  const size_t es = dtype == 0 ? 4 : 2;
  int bad = 0;
  set_threads(threads);
#pragma omp parallel for schedule(static) reduction(| : bad)
  for (int64_t bh = 0; bh < (int64_t)B * H_kv; ++bh) {
    const int b = (int)(bh / H_kv), hk = (int)(bh % H_kv);
    const int n = lengths[b];
    char* dk = (char*)out_k + (size_t)bh * lpad * D * es;
    char* dv = (char*)out_v + (size_t)bh * lpad * D * es;
    memset(dk, 0, (size_t)lpad * D * es);
    memset(dv, 0, (size_t)lpad * D * es);
    if (n < 0 || n > lpad || (int64_t)(n + bs - 1) / bs > max_blocks) {
      bad = 1;
      continue;
    }
    for (int t = 0; t < n; ++t) {
      const int32_t blk = table[(int64_t)b * bt_stride + t / bs];
      if (blk < 0 || blk >= n_blocks) {
        bad = 1;
        break;
      }
      memcpy(dk + (size_t)t * D * es, (const char*)k + pool_index(ks, blk, t % bs, hk, 0) * es, D * es);
      memcpy(dv + (size_t)t * D * es, (const char*)v + pool_index(vs, blk, t % bs, hk, 0) * es, D * es);
    }
  }
  return bad ? -1 : 0;
}

/*
 * Seat decode over dense slabs (B, H_kv, lpad, D): column c of row b is live iff
 * c < lengths[b]; a row with no live column attends every column with zero bias (the
 * reference's dead-row rule). Rounds to `dtype` after q*scale, after q.k + bias, after the
 * softmax and for the output, accumulating each dot product in fp32.
 */
__attribute__((target_clones("avx2", "default")))
void oracle_seat_decode(const void* q, const void* slab_k, const void* slab_v, const int32_t* lengths, int B,
                        int H, int H_kv, int D, int lpad, int dtype, void* out, int threads) {
  const int G = H / H_kv;
  const float scale = 1.0f / sqrtf((float)D);
  set_threads(threads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t bh = 0; bh < (int64_t)B * H_kv; ++bh) {
    const int b = (int)(bh / H_kv), hk = (int)(bh % H_kv);
    const int n = lengths[b];
    const int alive = n > 0;
    float* qf = (float*)malloc(sizeof(float) * (size_t)D);
    float* sc = (float*)malloc(sizeof(float) * (size_t)lpad);
    float* ctx = (float*)malloc(sizeof(float) * (size_t)D);
    const int64_t base = bh * (int64_t)lpad * D;
    for (int g = 0; g < G; ++g) {
      const int64_t qrow = ((int64_t)b * H + hk * G + g) * D;
      for (int d = 0; d < D; ++d) qf[d] = round_to(load_elem(q, qrow + d, dtype) * scale, dtype);
      float mx = -INFINITY;
      for (int c = 0; c < lpad; ++c) {
        float s = 0.f;
        for (int d = 0; d < D; ++d) s += qf[d] * load_elem(slab_k, base + (int64_t)c * D + d, dtype);
        const float bias = (!alive || c < n) ? 0.f : -INFINITY;
        s = round_to(s + bias, dtype);
        sc[c] = s;
        if (s > mx) mx = s;
      }
      float sum = 0.f;
      for (int c = 0; c < lpad; ++c) {
        sc[c] = expf(sc[c] - mx);
        sum += sc[c];
      }
      for (int c = 0; c < lpad; ++c) sc[c] = round_to(sc[c] / sum, dtype);
      for (int d = 0; d < D; ++d) ctx[d] = 0.f;
      for (int c = 0; c < lpad; ++c) {
        const float p = sc[c];
        if (p == 0.f) continue;
        for (int d = 0; d < D; ++d) ctx[d] += p * load_elem(slab_v, base + (int64_t)c * D + d, dtype);
      }
      for (int d = 0; d < D; ++d) store_elem(out, qrow + d, dtype, ctx[d]);
    }
    free(qf);
    free(sc);
    free(ctx);
  }
}

/* Round-trip helpers the tests use to pin the conversions against torch. */
/* GPT-NeoX rotary embedding of rows of length head_dim (model/layers.py:59-117,
 * apply_rotary_emb / apply_rotary_emb_partial): pairs (i, i + rot_dim / 2) over the first
 * rot_dim elements, the tail copied. Row r uses cos/sin + r * cs_stride. As torch's
 * elementwise ops in the row dtype: each product rounded to the dtype, then the difference
 * (first half) or sum (second half) rounded again. Build with -ffp-contract=off. */
void oracle_rope(const void* x, const void* cos_t, const void* sin_t, void* out, int64_t n_rows,
                 int head_dim, int rot_dim, int64_t cs_stride, int64_t rows_per_table_row, int dtype) {
  const int half = rot_dim / 2;
  for (int64_t r = 0; r < n_rows; ++r) {
    const int64_t t = (r / rows_per_table_row) * cs_stride;
    const int64_t base = r * head_dim;
    for (int e = 0; e < head_dim; ++e) {
      float y;
      if (e >= rot_dim) {
        y = load_elem(x, base + e, dtype);
      } else {
        const int i = e < half ? e : e - half;
        const float x1 = load_elem(x, base + i, dtype), x2 = load_elem(x, base + i + half, dtype);
        const float c = load_elem(cos_t, t + i, dtype), s = load_elem(sin_t, t + i, dtype);
        if (e < half) {
          const float a = round_to(x1 * c, dtype), b = round_to(x2 * s, dtype);
          y = a - b;
        } else {
          const float a = round_to(x1 * s, dtype), b = round_to(x2 * c, dtype);
          y = a + b;
        }
      }
      store_elem(out, base + e, dtype, y);
    }
  }
}

void oracle_convert(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n) {
  for (int64_t i = 0; i < n; ++i) store_elem(dst, i, dst_dtype, load_elem(src, i, src_dtype));
}

int oracle_max_threads(void) { return omp_get_max_threads(); }
