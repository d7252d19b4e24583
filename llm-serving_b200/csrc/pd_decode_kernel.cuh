// pd_decode_kernel.cuh -- paged GQA decode attention for sm_100a.
//
// What it computes (model/triton_decode.py:544-643 of the reference): for every row b and
// query head h, out[b, h] = softmax(q[b, h] . K^T * scale) V over the first seqlen[b]
// logical tokens of the row, token t living at pool block block_table[b, t / bs], slot
// t % bs. Scores are formed in fp32 and scaled by scale * log2(e) so the online softmax
// uses exp2; the result is acc / max(l, 1), which makes a zero-length row exactly zero.
//
// How (B200 design, not the reference's):
//  * Work unit = one KV tile of TILE tokens of one (row, kv head, q-head chunk) item;
//    TILE * head_dim * sizeof(T) = 4 KB for K (and again for V). The units of all items
//    are laid end to end (row-major, kv head, q-head chunk, tile) and cut into equal
//    contiguous ranges, one per worker. Every worker gets the same number of KV bytes
//    (+-1 tile) whatever the length skew, and a long row is spread over many workers.
//  * Worker = one warp. It owns a private ring of `stages` shared-memory stages, each
//    filled by two 4-D TMA tile loads (K and V, box = head_dim x 1 head x box_tokens x 1
//    block) that complete on the stage's mbarrier. Lane 0 issues; the warp consumes tile
//    k while tiles k+1 .. k+stages-1 are in flight, then refills the stage it just read.
//    There is no block-level synchronisation after the prologue.
//  * Tile math, tensor-core consumer (16-bit K/V, head_dim 64..256, the default there):
//    S^T = K q^T and O^T += V^T P^T as warp-level mma.sync tiles fed by ldmatrix from
//    128-byte-swizzled stages (pd_decode_mma.cuh). The tensor cores are not there for
//    flops -- a decode step is a GEMV at 2 flop/byte per q head -- but to cut the issue
//    slots per tile, which otherwise bound wide heads with several q heads per kv head.
//  * Tile math, CUDA-core consumer (every dtype and head size): lanes span head_dim (16 B
//    per lane per row), a warp-wide load covers 32/LPR rows. Partial dot products for all
//    (token, q head) pairs of the tile are finished by a butterfly reduce-scatter, so each
//    shuffle carries useful sums. Online softmax in fp32 per q head, then every lane
//    fetches the probabilities of its own rows by shuffle and accumulates P.V in fp32
//    registers.
//  * A worker whose range covers a whole item writes the output directly. A split item
//    leaves (m, l, acc) in the workspace; the last of its workers to finish (arrival
//    counter, __threadfence) merges the pieces with the log-sum-exp rule, so split-KV costs
//    no extra launch. Counters are tagged with the launch's epoch, which the kernel keeps in
//    the workspace header and advances itself when its last warp leaves: the workspace never
//    needs clearing, and a launch replayed from a CUDA graph gets a fresh epoch every time.
//  * Block-table entries are fetched 32 at a time into one register per lane (plus the
//    next 32 prefetched), so a TMA issue never waits on a dependent global load inside a
//    row. Table entries past ceil(seqlen / bs) are never read; an entry outside the pool
//    makes TMA fill zeros instead of faulting.
//  * Every mbarrier wait is bounded (1 s of %globaltimer). On expiry the warp records
//    DEVERR_WAIT_TIMEOUT, drains its in-flight copies (bounded again) and returns.
#pragma once

#include "pd_common.cuh"
#include "pd_decode_mma.cuh"

namespace pd {

template <typename T, int D, int GT>
struct DecodeCfg {
  static constexpr int ES = int(sizeof(T));
  static constexpr int ROW_BYTES = D * ES;
  static constexpr int CHUNKS = ROW_BYTES / 16;  // 16 B chunks per K/V row
  static_assert(CHUNKS >= 1, "head_dim * sizeof(T) must be at least 16 bytes");
  static constexpr int LPR = CHUNKS >= 32 ? 32 : CHUNKS;  // lanes per row
  static constexpr int LOG_LPR = ilog2(LPR);
  static constexpr int CPL = CHUNKS / LPR;  // chunks per lane per row
  static constexpr int EPC = 16 / ES;       // elements per chunk
  static constexpr int EPL = CPL * EPC;     // elements per lane per row
  static constexpr int PPL = EPL / 2;       // element pairs per lane per row (packed fp32 math)
  static constexpr int RPL = 32 / LPR;      // rows covered by one warp-wide load
  static constexpr int LOG_RPL = ilog2(RPL);
  static constexpr int TILE_BYTES = 4096;   // K bytes per stage (same again for V)
  static constexpr int TILE = TILE_BYTES / ROW_BYTES;  // tokens per stage
  static constexpr int LOG_TILE = ilog2(TILE);
  static constexpr int NT = TILE / RPL;  // row slots per lane
  static constexpr int NV = NT * GT;     // partial scores per lane before reduction
  static constexpr int LOG_NV = ilog2(NV);
  static constexpr int SL = LOG_LPR < LOG_NV ? LOG_LPR : LOG_NV;  // scatter levels
  static constexpr int AL = LOG_LPR - SL;                          // all-reduce levels
  static constexpr int R = NV >> SL;  // reduced scores held per lane
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static_assert(TILE >= RPL, "tile smaller than one warp load");
  static_assert((1 << LOG_TILE) == TILE, "tile must be a power of two");
};

// Consumer of a worker's tiles: the CUDA-core path above (MMA = false, every dtype and head
// size) or the tensor-core worker of pd_decode_mma.cuh (16-bit K/V, head_dim 64..256).
struct NoMmaWorker {};
template <bool MMA, typename T, int D, int GT>
struct ConsumerSel {
  using W = NoMmaWorker;
  static constexpr int R = DecodeCfg<T, D, GT>::R;
};
template <typename T, int D, int GT>
struct ConsumerSel<true, T, D, GT> {
  using W = MmaWorker<T, D, GT>;
  static constexpr int R = MmaCfg<T, D, GT>::R;
};

// Position of a worker inside the unit sequence.
struct Cursor {
  int b;      // row
  int item;   // kv head * n_gchunks + q-head chunk within the row
  int h;      // kv head (= item / n_gchunks)
  int gc;     // q-head chunk (= item % n_gchunks)
  int tile;   // tile within the item
  int ntile;  // tiles of this row's items
  int len;    // clamped seqlen of the row
};

__device__ __forceinline__ void cursor_advance(Cursor& c, const int* pre, const int* lens, int batch,
                                               int items_per_row, int n_gchunks) {
  if (++c.tile < c.ntile) return;
  c.tile = 0;
  if (++c.gc == n_gchunks) {
    c.gc = 0;
    ++c.h;
  }
  if (++c.item < items_per_row) return;
  c.item = 0;
  c.h = 0;
  c.gc = 0;
  do {
    ++c.b;
  } while (c.b < batch && pre[c.b + 1] == pre[c.b]);
  if (c.b < batch) {
    c.ntile = pre[c.b + 1] - pre[c.b];
    c.len = lens[c.b];
  }
}

// Column-mode advance: the item (kv head, q-head chunk) stays fixed, the cursor walks the
// row's tiles and then the next rows' (rows with no tiles are skipped).
__device__ __forceinline__ void cursor_advance_col(Cursor& c, const int* pre, const int* lens, int batch) {
  if (++c.tile < c.ntile) return;
  c.tile = 0;
  do {
    ++c.b;
  } while (c.b < batch && pre[c.b + 1] == pre[c.b]);
  if (c.b < batch) {
    c.ntile = pre[c.b + 1] - pre[c.b];
    c.len = lens[c.b];
  }
}

// Tag that a launch of epoch `epoch` writes into the high word of its counters. It is odd, so
// it never equals the high word of memory in the states stale memory is usually found in:
// zero-filled (a fresh allocation, a zeroed buffer, the library's static scratch array) or
// holding float partials (+-0, +-inf and 1.0 all have even bit patterns). The even `salt`
// (host-chosen per workspace layout and half) separates the tags of different layouts that
// reuse one buffer, and tags of consecutive epochs differ, so the counters a finished launch
// leaves behind never carry the next launch's tag either.
__device__ __forceinline__ uint32_t counter_tag(uint32_t epoch, uint32_t salt) {
  return ((epoch << 1) | 1u) ^ salt;
}

// ---- step cache of the work split ------------------------------------------------------
// A launch's split -- each warp's range of units (or of columns), its starting cursor, and the
// first two 32-entry windows of that row's block table -- depends only on the clamped lengths
// and the plan's geometry. The layers of a decode step share both, so the first layer of a
// step computes the split and records it per warp, and the later layers, whose lengths hash to
// the recorded key, take it from the record (loaded in the same round trip as the lengths)
// instead of recomputing it and then waiting on the block table. A record's key is never 0,
// so zero-filled memory never matches.
constexpr int STEP_REC_BYTES = 320;
constexpr int STEP_WIN_OFF = 64;  // 64 int32 table entries (the window and the next one)
struct StepHeader {               // bytes 0..47 of a record
  long long u0, u1;
  int b, item, tile, workers;
  int win_row, win_base;
  unsigned long long key;
};

__device__ __forceinline__ unsigned long long mix64(unsigned long long x) {  // SplitMix64 finaliser
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Arrival on the counter shared by the pieces of one split item; returns how many pieces of
// this launch arrived before. Counters live in workspace memory that is never cleared and hold
// (tag << 32) | count. Every launch re-tags its item counters with its own tag in the
// prologue (each CTA a share of them), so an arrival is one acquire-release add (it releases
// the partial the caller's warp stored, and the last piece's acquires the others'), with no
// contention beyond the hardware's. An arrival that beats its counter's re-tag sees another tag; its
// add lands on a value the re-tag overwrites, so it waits for the re-tag and adds again
// (bounded: on expiry it records DEVERR_WAIT_TIMEOUT and returns -1, i.e. "not last").
__device__ __forceinline__ int take_ticket(unsigned long long* counter, uint32_t tag, unsigned* err,
                                           unsigned long long limit_ns) {
  unsigned long long t0 = 0;
  for (;;) {
    const unsigned long long old = atom_add_acq_rel_gpu(counter, 1ull);
    if (uint32_t(old >> 32) == tag) return int(uint32_t(old));
    const unsigned long long now = global_timer_ns();
    if (t0 == 0 && limit_ns >= TEST_LIMIT_NS) {
      t0 = now;
    } else if (now - t0 > limit_ns) {
      atomicOr(err, DEVERR_WAIT_TIMEOUT);
      return -1;
    }
    __nanosleep(128);
  }
}

// Leaving the launch (lane 0 of every warp, on every path): one arrival on the exit counter.
// The last of the launch's `total_warps` arrivals advances the workspace epoch for the next
// launch. An arrival that beats CTA 0's re-tag of the counter sees another tag; like
// take_ticket it waits (bounded) for the re-tag and arrives again.
__device__ __forceinline__ void leave_launch(unsigned long long* exit_counter, unsigned* epoch_word,
                                             uint32_t epoch, uint32_t salt, unsigned total_warps,
                                             unsigned* err) {
  const uint32_t tag = counter_tag(epoch, salt);
  unsigned long long t0 = 0;
  for (;;) {
    const unsigned long long old = atomicAdd(exit_counter, 1ull);
    if (uint32_t(old >> 32) == tag) {
      if (uint32_t(old) == total_warps - 1u) atomicExch(epoch_word, epoch + 1u);
      return;
    }
    const unsigned long long now = global_timer_ns();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > WAIT_LIMIT_NS) {
      atomicOr(err, DEVERR_WAIT_TIMEOUT);
      return;
    }
    __nanosleep(128);
  }
}

// Worker that owns unit u when `units` units are cut into `workers` ranges
// [w*units/workers, (w+1)*units/workers).
__device__ __forceinline__ int worker_of(int64_t u, int64_t units, int workers) {
  return int(((u + 1) * int64_t(workers) - 1) / units);
}

// One launch's work for this thread's warp. It returns on several paths (no work, a failed
// wait, the end of the warp's range); pd_decode_kernel then lets the warp leave the launch.
// The launch's epoch sits in the first word of the shared arrays (written by thread 0 in the
// prologue, read after its block barriers).
//
// CTA = false: every warp runs its own TMA pipeline (per-warp stages, unit or column split).
// CTA = true (used when a row has exactly one item per consumer warp): the CTA shares its
// stages. The last warp is the producer: per column it loads the whole K and V boxes of all
// kv heads (one TMA copy each per block part) into a shared stage, and the consumer warps --
// warp j streams item j -- read their head's rows from it and release the stage on an
// "empty" barrier. Contiguous block-sized copies keep the DRAM stream dense.
template <typename T, int D, int GT, bool CTA, bool MMA>
__device__ __forceinline__ uint32_t decode_body(const DecodeParams& p, const CUtensorMap& kmap,
                                                const CUtensorMap& vmap, unsigned char* smem) {
  using C = DecodeCfg<T, D, GT>;
  using E = Elem<T>;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = (blockDim.x >> 5) - (CTA ? 1 : 0);  // consumer warps
  const bool producer = CTA && warp == nwarps;
  const int S = p.stages;
  const int B = p.batch;
  // Shared-stage geometry (CTA mode): a stage holds TILE tokens of every kv head for K, then V.
  const int kv_stage_bytes = CTA ? p.n_kv_head * C::TILE_BYTES : C::TILE_BYTES;  // K (or V) part
  const int row_stride = CTA ? p.n_kv_head * C::ROW_BYTES : C::ROW_BYTES;       // token to token

  // Dynamic shared memory:
  // [mbarriers | epoch | warp_sums[32] | key_lo[32] | key_hi[32] | grp_cnt[32] | lens[B] | pre[B+1] |
  //  apos[B] | pad | stages].
  // mbarriers: per-warp mode S per warp; CTA mode full[S] then empty[S].
  // The stage region is re-aligned to 1024 B at run time (the host adds the slack).
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  const uint32_t* s_epoch = reinterpret_cast<const uint32_t*>(smem + p.smem_arrays_off);
  int* warp_sums = reinterpret_cast<int*>(smem + p.smem_arrays_off) + 1;
  unsigned* key_lo = reinterpret_cast<unsigned*>(warp_sums + 32);  // per warp: XOR of its rows' hashes
  unsigned* key_hi = key_lo + 32;
  int* grp_cnt = reinterpret_cast<int*>(key_hi + 32);  // arrivals per CTA group (unit mode), by first warp
  int* lens = grp_cnt + 32;
  int* pre = lens + B;  // B + 1 entries: exclusive prefix of tiles per row
  int* apos = pre + B + 1;  // fused append: position to take from the source, or -1
  const uint32_t smem_base = smem_addr(smem);
  unsigned char* stage_base =
      smem + (((smem_base + uint32_t(p.smem_stage_off) + 1023u) & ~1023u) - smem_base);

  if (tid == 0) {
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  // The stage mbarriers are initialised before this thread has any memory operation in
  // flight: the init fence is a release and would otherwise wait for them (the counter
  // re-tags below). Shared stages: thread 0, made visible by the prologue's block barriers.
  if (CTA) {
    if (tid == 0) {
      for (int s = 0; s < S; ++s) {
        mbar_init(smem_addr(bars + s), 1);
        mbar_init(smem_addr(bars + S + s), nwarps);
      }
      fence_barrier_init();
    }
  } else if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(smem_addr(bars + warp * S + s), 1);
    fence_barrier_init();
  }

  // ---- fused append: store every row's new K/V rows in the pools (16 B per thread) -----
  // Every thread runs this exactly once, on whichever path it takes: a worker warp right
  // after issuing its first TMA copies (the stores and their dependent loads then overlap
  // the first DRAM round trip), any other warp before it leaves. Tiles may see the old
  // bytes of these slots (their copies are not ordered after the stores); the consumer
  // overwrites those rows from the source, so the result never depends on which bytes a
  // copy saw.
  // Chunk c of row b's appended K row, rotated when the launch carries rotary tables (the
  // patch below computes the same bits for the tile that reads it).
  auto appended_k_chunk = [&](const T* ksrc, int b, int c) -> uint4 {
    const T* cs = reinterpret_cast<const T*>(p.rope_cos) + int64_t(b) * p.rope_stride;
    const T* sn = reinterpret_cast<const T*>(p.rope_sin) + int64_t(b) * p.rope_stride;
    return rope_chunk(ksrc, cs, sn, c * C::EPC, p.rope_dim);
  };
  auto store_appended = [&]() {
    if (!p.append) return;
    constexpr int CH = C::CHUNKS;
    const int64_t tasks = int64_t(B) * p.n_kv_head * 2 * CH;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + tid; i < tasks; i += int64_t(gridDim.x) * blockDim.x) {
      const int c = int(i % CH);
      int64_t r = i / CH;
      const int kv = int(r & 1);
      r >>= 1;
      const int h = int(r % p.n_kv_head);
      const int b = int(r / p.n_kv_head);
      const int64_t pos = __ldg(p.app_pos + b);
      const int64_t page = pos >= 0 ? (pos >> p.log2_bs) : -1;
      const bool report = c == 0 && kv == 0 && h == 0;
      if (page < 0 || page >= p.max_blocks) {
        if (report) atomicOr(p.err, DEVERR_APPEND_RANGE);
        continue;
      }
      const int64_t blk = __ldg(p.table + int64_t(b) * p.bt_stride + page);
      if (blk < 0 || blk >= p.n_blocks) {
        if (report) atomicOr(p.err, DEVERR_APPEND_RANGE);
        continue;
      }
      const int64_t off = pos & (p.block_size - 1);
      const T* src = kv ? reinterpret_cast<const T*>(p.app_v) + int64_t(b) * p.app_v_sb + int64_t(h) * p.app_v_sh
                        : reinterpret_cast<const T*>(p.app_k) + int64_t(b) * p.app_k_sb + int64_t(h) * p.app_k_sh;
      T* dst = kv ? reinterpret_cast<T*>(p.pool_v) + blk * p.pv_sb + off * p.pv_sn + int64_t(h) * p.pv_sh
                  : reinterpret_cast<T*>(p.pool_k) + blk * p.pk_sb + off * p.pk_sn + int64_t(h) * p.pk_sh;
      *reinterpret_cast<uint4*>(dst + c * C::EPC) =
          !kv && p.rope_cos ? appended_k_chunk(src, b, c) : __ldg(reinterpret_cast<const uint4*>(src + c * C::EPC));
    }
  };

  // ---- this warp's step record, loaded alongside the lengths --------------------------
  const bool use_step = !CTA && p.step_rec != nullptr;
  unsigned char* my_rec =
      use_step ? p.step_rec + (size_t(blockIdx.x) * (blockDim.x >> 5) + warp) * STEP_REC_BYTES : nullptr;
  uint4 rec_a = make_uint4(0u, 0u, 0u, 0u), rec_b = rec_a, rec_c = rec_a;
  int rec_win0 = 0, rec_win1 = 0;
  if (use_step) {
    if (lane == 0) {
      rec_a = ld_cg_v4(my_rec);
      rec_b = ld_cg_v4(my_rec + 16);
      rec_c = ld_cg_v4(my_rec + 32);
    }
    if (p.step_table) {
      rec_win0 = __ldcg(reinterpret_cast<const int*>(my_rec + STEP_WIN_OFF) + lane);
      rec_win1 = __ldcg(reinterpret_cast<const int*>(my_rec + STEP_WIN_OFF) + 32 + lane);
    }
  }

  // ---- prologue: clamp lengths, tiles per row, block-wide exclusive scan -------------
  unsigned long long launch_key = 0;  // the step key of these lengths (step cache)
  {
    // The launch's epoch (thread 0) is loaded alongside the lengths, not before them.
    const unsigned ep = tid == 0 ? *reinterpret_cast<volatile unsigned*>(p.epoch_word) : 0u;
    const int per = (B + blockDim.x - 1) / blockDim.x;
    const int b0 = min(B, tid * per);
    const int b1 = min(B, b0 + per);
    int local = 0;
    unsigned long long key = 0;
    for (int b = b0; b < b1; ++b) {
      int len = __ldg(p.seqlen + b);
      const int64_t pos = p.append ? __ldg(p.app_pos + b) : -1;
      len = len < 0 ? 0 : (len > p.capacity ? p.capacity : len);
      lens[b] = len;
      key ^= mix64(p.step_salt ^ ((unsigned long long)(unsigned)b << 32 | (unsigned)len));
      // Fused append: the tile holding the appended token takes it from the source when the
      // row reads that position (a position inside [0, len) is inside the table).
      if (p.append) apos[b] = pos >= 0 && pos < len ? int(pos) : -1;
      local += (len + C::TILE - 1) >> C::LOG_TILE;
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(FULL_MASK, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    if (tid == 0) *reinterpret_cast<uint32_t*>(smem + p.smem_arrays_off) = ep;
    if (tid < 32) grp_cnt[tid] = 0;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) key ^= __shfl_xor_sync(FULL_MASK, key, o);
    if (lane == 0) {
      key_lo[warp] = unsigned(key);
      key_hi[warp] = unsigned(key >> 32);
    }
    __syncthreads();
    if (warp == 0) {
      int v = lane < int(blockDim.x >> 5) ? warp_sums[lane] : 0;  // every warp's share
      int vi = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(FULL_MASK, vi, o);
        if (lane >= o) vi += y;
      }
      warp_sums[lane] = vi - v;  // exclusive warp offsets
      if (lane == 31) pre[B] = vi;
    }
    __syncthreads();
    int run = warp_sums[warp] + incl - local;
    for (int b = b0; b < b1; ++b) {
      pre[b] = run;
      run += (lens[b] + C::TILE - 1) >> C::LOG_TILE;
    }
    __syncthreads();
    if (use_step) {
      for (int i = 0; i < int(blockDim.x >> 5); ++i)
        launch_key ^= (unsigned long long)key_hi[i] << 32 | key_lo[i];
      launch_key = mix64(launch_key ^ p.step_salt) | 1ull;
    }
  }
  const uint32_t epoch = *s_epoch;

  // Re-tag this launch's item counters (this CTA's share) and, in CTA 0, the exit counter
  // with the launch's tag (counter_tag). Arrivals come at least one tile later. (The workspace belongs to
  // this launch alone: an overlapped launch gets the other half of its plan's workspace from
  // the one it overlaps.)
  {
    const int64_t n_items = int64_t(B) * p.n_kv_head * p.n_gchunks;
    const unsigned long long tag = (unsigned long long)counter_tag(epoch, p.tag_salt) << 32;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + tid; i < n_items; i += int64_t(gridDim.x) * blockDim.x)
      atomicExch(p.counters + i, tag);
    if (blockIdx.x == 0 && tid == 0) atomicExch(p.exit_counter, tag);
  }

  // ---- the dependency point ------------------------------------------------------------
  // Everything before it -- the prologue, the work split, the first K/V copies -- reads only
  // the lengths, positions, block table, pools and this launch's workspace, none of which the
  // preceding kernel of an overlapped launch writes. Each warp passes this point once, on
  // whichever path it takes, before it reads q or the appended rows or writes any output:
  // it waits for the preceding grid, writes its share of the zero-length rows' outputs and
  // lets the next launch start.
  auto enter_dependent = [&]() {
    griddep_wait();
    // zero-length rows: exact zeros (mode 0) or an empty triple (mode 1)
    for (int b = blockIdx.x; b < B; b += gridDim.x) {
      if (lens[b] != 0) continue;
      for (int i = tid; i < p.n_head * D; i += blockDim.x) {
        const int h = i / D, d = i - h * D;
        if (p.mode == 0) {
          T* o = reinterpret_cast<T*>(p.out) + int64_t(b) * p.o_sb + int64_t(h) * p.o_sh + d;
          *o = E::from_float(0.f);
        } else {
          p.part_acc[(int64_t(b) * p.n_head + h) * D + d] = 0.f;
          if (d == 0) {
            p.part_m[int64_t(b) * p.n_head + h] = -INFINITY;
            p.part_l[int64_t(b) * p.n_head + h] = 0.f;
          }
        }
      }
    }
    griddep_launch_dependents();
  };

  const int items_per_row = p.n_kv_head * p.n_gchunks;
  const int64_t units = int64_t(items_per_row) * pre[B];
  if (units == 0) {
    enter_dependent();
    store_appended();
    return epoch;
  }

  // ---- this warp's share of the work -----------------------------------------------------
  // Column mode (a row has exactly one item per warp): the (row, tile) columns are cut into
  // one contiguous range per CTA, and warp j streams item j over the CTA's columns. The
  // block's kv heads are then requested by the CTA's warps at about the same time, which is
  // what keeps DRAM pages open. Otherwise (unit mode) the units (row, item, tile) are cut
  // into one contiguous range per warp.
  const bool colmode = CTA || items_per_row == nwarps;
  const int64_t ncols = pre[B];
  // Column mode cuts *virtual* columns: each row is preceded by row_cost extra ones (what a
  // row switch costs a warp -- a table window, a q load, a partial store -- in tile times),
  // so a range that crosses into a new row gets that many fewer real tiles. vpre(b) is the
  // first virtual column of row b; its real tiles start row_cost later.
  const int rc = colmode ? p.row_cost : 0;
  auto vpre = [&](int b) -> int64_t { return int64_t(pre[b]) + int64_t(rc) * b; };
  const int64_t vcols = colmode ? vpre(B) : 0;
  // Ranges in use: never more than virtual columns, so that no range is empty.
  const int col_parts = int(vcols < int64_t(gridDim.x) ? vcols : int64_t(gridDim.x));
  // Real column at virtual column v (0 <= v <= vcols); a row's extra columns map to its first tile.
  auto real_col = [&](int64_t v) -> int64_t {
    if (v >= vcols) return ncols;
    int lo = 0, hi = B;  // first row i with vpre(i) > v
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (vpre(mid) > v) hi = mid; else lo = mid + 1;
    }
    const int64_t t = v - vpre(lo - 1) - rc;
    return pre[lo - 1] + (t > 0 ? t : 0);
  };
  auto range_start = [&](int c) -> int64_t { return real_col(int64_t(c) * vcols / col_parts); };
  int workers = 0, w = 0;     // unit mode: worker count and this warp's worker id
  int64_t u0 = 0, u1 = 0;     // unit mode: range of units; column mode: range of real columns
  // Step cache: this warp's record holds the split of these very lengths.
  const bool cached =
      use_step && __shfl_sync(FULL_MASK, lane == 0 && ((unsigned long long)rec_c.w << 32 | rec_c.z) == launch_key, 0);
  if (cached) {
    u0 = __shfl_sync(FULL_MASK, (long long)rec_a.y << 32 | rec_a.x, 0);
    u1 = __shfl_sync(FULL_MASK, (long long)rec_a.w << 32 | rec_a.z, 0);
    workers = __shfl_sync(FULL_MASK, int(rec_b.w), 0);
  } else if (colmode) {
    if (int(blockIdx.x) < col_parts) {
      u0 = range_start(int(blockIdx.x));
      u1 = range_start(int(blockIdx.x) + 1);
    }
  } else {
    // Never more workers than units: every worker range must be non-empty, because a split
    // item is merged when all workers overlapping it have arrived.
    workers = int(gridDim.x) * nwarps;
    if (int64_t(workers) > units) workers = int(units);
    if (p.min_tiles > 1) {
      const int64_t want = (units + p.min_tiles - 1) / p.min_tiles;
      if (want < workers) workers = int(want < 1 ? 1 : want);
    }
    // With at most one item per worker, a multiple of the item count makes every item
    // boundary a range boundary when the rows are equally long: no range then straddles two
    // items, so items have fewer pieces and every piece is a single segment. Taken when it
    // idles at most 1/20 of the workers.
    {
      const int64_t n_items = int64_t(B) * items_per_row;
      if (n_items <= workers) {
        const int aligned = int((workers / n_items) * n_items);
        if (int64_t(aligned) * 20 >= int64_t(workers) * 19) workers = aligned;
      }
    }
  }
  // Unit mode, worker numbering. When (nearly) every warp is a worker, consecutive workers
  // share a CTA ("grouped"): the pieces of a split item then sit in few CTAs, and the pieces
  // that end a range are folded in shared memory by the last warp of their CTA before one
  // piece per CTA goes to the global merge. Otherwise low worker ids are spread over all SMs.
  const bool grouped = !colmode && int64_t(workers) * 20 >= int64_t(gridDim.x) * nwarps * 19;
  if (!colmode) {
    w = grouped ? int(blockIdx.x) * nwarps + warp : warp * int(gridDim.x) + int(blockIdx.x);
    if (!cached) {
      u0 = w < workers ? int64_t(w) * units / workers : 0;
      u1 = w < workers ? int64_t(w + 1) * units / workers : 0;
    }
  }
  // Records this launch's split of its warp (when it computed it): header by lane 0, the
  // table windows the first copies used by every lane, made visible before the launch lets the
  // next one start (enter_dependent).
  auto write_record = [&](int rb, int ritem, int rtile, int wrow, int wbase, int wcur, int wnxt) {
    if (!use_step || cached) return;
    if (lane == 0) {
      StepHeader hd;
      hd.u0 = u0;
      hd.u1 = u1;
      hd.b = rb;
      hd.item = ritem;
      hd.tile = rtile;
      hd.workers = workers;
      hd.win_row = wrow;
      hd.win_base = wbase;
      hd.key = launch_key;
      *reinterpret_cast<StepHeader*>(my_rec) = hd;
    }
    reinterpret_cast<int*>(my_rec + STEP_WIN_OFF)[lane] = wcur;
    reinterpret_cast<int*>(my_rec + STEP_WIN_OFF)[32 + lane] = wnxt;
    __threadfence();
  };
  if (u0 >= u1) {
    write_record(0, 0, 0, -1, 0, 0, 0);
    enter_dependent();
    store_appended();
    return epoch;
  }
  const int64_t nunits = u1 - u0;
  // Partial-result slot pair of this warp (two: its range's first and last segment).
  const int wslot = colmode ? int(blockIdx.x) * nwarps + warp : w;
  auto advance = [&](Cursor& c) {
    if (colmode) cursor_advance_col(c, pre, lens, B);
    else cursor_advance(c, pre, lens, B, items_per_row, p.n_gchunks);
  };

  // Stage s of this warp: K at stage_k(s), V at stage_k(s) + kv_stage_bytes. Its "full"
  // barrier completes when the stage's copies land; in CTA mode the consumers' arrivals on
  // its "empty" barrier hand it back to the producer.
  uint64_t* my_bars = CTA ? bars : bars + warp * S;
  uint64_t* empty_bars = bars + S;  // CTA mode only
  unsigned char* my_stages = CTA ? stage_base : stage_base + size_t(warp) * S * C::STAGE_BYTES;
  const size_t stage_stride = CTA ? size_t(2) * kv_stage_bytes : size_t(C::STAGE_BYTES);
  if (CTA) {
    __syncthreads();  // the CTA's warps share one range: all of them are here
  } else {
    __syncwarp();
  }

  // Locate u0: the last row whose first unit (column) is <= u0 (rows with no tiles are skipped).
  Cursor cur;
  if (cached) {
    cur.b = __shfl_sync(FULL_MASK, int(rec_b.x), 0);
    cur.item = __shfl_sync(FULL_MASK, int(rec_b.y), 0);
    cur.tile = __shfl_sync(FULL_MASK, int(rec_b.z), 0);
    cur.ntile = pre[cur.b + 1] - pre[cur.b];
    cur.len = lens[cur.b];
    cur.h = cur.item / p.n_gchunks;
    cur.gc = cur.item - cur.h * p.n_gchunks;
  } else {
    const int per_row = colmode ? 1 : items_per_row;
    int lo = 0, hi = B;  // find first i with per_row * pre[i] > u0
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (int64_t(per_row) * pre[mid] > u0) hi = mid; else lo = mid + 1;
    }
    cur.b = lo - 1;
    cur.ntile = pre[cur.b + 1] - pre[cur.b];
    cur.len = lens[cur.b];
    const int64_t r = u0 - int64_t(per_row) * pre[cur.b];
    cur.item = colmode ? (producer ? 0 : warp) : int(r / cur.ntile);
    cur.tile = int(r - int64_t(colmode ? 0 : cur.item) * cur.ntile);
    cur.h = cur.item / p.n_gchunks;
    cur.gc = cur.item - cur.h * p.n_gchunks;
  }

  // ---- producer: block-table window + TMA issue ---------------------------------------
  const int bs = p.block_size;
  const int box_tokens = p.box_tokens;
  const int log2_box = p.log2_box;
  const int nbox = C::TILE >> log2_box;
  const uint32_t box_bytes = uint32_t(box_tokens) * uint32_t(row_stride);  // one copy
  int win_row = -1, win_base = 0, win_cur = 0, win_nxt = 0;
  if (cached && p.step_table) {  // the recorded windows of this row's table (a fixed table)
    const int rrow = __shfl_sync(FULL_MASK, int(rec_c.x), 0);
    if (rrow >= 0) {
      win_row = rrow;
      win_base = __shfl_sync(FULL_MASK, int(rec_c.y), 0);
      win_cur = rec_win0;
      win_nxt = rec_win1;
    }
  }

  auto table_entry = [&](int row, int page, int npages) -> int {
    if (page < npages && page < p.max_blocks) return __ldg(p.table + int64_t(row) * p.bt_stride + page);
    return 0;
  };
  // Warp-collective: all lanes call with the same (row, page).
  auto block_of = [&](int row, int page, int npages) -> int {
    if (row != win_row || page < win_base || page >= win_base + 32) {
      if (row == win_row && page >= win_base + 32 && page < win_base + 64) {
        win_cur = win_nxt;
        win_base += 32;
      } else {
        win_row = row;
        win_base = page & ~31;
        win_cur = table_entry(row, win_base + lane, npages);
      }
      win_nxt = table_entry(row, win_base + 32 + lane, npages);
    }
    return __shfl_sync(FULL_MASK, win_cur, page - win_base);
  };

  const uint64_t kv_policy = l2_policy_evict_first();
  auto issue = [&](const Cursor& c, int s) {
    const int h = c.h;
    const int tok0 = c.tile << C::LOG_TILE;
    const int remain = c.len - tok0;  // >= 1
    const int nvalid = min(nbox, (remain + box_tokens - 1) >> log2_box);
    const int npages = (c.len + bs - 1) >> p.log2_bs;
    const uint32_t bar = smem_addr(my_bars + s);
    const uint32_t kdst = smem_addr(my_stages + size_t(s) * stage_stride);
    const uint32_t vdst = kdst + uint32_t(kv_stage_bytes);
    if (lane == 0) mbar_arrive_expect_tx(bar, 2u * uint32_t(nvalid) * box_bytes);
    for (int j = 0; j < nvalid; ++j) {
      const int tok = tok0 + j * box_tokens;
      const int page = tok >> p.log2_bs;
      const int off = tok & (bs - 1);
      const int blk = block_of(c.b, page, npages);
      if (lane == 0) {
        // K/V bytes are read once per launch: evict-first keeps the stream from evicting the
        // split partials that the merges read back at the end.
        if constexpr (MMA) {  // swizzled map: (64 elements, token, head, 128-byte piece, block)
          tma_load_5d_hint(kdst + j * box_bytes, &kmap, bar, 0, off, h, 0, blk, kv_policy);
          tma_load_5d_hint(vdst + j * box_bytes, &vmap, bar, 0, off, h, 0, blk, kv_policy);
        } else {
          tma_load_4d_hint(kdst + j * box_bytes, &kmap, bar, 0, CTA ? 0 : h, off, blk, kv_policy);
          tma_load_4d_hint(vdst + j * box_bytes, &vmap, bar, 0, CTA ? 0 : h, off, blk, kv_policy);
        }
      }
    }
  };

  // Pulls the q rows of the item that cursor c opens into L2, so that start_segment, a few
  // tiles later, does not wait on DRAM.
  auto prefetch_q = [&](const Cursor& c) {
    constexpr int LINES = (C::ROW_BYTES + 127) / 128;  // 128-byte lines per q row
    if (lane < GT * LINES) {
      const int hq = c.h * p.group + c.gc * GT + lane / LINES;
      prefetch_l2(reinterpret_cast<const unsigned char*>(p.q) +
                  (int64_t(c.b) * p.q_sb + int64_t(hq) * p.q_sh) * C::ES + (lane % LINES) * 128);
    }
  };

  Cursor pc = cur;
  int64_t issued = 0;
  if (producer) {
    // CTA mode: the producer streams the CTA's columns into the shared stages. Stage s is
    // reused once all consumer warps released its previous column (empty barrier).
    for (; issued < nunits; ++issued) {
      const int s = int(issued % S);
      if (issued >= S &&
          !warp_wait_phase(smem_addr(empty_bars + s), uint32_t(((issued / S) - 1) & 1), p.wait_ns)) {
        if (lane == 0) atomicOr(p.err, DEVERR_WAIT_TIMEOUT);
        break;
      }
      issue(pc, s);
      advance(pc);
      if (issued + 1 == (nunits < S ? nunits : S)) {
        enter_dependent();
        store_appended();
      }
    }
    if (issued < (nunits < S ? nunits : S)) {
      enter_dependent();
      store_appended();
    }
    // Leave only once the copies issued last have landed (bounded): the CTA must not retire
    // with a copy in flight, whatever the consumers did.
    const int64_t from = issued > S ? issued - S : 0;
    for (int64_t j = from; j < issued; ++j)
      warp_wait_phase(smem_addr(my_bars + int(j % S)), uint32_t((j / S) & 1), DRAIN_LIMIT_NS);
    return epoch;
  }
  if (!CTA) {
    const int64_t first = nunits < S ? nunits : S;
    for (; issued < first; ++issued) {
      issue(pc, int(issued));
      advance(pc);
      if (pc.tile == 0 && issued + 1 < nunits) prefetch_q(pc);
    }
    write_record(cur.b, cur.item, cur.tile, win_row, win_base, win_cur, win_nxt);
  }
  enter_dependent();
  store_appended();
  // This warp's rows inside a stage: per-warp stages hold only its head; shared stages hold
  // every kv head, and the warp's item fixes its head (column mode).
  const int head_off = CTA ? (warp / p.n_gchunks) * C::ROW_BYTES : 0;

  // ---- consumer state -----------------------------------------------------------------
  const int rg = lane >> C::LOG_LPR;        // row group of this lane
  const int pl = lane & (C::LPR - 1);       // position within the row group
  const int hold_q = pl >> C::AL;           // reduced-score block held by this lane
  const bool primary = (pl & ((1 << C::AL) - 1)) == 0;
  // Held score j of this lane is (tile row hold_row[j], q head hold_g[j]): index
  // j + R * hold_q = (row slot i) * GT + g, row = i * RPL + rg. Lane constants.
  int hold_row[C::R], hold_g[C::R];
#pragma unroll
  for (int j = 0; j < C::R; ++j) {
    const int idx = j + C::R * hold_q;
    hold_row[j] = (idx / GT) * C::RPL + rg;
    hold_g[j] = idx % GT;
  }

  // Tensor-core consumer (MMA): its own fragments and running state; RR scores per lane.
  using Sel = ConsumerSel<MMA, T, D, GT>;
  constexpr int RR = Sel::R;
  typename Sel::W mw;
  const uint32_t stages_addr = smem_addr(my_stages);
  if constexpr (MMA) mw.init(lane, p.box_tokens, p.log2_box);

  // q and the P.V accumulators as pairs of consecutive head_dim elements: every multiply-add
  // below is a packed fp32 FMA (two lanes of fp32 per instruction, same rounding as fmaf).
  float2 qf[GT][C::PPL];
  float2 acc[GT][C::PPL];
  auto acc_at = [&](int g, int e) -> float& { return (e & 1) ? acc[g][e >> 1].y : acc[g][e >> 1].x; };
  float m_run[GT], l_run[GT];
  int seg_first_tile = 0;
  bool first_segment = true;
  // Split segments of this range whose partials are stored and whose arrival comes after the
  // loop: a range holds at most two (its first and its last segment).
  int n_pend = 0;
  int pend_b0 = 0, pend_item0 = 0, pend_b1 = 0, pend_item1 = 0;
  bool early = false;                 // the first pending segment already arrived (lane 0's
  unsigned long long early_old = 0;   // add returned early_old)

  // Phase A of a tile: q.K for every (row, q head) of the stage, reduce-scattered so this
  // lane ends with its R held scores, scaled to log2 units and masked past valid_rows.
  auto tile_scores = [&](int stage, int valid_rows, float (&sc)[RR]) {
    if constexpr (MMA) {
      mw.scores(stages_addr + uint32_t(stage) * uint32_t(stage_stride), valid_rows, p.scale_log2, sc);
    } else {
      const unsigned char* ks = my_stages + size_t(stage) * stage_stride + head_off;
      float sv[C::NV];
#pragma unroll
      for (int i = 0; i < C::NT; ++i) {
        const int row = i * C::RPL + rg;
        float2 kf[C::PPL];
#pragma unroll
        for (int c = 0; c < C::CPL; ++c) {
          const uint4 raw = *reinterpret_cast<const uint4*>(ks + row * row_stride + (c * C::LPR + pl) * 16);
          E::unpack_pairs(raw, &kf[c * (C::EPC / 2)]);
        }
#pragma unroll
        for (int g = 0; g < GT; ++g) {
          float2 a = __fmul2_rn(qf[g][0], kf[0]);
#pragma unroll
          for (int e = 1; e < C::PPL; ++e) a = __ffma2_rn(qf[g][e], kf[e], a);
          sv[i * GT + g] = a.x + a.y;
        }
      }
#pragma unroll
      for (int lv = 0; lv < C::SL; ++lv) {  // butterfly reduce-scatter over the row group
        const int o = C::LPR >> (lv + 1);
        const int half = C::NV >> (lv + 1);
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < half; ++j) {
          const float send = up ? sv[j] : sv[j + half];
          const float keep = up ? sv[j + half] : sv[j];
          sv[j] = keep + __shfl_xor_sync(FULL_MASK, send, o);
        }
      }
#pragma unroll
      for (int lv = C::SL; lv < C::LOG_LPR; ++lv) sv[0] += __shfl_xor_sync(FULL_MASK, sv[0], C::LPR >> (lv + 1));
#pragma unroll
      for (int j = 0; j < C::R; ++j) {
        const float x = sv[j] * p.scale_log2;
        sc[j] = hold_row[j] < valid_rows ? x : -INFINITY;
      }
    }
  };

  // Phase B, part 1: the online-softmax max update. m' = max(m, tile max) and
  // alpha = exp2(m - m') is the identity when no score of the tile exceeds the running max,
  // so the warp max and the rescale run only when one does (same arithmetic as always).
  auto tile_max_update = [&](const float (&sc)[RR]) {
    if constexpr (MMA) {
      mw.max_update(sc);
    } else {
      bool exceeds = false;
#pragma unroll
      for (int j = 0; j < C::R; ++j) {
#pragma unroll
        for (int g = 0; g < GT; ++g)
          if (hold_g[j] == g) exceeds |= sc[j] > m_run[g];
      }
      if (__builtin_expect(__any_sync(FULL_MASK, exceeds), 0)) {
        float tmax[GT];
#pragma unroll
        for (int g = 0; g < GT; ++g) tmax[g] = -INFINITY;
#pragma unroll
        for (int j = 0; j < C::R; ++j) {
#pragma unroll
          for (int g = 0; g < GT; ++g)
            if (hold_g[j] == g) tmax[g] = fmaxf(tmax[g], sc[j]);
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
#pragma unroll
          for (int g = 0; g < GT; ++g) tmax[g] = fmaxf(tmax[g], __shfl_xor_sync(FULL_MASK, tmax[g], o));
        }
#pragma unroll
        for (int g = 0; g < GT; ++g) {
          const float mn = fmaxf(m_run[g], tmax[g]);  // finite: the tile has a live row
          const float alpha = exp2f(m_run[g] - mn);
          m_run[g] = mn;
          l_run[g] *= alpha;
          const float2 alpha2 = make_float2(alpha, alpha);
#pragma unroll
          for (int e = 0; e < C::PPL; ++e) acc[g][e] = __fmul2_rn(acc[g][e], alpha2);
        }
      }
      }
  };

  // Phase B, part 2: probabilities, their shuffle to the lanes that own each row's V chunk,
  // and P.V into the fp32 accumulators. Rows at or past valid_rows contribute exact zeros
  // (their V is zeroed too, so stale bytes -- even NaN patterns -- never reach acc).
  auto tile_pv = [&](int stage, const float (&sc)[RR], int valid_rows, bool full) {
    if constexpr (MMA) {
      mw.pv(stages_addr + uint32_t(stage) * uint32_t(stage_stride) + uint32_t(kv_stage_bytes), sc, valid_rows, full);
    } else {
      float pj[C::R];
#pragma unroll
      for (int j = 0; j < C::R; ++j) {
        float mj = m_run[0];
#pragma unroll
        for (int g = 1; g < GT; ++g)
          if (hold_g[j] == g) mj = m_run[g];
        pj[j] = exp2f(sc[j] - mj);
        if (primary) {
#pragma unroll
          for (int g = 0; g < GT; ++g)
            if (hold_g[j] == g) l_run[g] += pj[j];
        }
      }
      const unsigned char* vs = my_stages + size_t(stage) * stage_stride + kv_stage_bytes + head_off;
#pragma unroll
      for (int i = 0; i < C::NT; ++i) {
        const int row = i * C::RPL + rg;
        float2 vf[C::PPL];
#pragma unroll
        for (int c = 0; c < C::CPL; ++c) {
          const uint4 raw = *reinterpret_cast<const uint4*>(vs + row * row_stride + (c * C::LPR + pl) * 16);
          E::unpack_pairs(raw, &vf[c * (C::EPC / 2)]);
        }
        if (!full) {
          const bool live = row < valid_rows;
#pragma unroll
          for (int e = 0; e < C::PPL; ++e) vf[e] = live ? vf[e] : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int g = 0; g < GT; ++g) {
          const int idx = i * GT + g;
          const int src = (rg << C::LOG_LPR) + ((idx / C::R) << C::AL);
          const float pv = __shfl_sync(FULL_MASK, pj[idx % C::R], src);
          const float2 pv2 = make_float2(pv, pv);
#pragma unroll
          for (int e = 0; e < C::PPL; ++e) acc[g][e] = __ffma2_rn(pv2, vf[e], acc[g][e]);
        }
      }
    }
  };

  auto start_segment = [&](const Cursor& c) {
    if constexpr (MMA) {
      mw.start(reinterpret_cast<const T*>(p.q) + int64_t(c.b) * p.q_sb, p.q_sh, c.h * p.group + c.gc * GT);
    } else {
      const int hq = c.h * p.group + c.gc * GT;
      const T* qrow = reinterpret_cast<const T*>(p.q) + int64_t(c.b) * p.q_sb;
#pragma unroll
      for (int g = 0; g < GT; ++g) {
#pragma unroll
        for (int cc = 0; cc < C::CPL; ++cc) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(qrow + int64_t(hq + g) * p.q_sh +
                                                                   (cc * C::LPR + pl) * C::EPC));
          E::unpack_pairs(raw, &qf[g][cc * (C::EPC / 2)]);
        }
        m_run[g] = -INFINITY;
        l_run[g] = 0.f;
#pragma unroll
        for (int e = 0; e < C::PPL; ++e) acc[g][e] = make_float2(0.f, 0.f);
      }
    }
  };

  // Fused append: after tile c's copies landed in `stage`, overwrite the appended token's
  // K and V rows with the source rows (16 B per lane), so the tile holds the new token
  // whatever the copy read from the pool. (Tensor-core stages hold the row in swizzled
  // 16-byte units; unit u of token t sits at mw.unit_addr(0, t, u).)
  auto patch = [&](const Cursor& c, int stage) {
    if (!p.append) return;
    const int ap = apos[c.b];
    if (ap < 0 || (ap >> C::LOG_TILE) != c.tile) return;
    const int t = ap & (C::TILE - 1);
    unsigned char* ktile = my_stages + size_t(stage) * stage_stride;
    unsigned char* krow = ktile + t * row_stride + head_off;
    unsigned char* vrow = krow + kv_stage_bytes;
    const T* ksrc = reinterpret_cast<const T*>(p.app_k) + int64_t(c.b) * p.app_k_sb + int64_t(c.h) * p.app_k_sh;
    const T* vsrc = reinterpret_cast<const T*>(p.app_v) + int64_t(c.b) * p.app_v_sb + int64_t(c.h) * p.app_v_sh;
    for (int i = lane; i < 2 * C::CHUNKS; i += 32) {
      const bool isv = i >= C::CHUNKS;
      const int ci = isv ? i - C::CHUNKS : i;
      const uint4 x = !isv && p.rope_cos ? appended_k_chunk(ksrc, c.b, ci)
                                         : __ldg(reinterpret_cast<const uint4*>((isv ? vsrc : ksrc) + ci * C::EPC));
      if constexpr (MMA) {
        *reinterpret_cast<uint4*>(ktile + (isv ? kv_stage_bytes : 0) + mw.unit_addr(0u, t, ci)) = x;
      } else {
        *reinterpret_cast<uint4*>((isv ? vrow : krow) + ci * 16) = x;
      }
    }
    fence_proxy_async_smem();  // the stage is refilled by TMA later
    __syncwarp();
  };

  auto fail_and_drain = [&](int64_t from) {
    if (lane == 0) atomicOr(p.err, DEVERR_WAIT_TIMEOUT);
    if (!CTA) {  // shared stages' copies are the producer's; it waits for them before it leaves
      for (int64_t j = from; j < issued; ++j)
        warp_wait_phase(smem_addr(my_bars + int(j % S)), uint32_t((j / S) & 1), DRAIN_LIMIT_NS);
    }
  };

  // Unit mode: the workers whose ranges overlap item (b, item) are w_a .. w_b. Every piece ends
  // its worker's range except possibly w_b's: when w_b's range runs past the item (mid), the
  // item is that range's first segment, parked in slot 0 and arrived at once. w_t is the last
  // worker whose piece ends its range (slot 1, or its CTA group's shared memory when grouped).
  struct ItemSpan {
    int w_a, w_b, w_t;
    bool mid;
  };
  auto item_span = [&](int b, int item) -> ItemSpan {
    const int nt = pre[b + 1] - pre[b];
    const int64_t us = int64_t(items_per_row) * pre[b] + int64_t(item) * nt;
    ItemSpan r;
    r.w_a = worker_of(us, units, workers);
    r.w_b = worker_of(us + nt - 1, units, workers);
    r.mid = int64_t(r.w_b + 1) * units / workers > us + nt;
    r.w_t = r.mid ? r.w_b - 1 : r.w_b;
    return r;
  };
  // Pieces of a split item that reach the global merge (unit mode): one per CTA group of
  // range-ending pieces (grouped numbering) or one per range-ending piece, then the mid piece.
  auto global_reps = [&](const ItemSpan& sp) -> int {
    return grouped ? sp.w_t / nwarps - sp.w_a / nwarps + 1 : sp.w_t - sp.w_a + 1;
  };
  // A range-ending piece parked in shared memory: warp j's own stages hold its accumulators
  // (GT x D floats, head-major) followed by m[GT] and l[GT].
  auto smem_piece = [&](int j) -> float* {
    return reinterpret_cast<float*>(stage_base + size_t(j) * S * C::STAGE_BYTES);
  };

  // Where the pieces of a fold live. One fold routine serves every kind, so that its code
  // exists once in the kernel. kind 0: column mode, the slot pairs of CTAs a = c_first ..
  // (b = whether the first CTA's range starts at the row, c = the item's warp); kind 1: unit
  // mode, the item's global pieces (a = w_a, b = nreps, c = w_b; see merge_if_last); kind 2: the
  // range-ending pieces of a CTA group in the stages of warps a, a + 1, ...
  struct FoldSrc {
    int kind, a, b, c;
  };
  auto piece_ptr = [&](const FoldSrc& src, int i, const float*& ml, const float*& acc) {
    if (src.kind == 2) {
      acc = smem_piece(src.a + i);
      ml = acc + GT * D;
      return;
    }
    int64_t sl;
    if (src.kind == 0) {
      sl = (int64_t(src.a + i) * nwarps + src.c) * 2 + (i == 0 && !src.b ? 1 : 0);
    } else if (i >= src.b) {
      sl = int64_t(src.c) * 2;
    } else {
      const int rep = grouped ? (i == 0 ? src.a : (src.a / nwarps + i) * nwarps) : src.a + i;
      sl = int64_t(rep) * 2 + 1;
    }
    ml = p.ws_ml + sl * (2 * GT);
    acc = p.ws_acc + sl * (GT * D);
  };

  // Folds npieces partial triples of item (mb, mitem) in piece order (piece i's m at ml, its l
  // at ml + GT, its accumulators at acc, from piece_ptr) with a running maximum, and writes the
  // result: the normalised output (mode 0) or the item's triple (mode 1) when dst_ml is null,
  // otherwise one partial triple at dst_ml / dst_acc (a CTA group's piece). Each lane owns NG
  // consecutive float4 groups of the GT x D output and folds the pieces in batches of MB,
  // every load of a batch in flight together.
  auto fold_pieces = [&](int mb, int mitem, int npieces, const FoldSrc& src, float* dst_ml, float* dst_acc) {
    const bool from_global = src.kind != 2;
    const int mh = mitem / p.n_gchunks;
    const int mhq0 = mh * p.group + (mitem - mh * p.n_gchunks) * GT;
    // The item's output is GROUPS float4 groups, head-major; lane l owns groups t * 32 + l,
    // so each load instruction of the warp reads 512 contiguous bytes of a partial. Every lane
    // keeps the running maximum and normaliser of all GT heads (from broadcast loads).
    constexpr int GROUPS = GT * (D / 4);
    constexpr int GPH = D / 4;                           // groups per head
    constexpr int NG = GROUPS >= 32 ? GROUPS / 32 : 1;   // groups per lane
    constexpr int GB = NG < 8 ? NG : 8;                  // groups per pass
    constexpr int MB = GB >= 8 ? (GT >= 8 ? 2 : 4) : 16 / GB;  // pieces per batch
    auto head_of = [&](int t) -> int {  // head of the lane's group t (static when GPH >= 32)
      return (t * 32) / GPH + (GPH >= 32 ? 0 : lane / GPH);
    };
    auto pick = [&](const float (&v)[GT], int g) -> float {
      float r = v[0];
#pragma unroll
      for (int gg = 1; gg < GT; ++gg)
        if (g == gg) r = v[gg];
      return r;
    };
    auto ld1 = [&](const float* q) -> float { return from_global ? __ldcg(q) : *q; };
    auto ld4 = [&](const float* q) -> float4 {
      return from_global ? __ldcg(reinterpret_cast<const float4*>(q)) : *reinterpret_cast<const float4*>(q);
    };
    const int64_t hrow0 = int64_t(mb) * p.n_head + mhq0;
    for (int t0 = 0; t0 < NG; t0 += GB) {
      float M[GT], L[GT];
#pragma unroll
      for (int g = 0; g < GT; ++g) {
        M[g] = -INFINITY;
        L[g] = 0.f;
      }
      float4 a[GB];
#pragma unroll
      for (int t = 0; t < GB; ++t) a[t] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int i0 = 0; i0 < npieces; i0 += MB) {
        float mj[MB][GT], lj[MB][GT];
        float4 x[MB][GB];
#pragma unroll
        for (int j = 0; j < MB; ++j) {
          const int i = i0 + j < npieces ? i0 + j : npieces - 1;
          const float* mlp;
          const float* ap;
          piece_ptr(src, i, mlp, ap);
#pragma unroll
          for (int g = 0; g < GT; ++g) {
            mj[j][g] = ld1(mlp + g);
            lj[j][g] = ld1(mlp + GT + g);
          }
#pragma unroll
          for (int t = 0; t < GB; ++t) {
            const int jg = (t0 + t) * 32 + lane;
            x[j][t] = ld4(ap + 4 * (jg < GROUPS ? jg : 0));
          }
        }
        float Mn[GT], rs[GT];
#pragma unroll
        for (int g = 0; g < GT; ++g) {
          Mn[g] = M[g];
#pragma unroll
          for (int j = 0; j < MB; ++j)
            if (i0 + j < npieces) Mn[g] = fmaxf(Mn[g], mj[j][g]);
          rs[g] = M[g] == Mn[g] ? 1.f : exp2f(M[g] - Mn[g]);
          L[g] *= rs[g];
        }
#pragma unroll
        for (int t = 0; t < GB; ++t) {
          const float r = pick(rs, head_of(t0 + t));
          a[t].x *= r;
          a[t].y *= r;
          a[t].z *= r;
          a[t].w *= r;
        }
#pragma unroll
        for (int j = 0; j < MB; ++j) {
          if (i0 + j >= npieces) continue;
          float f[GT];
#pragma unroll
          for (int g = 0; g < GT; ++g) {
            f[g] = mj[j][g] == -INFINITY ? 0.f : exp2f(mj[j][g] - Mn[g]);
            L[g] = fmaf(f[g], lj[j][g], L[g]);
          }
#pragma unroll
          for (int t = 0; t < GB; ++t) {
            const float ft = pick(f, head_of(t0 + t));
            a[t].x = fmaf(ft, x[j][t].x, a[t].x);
            a[t].y = fmaf(ft, x[j][t].y, a[t].y);
            a[t].z = fmaf(ft, x[j][t].z, a[t].z);
            a[t].w = fmaf(ft, x[j][t].w, a[t].w);
          }
        }
#pragma unroll
        for (int g = 0; g < GT; ++g) M[g] = Mn[g];
      }
#pragma unroll
      for (int t = 0; t < GB; ++t) {
        const int jg = (t0 + t) * 32 + lane;
        if (jg >= GROUPS) continue;
        const int g = head_of(t0 + t);
        const int col = (jg % GPH) * 4;
        if (dst_ml != nullptr) {  // a CTA group's piece, same layout as the pieces
          *reinterpret_cast<float4*>(dst_acc + g * D + col) = a[t];
          if (col == 0) {
            dst_ml[g] = pick(M, g);
            dst_ml[GT + g] = pick(L, g);
          }
        } else if (p.mode == 0) {
          const float inv = 1.f / fmaxf(pick(L, g), 1.f);
          T* o = reinterpret_cast<T*>(p.out) + int64_t(mb) * p.o_sb + int64_t(mhq0 + g) * p.o_sh + col;
          o[0] = E::from_float(a[t].x * inv);
          o[1] = E::from_float(a[t].y * inv);
          o[2] = E::from_float(a[t].z * inv);
          o[3] = E::from_float(a[t].w * inv);
        } else {
          *reinterpret_cast<float4*>(p.part_acc + (hrow0 + g) * D + col) = a[t];
          if (col == 0) {  // the lane that owns the head's first column
            p.part_m[hrow0 + g] = pick(M, g);
            p.part_l[hrow0 + g] = pick(L, g);
          }
        }
      }
    }
  };

  // Merge of split item (mb, mitem) by the piece that arrived last (ticket == pieces - 1), from
  // the pieces' workspace slots in piece order.
  // `acquired`: the ticket came from an acquire-release arrival (take_ticket) of this warp's
  // lane 0, so the other pieces' partials are visible to the warp after a __syncwarp; an early
  // arrival is release-only, and its merge fences instead.
  auto acquire_pieces = [&](bool acquired) {
    if (acquired) {
      __syncwarp();
    } else {
      __threadfence();
    }
  };
  auto merge_if_last = [&](int mb, int mitem, int ticket, bool acquired) {
    if (colmode) {
      // Column mode: the pieces are the CTAs whose column ranges overlap the item's row (slot
      // pair of that CTA's warp mitem): the ranges holding the row's real tiles, virtual
      // columns [vpre(mb) + row_cost, vpre(mb + 1)); a range of only the extra columns is not a
      // piece. A CTA's first segment sits in slot 0 of its pair, a later one in slot 1.
      const int mntile = pre[mb + 1] - pre[mb];
      const int64_t us = vpre(mb) + rc;
      const int c_first = worker_of(us, vcols, col_parts);
      const int c_last = worker_of(us + mntile - 1, vcols, col_parts);
      if (ticket != c_last - c_first) return;
      acquire_pieces(acquired);  // the other pieces' partials
      const bool first_starts_here = range_start(c_first) == pre[mb];
      fold_pieces(mb, mitem, c_last - c_first + 1, FoldSrc{0, c_first, first_starts_here ? 1 : 0, mitem}, nullptr,
                  nullptr);
      return;
    }
    const ItemSpan sp = item_span(mb, mitem);
    const int nreps = global_reps(sp);
    if (ticket != nreps + (sp.mid ? 1 : 0) - 1) return;
    acquire_pieces(acquired);  // the other pieces' partials
    // Piece i < nreps: the range-ending piece(s) of the i-th CTA group (grouped) or worker,
    // in slot 1 of its first worker; then the mid piece in slot 0 of w_b.
    fold_pieces(mb, mitem, nreps + (sp.mid ? 1 : 0), FoldSrc{1, sp.w_a, nreps, sp.w_b}, nullptr, nullptr);
  };

  // ---- pipelined tile loop: scores of tile k+1 overlap softmax + P.V of tile k ---------
  int s = 0;              // stage of tile k (= k % S)
  uint32_t parity = 0u;   // mbarrier phase parity of tile k (= (k / S) & 1)
  float sc_cur[RR], sc_nxt[RR];
  if (!warp_wait_phase(smem_addr(my_bars), 0u, p.wait_ns)) {
    fail_and_drain(0);
    return epoch;
  }
  patch(cur, 0);
  start_segment(cur);
  seg_first_tile = cur.tile;
  tile_scores(0, cur.len - (cur.tile << C::LOG_TILE), sc_cur);

  for (int64_t k = 0; k < nunits; ++k) {
    const bool has_next = k + 1 < nunits;
    Cursor nxt = cur;
    advance(nxt);
    const int s_n = s + 1 == S ? 0 : s + 1;
    const uint32_t parity_n = s + 1 == S ? parity ^ 1u : parity;
    if (!CTA && has_next) {
      if (!warp_wait_phase(smem_addr(my_bars + s_n), parity_n, p.wait_ns)) {
        fail_and_drain(k + 1);
        return epoch;
      }
      patch(nxt, s_n);
    }
    const int tok0 = cur.tile << C::LOG_TILE;
    const int valid_rows = cur.len - tok0;  // rows [0, valid_rows) of tile k are live
    const bool full_tile = valid_rows >= C::TILE;
    const int hq0 = cur.h * p.group + cur.gc * GT;  // first q head of this item

    tile_max_update(sc_cur);
    // Per-warp stages: phase A of tile k+1 (when it exists; its stage is not being written
    // otherwise) and phase B of tile k are independent chains, run side by side. Shared
    // stages: a warp holds one stage at a time, so that more of them are in flight; the
    // CTA's other warps cover the latency instead.
    if (!CTA) tile_scores(s_n, nxt.len - (nxt.tile << C::LOG_TILE), sc_nxt);
    if (__builtin_expect(full_tile, 1)) {
      tile_pv(s, sc_cur, valid_rows, true);
    } else {
      tile_pv(s, sc_cur, valid_rows, false);
    }
    __syncwarp();

    if (CTA) {
      // Hand the stage just consumed back to the producer, then take the next one.
      if (lane == 0) mbar_arrive(smem_addr(empty_bars + s));
      if (has_next) {
        if (!warp_wait_phase(smem_addr(my_bars + s_n), parity_n, p.wait_ns)) {
          fail_and_drain(k + 1);
          return epoch;
        }
        patch(nxt, s_n);
        tile_scores(s_n, nxt.len - (nxt.tile << C::LOG_TILE), sc_nxt);
      }
    } else if (issued < nunits) {
      // Refill the stage just consumed with the tile `stages` ahead.
      issue(pc, s);
      advance(pc);
      ++issued;
      if (pc.tile == 0 && issued < nunits) prefetch_q(pc);
    }

    // ---- segment end ---------------------------------------------------------------------
    const bool seg_end = (k == nunits - 1) || (cur.tile == cur.ntile - 1);
    if (__builtin_expect(seg_end, 0)) {
      const bool whole = seg_first_tile == 0 && cur.tile == cur.ntile - 1;
      // Split item: (m, l, acc) go to this worker's slot and the last arrival merges. Column
      // mode: a range's first segment in slot 0, a later one in slot 1. Unit mode: a segment
      // that ends inside the range in slot 0, the one that ends the range in slot 1 -- or, with
      // grouped numbering when other warps of this CTA hold pieces of the item too, in this
      // warp's own stages (no copy is in flight any more), folded there by the group's last.
      const bool last_seg = k == nunits - 1;
      const int64_t slot = int64_t(wslot) * 2 + (colmode ? (first_segment ? 0 : 1) : (last_seg ? 1 : 0));
      bool local_piece = false;
      if (!colmode && grouped && last_seg && !whole) {
        const ItemSpan sp = item_span(cur.b, cur.item);
        const int cta0 = int(blockIdx.x) * nwarps;
        local_piece = min(sp.w_t, cta0 + nwarps - 1) > max(sp.w_a, cta0);
      }
      float* const piece_ml = local_piece ? smem_piece(warp) + GT * D : p.ws_ml + slot * (2 * GT);
      float* const piece_acc = local_piece ? smem_piece(warp) : p.ws_acc + slot * (GT * D);
      if constexpr (MMA) {
        float lt[2];
        mw.total_l(lt);
        if (whole) {
          if (p.mode == 0) {
            mw.store_out(reinterpret_cast<T*>(p.out) + int64_t(cur.b) * p.o_sb + int64_t(hq0) * p.o_sh, p.o_sh, lt);
          } else {
            const int64_t hrow = int64_t(cur.b) * p.n_head + hq0;
            mw.store_ml(p.part_m + hrow, p.part_l + hrow, lt);
            mw.store_acc(p.part_acc + hrow * D);
          }
        } else {
          mw.store_ml(piece_ml, piece_ml + GT, lt);
          mw.store_acc(piece_acc);
        }
      } else {
        float l_tot[GT];
#pragma unroll
        for (int g = 0; g < GT; ++g) {
          float x = l_run[g];
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(FULL_MASK, x, o);
          l_tot[g] = x;
        }
#pragma unroll
        for (int o = C::LPR; o < 32; o <<= 1) {
#pragma unroll
          for (int g = 0; g < GT; ++g) {
#pragma unroll
            for (int e = 0; e < C::PPL; ++e) {
              acc[g][e].x += __shfl_xor_sync(FULL_MASK, acc[g][e].x, o);
              acc[g][e].y += __shfl_xor_sync(FULL_MASK, acc[g][e].y, o);
            }
          }
        }
        if (whole) {
          if (p.mode == 0) {
            if (rg == 0) {
              T* orow = reinterpret_cast<T*>(p.out) + int64_t(cur.b) * p.o_sb;
#pragma unroll
              for (int g = 0; g < GT; ++g) {
                const float inv = 1.f / fmaxf(l_tot[g], 1.f);
#pragma unroll
                for (int c = 0; c < C::CPL; ++c) {
                  float o[C::EPC];
#pragma unroll
                  for (int e = 0; e < C::EPC; ++e) o[e] = acc_at(g, c * C::EPC + e) * inv;
                  *reinterpret_cast<uint4*>(orow + int64_t(hq0 + g) * p.o_sh + (c * C::LPR + pl) * C::EPC) =
                      E::pack(o);
                }
              }
            }
          } else {
            const int64_t hrow = int64_t(cur.b) * p.n_head + hq0;
            if (lane == 0) {
#pragma unroll
              for (int g = 0; g < GT; ++g) {
                p.part_m[hrow + g] = m_run[g];
                p.part_l[hrow + g] = l_tot[g];
              }
            }
            if (rg == 0) {
#pragma unroll
              for (int g = 0; g < GT; ++g) {
#pragma unroll
                for (int c = 0; c < C::CPL; ++c) {
                  float* dst = p.part_acc + (hrow + g) * D + (c * C::LPR + pl) * C::EPC;
#pragma unroll
                  for (int e = 0; e < C::EPC; e += 4)
                    *reinterpret_cast<float4*>(dst + e) =
                        make_float4(acc_at(g, c * C::EPC + e), acc_at(g, c * C::EPC + e + 1),
                                    acc_at(g, c * C::EPC + e + 2), acc_at(g, c * C::EPC + e + 3));
                }
              }
            }
          }
        } else {
          // Split item: park (m, l, acc) in this worker's slot, then the last arrival merges.
          float* ml = piece_ml;
          float* wa = piece_acc;
          if (lane == 0) {
#pragma unroll
            for (int g = 0; g < GT; ++g) {
              ml[g] = m_run[g];
              ml[GT + g] = l_tot[g];
            }
          }
          if (rg == 0) {
#pragma unroll
            for (int g = 0; g < GT; ++g) {
#pragma unroll
              for (int c = 0; c < C::CPL; ++c) {
                float* dst = wa + g * D + (c * C::LPR + pl) * C::EPC;
#pragma unroll
                for (int e = 0; e < C::EPC; e += 4)
                  *reinterpret_cast<float4*>(dst + e) =
                      make_float4(acc_at(g, c * C::EPC + e), acc_at(g, c * C::EPC + e + 1),
                                  acc_at(g, c * C::EPC + e + 2), acc_at(g, c * C::EPC + e + 3));
              }
            }
          }
        }
      }
      if (!whole) {
        // Arrive on the item's counter. A segment that ends inside the range arrives now, with
        // a release-ordered add whose answer is read only after the loop (the warp keeps
        // streaming); the other pieces of its item end later, so one of them usually merges.
        // The range's last segment arrives after the loop. (Only a range's first and last
        // segments can be split, so two slots suffice.)
        if (k != nunits - 1) {
          __syncwarp();  // every lane's partial stores precede lane 0's release
          if (lane == 0)
            early_old = atom_add_release_gpu(p.counters + int64_t(cur.b) * items_per_row + cur.item, 1ull);
          early = true;
        }
        if (n_pend == 0) {
          pend_b0 = cur.b;
          pend_item0 = cur.item;
        } else {
          pend_b1 = cur.b;
          pend_item1 = cur.item;
        }
        ++n_pend;
      }
      first_segment = false;
    }
    if (has_next && __builtin_expect(nxt.tile == 0, 0)) {
      // Tile k+1 opens a new item: its scores above used the old q. Reload and redo.
      start_segment(nxt);
      seg_first_tile = 0;
      tile_scores(s_n, nxt.len, sc_nxt);
    }
#pragma unroll
    for (int j = 0; j < RR; ++j) sc_cur[j] = sc_nxt[j];
    cur = nxt;
    s = s_n;
    parity = parity_n;
  }

  // ---- arrivals of this range's split segments; the last piece of an item merges it ----
  if (n_pend > 0 && colmode) {
    // Every lane's partial stores precede lane 0's arrivals, which release them.
    __syncwarp();
    int t0 = 0, t1 = 0, early_ok = 0;
    if (lane == 0) {
      // An early add that beat the counter's re-tag was overwritten by it: arrive again.
      const uint32_t tag = counter_tag(epoch, p.tag_salt);
      early_ok = early && uint32_t(early_old >> 32) == tag;
      t0 = early_ok ? int(uint32_t(early_old))
                    : take_ticket(p.counters + int64_t(pend_b0) * items_per_row + pend_item0, tag, p.err, p.wait_ns);
      if (n_pend > 1) t1 = take_ticket(p.counters + int64_t(pend_b1) * items_per_row + pend_item1, tag, p.err, p.wait_ns);
    }
    early_ok = __shfl_sync(FULL_MASK, early_ok, 0);
    merge_if_last(pend_b0, pend_item0, __shfl_sync(FULL_MASK, t0, 0), !early_ok);
    if (n_pend > 1) merge_if_last(pend_b1, pend_item1, __shfl_sync(FULL_MASK, t1, 0), true);
  } else if (n_pend > 0) {
    // Unit mode: the range's first segment when it ended inside the range (the mid piece,
    // arrived early) and/or the segment that ends the range (the tail piece).
    const uint32_t tag = counter_tag(epoch, p.tag_salt);
    const bool has_mid = early;
    const bool has_tail = n_pend > 1 || !early;
    const int tb = n_pend > 1 ? pend_b1 : pend_b0;
    const int ti = n_pend > 1 ? pend_item1 : pend_item0;
    int t_mid = -1, t_tail = -1, mid_acq = 0;
    if (has_mid) {
      const bool stale = uint32_t(early_old >> 32) != tag;  // lane 0's view; others unused
      if (lane == 0)
        t_mid = !stale ? int(uint32_t(early_old))
                       : take_ticket(p.counters + int64_t(pend_b0) * items_per_row + pend_item0, tag, p.err,
                                     p.wait_ns);
      mid_acq = stale;  // a re-arrival through take_ticket acquires
    }
    if (has_tail) {
      const ItemSpan sp = item_span(tb, ti);
      const int cta0 = int(blockIdx.x) * nwarps;
      const int m0 = max(sp.w_a, cta0) - cta0;
      const int m1 = min(sp.w_t, cta0 + nwarps - 1) - cta0;
      bool arrive = true;  // this warp arrives on the item's counter with a piece in slot 1
      if (grouped && m1 > m0) {
        // The pieces of warps m0..m1 of this CTA sit in their stages: the last of them to
        // arrive folds them, in warp order, into the CTA group's piece -- or into the output
        // when the group holds the whole item.
        __threadfence_block();
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(grp_cnt + m0, 1);
        old = __shfl_sync(FULL_MASK, old, 0);
        arrive = old == m1 - m0;
        if (arrive) {
          __threadfence_block();
          const bool whole_item = global_reps(sp) == 1 && !sp.mid;
          const int64_t rslot = int64_t(cta0 + m0) * 2 + 1;
          fold_pieces(tb, ti, m1 - m0 + 1, FoldSrc{2, m0, 0, 0}, whole_item ? nullptr : p.ws_ml + rslot * (2 * GT),
                      whole_item ? nullptr : p.ws_acc + rslot * (GT * D));
          arrive = !whole_item;
        }
      }
      if (arrive) {
        __syncwarp();  // every lane's partial stores precede lane 0's releasing arrival
        if (lane == 0) t_tail = take_ticket(p.counters + int64_t(tb) * items_per_row + ti, tag, p.err, p.wait_ns);
      }
    }
    t_mid = __shfl_sync(FULL_MASK, t_mid, 0);
    t_tail = __shfl_sync(FULL_MASK, t_tail, 0);
    mid_acq = __shfl_sync(FULL_MASK, mid_acq, 0);
    if (t_mid >= 0) merge_if_last(pend_b0, pend_item0, t_mid, mid_acq != 0);
    if (t_tail >= 0) merge_if_last(tb, ti, t_tail, true);
  }
  return epoch;
}

template <typename T, int D, int GT, bool CTA, bool MMA>
__global__ void __launch_bounds__(CTA ? 288 : 256, 1)
    pd_decode_kernel(const __grid_constant__ DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const uint32_t epoch = decode_body<T, D, GT, CTA, MMA>(p, kmap, vmap, smem);
  __syncwarp();
  if ((threadIdx.x & 31) == 0)
    leave_launch(p.exit_counter, p.epoch_word, epoch, p.tag_salt, gridDim.x * (blockDim.x >> 5), p.err);
}

template <typename T, int D, int GT, bool CTA = false, bool MMA = false>
cudaError_t launch_decode(const DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                          dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl) {
  auto fn = pd_decode_kernel<T, D, GT, CTA, MMA>;
  static int attr_smem[64] = {0};  // per-device dynamic-smem opt-in already granted
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 64 && attr_smem[dev] < int(smem)) {
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    attr_smem[dev] = int(smem);
  }
  if (!pdl) {
    fn<<<grid, block, smem, stream>>>(p, kmap, vmap);
    return cudaGetLastError();
  }
  // Programmatic dependent launch: the kernel may start while the previous kernel of the
  // stream finishes; it runs its prologue and first K/V copies, then waits for that kernel
  // (griddep_wait) before it reads q or the appended rows or writes any output.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, p, kmap, vmap);
}

}  // namespace pd
