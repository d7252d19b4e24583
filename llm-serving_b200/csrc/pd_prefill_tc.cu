// pd_prefill_tc.cu -- block-table-aware chunked-prefill attention on the 5th-generation tensor
// cores (tcgen05 / TMEM) for sm_100a: bf16 / fp16 pools, head_dim 64, 128 or 256, 1, 2, 4 or 8
// q heads per kv head, block_size >= 8.
//
// What it computes is pd_prefill's contract (pd_prefill.cu has the mma.sync kernel of the same
// function): row b's chunk of Sq query tokens, packed in q[cu_q[b] .. cu_q[b+1]), attends
// causally -- bottom-right aligned, query token i at position Lk - Sq + i -- to the row's Lk =
// seqlen_k[b] keys in the paged pool, softmax(q k^T * scale) in fp32 and P.V with fp32
// accumulation (P carried as a hi + lo pair of 16-bit operands, about 2^-17 relative).
//
// How (one CTA = 128 query rows of one row's chunk and one kv head; a query row is a
// (token, q head) pair of the kv head's group, token-major, so the group's heads share every
// K/V tile):
//  * warp 8 streams K and V tiles of KT keys (128 up to head_dim 128, 64 at 256) by TMA from the
//    pool's 128-byte-swizzled map into two rings of shared-memory stages. With the engine's pool
//    layout one copy carries a block part of every 64-element piece and lands as 8-token
//    groups of all pieces (4 KB per 16 tokens at head_dim 128: a copy costs the TMA unit ~75
//    cycles whatever its size up to a few KB, so 2 KB copies capped a CTA at ~28 bytes per
//    cycle); other pool strides take one copy per (block part, piece). Either way every
//    piece's 8-row groups are evenly spaced -- the K-major (K) and MN-major (V) operand layouts
//    of the MMA. A K stage is refilled as soon as its S MMA has read it, a V stage once its
//    P.V has; the block table is read 32 entries at a time;
//  * warp 9, lane 0 issues the MMAs: S_j = Q K_j^T (M 128, N KT, K head_dim; both operands in
//    shared memory) into TMEM buffer j % 3, and O += P_hi V_j + P_lo V_j (M 128, N head_dim,
//    K KT) into the TMEM O accumulator with P read from TMEM -- the softmax writes P over the
//    S it came from -- and V from shared memory. S_{j+1} is issued before P.V_j, so the tensor
//    cores work while the softmax runs; a buffer takes S_{j+3} once P.V_j has read its P.
//    Completion is signalled with tcgen05.commit on mbarriers;
//  * warps 0-7, two threads per query row (TMEM lane = row; warps w and w + 4 take the two
//    halves of each key tile): they load the Q tile, then per key tile read their half row of
//    S from TMEM, mask it (causal and row end), agree on the running max with the partner,
//    and write P = 2^(s - m) as 16-bit hi and lo halves into the same TMEM columns, summing
//    the normaliser. The running max is rescaled lazily: only when a row's tile max exceeds it
//    by more than 2^8 is O rescaled in TMEM (P then stays below 2^8, which the hi + lo operands
//    carry exactly as well as smaller values); the final out = O / max(l, 1) is unchanged.
//  * Set-up: warp 9 initialises the barriers and allocates TMEM at entry, before any thread
//    waits on memory; the Q rows and the block table are loaded only after the CTA barrier
//    that follows (a barrier waits for its threads' loads in flight).
//  * Key tiles past the CTA's last query position are never loaded. V rows past the row end
//    are zeroed in shared memory before use, so stale or NaN pool bytes never reach O.
//  * Every wait is bounded (the launch's wait limit). A role whose wait runs out records
//    DEVERR_WAIT_TIMEOUT and raises the CTA's abort flag; every role then stops, the TMA lane
//    waits for its copies in flight and the MMA lane for its MMAs (fixed 0.1 s limits), and
//    the CTA frees its TMEM and returns. TMEM allocation itself cannot wait: at most one CTA of
//    this kernel fits on an SM (shared memory) and it takes at most 512 columns.
#include "paged_decode.h"
#include "pd_common.cuh"
#include "pd_internal.h"
#include "pd_tcgen05.cuh"

#include <type_traits>

namespace pd {

namespace {

constexpr int TC_ROWS = 128;    // query rows per CTA (the MMA's M)
constexpr int TC_SOFTMAX = 256; // softmax warps 0-7: two threads per query row, half a tile each
constexpr int TC_THREADS = 320; // + TMA warp 8, MMA warp 9
constexpr int TC_TMA_WARP = 8;
constexpr int TC_MMA_WARP = 9;
constexpr float TC_RESCALE = 8.f;  // log2 headroom before the running max is moved

template <int D>
struct TcCfg {
  static_assert(D == 64 || D == 128 || D == 256, "head_dim 64, 128 or 256");
  // Keys per tile (the S MMA's N): 128 up to head_dim 128 -- fewer, larger MMAs, since every
  // tcgen05.mma costs at least ~94 cycles to issue whatever its N -- and 64 at head_dim 256
  // (shared memory).
  static constexpr int KT = D <= 128 ? 128 : 64;
  static constexpr int HK = KT / 2;                     // keys per softmax thread
  static constexpr int PIECES = D / 64;                 // 128-byte pieces of a K/V/Q row
  static constexpr int STAGES = D == 64 ? 4 : (D == 128 ? 3 : 2);  // stages of each K/V ring
  static constexpr int NSB = 3;                         // TMEM S/P buffers
  // S_{j+SLEAD} is issued before P.V_j, and K_{j+KLEAD} copied before V_j. Measured on the
  // bench's prefill cases over (SLEAD, KLEAD) = (1, 0), (1, 1), (2, 0), (2, 1), (2, 2): (1, 0) is
  // fastest up to head_dim 128, where a K copy ahead of V delays the P.V that waits for V;
  // (1, 1) at 256.
  static constexpr int SLEAD = 1;
  static constexpr int KLEAD = D <= 128 ? 0 : 1;
  static_assert(SLEAD < NSB && KLEAD <= STAGES && KLEAD <= 2, "lookahead");
  static constexpr int Q_BYTES = TC_ROWS * D * 2;
  static constexpr int KV_BYTES = KT * D * 2;           // one K (or V) tile
  static constexpr int TMEM_COLS = 512;
  static constexpr int O_COL = NSB * KT;                // S/P buffers at columns 0, KT, 2 KT
  static_assert(O_COL + D <= TMEM_COLS, "TMEM columns");
  // shared memory: [barriers, flags, the pair exchange: 2 KB | Q | STAGES x K | STAGES x V]
  static constexpr int OFF_Q = 2048;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int SMEM = OFF_V + STAGES * KV_BYTES + 1024;  // + run-time 1 KB alignment
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

// Barrier slots (8 bytes each) in the first KB of shared memory.
struct TcBars {
  static constexpr int K_FULL = 0;    // [6] K tile landed (TMA transaction bytes)
  static constexpr int V_FULL = 6;    // [6] V tile landed
  static constexpr int K_EMPTY = 12;  // [6] S = Q K^T of the stage's tile completed (commit)
  static constexpr int V_EMPTY = 18;  // [6] P.V of the stage's tile completed (commit)
  static constexpr int S_FULL = 24;   // [3] S buffer written (commit)
  static constexpr int P_FULL = 27;   // [3] P written over the buffer's S (and O rescaled): one arrival per softmax warp
  static constexpr int O_DONE = 30;   // [3] P.V of the tile that read buffer i's P completed (commit)
  static constexpr int Q_FULL = 33;   // Q tile written: one arrival per softmax warp
  static constexpr int DRAIN = 34;    // every MMA of the CTA completed (commit at exit)
  static constexpr int TMEM_SLOT = 344;  // byte offset: TMEM base address written by tcgen05.alloc
  static constexpr int ABORT = 352;      // byte offset: a role's wait ran out
  static constexpr int MAXES = 1024;     // byte offset: bf16 [2 parities][2 halves][128 rows]
};
static_assert((TcBars::DRAIN + 1) * 8 <= TcBars::TMEM_SLOT, "barrier slots");

// Single-thread bounded mbarrier wait (the TMA and MMA lanes run alone in their warps).
__device__ __forceinline__ bool thread_wait_phase(uint32_t bar, uint32_t parity, unsigned long long limit_ns) {
  if (limit_ns < TEST_LIMIT_NS) return false;
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (unsigned it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0 && global_timer_ns() - t0 > limit_ns) return false;
  }
}

// Named barrier `id` over `threads` threads (whole warps) with an OR of `pred` over them: every
// participant gets the same answer, so a failure seen by one warp stops all of them together.
__device__ __forceinline__ bool bar_any(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// 2^x by the hardware approximation (ex2.approx, subnormal results flushed to zero). Here x <= 8
// (the running max's headroom), and a probability below 2^-126 changes no fp32 sum it joins.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Offset of 16-byte unit u of row r in a 128-byte-swizzled piece (rows of 128 bytes).
__device__ __forceinline__ uint32_t sw128(int r, int u) { return uint32_t(r * 128 + ((u ^ (r & 7)) << 4)); }

template <typename T, int D, int G>
__global__ void __launch_bounds__(TC_THREADS, 1)
    pd_prefill_tc_kernel(const __grid_constant__ PrefillParams p, const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap) {
  using C = TcCfg<D>;
  using E = Elem<T>;
  constexpr int TQ = TC_ROWS / G;  // query tokens per CTA
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t raw = smem_addr(smem_raw);
  unsigned char* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const uint32_t sbase = smem_addr(smem);
  auto bar = [&](int slot) -> uint32_t { return sbase + uint32_t(slot) * 8u; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + TcBars::ABORT);
  const unsigned long long wait_ns = p.wait_ns;

  // Set-up first, before anything waits on memory, by the MMA warp: it has no loads in flight,
  // so the fence after the barrier initialisation waits for none (the same fence in a thread
  // that has just issued its Q loads waits for them), and TMEM allocation starts at entry. Every
  // CTA allocates; one without work frees the columns at the common exit.
  if (warp == TC_MMA_WARP) {
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      for (int s = 0; s < C::STAGES; ++s) {
        mbar_init(bar(TcBars::K_FULL + s), 1);
        mbar_init(bar(TcBars::V_FULL + s), 1);
        mbar_init(bar(TcBars::K_EMPTY + s), 1);
        mbar_init(bar(TcBars::V_EMPTY + s), 1);
      }
      for (int i = 0; i < C::NSB; ++i) {
        mbar_init(bar(TcBars::S_FULL + i), 1);
        mbar_init(bar(TcBars::P_FULL + i), TC_SOFTMAX / 32);
        mbar_init(bar(TcBars::O_DONE + i), 1);
      }
      mbar_init(bar(TcBars::Q_FULL), TC_SOFTMAX / 32);
      mbar_init(bar(TcBars::DRAIN), 1);
      *abort_flag = 0;
      fence_barrier_init();
    }
    __syncwarp();
    tc::tmem_alloc(sbase + TcBars::TMEM_SLOT, C::TMEM_COLS);
    tc::tmem_relinquish();
  }

  // 1-D grid, query tile slowest: the CTAs of the last (heaviest, causal) query tiles of every
  // (row, kv head) are launched first, so the lighter ones fill the later waves.
  const int pairs = p.batch * p.n_kv_head;
  const int b = int(blockIdx.x) % p.batch;
  const int h = (int(blockIdx.x) / p.batch) % p.n_kv_head;
  const int qtile = p.q_tiles - 1 - int(blockIdx.x) / pairs;
  const int q_begin = __ldg(p.cu_q + b);
  const int sq = __ldg(p.cu_q + b + 1) - q_begin;
  int lk = __ldg(p.seqlen_k + b);
  lk = lk < 0 ? 0 : (lk > p.capacity ? p.capacity : lk);
  const int tok0 = qtile * TQ;
  const bool has_rows = sq > 0 && tok0 < sq;
  const int ntok = !has_rows ? 0 : (sq - tok0 < TQ ? sq - tok0 : TQ);
  const int ctx = lk - sq;
  int kend = ctx + tok0 + ntok;  // keys this CTA needs: 0 .. kend - 1
  if (kend > lk) kend = lk;
  if (kend < 0 || !has_rows) kend = 0;
  const int ntiles = (kend + C::KT - 1) / C::KT;
  T* og = reinterpret_cast<T*>(p.out);

  if (has_rows && ntiles == 0) {  // no visible key for any row of the CTA: exact zeros
    if (tid < TC_ROWS && tid / G < ntok) {
      T* dst = og + int64_t(q_begin + tok0 + tid / G) * p.o_st + int64_t(h * G + tid % G) * p.o_sh;
      for (int u = 0; u < D / 8; ++u) reinterpret_cast<uint4*>(dst)[u] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  const bool run = ntiles > 0;

  // A barrier waits for the loads its threads have in flight, so the Q rows and the block
  // table are loaded after this one, by the roles that use them.
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + TcBars::TMEM_SLOT);

  const uint32_t q_addr = sbase + C::OFF_Q;
  auto k_addr = [&](int s) -> uint32_t { return sbase + uint32_t(C::OFF_K + s * C::KV_BYTES); };
  auto v_addr = [&](int s) -> uint32_t { return sbase + uint32_t(C::OFF_V + s * C::KV_BYTES); };
  auto fail = [&]() {
    *abort_flag = 1;
    atomicOr(p.err, DEVERR_WAIT_TIMEOUT);
  };
  // Where row r (a key) of 128-byte piece pc of a K/V tile sits: 8-row groups `gstride` bytes
  // apart, pieces `pstride` apart. Grouped copies land [group][piece][8 rows]; one-piece copies
  // land piece-major, [piece][row].
  const uint32_t gstride = p.grouped ? uint32_t(C::PIECES * 1024) : 1024u;
  const uint32_t pstride = p.grouped ? 1024u : uint32_t(C::KT * 128);

  if (!run) {
    // no key tile: nothing to stream (the rows, if any, were zeroed above)
  } else if (warp == TC_TMA_WARP) {
    // ---------------------------------------------------------------- TMA producer
    // The whole warp runs the loop (its waits are warp-collective) and keeps the row's block
    // table in a 32-entry register window, the next window prefetched, so no copy waits on a
    // dependent table load; lane 0 issues the copies. K tile j is issued once the S MMA of tile
    // j - STAGES has read its stage, V tile j once the P.V of tile j - STAGES has.
    const int bs = p.block_size;
    const int bt = p.box_tokens;  // tokens per copy: min(block_size, KT)
    // Both are powers of two (pd_prefill checks): this warp's per-tile work is one dependent
    // chain, so its page and box arithmetic uses shifts, not integer divisions.
    const int bs_log = __ffs(bs) - 1, bt_log = __ffs(bt) - 1;
    const int npages = (lk + bs - 1) >> bs_log;
    const uint32_t box_bytes = uint32_t(bt) * 128u;  // one piece of one box
    const int32_t* trow = p.table + int64_t(b) * p.bt_stride;
    auto entry = [&](int page) -> int {
      return page >= 0 && page < npages && page < p.max_blocks ? __ldg(trow + page) : 0;
    };
    // Window [win_base, win_base + 64) of the table: lane l holds entries win_base + l and + 32 + l,
    // and the 32 after them are already loading (a window advance never waits on a table read;
    // the first of those loads goes out after the first tile's copies, which then do not wait
    // for it).
    // Tiles start on KT-token boundaries, so a tile spans at most KT / block_size <= 16 pages (a
    // block of KT tokens or more holds a whole tile); once the window starts at or below the
    // tile's first page and within 32 of it, every page of the tile is inside.
    int win_base = 0, win_cur = entry(lane), win_nxt = entry(32 + lane), win_far = 0;
    bool far_pending = true;  // win_far is loaded once the first tile's copies are out
    auto advance_window = [&](int first_page) {  // warp-collective
      while (first_page >= win_base + 32) {
        if (far_pending) {
          win_far = entry(win_base + 64 + lane);
          far_pending = false;
        }
        win_base += 32;
        win_cur = win_nxt;
        win_nxt = win_far;
        win_far = entry(win_base + 64 + lane);
      }
    };
    auto block_of = [&](int page) -> int {  // per-lane page inside the window
      const int i = page - win_base;
      const int lo = __shfl_sync(FULL_MASK, win_cur, i & 31);
      const int hi = __shfl_sync(FULL_MASK, win_nxt, i & 31);
      return i < 32 ? lo : hi;
    };
    // The copies of one K (or V) tile, issued in parallel: lane c issues copy c. Grouped: one
    // copy per box of bt tokens and every piece (boxes <= KT / 8 <= 16), at group coordinate
    // block * bs / 8 + (token in block) / 8. One-piece: one copy per (box, piece) (boxes *
    // PIECES <= 32: 16 x 2 pieces up to head_dim 128, 8 x 4 at 256). `blk` is the block of this
    // lane's box.
    const int my_box = p.grouped ? lane : lane / C::PIECES;
    const int my_piece = p.grouped ? 0 : lane - my_box * C::PIECES;
    auto issue_tile = [&](int t, bool is_k, int blk) {
      const int t0 = t * C::KT;
      const int covered = kend - t0 < C::KT ? kend - t0 : C::KT;
      const int boxes = (covered + bt - 1) >> bt_log;
      const int s = t % C::STAGES;
      const uint32_t full = bar((is_k ? TcBars::K_FULL : TcBars::V_FULL) + s);
      const uint32_t dst0 = is_k ? k_addr(s) : v_addr(s);
      const CUtensorMap* map = is_k ? &kmap : &vmap;
      // Lane 0's expect-tx need not precede the other lanes' copies: until that single arrival
      // the phase cannot complete, whatever the transaction count (which may go negative)
      // reads. No warp barrier here, since one would wait for the table loads in flight.
      if (lane == 0) mbar_arrive_expect_tx(full, uint32_t(boxes) * box_bytes * C::PIECES);
      const int tok = t0 + (my_box << bt_log);
      const int in_block = tok & (bs - 1);
      if (my_box < boxes) {
        if (p.grouped)
          tma_load_5d(dst0 + uint32_t((my_box << bt_log) * 128 * C::PIECES), map, full, 0, 0, 0, h,
                      (blk << (bs_log - 3)) + (in_block >> 3));
        else
          tma_load_5d(dst0 + uint32_t(my_piece * C::KT * 128 + (my_box << bt_log) * 128), map, full, 0, in_block, h,
                      my_piece, blk);
      }
    };
    // K runs KLEAD tiles ahead of V (the MMA lane consumes S_{j+SLEAD} before P.V_j).
    // Each K issue looks up its boxes' blocks and keeps them for the tile's V (a 3-entry ring:
    // K_t is issued after V_{t-3}). K_t goes into its stage once S_{t - STAGES} has read it, V_t
    // once P.V_{t - STAGES} has.
    int ring0 = 0, ring1 = 0, ring2 = 0;
    auto issue_k = [&](int t) -> bool {
      const int s = t % C::STAGES;
      if (t >= C::STAGES &&
          !warp_wait_phase(bar(TcBars::K_EMPTY + s), uint32_t((t / C::STAGES - 1) & 1), wait_ns))
        return false;
      advance_window((t * C::KT) >> bs_log);
      const int blk = block_of((t * C::KT + (my_box << bt_log)) >> bs_log);
      const int r3 = t % 3;
      ring0 = r3 == 0 ? blk : ring0;
      ring1 = r3 == 1 ? blk : ring1;
      ring2 = r3 == 2 ? blk : ring2;
      issue_tile(t, true, blk);
      return true;
    };
    auto issue_v = [&](int t) -> bool {
      const int s = t % C::STAGES;
      if (t >= C::STAGES &&
          !warp_wait_phase(bar(TcBars::V_EMPTY + s), uint32_t((t / C::STAGES - 1) & 1), wait_ns))
        return false;
      const int r3 = t % 3;
      issue_tile(t, false, r3 == 0 ? ring0 : (r3 == 1 ? ring1 : ring2));
      return true;
    };
    int k_issued = 0, v_issued = 0;
    bool ok = true;
    for (int t = 0; ok && t < C::KLEAD && t < ntiles; ++t) {
      ok = issue_k(t);
      if (ok) k_issued = t + 1;
    }
    for (int j = 0; ok && j < ntiles; ++j) {
      if (__any_sync(FULL_MASK, *abort_flag != 0)) break;
      if (j + C::KLEAD < ntiles) {
        if (!issue_k(j + C::KLEAD)) {
          ok = false;
          break;
        }
        k_issued = j + C::KLEAD + 1;
      }
      if (!issue_v(j)) {
        ok = false;
        break;
      }
      v_issued = j + 1;
      if (far_pending) {
        win_far = entry(win_base + 64 + lane);
        far_pending = false;
      }
    }
    if (!ok && lane == 0) fail();
    // never leave with a copy in flight: the last STAGES tiles' copies must have landed
    for (int j = k_issued > C::STAGES ? k_issued - C::STAGES : 0; j < k_issued; ++j)
      warp_wait_phase(bar(TcBars::K_FULL + j % C::STAGES), uint32_t((j / C::STAGES) & 1), DRAIN_LIMIT_NS);
    for (int j = v_issued > C::STAGES ? v_issued - C::STAGES : 0; j < v_issued; ++j)
      warp_wait_phase(bar(TcBars::V_FULL + j % C::STAGES), uint32_t((j / C::STAGES) & 1), DRAIN_LIMIT_NS);
  } else if (warp == TC_MMA_WARP) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = tc::instr_desc_f16(BF16, TC_ROWS, C::KT, false, false);
      constexpr uint32_t IDESC_PV = tc::instr_desc_f16(BF16, TC_ROWS, D, false, true);
      const uint32_t o_tmem = tmem + C::O_COL;
      bool ok = thread_wait_phase(bar(TcBars::Q_FULL), 0u, wait_ns);
      // Descriptors are built once; a step's operand is the base descriptor plus the step's byte
      // offset >> 4 in the start-address field (every operand lies below 256 KB of shared
      // memory, so the 14-bit field never carries into the next one).
      const uint64_t q_desc = tc::smem_desc(q_addr, 16u, 1024u);
      // K: K-major B operand (rows = keys), 8-row groups gstride apart, the next 64 elements of
      // head_dim pstride further. V: MN-major B operand, 64-element head_dim blocks pstride
      // apart (leading byte offset), 8-key groups gstride apart (stride byte offset).
      const uint64_t k_desc0 = tc::smem_desc(k_addr(0), 16u, gstride);
      const uint64_t v_desc0 = tc::smem_desc(v_addr(0), pstride, gstride);
      // S_t = Q K_t^T into buffer t % 3 (head_dim / 16 steps of K = 16: 32 bytes of a row), once
      // P.V of tile t - 3 has read the P that buffer held.
      auto issue_s = [&](int t) -> bool {
        const int s = t % C::STAGES;
        const int sb = t % C::NSB;
        if (!thread_wait_phase(bar(TcBars::K_FULL + s), uint32_t((t / C::STAGES) & 1), wait_ns)) return false;
        if (t >= C::NSB && !thread_wait_phase(bar(TcBars::O_DONE + sb), uint32_t((t / C::NSB - 1) & 1), wait_ns))
          return false;
        tc::fence_after_sync();
        const uint64_t k_desc = k_desc0 + uint64_t((s * C::KV_BYTES) >> 4);
        const uint32_t d_tmem = tmem + uint32_t(sb * C::KT);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint64_t a = q_desc + uint64_t(((ks >> 2) * 16384 + (ks & 3) * 32) >> 4);  // Q piece: 128 x 128 B
          const uint64_t bd = k_desc + uint64_t(((ks >> 2) * pstride + (ks & 3) * 32) >> 4);
          tc::mma_f16_ss(d_tmem, a, bd, IDESC_S, ks > 0);
        }
        tc::commit(bar(TcBars::S_FULL + sb));
        tc::commit(bar(TcBars::K_EMPTY + s));
        return true;
      };
      for (int t = 0; ok && t < C::SLEAD && t < ntiles; ++t) ok = issue_s(t);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (*abort_flag) break;
        // S_{j+SLEAD} goes ahead of P.V_j, so the tensor pipe has work while the softmax of tile j
        // runs (S_t reuses the buffer P.V_{t-3} has read).
        if (j + C::SLEAD < ntiles && !issue_s(j + C::SLEAD)) {
          ok = false;
          break;
        }
        const int sb = j % C::NSB;
        const int s = j % C::STAGES;
        if (!thread_wait_phase(bar(TcBars::P_FULL + sb), uint32_t((j / C::NSB) & 1), wait_ns) ||
            !thread_wait_phase(bar(TcBars::V_FULL + s), uint32_t((j / C::STAGES) & 1), wait_ns)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        // O += P_hi V + P_lo V in steps of K = 16 keys (8 TMEM columns of P, two 8-row groups of
        // V). Half h of
        // the buffer (columns h KT/2 ..) holds keys h KT/2 .. of the tile: hi in its first KT/4
        // columns, lo in the next KT/4.
        const uint64_t v_desc = v_desc0 + uint64_t((s * C::KV_BYTES) >> 4);
        const uint32_t p_tmem = tmem + uint32_t(sb * C::KT);
#pragma unroll
        for (int part = 0; part < 2; ++part) {  // P_hi, then P_lo
#pragma unroll
          for (int kk = 0; kk < C::KT / 16; ++kk) {
            const int hh = kk / (C::HK / 16), within = kk % (C::HK / 16);
            tc::mma_f16_ts(o_tmem, p_tmem + uint32_t(hh * C::HK + part * (C::HK / 2) + within * 8),
                           v_desc + uint64_t((kk * 2 * gstride) >> 4), IDESC_PV, j > 0 || part > 0 || kk > 0);
          }
        }
        tc::commit(bar(TcBars::O_DONE + sb));
        tc::commit(bar(TcBars::V_EMPTY + s));
      }
      if (!ok) fail();
      // never leave with an MMA in flight (TMEM is freed and shared memory reused after exit)
      tc::commit(bar(TcBars::DRAIN));
      thread_wait_phase(bar(TcBars::DRAIN), 0u, DRAIN_LIMIT_NS);
    }
  } else {
    // ---------------------------------------------------------------- softmax warps 0-7
    // Warps w and w + 4 share the query rows of TMEM lanes 32 (w % 4) .. + 31: half = w / 4 takes
    // keys HK half .. + HK - 1 of every tile (and columns D/2 half .. of O for rescales and output).
    // Per tile the pair posts its halves' maxima, rounded down to bf16, and waits for the other's
    // (an mbarrier of 64 arrivals, bounded): both threads of a row then take the same running max.
    // Rounding down keeps the running max at or below the row's true maximum, so the largest
    // probability is at least 1 and l >= 1 for every row with a visible key -- the reference's
    // out = acc / max(l, 1) (model/triton_decode.py:639) then divides by l itself.
    const int half = warp >> 2;
    const int r = (warp & 3) * 32 + lane;  // query row = TMEM lane
    const int i = r / G;
    const int hq = h * G + r % G;
    {  // this thread's half of the Q row -> the swizzled K-major Q tile (zeros past the chunk)
      const T* src = reinterpret_cast<const T*>(p.q) + int64_t(q_begin + tok0 + i) * p.q_st + int64_t(hq) * p.q_sh;
      uint4 qv[D / 16];
#pragma unroll
      for (int uu = 0; uu < D / 16; ++uu)
        qv[uu] = i < ntok ? __ldg(reinterpret_cast<const uint4*>(src) + half * (D / 16) + uu)
                          : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int uu = 0; uu < D / 16; ++uu) {
        const int u = half * (D / 16) + uu;
        *reinterpret_cast<uint4*>(smem + C::OFF_Q + (u >> 3) * 16384 + sw128(r, u & 7)) = qv[uu];
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(TcBars::Q_FULL));
    }
    const int row_last = i < ntok ? ctx + tok0 + i : kend - 1;  // padding rows: any finite row
    const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
    __nv_bfloat16* maxes = reinterpret_cast<__nv_bfloat16*>(smem + TcBars::MAXES);
    const int pair_bar = 1 + (warp & 3);  // the warp pair's named barrier (0 is __syncthreads)
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;  // this warp's own waits so far (warp-uniform)
    // P.V of tile t has completed. Tile t's phase on its buffer's barrier is t / 3; the barrier
    // cannot pass it before this warp writes P_{t+3}, and the phase before it (P.V of tile
    // t - 3) completed before S_t was issued, which this warp has seen, so the parity test is
    // unambiguous.
    auto wait_pv = [&](int t) -> bool {
      return warp_wait_phase(bar(TcBars::O_DONE + t % C::NSB), uint32_t((t / C::NSB) & 1), wait_ns);
    };
    // Every exit from the loop is taken by both warps of a pair at the same pair barrier (a wait
    // that runs out later in a tile only skips that tile's work, and the next barrier stops
    // both), so neither warp is ever left waiting for the other.
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j % C::NSB;
      bool bad = __any_sync(FULL_MASK, !ok || *abort_flag != 0);
      if (!bad && !warp_wait_phase(bar(TcBars::S_FULL + sb), uint32_t((j / C::NSB) & 1), wait_ns)) bad = true;
      // this thread's half row of S: columns half KT/2 .. + KT/2 - 1 of the buffer
      const uint32_t s_tmem = lane_base + uint32_t(sb * C::KT + half * C::HK);
      const int c0 = j * C::KT + half * C::HK;  // key of its first column
      float s[C::HK];
      __nv_bfloat16 mine = __float2bfloat16_rd(-INFINITY);
      if (!bad) {
        tc::fence_after_sync();
        uint32_t raw_s[C::HK];
#pragma unroll
        for (int c = 0; c < C::HK; c += 32)
          tc::ld_32x32b_x32(s_tmem + uint32_t(c), *reinterpret_cast<uint32_t(*)[32]>(raw_s + c));
        tc::wait_ld();
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // independent chains
        if (c0 + C::HK - 1 <= row_last) {  // every key of this half is visible to the row
#pragma unroll
          for (int c = 0; c < C::HK; ++c) {
            s[c] = __uint_as_float(raw_s[c]) * p.scale_log2;
            mx[c & 3] = fmaxf(mx[c & 3], s[c]);
          }
        } else {  // the causal edge (or the row end) crosses it
#pragma unroll
          for (int c = 0; c < C::HK; ++c) {
            const float x = __uint_as_float(raw_s[c]) * p.scale_log2;
            s[c] = c0 + c <= row_last ? x : -INFINITY;
            mx[c & 3] = fmaxf(mx[c & 3], s[c]);
          }
        }
        // post this half's maximum, rounded down (never above the true one)
        mine = __float2bfloat16_rd(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])));
        maxes[((j & 1) * 2 + half) * TC_ROWS + r] = mine;
      }
      // Both halves have read their S (so P may overwrite it) and posted their maxima. The
      // partner can post tile j + 1's only after this warp reaches the next barrier, so two
      // parities of slots suffice.
      if (bar_any(pair_bar, 64, bad)) {
        ok = false;
        break;
      }
      const float tmax = fmaxf(__bfloat162float(mine), __bfloat162float(maxes[((j & 1) * 2 + (half ^ 1)) * TC_ROWS + r]));
      const bool move = tmax > m_run + TC_RESCALE || (m_run == -INFINITY && tmax > -INFINITY);
      const float alpha = !move ? 1.f : (m_run == -INFINITY ? 0.f : exp2f(m_run - tmax));
      const bool rescale = j > 0 && __any_sync(FULL_MASK, move);
      if (rescale) {  // O *= alpha per row (this half's columns), once P.V of tile j - 1 landed
        if (!wait_pv(j - 1)) {
          ok = false;
        } else {
          tc::fence_after_sync();
#pragma unroll 1
          for (int oc = half * (D / 2); oc < (half + 1) * (D / 2); oc += 32) {
            uint32_t o[32];
            tc::ld_32x32b_x32(lane_base + uint32_t(C::O_COL + oc), o);
            tc::wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tc::st_32x32b_x32(lane_base + uint32_t(C::O_COL + oc), o);
          }
          tc::wait_st();
        }
      }
      if (!ok) continue;  // the next pair barrier stops both warps
      if (move) m_run = tmax;
      l_run *= alpha;
      const float m_use = m_run == -INFINITY ? 0.f : m_run;
      // P = 2^(s - m) as hi + lo 16-bit pairs, written over this thread's own S columns (read
      // above): hi in the first KT/4 columns, lo in the next KT/4, two keys per column, the lower
      // key in the low half -- the K-major A layout of the P.V MMA.
      float ls[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial sums
#pragma unroll
      for (int uu = 0; uu < C::HK / 8; ++uu) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = ex2_ftz(s[uu * 8 + 2 * e] - m_use);
          const float p1 = ex2_ftz(s[uu * 8 + 2 * e + 1] - m_use);
          ls[e] += p0 + p1;
          hw[e] = E::pack2(p0, p1);
          float hf[2];
          E::unpack2(hw[e], hf);
          lw[e] = E::pack2(p0 - hf[0], p1 - hf[1]);
        }
        tc::st_32x32b_x4(s_tmem + uint32_t(uu * 4), hw[0], hw[1], hw[2], hw[3]);
        tc::st_32x32b_x4(s_tmem + uint32_t(C::HK / 2 + uu * 4), lw[0], lw[1], lw[2], lw[3]);
      }
      l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // The last tile: V rows past the row end must be zero (P is 0 there, but 0 * NaN is not).
      const int valid = kend - j * C::KT;
      if (valid < C::KT) {
        const int s_st = j % C::STAGES;
        if (!warp_wait_phase(bar(TcBars::V_FULL + s_st), uint32_t((j / C::STAGES) & 1), wait_ns)) {
          ok = false;
          continue;
        }
        unsigned char* vs = smem + C::OFF_V + s_st * C::KV_BYTES;
        const int zrows = C::KT - valid;
        for (int idx = half * TC_ROWS + r; idx < zrows * 8 * C::PIECES; idx += TC_SOFTMAX) {
          const int pc = idx / (zrows * 8);
          const int rem = idx - pc * zrows * 8;
          const int row = valid + rem / 8;
          *reinterpret_cast<uint4*>(vs + (row >> 3) * gstride + pc * pstride + (row & 7) * 128 + ((rem & 7) << 4)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(TcBars::P_FULL + sb));
    }
    if (!ok) fail();
    // ---- epilogue: out = O / max(l, 1) for the rows of the chunk; l is the sum of the pair's
    // halves, exchanged through K stage 0 (free once the last P.V has completed: every copy has
    // landed and been read by then). Both warps of the pair reach this barrier exactly once.
    const bool good = ok && wait_pv(ntiles - 1);
    float* lsum = reinterpret_cast<float*>(smem + C::OFF_K);
    if (good) lsum[half * TC_ROWS + r] = l_run;
    if (bar_any(pair_bar, 64, !good)) {
      if (ok && !good) fail();
    } else {
      tc::fence_after_sync();
      const float inv = 1.f / fmaxf(l_run + lsum[(half ^ 1) * TC_ROWS + r], 1.f);
      T* dst = og + int64_t(q_begin + tok0 + i) * p.o_st + int64_t(hq) * p.o_sh;
#pragma unroll 1
      for (int oc = half * (D / 2); oc < (half + 1) * (D / 2); oc += 32) {
        uint32_t o[32];
        tc::ld_32x32b_x32(lane_base + uint32_t(C::O_COL + oc), o);
        tc::wait_ld();
        if (i < ntok) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w;
            w.x = E::pack2(__uint_as_float(o[8 * u + 0]) * inv, __uint_as_float(o[8 * u + 1]) * inv);
            w.y = E::pack2(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv);
            w.z = E::pack2(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv);
            w.w = E::pack2(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + oc + 8 * u) = w;
          }
        }
      }
    }
  }

  // ---- every role is done with TMEM and shared memory: free the TMEM columns
  tc::fence_before_sync();
  __syncthreads();
  if (warp == TC_MMA_WARP) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <typename T, int D, int G>
cudaError_t launch_tc_t(const PrefillParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, int max_seqlen_q,
                        int batch, int n_kv_head, cudaStream_t stream) {
  using C = TcCfg<D>;
  auto fn = pd_prefill_tc_kernel<T, D, G>;
  static int attr_smem[64] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 64 && attr_smem[dev] < C::SMEM) {
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (err != cudaSuccess) return err;
    attr_smem[dev] = C::SMEM;
  }
  constexpr int TQ = TC_ROWS / G;
  PrefillParams q = p;
  q.batch = batch;
  q.n_kv_head = n_kv_head;
  q.q_tiles = (max_seqlen_q + TQ - 1) / TQ;
  const int64_t ctas = int64_t(q.q_tiles) * batch * n_kv_head;
  if (ctas > 0x7fffffff) return cudaErrorInvalidValue;
  fn<<<dim3(unsigned(ctas)), TC_THREADS, C::SMEM, stream>>>(q, kmap, vmap);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_tc_g(const PrefillParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, int group,
                        int max_seqlen_q, int batch, int n_kv_head, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_tc_t<T, D, 1>(p, kmap, vmap, max_seqlen_q, batch, n_kv_head, stream);
    case 2: return launch_tc_t<T, D, 2>(p, kmap, vmap, max_seqlen_q, batch, n_kv_head, stream);
    case 4: return launch_tc_t<T, D, 4>(p, kmap, vmap, max_seqlen_q, batch, n_kv_head, stream);
    case 8: return launch_tc_t<T, D, 8>(p, kmap, vmap, max_seqlen_q, batch, n_kv_head, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

int prefill_tc_tile_tokens(int head_dim) { return head_dim <= 128 ? TcCfg<128>::KT : TcCfg<256>::KT; }

cudaError_t launch_prefill_tc(const PrefillParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, int dtype,
                              int head_dim, int group, int max_seqlen_q, int batch, int n_kv_head,
                              cudaStream_t stream) {
  if (dtype == PD_BF16) {
    if (head_dim == 64)
      return launch_tc_g<__nv_bfloat16, 64>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
    if (head_dim == 256)
      return launch_tc_g<__nv_bfloat16, 256>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
    return launch_tc_g<__nv_bfloat16, 128>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
  }
  if (head_dim == 64) return launch_tc_g<__half, 64>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
  if (head_dim == 256) return launch_tc_g<__half, 256>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
  return launch_tc_g<__half, 128>(p, kmap, vmap, group, max_seqlen_q, batch, n_kv_head, stream);
}

}  // namespace pd
