// pd_api.cu -- the extern "C" boundary declared in include/paged_decode.h.
//
// Host-side argument checks, TMA descriptor encoding for the paged pools, workspace layout,
// launch-shape selection and the plan handle. All device work is in pd_decode_*.cu,
// pd_append.cu and pd_merge.cu.
#include <atomic>
#include <cstdio>
#include <mutex>
#include <new>
#include <vector>

#include "paged_decode.h"
#include "pd_internal.h"

namespace pd {

__device__ unsigned g_error_word = 0;

namespace {

constexpr int kAbiVersion = 1;
constexpr int kMaxDevices = 64;
constexpr int kMaxSmemPerBlock = 232448;  // 227 KB opt-in limit on sm_100

struct Tuning {
  int warps = 8;
  int stages = 3;
  int ctas_per_sm = 1;
  int min_tiles = 4;
};
Tuning g_tuning;
std::mutex g_mutex;
// Decode kernel choice: 0 = per-warp kernel, tensor-core tile math where it applies (the
// default), 1 = shared-stage (CTA) kernel wherever a row has exactly one item per consumer
// warp, 2 = per-warp kernel with CUDA-core tile math everywhere. cta_stages 0 = sized from
// shared memory.
int g_decode_mode = 0;
int g_cta_stages = 0;
int g_row_cost = 3;  // column split: virtual columns charged per row start
// Prefill kernel choice: 0 = tcgen05 / TMEM kernel (default), 1 = mma.sync kernel.
int g_prefill_mode = 0;
constexpr int kCtaConsumerWarps = 8;

thread_local char g_last_error[256] = "";
// Workspace bytes the last prepare() on this thread found missing (PD_ERR_WORKSPACE).
thread_local size_t g_last_ws_need = 0;

// Kernels launched by this library in this process (pd_launch_count).
std::atomic<unsigned long long> g_launches{0};

// Limit of the kernels' mbarrier and arrival-counter waits, read at every launch
// (pd_set_wait_limit).
std::atomic<unsigned long long> g_wait_limit_ns{WAIT_LIMIT_NS};

// Records a failed CUDA call for pd_last_error_string and returns PD_ERR_CUDA.
int cuda_fail(cudaError_t e, const char* where) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorName(e),
           cudaGetErrorString(e));
  return PD_ERR_CUDA;
}

int g_sm_count[kMaxDevices] = {0};
unsigned* g_err_ptr[kMaxDevices] = {nullptr};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

int elem_size(int dtype) { return dtype == PD_F32 ? 4 : 2; }
bool valid_dtype(int dtype) { return dtype == PD_F32 || dtype == PD_F16 || dtype == PD_BF16; }
bool pow2(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }
int ilog2_host(int64_t x) {
  int r = 0;
  while ((int64_t(1) << (r + 1)) <= x) ++r;
  return r;
}
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int current_device(int* dev) {
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= kMaxDevices) return PD_ERR_CUDA;
  return PD_OK;
}

int sm_count(int dev) {
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      return 0;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

unsigned* error_word(int dev) {
  if (g_err_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<unsigned*>(p);
  }
  return g_err_ptr[dev];
}

int load_encoder() {
  if (g_encode) return PD_OK;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_encode) return PD_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr)
    return PD_ERR_CUDA;
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  return PD_OK;
}

// Decode-kernel geometry that the host needs (mirrors DecodeCfg in pd_decode_kernel.cuh).
struct Geometry {
  int d_index;   // 0..5 for head_dim 8..256
  int gt;        // q heads per worker item
  int gt_index;  // 0..3 for gt 1, 2, 4, 8
  int n_gchunks;
  int tile;        // tokens per stage
  int box_tokens;  // tokens per TMA box
  bool cta;        // shared-stage kernel: one consumer warp per item of a row
  bool mma;        // per-warp kernel with tensor-core tile math (swizzled 5-D pool maps)
  int box_heads;   // kv heads per TMA box: all of them in the shared-stage kernel, else 1
  int stage_bytes; // K + V bytes of one stage (of one warp, or of the CTA when shared)
};

int geometry(int n_head, int n_kv_head, int head_dim, int block_size, int dtype, Geometry* g) {
  if (!valid_dtype(dtype)) return PD_ERR_INVALID;
  if (n_kv_head < 1 || n_head < 1 || n_head % n_kv_head != 0) return PD_ERR_INVALID;
  if (!pow2(head_dim) || !pow2(block_size)) return PD_ERR_INVALID;
  if (head_dim < 8 || head_dim > 256) return PD_ERR_UNSUPPORTED;
  const int group = n_head / n_kv_head;
  int gt = 8;
  while (group % gt != 0) gt >>= 1;
  g->gt = gt;
  g->gt_index = ilog2_host(gt);
  g->n_gchunks = group / gt;
  g->d_index = ilog2_host(head_dim) - 3;
  const int row_bytes = head_dim * elem_size(dtype);
  g->tile = 4096 / row_bytes;
  g->box_tokens = block_size < g->tile ? block_size : g->tile;
  int mode;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    mode = g_decode_mode;
  }
  g->cta = mode == 1 && n_kv_head * g->n_gchunks == kCtaConsumerWarps && gt <= 4 &&
           (dtype == PD_BF16 || dtype == PD_F16) && head_dim >= 64;
  g->mma = !g->cta && mode != 2 && (dtype == PD_BF16 || dtype == PD_F16) && head_dim >= 64 &&
           g->box_tokens >= 8;
  g->box_heads = g->cta ? n_kv_head : 1;
  g->stage_bytes = 2 * 4096 * g->box_heads;
  return PD_OK;
}

DecodeLaunchFn launcher_for(int dtype, const Geometry& g) {
  if (g.cta) return dtype == PD_BF16 ? decode_launcher_cta_bf16(g.d_index, g.gt_index)
                                     : decode_launcher_cta_f16(g.d_index, g.gt_index);
  if (g.mma) return dtype == PD_BF16 ? decode_launcher_mma_bf16(g.d_index, g.gt_index)
                                     : decode_launcher_mma_f16(g.d_index, g.gt_index);
  switch (dtype) {
    case PD_F32: return decode_launcher_f32(g.d_index, g.gt_index);
    case PD_F16: return decode_launcher_f16(g.d_index, g.gt_index);
    case PD_BF16: return decode_launcher_bf16(g.d_index, g.gt_index);
  }
  return nullptr;
}

struct Launch {
  int grid;
  int warps;
  int stages;
  int min_tiles;
  int rows_per_launch;  // batch chunk that fits the shared-memory prefix arrays
  int arrays_off;
  int stage_off;
  size_t smem;
};

// Per-warp kernel: `stages` stages and barriers per warp. Shared-stage kernel: `stages` shared
// stages with a full and an empty barrier each.
size_t smem_for(bool cta, int warps, int stages, int rows, int stage_bytes, int* arrays_off, int* stage_off) {
  const size_t bars = round_up(size_t(cta ? 2 : warps) * stages * 8, 16);
  const size_t arrays = round_up(size_t(1 + 32 + 64 + 32 + 3 * rows + 1) * 4, 16);
  *arrays_off = int(bars);
  *stage_off = int(bars + arrays);
  return bars + arrays + 1024 /* run-time re-alignment slack */ + size_t(cta ? 1 : warps) * stages * stage_bytes;
}

int launch_shape(int dev, int batch, const Geometry& g, Launch* L) {
  Tuning t;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    t = g_tuning;
  }
  const int sms = sm_count(dev);
  if (sms <= 0) return PD_ERR_CUDA;
  int cta_stages;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    cta_stages = g_cta_stages;
  }
  L->warps = g.cta ? kCtaConsumerWarps + 1 : t.warps;  // shared stages: consumers + a producer
  L->stages = g.cta ? (cta_stages > 0 ? cta_stages : std::min(8, std::max(2, 196608 / g.stage_bytes)))
                    : t.stages;
  L->min_tiles = t.min_tiles;
  const int ctas_per_sm = g.cta ? 1 : t.ctas_per_sm;
  L->grid = sms * ctas_per_sm;
  int rows = batch < 1 ? 1 : batch;
  if (rows > 4096) rows = 4096;
  for (;;) {
    L->smem = smem_for(g.cta, L->warps, L->stages, rows, g.stage_bytes, &L->arrays_off, &L->stage_off);
    if (L->smem * size_t(ctas_per_sm) <= size_t(kMaxSmemPerBlock)) break;
    if (rows <= 256) return PD_ERR_INVALID;  // tuning asks for more shared memory than exists
    rows /= 2;
  }
  L->rows_per_launch = rows;
  return PD_OK;
}

// Workspace: [header 256 B: epoch word (u32) at 0, exit counter (u64) at 8 | item arrival
// counters (u64) | partial (m, l) slots | partial accumulator slots | step records]. The header
// is the kernel's own launch bookkeeping; nothing in the workspace needs to start at zero. The
// step records (one per physical warp) cache a plan's work split across the layers of a step.
struct WorkspaceLayout {
  size_t counters_off;
  size_t ml_off, acc_off, step_off, total;
};
constexpr size_t kStepRecordBytes = 320;  // STEP_REC_BYTES in pd_decode_kernel.cuh

WorkspaceLayout workspace_layout(int batch, int n_kv_head, const Geometry& g, int head_dim,
                                 const Launch& L) {
  WorkspaceLayout w;
  const int rows = batch < L.rows_per_launch ? batch : L.rows_per_launch;
  w.counters_off = 256;
  const size_t workers = size_t(L.grid) * L.warps;
  w.ml_off = w.counters_off + round_up(size_t(rows < 1 ? 1 : rows) * n_kv_head * g.n_gchunks * 8, 256);
  w.acc_off = w.ml_off + round_up(workers * 2 * 2 * g.gt * 4, 256);
  w.step_off = w.acc_off + round_up(workers * 2 * size_t(g.gt) * head_dim * 4, 256);
  w.total = w.step_off + round_up(workers * kStepRecordBytes, 256);
  return w;
}

// Pool map of the decode kernels. Plain: 4-D (head_dim, head, token-in-block, block), box
// (head_dim, box_heads, box_tokens, 1). Swizzled (tensor-core kernel, 16-bit head_dim >= 64):
// 5-D (64 elements, token-in-block, head, 128-byte piece, block) with the 128-byte swizzle and
// box (64, box_tokens, 1, head_dim / 64, 1), so a box lands piece-major: shared row
// piece * box_tokens + token, 16-byte units XOR-permuted by the row index.
// Swizzled pool views (the tensor-core kernels'):
//  * SW_ROWS: (64 elements, token-in-block, head, 128-byte piece, block), a box = box_tokens rows
//    of every piece (the decode kernel);
//  * SW_ONE_PIECE: the same view, a box = one piece of box_tokens rows, so a kernel can place
//    every piece of a tile where it wants it;
//  * SW_GROUPED: (64 elements, 8 tokens, 128-byte piece, head, 8-token group of the pool), a box
//    = box_tokens / 8 groups of every piece. It lands as [group][piece][8 rows of 128 bytes], so
//    every piece's 8-row groups are evenly spaced (pieces x 1 KB apart) and a box carries all
//    pieces at once -- 2x-4x larger copies than one-piece boxes. Needs the pool's blocks evenly
//    spaced at block_size tokens (block stride = block_size x token stride) and block_size a
//    multiple of 8.
enum SwizzledView { SW_ROWS = 0, SW_ONE_PIECE = 1, SW_GROUPED = 2 };

int encode_pool(CUtensorMap* map, const void* base, int64_t n_blocks, int block_size, int n_kv_head,
                int head_dim, const int64_t* strides, int dtype, int box_tokens, int box_heads,
                bool swizzle, int view = SW_ROWS) {
  if (load_encoder() != PD_OK) return PD_ERR_CUDA;
  const int es = elem_size(dtype);
  if (!aligned16(base)) return PD_ERR_INVALID;
  for (int i = 0; i < 3; ++i) {
    if (strides[i] <= 0 || (strides[i] * es) % 16 != 0 || strides[i] * es >= (int64_t(1) << 40))
      return PD_ERR_INVALID;
  }
  CUtensorMapDataType t = dtype == PD_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                          : dtype == PD_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                            : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (swizzle && view == SW_GROUPED) {
    if (es != 2 || head_dim % 64 != 0 || box_heads != 1 || block_size % 8 != 0 || box_tokens % 8 != 0 ||
        strides[0] != int64_t(block_size) * strides[1])
      return PD_ERR_INVALID;
    const cuuint64_t dims[5] = {64u, 8u, cuuint64_t(head_dim / 64), cuuint64_t(n_kv_head),
                                cuuint64_t(n_blocks) * cuuint64_t(block_size / 8)};
    // Byte strides of dims 1..4: token, 128-byte piece, head, 8-token group.
    const cuuint64_t gstr[4] = {cuuint64_t(strides[1] * es), 128u, cuuint64_t(strides[2] * es),
                                cuuint64_t(strides[1] * es) * 8u};
    const cuuint32_t box[5] = {64u, 8u, cuuint32_t(head_dim / 64), 1u, cuuint32_t(box_tokens / 8)};
    const cuuint32_t estr[5] = {1u, 1u, 1u, 1u, 1u};
    CUresult r = g_encode(map, t, 5, const_cast<void*>(base), dims, gstr, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? PD_OK : PD_ERR_INVALID;
  }
  if (swizzle) {
    if (es != 2 || head_dim % 64 != 0 || box_heads != 1) return PD_ERR_INVALID;
    const cuuint64_t dims[5] = {64u, cuuint64_t(block_size), cuuint64_t(n_kv_head), cuuint64_t(head_dim / 64),
                                cuuint64_t(n_blocks)};
    // Byte strides of dims 1..4: token-in-block, head, 128-byte piece, block.
    const cuuint64_t gstr[4] = {cuuint64_t(strides[1] * es), cuuint64_t(strides[2] * es), 128u,
                                cuuint64_t(strides[0] * es)};
    const cuuint32_t box[5] = {64u, cuuint32_t(box_tokens), 1u,
                               view == SW_ONE_PIECE ? 1u : cuuint32_t(head_dim / 64), 1u};
    const cuuint32_t estr[5] = {1u, 1u, 1u, 1u, 1u};
    CUresult r = g_encode(map, t, 5, const_cast<void*>(base), dims, gstr, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? PD_OK : PD_ERR_INVALID;
  }
  const cuuint64_t dims[4] = {cuuint64_t(head_dim), cuuint64_t(n_kv_head), cuuint64_t(block_size),
                              cuuint64_t(n_blocks)};
  // Byte strides of dims 1..3: head, token-in-block, block.
  const cuuint64_t gstr[3] = {cuuint64_t(strides[2] * es), cuuint64_t(strides[1] * es),
                              cuuint64_t(strides[0] * es)};
  const cuuint32_t box[4] = {cuuint32_t(head_dim), cuuint32_t(box_heads), cuuint32_t(box_tokens), 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = g_encode(map, t, 4, const_cast<void*>(base), dims, gstr, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PD_OK : PD_ERR_INVALID;
}

// Even 32-bit salt of a workspace layout and half for the counters' tags: two layouts (or the two
// halves of one plan's workspace) that reuse the same bytes get unrelated tags, so a counter
// one of them left behind does not carry a tag the other is using.
uint32_t layout_salt(const WorkspaceLayout& w, int batch, int items_per_row, int half) {
  uint64_t x = uint64_t(w.total) * 0x9E3779B97F4A7C15ull;
  x ^= (uint64_t(uint32_t(batch)) << 32 | uint32_t(items_per_row)) * 0xC2B2AE3D27D4EB4Full;
  x ^= uint64_t(half + 1) * 0x165667B19E3779F9ull;
  x ^= x >> 29;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 32;
  return uint32_t(x) & ~1u;
}

// Everything fixed for one (pool layout, table, seqlen, batch) -- shared by pd_decode,
// pd_decode_partials and the plan.
struct Prepared {
  Geometry g;
  Launch L;
  WorkspaceLayout ws;
  DecodeLaunchFn fn;
  DecodeParams base;  // q/out/partials pointers filled per launch
  // The workspace holds `halves` (1 or 2) copies of the layout, half_bytes apart. With two,
  // consecutive launches alternate between them, so a launch that overlaps the previous one
  // (programmatic dependent launch) never shares its counters, epoch or partials.
  int halves = 1;
  size_t half_bytes = 0;
};

int prepare(Prepared* P, int64_t n_blocks, int32_t block_size, const int32_t* block_table,
            int64_t bt_stride, int32_t max_blocks, const int32_t* seqlen, int32_t batch,
            int32_t n_head, int32_t n_kv_head, int32_t head_dim, int32_t dtype, float scale_log2,
            void* workspace, size_t workspace_bytes) {
  if (batch < 0 || max_blocks < 0 || n_blocks < 1) return PD_ERR_INVALID;
  int st = geometry(n_head, n_kv_head, head_dim, block_size, dtype, &P->g);
  if (st != PD_OK) return st;
  P->fn = launcher_for(dtype, P->g);
  if (P->fn == nullptr) return PD_ERR_UNSUPPORTED;
  int dev = 0;
  if (current_device(&dev) != PD_OK) return PD_ERR_CUDA;
  st = launch_shape(dev, batch, P->g, &P->L);
  if (st != PD_OK) return st;
  P->ws = workspace_layout(batch, n_kv_head, P->g, head_dim, P->L);
  if (batch > 0) {
    if (workspace == nullptr || workspace_bytes < P->ws.total) {
      g_last_ws_need = P->ws.total;
      snprintf(g_last_error, sizeof(g_last_error),
               "workspace of %zu bytes is smaller than the %zu bytes this shape needs", workspace_bytes,
               P->ws.total);
      return PD_ERR_WORKSPACE;
    }
    P->half_bytes = round_up(P->ws.total, 256);
    P->halves = workspace_bytes >= 2 * P->half_bytes ? 2 : 1;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) {
      snprintf(g_last_error, sizeof(g_last_error), "workspace is not 256-byte aligned");
      return PD_ERR_WORKSPACE;
    }
    if (block_table == nullptr && max_blocks > 0) return PD_ERR_INVALID;
    if (seqlen == nullptr) return PD_ERR_INVALID;
  }
  if (max_blocks > 0 && bt_stride < max_blocks) return PD_ERR_INVALID;
  const int64_t capacity = int64_t(max_blocks) * block_size;
  if (capacity > (int64_t(1) << 30)) return PD_ERR_INVALID;
  unsigned* err = error_word(dev);
  if (err == nullptr) return PD_ERR_CUDA;

  DecodeParams& p = P->base;
  p = DecodeParams{};
  p.table = block_table;
  p.bt_stride = bt_stride;
  p.seqlen = seqlen;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  p.epoch_word = reinterpret_cast<unsigned*>(ws);
  p.exit_counter = reinterpret_cast<unsigned long long*>(ws + 8);
  p.tag_salt = layout_salt(P->ws, batch, n_kv_head * P->g.n_gchunks, 0);
  p.step_rec = nullptr;  // plans switch the step cache on (pd_plan_create)
  p.step_table = 0;

  p.counters = reinterpret_cast<unsigned long long*>(ws + P->ws.counters_off);
  p.ws_ml = reinterpret_cast<float*>(ws + P->ws.ml_off);
  p.ws_acc = reinterpret_cast<float*>(ws + P->ws.acc_off);
  p.err = err;
  p.max_blocks = max_blocks;
  p.capacity = int32_t(capacity);
  p.batch = batch;
  p.n_head = n_head;
  p.n_kv_head = n_kv_head;
  p.group = n_head / n_kv_head;
  p.n_gchunks = P->g.n_gchunks;
  p.block_size = block_size;
  p.log2_bs = ilog2_host(block_size);
  p.box_tokens = P->g.box_tokens;
  p.log2_box = ilog2_host(P->g.box_tokens);
  p.stages = P->L.stages;
  p.min_tiles = P->L.min_tiles;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    p.row_cost = g_row_cost;
  }
  p.smem_arrays_off = P->L.arrays_off;
  p.smem_stage_off = P->L.stage_off;
  p.scale_log2 = scale_log2;
  {  // everything besides the lengths that the work split depends on
    uint64_t x = 0x243F6A8885A308D3ull;
    const int64_t shape[] = {batch, n_head, n_kv_head, head_dim, dtype, block_size, max_blocks,
                             P->L.grid, P->L.warps, P->L.stages, P->L.min_tiles, P->L.rows_per_launch,
                             P->g.gt, P->g.mma, P->g.cta, p.row_cost};
    for (int64_t v : shape) {
      x = (x ^ uint64_t(v)) * 0x100000001B3ull;
      x ^= x >> 29;
    }
    p.step_salt = x;
  }
  return PD_OK;
}

// Rotary tables: a positive even width that fits the head, row stride >= width / 2, and
// one dtype for the K source, the pool and the tables.
bool rope_args_ok(const void* rope_cos, const void* rope_sin, int64_t rope_stride, int32_t rotary_dim,
                         int32_t head_dim, int32_t src_dtype, int32_t pool_dtype) {
  return rope_cos != nullptr && rope_sin != nullptr && rotary_dim >= 2 && rotary_dim % 2 == 0 &&
         rotary_dim <= head_dim && rope_stride >= rotary_dim / 2 && src_dtype == pool_dtype;
}

int check_rows(const void* ptr, int64_t sb, int64_t sh, int dtype) {
  const int es = elem_size(dtype);
  if (ptr == nullptr || !aligned16(ptr)) return PD_ERR_INVALID;
  if ((sb * es) % 16 != 0 || (sh * es) % 16 != 0) return PD_ERR_INVALID;
  return PD_OK;
}

// The new token of every row for a fused append + decode launch (pd_plan_run_append).
struct AppendArgs {
  const void* k;
  int64_t k_sb, k_sh;
  const void* v;
  int64_t v_sb, v_sh;
  const int64_t* pos;
  void* pool_k;
  void* pool_v;
  const int64_t* k_strides;  // pool element strides: block, token, head
  const int64_t* v_strides;
  int64_t n_blocks;
  const void* rope_cos;  // rotary tables of the appended K rows, or nullptr
  const void* rope_sin;
  int64_t rope_stride;
  int32_t rope_dim;
};

// Launches the decode kernel over the batch in chunks of rows_per_launch rows.
int run_prepared(const Prepared& P, const CUtensorMap& kmap, const CUtensorMap& vmap, const void* q,
                 int64_t q_sb, int64_t q_sh, void* out, int64_t o_sb, int64_t o_sh, float* pm,
                 float* pl, float* pacc, int mode, int dtype, cudaStream_t stream,
                 const AppendArgs* app = nullptr, bool overlap = false, uint32_t* seq = nullptr) {
  const int batch = P.base.batch;
  const int es = elem_size(dtype);
  for (int b0 = 0; b0 < batch; b0 += P.L.rows_per_launch) {
    const int rows = batch - b0 < P.L.rows_per_launch ? batch - b0 : P.L.rows_per_launch;
    DecodeParams p = P.base;
    if (P.halves == 2 && seq != nullptr && ((*seq)++ & 1u)) {  // the workspace's second half
      const size_t h = P.half_bytes;
      p.epoch_word = reinterpret_cast<unsigned*>(reinterpret_cast<unsigned char*>(p.epoch_word) + h);
      p.exit_counter = reinterpret_cast<unsigned long long*>(reinterpret_cast<unsigned char*>(p.exit_counter) + h);
      p.counters = reinterpret_cast<unsigned long long*>(reinterpret_cast<unsigned char*>(p.counters) + h);
      p.ws_ml = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(p.ws_ml) + h);
      p.ws_acc = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(p.ws_acc) + h);
      p.tag_salt = layout_salt(P.ws, P.base.batch, P.base.n_kv_head * P.base.n_gchunks, 1);
    }
    p.batch = rows;
    p.mode = mode;
    p.wait_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
    p.q = static_cast<const unsigned char*>(q) + int64_t(b0) * q_sb * es;
    p.q_sb = q_sb;
    p.q_sh = q_sh;
    if (mode == 0) {
      p.out = static_cast<unsigned char*>(out) + int64_t(b0) * o_sb * es;
      p.o_sb = o_sb;
      p.o_sh = o_sh;
    } else {
      // m, l are (B, H) and acc is (B, H, D), all contiguous: offset by b0 rows.
      const int64_t head_dim = int64_t(8) << P.g.d_index;
      p.part_m = pm + int64_t(b0) * p.n_head;
      p.part_l = pl + int64_t(b0) * p.n_head;
      p.part_acc = pacc + int64_t(b0) * p.n_head * head_dim;
    }
    if (P.base.table) p.table = P.base.table + int64_t(b0) * P.base.bt_stride;
    p.seqlen = P.base.seqlen + b0;
    if (app != nullptr) {
      p.append = 1;
      p.app_k = static_cast<const unsigned char*>(app->k) + int64_t(b0) * app->k_sb * es;
      p.app_v = static_cast<const unsigned char*>(app->v) + int64_t(b0) * app->v_sb * es;
      p.app_k_sb = app->k_sb;
      p.app_k_sh = app->k_sh;
      p.app_v_sb = app->v_sb;
      p.app_v_sh = app->v_sh;
      p.app_pos = app->pos + b0;
      p.pool_k = app->pool_k;
      p.pool_v = app->pool_v;
      p.pk_sb = app->k_strides[0];
      p.pk_sn = app->k_strides[1];
      p.pk_sh = app->k_strides[2];
      p.pv_sb = app->v_strides[0];
      p.pv_sn = app->v_strides[1];
      p.pv_sh = app->v_strides[2];
      p.n_blocks = app->n_blocks;
      if (app->rope_cos != nullptr) {
        p.rope_cos = static_cast<const unsigned char*>(app->rope_cos) + int64_t(b0) * app->rope_stride * es;
        p.rope_sin = static_cast<const unsigned char*>(app->rope_sin) + int64_t(b0) * app->rope_stride * es;
        p.rope_stride = app->rope_stride;
        p.rope_dim = app->rope_dim;
      }
    }
    const size_t smem = smem_for(P.g.cta, P.L.warps, P.L.stages, rows, P.g.stage_bytes, &p.smem_arrays_off,
                                 &p.smem_stage_off);
    cudaError_t e = P.fn(p, kmap, vmap, dim3(P.L.grid), dim3(P.L.warps * 32), smem, stream, overlap);
    if (e != cudaSuccess) return cuda_fail(e, "decode launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  return PD_OK;
}

int decode_common(const void* q, int64_t q_sb, int64_t q_sh, const void* k_cache, const void* v_cache,
                  int64_t n_blocks, int32_t block_size, const int64_t* k_strides,
                  const int64_t* v_strides, const int32_t* block_table, int64_t bt_stride,
                  int32_t max_blocks, const int32_t* seqlen, void* out, int64_t o_sb, int64_t o_sh,
                  float* pm, float* pl, float* pacc, int mode, int32_t batch, int32_t n_head,
                  int32_t n_kv_head, int32_t head_dim, int32_t dtype, float scale_log2,
                  void* workspace, size_t workspace_bytes, void* stream) {
  if (k_strides == nullptr || v_strides == nullptr) return PD_ERR_INVALID;
  Prepared P;
  int st = prepare(&P, n_blocks, block_size, block_table, bt_stride, max_blocks, seqlen, batch,
                   n_head, n_kv_head, head_dim, dtype, scale_log2, workspace, workspace_bytes);
  if (st != PD_OK) return st;
  if (batch == 0) return PD_OK;
  if (check_rows(q, q_sb, q_sh, dtype) != PD_OK) return PD_ERR_INVALID;
  if (mode == 0 && check_rows(out, o_sb, o_sh, dtype) != PD_OK) return PD_ERR_INVALID;
  if (mode == 1 && (pm == nullptr || pl == nullptr || pacc == nullptr || !aligned16(pacc)))
    return PD_ERR_INVALID;
  CUtensorMap kmap, vmap;
  st = encode_pool(&kmap, k_cache, n_blocks, block_size, n_kv_head, head_dim, k_strides, dtype,
                   P.g.box_tokens, P.g.box_heads, P.g.mma);
  if (st != PD_OK) return st;
  st = encode_pool(&vmap, v_cache, n_blocks, block_size, n_kv_head, head_dim, v_strides, dtype,
                   P.g.box_tokens, P.g.box_heads, P.g.mma);
  if (st != PD_OK) return st;
  return run_prepared(P, kmap, vmap, q, q_sb, q_sh, out, o_sb, o_sh, pm, pl, pacc, mode, dtype,
                      static_cast<cudaStream_t>(stream));
}

}  // namespace
}  // namespace pd

using namespace pd;

struct pd_plan {
  Prepared P;
  int32_t n_layer;
  int32_t dtype;
  int64_t q_sb, q_sh;
  int64_t n_blocks;
  int64_t k_strides[3], v_strides[3];
  std::vector<CUtensorMap> kmaps;
  std::vector<CUtensorMap> vmaps;
  std::vector<void*> k_pools;  // for the fused append's stores
  std::vector<void*> v_pools;
  int32_t overlap = 0;  // launches may overlap the previous kernel (pd_plan_set_overlap)
  mutable uint32_t seq = 0;  // launches made: selects the workspace half of the next one
};

extern "C" {

const char* pd_status_string(int status) {
  switch (status) {
    case PD_OK: return "ok";
    case PD_ERR_INVALID: return "invalid argument";
    case PD_ERR_UNSUPPORTED: return "unsupported shape";
    case PD_ERR_CUDA: return "CUDA error";
    case PD_ERR_WORKSPACE: return "workspace missing or too small";
  }
  return "unknown status";
}

int pd_abi_version(void) { return kAbiVersion; }

uint64_t pd_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* pd_last_error_string(void) { return g_last_error; }

int pd_device_error(unsigned int* bits, int clear) {
  if (bits == nullptr) return PD_ERR_INVALID;
  int dev = 0;
  if (current_device(&dev) != PD_OK) return PD_ERR_CUDA;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "pd_device_error synchronize");
  unsigned v = 0;
  e = cudaMemcpyFromSymbol(&v, g_error_word, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "pd_device_error read");
  *bits = v;
  if (clear && v != 0) {
    unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_error_word, &zero, sizeof(zero)) != cudaSuccess) return PD_ERR_CUDA;
  }
  return PD_OK;
}

size_t pd_decode_workspace_bytes(int32_t batch, int32_t n_head, int32_t n_kv_head, int32_t head_dim,
                                 int32_t dtype) {
  Geometry g;
  if (geometry(n_head, n_kv_head, head_dim, 16, dtype, &g) != PD_OK) return 0;
  int dev = 0;
  if (current_device(&dev) != PD_OK) return 0;
  Launch L;
  if (launch_shape(dev, batch, g, &L) != PD_OK) return 0;
  return workspace_layout(batch, n_kv_head, g, head_dim, L).total;
}

int pd_decode(const void* q, int64_t q_sb, int64_t q_sh, const void* k_cache, const void* v_cache,
              int64_t n_blocks, int32_t block_size, const int64_t* k_strides,
              const int64_t* v_strides, const int32_t* block_table, int64_t bt_stride,
              int32_t max_blocks, const int32_t* seqlen, void* out, int64_t o_sb, int64_t o_sh,
              int32_t batch, int32_t n_head, int32_t n_kv_head, int32_t head_dim, int32_t dtype,
              float scale_log2, void* workspace, size_t workspace_bytes, void* stream) {
  return decode_common(q, q_sb, q_sh, k_cache, v_cache, n_blocks, block_size, k_strides, v_strides,
                       block_table, bt_stride, max_blocks, seqlen, out, o_sb, o_sh, nullptr, nullptr,
                       nullptr, 0, batch, n_head, n_kv_head, head_dim, dtype, scale_log2, workspace,
                       workspace_bytes, stream);
}

int pd_prefill(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache, const void* v_cache,
               int64_t n_blocks, int32_t block_size, const int64_t* k_strides, const int64_t* v_strides,
               const int32_t* block_table, int64_t bt_stride, int32_t max_blocks,
               const int32_t* cu_seqlens_q, const int32_t* seqlen_k, void* out, int64_t o_st,
               int64_t o_sh, int32_t batch, int32_t max_seqlen_q, int32_t n_head, int32_t n_kv_head,
               int32_t head_dim, int32_t dtype, float scale_log2, void* stream) {
  if (!valid_dtype(dtype) || n_head < 1 || n_kv_head < 1 || n_head % n_kv_head != 0) return PD_ERR_INVALID;
  if (batch < 0 || max_seqlen_q < 0 || max_blocks < 0 || n_blocks < 1) return PD_ERR_INVALID;
  if (!pow2(block_size) || !pow2(head_dim)) return PD_ERR_INVALID;
  const int group = n_head / n_kv_head;
  if (!prefill_supported(dtype, head_dim, group) || block_size < 8) return PD_ERR_UNSUPPORTED;
  if (k_strides == nullptr || v_strides == nullptr) return PD_ERR_INVALID;
  if (max_blocks > 0 && bt_stride < max_blocks) return PD_ERR_INVALID;
  const int64_t capacity = int64_t(max_blocks) * block_size;
  if (capacity > (int64_t(1) << 30)) return PD_ERR_INVALID;
  if (batch == 0 || max_seqlen_q == 0) return PD_OK;
  if (cu_seqlens_q == nullptr || seqlen_k == nullptr || (block_table == nullptr && max_blocks > 0))
    return PD_ERR_INVALID;
  if (check_rows(q, q_st, q_sh, dtype) != PD_OK || check_rows(out, o_st, o_sh, dtype) != PD_OK)
    return PD_ERR_INVALID;
  int dev = 0;
  if (current_device(&dev) != PD_OK) return PD_ERR_CUDA;
  unsigned* err = error_word(dev);
  if (err == nullptr) return PD_ERR_CUDA;
  int mode;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    mode = g_prefill_mode;
  }
  const bool tc = mode == 0;
  const int tile_tokens = tc ? prefill_tc_tile_tokens(head_dim) : prefill_tile_tokens(head_dim);
  const int box_tokens = block_size < tile_tokens ? block_size : tile_tokens;
  // The tcgen05 kernel takes grouped boxes where the pools' blocks are evenly spaced (the
  // engine's layout), one-piece boxes otherwise.
  const bool grouped = tc && k_strides[0] == int64_t(block_size) * k_strides[1] &&
                       v_strides[0] == int64_t(block_size) * v_strides[1];
  const int view = !tc ? SW_ROWS : (grouped ? SW_GROUPED : SW_ONE_PIECE);
  CUtensorMap kmap, vmap;
  int st = encode_pool(&kmap, k_cache, n_blocks, block_size, n_kv_head, head_dim, k_strides, dtype, box_tokens,
                       1, true, view);
  if (st != PD_OK) return st;
  st = encode_pool(&vmap, v_cache, n_blocks, block_size, n_kv_head, head_dim, v_strides, dtype, box_tokens, 1,
                   true, view);
  if (st != PD_OK) return st;
  PrefillParams p{};
  p.grouped = grouped ? 1 : 0;
  p.q = q;
  p.q_st = q_st;
  p.q_sh = q_sh;
  p.out = out;
  p.o_st = o_st;
  p.o_sh = o_sh;
  p.cu_q = cu_seqlens_q;
  p.seqlen_k = seqlen_k;
  p.table = block_table;
  p.bt_stride = bt_stride;
  p.max_blocks = max_blocks;
  p.capacity = int32_t(capacity);
  p.block_size = block_size;
  p.box_tokens = box_tokens;
  p.scale_log2 = scale_log2;
  p.err = err;
  p.wait_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  const cudaError_t e = tc ? launch_prefill_tc(p, kmap, vmap, dtype, head_dim, group, max_seqlen_q, batch,
                                               n_kv_head, static_cast<cudaStream_t>(stream))
                           : launch_prefill(p, kmap, vmap, dtype, head_dim, group, max_seqlen_q, batch,
                                            n_kv_head, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return PD_OK;
}

int pd_decode_partials(const void* q, int64_t q_sb, int64_t q_sh, const void* k_cache,
                       const void* v_cache, int64_t n_blocks, int32_t block_size,
                       const int64_t* k_strides, const int64_t* v_strides,
                       const int32_t* block_table, int64_t bt_stride, int32_t max_blocks,
                       const int32_t* seqlen, float* m_out, float* l_out, float* acc_out,
                       int32_t batch, int32_t n_head, int32_t n_kv_head, int32_t head_dim,
                       int32_t dtype, float scale_log2, void* workspace, size_t workspace_bytes,
                       void* stream) {
  return decode_common(q, q_sb, q_sh, k_cache, v_cache, n_blocks, block_size, k_strides, v_strides,
                       block_table, bt_stride, max_blocks, seqlen, nullptr, 0, 0, m_out, l_out,
                       acc_out, 1, batch, n_head, n_kv_head, head_dim, dtype, scale_log2, workspace,
                       workspace_bytes, stream);
}

int pd_plan_create(pd_plan** plan, int32_t n_layer, const void* const* k_caches,
                   const void* const* v_caches, int64_t n_blocks, int32_t block_size,
                   const int64_t* k_strides, const int64_t* v_strides, const int32_t* block_table,
                   int64_t bt_stride, int32_t max_blocks, const int32_t* seqlen, int32_t batch,
                   int32_t n_head, int32_t n_kv_head, int32_t head_dim, int32_t dtype,
                   float scale_log2, void* workspace, size_t workspace_bytes) {
  if (plan == nullptr) return PD_ERR_INVALID;
  *plan = nullptr;
  if (n_layer < 1 || k_caches == nullptr || v_caches == nullptr || batch < 1) return PD_ERR_INVALID;
  if (k_strides == nullptr || v_strides == nullptr) return PD_ERR_INVALID;
  pd_plan* h = new (std::nothrow) pd_plan;
  if (h == nullptr) return PD_ERR_INVALID;
  int st = prepare(&h->P, n_blocks, block_size, block_table, bt_stride, max_blocks, seqlen, batch,
                   n_head, n_kv_head, head_dim, dtype, scale_log2, workspace, workspace_bytes);
  if (st != PD_OK) {
    delete h;
    return st;
  }
  h->n_layer = n_layer;
  h->dtype = dtype;
  // Step cache of the work split: one batch chunk per launch and the per-warp kernel.
  if (batch <= h->P.L.rows_per_launch && !h->P.g.cta)
    h->P.base.step_rec = static_cast<unsigned char*>(workspace) + h->P.ws.step_off;
  h->q_sh = head_dim;
  h->q_sb = int64_t(n_head) * head_dim;
  h->n_blocks = n_blocks;
  for (int i = 0; i < 3; ++i) {
    h->k_strides[i] = k_strides[i];
    h->v_strides[i] = v_strides[i];
  }
  h->kmaps.resize(n_layer);
  h->vmaps.resize(n_layer);
  h->k_pools.resize(n_layer);
  h->v_pools.resize(n_layer);
  for (int layer = 0; layer < n_layer; ++layer) {
    h->k_pools[layer] = const_cast<void*>(k_caches[layer]);
    h->v_pools[layer] = const_cast<void*>(v_caches[layer]);
    st = encode_pool(&h->kmaps[layer], k_caches[layer], n_blocks, block_size, n_kv_head, head_dim,
                     k_strides, dtype, h->P.g.box_tokens, h->P.g.box_heads, h->P.g.mma);
    if (st == PD_OK)
      st = encode_pool(&h->vmaps[layer], v_caches[layer], n_blocks, block_size, n_kv_head, head_dim,
                       v_strides, dtype, h->P.g.box_tokens, h->P.g.box_heads, h->P.g.mma);
    if (st != PD_OK) {
      delete h;
      return st;
    }
  }
  *plan = h;
  return PD_OK;
}

int pd_plan_run(const pd_plan* plan, int32_t layer, const void* q, void* out, void* stream) {
  if (plan == nullptr || layer < 0 || layer >= plan->n_layer) return PD_ERR_INVALID;
  if (check_rows(q, plan->q_sb, plan->q_sh, plan->dtype) != PD_OK) return PD_ERR_INVALID;
  if (check_rows(out, plan->q_sb, plan->q_sh, plan->dtype) != PD_OK) return PD_ERR_INVALID;
  return run_prepared(plan->P, plan->kmaps[layer], plan->vmaps[layer], q, plan->q_sb, plan->q_sh, out,
                      plan->q_sb, plan->q_sh, nullptr, nullptr, nullptr, 0, plan->dtype,
                      static_cast<cudaStream_t>(stream), nullptr, plan->overlap != 0, &plan->seq);
}

int pd_plan_set_static_table(pd_plan* plan, int32_t fixed) {
  if (plan == nullptr || fixed < 0 || fixed > 1) return PD_ERR_INVALID;
  plan->P.base.step_table = fixed;
  return PD_OK;
}

int pd_plan_set_overlap(pd_plan* plan, int32_t enable) {
  if (plan == nullptr || enable < 0 || enable > 1) return PD_ERR_INVALID;
  if (enable && plan->P.halves != 2) return PD_ERR_WORKSPACE;
  plan->overlap = enable;
  return PD_OK;
}

static int plan_run_append(const pd_plan* plan, int32_t layer, const void* q, void* out,
                           const void* k_new, int64_t k_sb, int64_t k_sh, const void* v_new,
                           int64_t v_sb, int64_t v_sh, const int64_t* pos, const void* rope_cos,
                           const void* rope_sin, int64_t rope_stride, int32_t rotary_dim, void* stream) {
  if (plan == nullptr || layer < 0 || layer >= plan->n_layer) return PD_ERR_INVALID;
  if (check_rows(q, plan->q_sb, plan->q_sh, plan->dtype) != PD_OK) return PD_ERR_INVALID;
  if (check_rows(out, plan->q_sb, plan->q_sh, plan->dtype) != PD_OK) return PD_ERR_INVALID;
  if (check_rows(k_new, k_sb, k_sh, plan->dtype) != PD_OK) return PD_ERR_INVALID;
  if (check_rows(v_new, v_sb, v_sh, plan->dtype) != PD_OK) return PD_ERR_INVALID;
  if (pos == nullptr || (reinterpret_cast<uintptr_t>(pos) & 7u) != 0) return PD_ERR_INVALID;
  AppendArgs app;
  app.k = k_new;
  app.k_sb = k_sb;
  app.k_sh = k_sh;
  app.v = v_new;
  app.v_sb = v_sb;
  app.v_sh = v_sh;
  app.pos = pos;
  app.pool_k = plan->k_pools[layer];
  app.pool_v = plan->v_pools[layer];
  app.k_strides = plan->k_strides;
  app.v_strides = plan->v_strides;
  app.n_blocks = plan->n_blocks;
  app.rope_cos = rope_cos;
  app.rope_sin = rope_sin;
  app.rope_stride = rope_stride;
  app.rope_dim = rotary_dim;
  return run_prepared(plan->P, plan->kmaps[layer], plan->vmaps[layer], q, plan->q_sb, plan->q_sh, out,
                      plan->q_sb, plan->q_sh, nullptr, nullptr, nullptr, 0, plan->dtype,
                      static_cast<cudaStream_t>(stream), &app, plan->overlap != 0, &plan->seq);
}

int pd_plan_run_append(const pd_plan* plan, int32_t layer, const void* q, void* out,
                       const void* k_new, int64_t k_sb, int64_t k_sh, const void* v_new,
                       int64_t v_sb, int64_t v_sh, const int64_t* pos, void* stream) {
  return plan_run_append(plan, layer, q, out, k_new, k_sb, k_sh, v_new, v_sb, v_sh, pos, nullptr, nullptr,
                         0, 0, stream);
}

int pd_plan_run_append_rope(const pd_plan* plan, int32_t layer, const void* q, void* out,
                            const void* k_new, int64_t k_sb, int64_t k_sh, const void* v_new,
                            int64_t v_sb, int64_t v_sh, const int64_t* pos, const void* rope_cos,
                            const void* rope_sin, int64_t rope_stride, int32_t rotary_dim, void* stream) {
  if (plan == nullptr) return PD_ERR_INVALID;
  const int32_t head_dim = int32_t(plan->q_sh);  // q rows are contiguous (B, H, D)
  if (!rope_args_ok(rope_cos, rope_sin, rope_stride, rotary_dim, head_dim, plan->dtype, plan->dtype))
    return PD_ERR_INVALID;
  return plan_run_append(plan, layer, q, out, k_new, k_sb, k_sh, v_new, v_sb, v_sh, pos, rope_cos, rope_sin,
                         rope_stride, rotary_dim, stream);
}

void pd_plan_destroy(pd_plan* plan) { delete plan; }

int pd_lse_merge(const float* m_parts, const float* l_parts, const float* acc_parts,
                 int64_t ml_part_stride, int64_t acc_part_stride, int32_t n_parts, int32_t batch,
                 int32_t n_head, int32_t head_dim, void* out, int64_t o_sb, int64_t o_sh,
                 int32_t dtype, void* stream) {
  if (!valid_dtype(dtype) || n_parts < 1 || batch < 0 || n_head < 1) return PD_ERR_INVALID;
  if (head_dim < 4 || head_dim % 4 != 0) return PD_ERR_UNSUPPORTED;
  if (batch == 0) return PD_OK;
  if (m_parts == nullptr || l_parts == nullptr || acc_parts == nullptr || out == nullptr ||
      !aligned16(acc_parts) || acc_part_stride % 4 != 0)
    return PD_ERR_INVALID;
  if (ml_part_stride < int64_t(batch) * n_head || acc_part_stride < int64_t(batch) * n_head * head_dim)
    return PD_ERR_INVALID;
  MergeParams p;
  p.m = m_parts;
  p.l = l_parts;
  p.acc = acc_parts;
  p.out = out;
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.ml_stride = ml_part_stride;
  p.acc_stride = acc_part_stride;
  p.n_parts = n_parts;
  p.batch = batch;
  p.n_head = n_head;
  p.head_dim = head_dim;
  const cudaError_t e = launch_merge(p, dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return PD_OK;
}

static int append_common(AppendParams& p, int32_t pool_dtype, int32_t src_dtype,
                         const int64_t* k_pool_strides, const int64_t* v_pool_strides,
                         const int64_t* k_strides, const int64_t* v_strides, void* stream) {
  if (!valid_dtype(pool_dtype) || !valid_dtype(src_dtype)) return PD_ERR_INVALID;
  if (p.n_tokens < 0 || p.n_kv_head < 1 || p.head_dim < 1 || p.block_size < 1 || p.n_blocks < 1)
    return PD_ERR_INVALID;
  if (p.n_tokens == 0) return PD_OK;
  if (!k_pool_strides || !v_pool_strides || !k_strides || !v_strides) return PD_ERR_INVALID;
  if (!p.k_pool || !p.v_pool || !p.k || !p.v) return PD_ERR_INVALID;
  int dev = 0;
  if (current_device(&dev) != PD_OK) return PD_ERR_CUDA;
  p.err = error_word(dev);
  if (p.err == nullptr) return PD_ERR_CUDA;
  p.kp_sb = k_pool_strides[0];
  p.kp_sn = k_pool_strides[1];
  p.kp_sh = k_pool_strides[2];
  p.vp_sb = v_pool_strides[0];
  p.vp_sn = v_pool_strides[1];
  p.vp_sh = v_pool_strides[2];
  p.k_s0 = k_strides[0];
  p.k_s1 = k_strides[1];
  p.v_s0 = v_strides[0];
  p.v_s1 = v_strides[1];
  // 8-wide vector path when every row start of every tensor is 16-byte aligned for both
  // element sizes involved.
  const int es_s = elem_size(src_dtype), es_d = elem_size(pool_dtype);
  auto ok_src = [&](const void* base, int64_t s0, int64_t s1) {
    return aligned16(base) && (s0 * es_s) % 16 == 0 && (s1 * es_s) % 16 == 0;
  };
  auto ok_dst = [&](const void* base, int64_t a, int64_t b, int64_t c) {
    return aligned16(base) && (a * es_d) % 16 == 0 && (b * es_d) % 16 == 0 && (c * es_d) % 16 == 0;
  };
  const bool vec = p.head_dim % 8 == 0 && ok_src(p.k, p.k_s0, p.k_s1) && ok_src(p.v, p.v_s0, p.v_s1) &&
                   ok_dst(p.k_pool, p.kp_sb, p.kp_sn, p.kp_sh) &&
                   ok_dst(p.v_pool, p.vp_sb, p.vp_sn, p.vp_sh);
  cudaError_t e = launch_append(p, src_dtype, pool_dtype, vec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "append launch");
  if (p.n_tokens > 0) g_launches.fetch_add(1, std::memory_order_relaxed);
  return PD_OK;
}

int pd_kv_append_slots(void* k_pool, void* v_pool, int64_t n_blocks, int32_t block_size,
                       const int64_t* k_pool_strides, const int64_t* v_pool_strides,
                       int32_t pool_dtype, const void* slot_ids, int32_t slot_dtype, const void* k,
                       const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       int32_t src_dtype, int64_t n_tokens, int32_t n_kv_head, int32_t head_dim,
                       void* stream) {
  if (slot_dtype != PD_SLOT_I32 && slot_dtype != PD_SLOT_I64) return PD_ERR_INVALID;
  if (slot_ids == nullptr && n_tokens > 0) return PD_ERR_INVALID;
  AppendParams p{};
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.n_blocks = n_blocks;
  p.slots = slot_ids;
  p.k = k;
  p.v = v;
  p.n_tokens = n_tokens;
  p.block_size = block_size;
  p.n_kv_head = n_kv_head;
  p.head_dim = head_dim;
  p.use_table = 0;
  p.slot_i64 = slot_dtype == PD_SLOT_I64;
  return append_common(p, pool_dtype, src_dtype, k_pool_strides, v_pool_strides, k_strides,
                       v_strides, stream);
}

int pd_kv_append_table(void* k_pool, void* v_pool, int64_t n_blocks, int32_t block_size,
                       const int64_t* k_pool_strides, const int64_t* v_pool_strides,
                       int32_t pool_dtype, const int32_t* block_table, int64_t bt_stride,
                       int32_t max_blocks, const int64_t* pos, const void* k,
                       const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       int32_t src_dtype, int32_t batch, int32_t n_kv_head, int32_t head_dim,
                       void* stream) {
  if (batch > 0 && (block_table == nullptr || pos == nullptr || max_blocks < 1)) return PD_ERR_INVALID;
  AppendParams p{};
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.n_blocks = n_blocks;
  p.table = block_table;
  p.bt_stride = bt_stride;
  p.max_blocks = max_blocks;
  p.pos = pos;
  p.k = k;
  p.v = v;
  p.n_tokens = batch;
  p.block_size = block_size;
  p.n_kv_head = n_kv_head;
  p.head_dim = head_dim;
  p.use_table = 1;
  return append_common(p, pool_dtype, src_dtype, k_pool_strides, v_pool_strides, k_strides,
                       v_strides, stream);
}

int pd_kv_append_table_rope(void* k_pool, void* v_pool, int64_t n_blocks, int32_t block_size,
                            const int64_t* k_pool_strides, const int64_t* v_pool_strides,
                            int32_t pool_dtype, const int32_t* block_table, int64_t bt_stride,
                            int32_t max_blocks, const int64_t* pos, const void* k,
                            const int64_t* k_strides, const void* v, const int64_t* v_strides,
                            int32_t src_dtype, int32_t batch, int32_t n_kv_head, int32_t head_dim,
                            const void* rope_cos, const void* rope_sin, int64_t rope_stride,
                            int32_t rotary_dim, void* stream) {
  if (!rope_args_ok(rope_cos, rope_sin, rope_stride, rotary_dim, head_dim, src_dtype, pool_dtype))
    return PD_ERR_INVALID;
  if (batch > 0 && (block_table == nullptr || pos == nullptr || max_blocks < 1)) return PD_ERR_INVALID;
  AppendParams p{};
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.n_blocks = n_blocks;
  p.table = block_table;
  p.bt_stride = bt_stride;
  p.max_blocks = max_blocks;
  p.pos = pos;
  p.k = k;
  p.v = v;
  p.n_tokens = batch;
  p.block_size = block_size;
  p.n_kv_head = n_kv_head;
  p.head_dim = head_dim;
  p.use_table = 1;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  p.rope_stride = rope_stride;
  p.rope_dim = rotary_dim;
  return append_common(p, pool_dtype, src_dtype, k_pool_strides, v_pool_strides, k_strides,
                       v_strides, stream);
}

int pd_set_decode_tuning(int32_t warps_per_cta, int32_t stages, int32_t ctas_per_sm,
                         int32_t min_tiles_per_warp) {
  std::lock_guard<std::mutex> lock(g_mutex);
  Tuning t = g_tuning;
  if (warps_per_cta > 0) t.warps = warps_per_cta;
  if (stages > 0) t.stages = stages;
  if (ctas_per_sm > 0) t.ctas_per_sm = ctas_per_sm;
  if (min_tiles_per_warp > 0) t.min_tiles = min_tiles_per_warp;
  if (t.warps > 8 || t.stages < 2 || t.stages > 16 || t.ctas_per_sm > 8) return PD_ERR_INVALID;
  if (size_t(t.warps) * t.stages * 8192 + 2048 > size_t(kMaxSmemPerBlock)) return PD_ERR_INVALID;
  g_tuning = t;
  return PD_OK;
}

int pd_set_decode_mode(int32_t mode, int32_t shared_stages, int32_t row_cost) {
  if (mode < 0 || mode > 2 || shared_stages < 0 || shared_stages > 8 || row_cost < -1 || row_cost > 64)
    return PD_ERR_INVALID;
  std::lock_guard<std::mutex> lock(g_mutex);
  g_decode_mode = mode;
  g_cta_stages = shared_stages;
  if (row_cost >= 0) g_row_cost = row_cost;
  return PD_OK;
}

int pd_get_decode_mode(int32_t* mode, int32_t* shared_stages, int32_t* row_cost) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (mode) *mode = g_decode_mode;
  if (shared_stages) *shared_stages = g_cta_stages;
  if (row_cost) *row_cost = g_row_cost;
  return PD_OK;
}

int pd_set_prefill_mode(int32_t mode) {
  if (mode < 0 || mode > 1) return PD_ERR_INVALID;
  std::lock_guard<std::mutex> lock(g_mutex);
  g_prefill_mode = mode;
  return PD_OK;
}

int pd_get_prefill_mode(void) {
  std::lock_guard<std::mutex> lock(g_mutex);
  return g_prefill_mode;
}

int pd_set_wait_limit(uint64_t limit_ns) {
  if (limit_ns > 10ull * WAIT_LIMIT_NS) return PD_ERR_INVALID;
  g_wait_limit_ns.store(limit_ns == 0 ? WAIT_LIMIT_NS : limit_ns, std::memory_order_relaxed);
  return PD_OK;
}

uint64_t pd_get_wait_limit(void) { return g_wait_limit_ns.load(std::memory_order_relaxed); }

int pd_get_decode_tuning(int32_t* warps_per_cta, int32_t* stages, int32_t* ctas_per_sm,
                         int32_t* min_tiles_per_warp) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (warps_per_cta) *warps_per_cta = g_tuning.warps;
  if (stages) *stages = g_tuning.stages;
  if (ctas_per_sm) *ctas_per_sm = g_tuning.ctas_per_sm;
  if (min_tiles_per_warp) *min_tiles_per_warp = g_tuning.min_tiles;
  return PD_OK;
}

// ---------------------------------------------------------------- decode without allocation
// Scratch for pd_decode_noalloc: a fixed array in this library's device image, so the call
// never allocates. Host code must not use `g_noalloc_scratch` as an address -- on the host the
// name stands for a shadow symbol, not device memory -- and instead passes the device address
// that cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[PD_NOALLOC_SCRATCH_BYTES];

static void* g_noalloc_ptr[kMaxDevices] = {nullptr};
static std::mutex g_noalloc_mutex;

// Device address of the scratch array on the current device, looked up on first use.
static int noalloc_scratch(void** ptr) {
  int dev = 0;
  if (current_device(&dev) != PD_OK) return PD_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return cuda_fail(e, "pd_decode_noalloc scratch lookup");
    g_noalloc_ptr[dev] = p;
  }
  *ptr = g_noalloc_ptr[dev];
  return PD_OK;
}

int pd_decode_noalloc(const void* q, int64_t q_sb, int64_t q_sh, const void* k_cache,
                      const void* v_cache, int64_t n_blocks, int32_t block_size,
                      const int64_t* k_strides, const int64_t* v_strides, const int32_t* block_table,
                      int64_t bt_stride, int32_t max_blocks, const int32_t* seqlen, void* out,
                      int64_t o_sb, int64_t o_sh, int32_t batch, int32_t n_head, int32_t n_kv_head,
                      int32_t head_dim, int32_t dtype, float scale_log2, void* stream) {
  void* scratch = nullptr;
  int st = noalloc_scratch(&scratch);
  if (st != PD_OK) return st;
  // The size check is the one pd_decode makes against its workspace, done by the same prepare()
  // that lays the scratch out, so the refusal always matches the layout actually used.
  st = decode_common(q, q_sb, q_sh, k_cache, v_cache, n_blocks, block_size, k_strides, v_strides,
                     block_table, bt_stride, max_blocks, seqlen, out, o_sb, o_sh, nullptr, nullptr,
                     nullptr, 0, batch, n_head, n_kv_head, head_dim, dtype, scale_log2, scratch,
                     size_t(PD_NOALLOC_SCRATCH_BYTES), stream);
  if (st == PD_ERR_WORKSPACE)
    snprintf(g_last_error, sizeof(g_last_error),
             "pd_decode_noalloc: this shape needs %zu bytes of scratch but the built-in scratch array "
             "holds %u; call pd_decode with a workspace instead",
             g_last_ws_need, unsigned(PD_NOALLOC_SCRATCH_BYTES));
  return st;
}

}  // extern "C"
