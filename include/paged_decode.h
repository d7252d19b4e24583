/*
 * paged_decode.h -- C ABI of the B200 (sm_100a) paged-KV decode path.
 *
 * This is the drop-in boundary for the block-table decode path of RAIN-LOJK/llm-serving.
 * The reference implements the path in Python + one Triton kernel; every entry point
 * below replaces one piece of it and names the reference interface it stands for
 * (paths are relative to the reference project root).
 *
 * Conventions
 *  - Plain pointers to device memory, element strides (not bytes), int32/int64 sizes.
 *    The head-dim stride of every tensor is 1.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Every function returns PD_OK (0) or a PD_ERR_* status; nothing aborts the process.
 *    Argument errors are detected on the host before any launch. Device-side problems
 *    (a bounded wait that ran out, an out-of-range slot or block id in the append path)
 *    never fault or trap: the kernel skips the access and records a bit in a per-device
 *    error word that pd_device_error() reads.
 *  - dtype codes: PD_F32, PD_F16, PD_BF16. q, K, V and out share one dtype.
 *  - K/V pools have the reference layout (n_blocks, block_size, n_kv_head, head_dim)
 *    (model/paged.py:115-123); block tables are int32 (B, max_blocks) with a unit
 *    column stride; seqlen is int32 (B,) (model/triton_decode.py:17-26).
 */
#ifndef PAGED_DECODE_H
#define PAGED_DECODE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status / dtypes */
#define PD_OK 0
#define PD_ERR_INVALID 1     /* bad argument (shape, stride, alignment, range)          */
#define PD_ERR_UNSUPPORTED 2 /* shape the library has no kernel for (e.g. head_dim 512) */
#define PD_ERR_CUDA 3        /* a CUDA runtime call or launch failed                     */
#define PD_ERR_WORKSPACE 4   /* workspace pointer missing or smaller than required      */

#define PD_F32 0
#define PD_F16 1
#define PD_BF16 2

/* Device error word bits (pd_device_error). */
#define PD_DEVERR_WAIT_TIMEOUT 1u  /* an mbarrier wait exceeded its time limit          */
#define PD_DEVERR_APPEND_RANGE 2u  /* append skipped a slot / block id outside the pool  */

/* Human-readable name of a status code (static storage). */
const char* pd_status_string(int status);

/* Library ABI version (increments on any signature change). */
int pd_abi_version(void);

/* Number of kernels this library has launched in this process, over all devices and
 * threads (a benchmark reports how many of its launches were this library's). */
uint64_t pd_launch_count(void);

/* Name and description of the last CUDA error a call on this thread returned as PD_ERR_CUDA
 * (static storage; "" when none). No reference counterpart: the Triton launch raises. */
const char* pd_last_error_string(void);

/* Reads the calling thread's current device's error word into *bits and, if `clear`,
 * resets it. Synchronises the device. No reference counterpart: the Triton kernel has no
 * device-side status (model/triton_decode.py:63-66 trusts the table instead). */
int pd_device_error(unsigned int* bits, int clear);

/* ---------------------------------------------------------------- decode
 *
 * pd_decode replaces `paged_decode(q, k_cache, v_cache, block_table, seqlen, *, scale)`
 * (model/triton_decode.py:250-328) after its validation: one launch of the decode kernel.
 *
 *   q        (B, H, D)       strides q_sb, q_sh (elements); 16-byte aligned rows
 *   k_cache  (n_blocks, block_size, H_kv, D) strides k_strides[0..2] (block, token, head)
 *   v_cache  same geometry, strides v_strides[0..2]
 *   block_table (B, max_blocks) int32, row stride bt_stride, unit column stride
 *   seqlen   (B,) int32; values are clamped to [0, max_blocks * block_size] on device
 *   out      (B, H, D)       strides o_sb, o_sh
 *   scale_log2 = scale * log2(e)  (model/triton_decode.py:291-292)
 *   workspace: device memory of at least pd_decode_workspace_bytes(...) bytes, 256-byte
 *     aligned, with any contents -- zero-filled, garbage, or left by earlier launches of any
 *     shape (no clearing needed: split rows are counted with per-launch epochs that the kernel
 *     keeps in the workspace and advances itself, and the counters' tags are odd and salted
 *     per layout, so stale memory never carries a live tag; launches replayed from a captured
 *     CUDA graph stay correct). One workspace must not be used by two launches that may run
 *     concurrently. After a launch that recorded PD_DEVERR_WAIT_TIMEOUT the workspace is
 *     still usable as is.
 *
 * Row b, head h reads only the first ceil(seqlen[b] / block_size) table entries;
 * zero-length rows produce exact zeros (model/triton_decode.py:639).
 */
size_t pd_decode_workspace_bytes(int32_t batch, int32_t n_head, int32_t n_kv_head,
                                 int32_t head_dim, int32_t dtype);

int pd_decode(const void* q, int64_t q_sb, int64_t q_sh,
              const void* k_cache, const void* v_cache, int64_t n_blocks, int32_t block_size,
              const int64_t* k_strides, const int64_t* v_strides,
              const int32_t* block_table, int64_t bt_stride, int32_t max_blocks,
              const int32_t* seqlen, void* out, int64_t o_sb, int64_t o_sh,
              int32_t batch, int32_t n_head, int32_t n_kv_head, int32_t head_dim,
              int32_t dtype, float scale_log2, void* workspace, size_t workspace_bytes,
              void* stream);

/* pd_decode_noalloc -- the same decode as pd_decode for callers that cannot allocate device
 * memory. No counterpart in the reference (it always runs inside PyTorch, which allocates).
 *
 * Who needs it: hosts that bind this C ABI without owning a device allocator -- for example
 * a Go, Java or Node serving process calling through cgo/JNI/N-API with only raw tensor
 * pointers handed to it -- and callers whose device memory is already fully reserved by
 * another allocator (PyTorch's caching allocator, an inference runtime's arena), where an
 * extra cudaMalloc can fail and cudaMalloc/cudaFree would synchronise the device.
 *
 * What differs from pd_decode: there is no workspace argument. The split-row scratch lives in
 * one fixed array of PD_NOALLOC_SCRATCH_BYTES (8 MiB) compiled into the library; every GPU
 * that loads the library holds that much device memory until the process exits. The call
 * itself performs no allocation of any kind. Its first call on a device, with that device
 * current, looks the array's device address up (cudaGetSymbolAddress) and caches it; make
 * that first call before capturing a stream. Shapes whose scratch need exceeds the array
 * (pd_decode_workspace_bytes(...) > PD_NOALLOC_SCRATCH_BYTES, e.g. head_dim 256 with 8 q
 * heads per kv head) are rejected with PD_ERR_WORKSPACE and a message in
 * pd_last_error_string(); use pd_decode with a workspace for those.
 *
 * The array keeps whatever the previous call left and starts out zero-filled; neither needs
 * clearing (split rows are counted with per-launch epochs and odd counter tags, which zeroed
 * or stale memory never carries). All calls on one device share the array, so two
 * calls whose kernels can overlap on the GPU (different streams without ordering between
 * them) race and may return wrong results: issue them on one stream or order them.
 */
#define PD_NOALLOC_SCRATCH_BYTES (8u << 20)

int pd_decode_noalloc(const void* q, int64_t q_sb, int64_t q_sh,
                      const void* k_cache, const void* v_cache, int64_t n_blocks,
                      int32_t block_size, const int64_t* k_strides, const int64_t* v_strides,
                      const int32_t* block_table, int64_t bt_stride, int32_t max_blocks,
                      const int32_t* seqlen, void* out, int64_t o_sb, int64_t o_sh,
                      int32_t batch, int32_t n_head, int32_t n_kv_head, int32_t head_dim,
                      int32_t dtype, float scale_log2, void* stream);

/* pd_prefill -- chunked-prefill attention reading the paged pool (block-table-aware prefill).
 *
 * Row b's new query tokens are q[cu_seqlens_q[b] .. cu_seqlens_q[b+1]) of a packed
 * (total_q, n_head, head_dim) tensor (token stride q_st, head stride q_sh, unit last stride,
 * 16-byte aligned rows); their K/V are already in the pool (appended as for decode). Query
 * token i of a chunk of Sq tokens sits at position seqlen_k[b] - Sq + i and attends causally
 * to keys 0 .. seqlen_k[b] - Sq + i of the row, token t at block block_table[b, t / bs],
 * slot t % bs: the causal convention of a varlen flash-attention call with a block table,
 * bottom-right aligned. softmax(q.k * scale) and P.V in fp32; out (same layout as q, its own
 * strides) in the pool dtype. A chunk of one token gives pd_decode's result.
 * max_seqlen_q must be at least the longest chunk (the grid is sized from it; the kernel does
 * not read cu_seqlens_q on the host): query tokens of a longer chunk past it are not written.
 * Supported: bf16 / fp16, head_dim 64, 128 or 256, 1, 2, 4 or 8 q heads per kv head, block_size
 * >= 8 (PD_ERR_UNSUPPORTED otherwise). No workspace. The reference has no counterpart: its
 * packed varlen prefill (flash_attn 2.8.3, model/attention/varlen.py:317-357; docs/decisions.md
 * D7) writes the paged pool but never reads it, so a chunk cannot attend to cached keys. */
int pd_prefill(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache, const void* v_cache,
               int64_t n_blocks, int32_t block_size, const int64_t* k_strides, const int64_t* v_strides,
               const int32_t* block_table, int64_t bt_stride, int32_t max_blocks,
               const int32_t* cu_seqlens_q, const int32_t* seqlen_k, void* out, int64_t o_st,
               int64_t o_sh, int32_t batch, int32_t max_seqlen_q, int32_t n_head, int32_t n_kv_head,
               int32_t head_dim, int32_t dtype, float scale_log2, void* stream);

/* ---------------------------------------------------------------- decode plan
 *
 * pd_plan_* replaces `PagedDecodePlan` / `paged_decode_plan` (model/triton_decode.py:
 * 331-538): every layer's pool is validated and its two TMA descriptors are encoded once;
 * pd_plan_run(layer, q, out) is the per-layer launch (model/triton_decode.py:500-520).
 * The block table and seqlen are held by address, so in-place updates are seen by the next
 * run (the reference's invariant, model/triton_decode.py:357-363). q and out of every run
 * are contiguous (B, H, D). The plan owns no device memory: `workspace` is the caller's
 * (same contract as pd_decode); with at least twice pd_decode_workspace_bytes(...) (each
 * half rounded up to 256 bytes) consecutive launches alternate between its two halves, which
 * pd_plan_set_overlap requires. The handle is host memory released by pd_plan_destroy.
 */
typedef struct pd_plan pd_plan;

int pd_plan_create(pd_plan** plan, int32_t n_layer, const void* const* k_caches,
                   const void* const* v_caches, int64_t n_blocks, int32_t block_size,
                   const int64_t* k_strides, const int64_t* v_strides,
                   const int32_t* block_table, int64_t bt_stride, int32_t max_blocks,
                   const int32_t* seqlen, int32_t batch, int32_t n_head, int32_t n_kv_head,
                   int32_t head_dim, int32_t dtype, float scale_log2, void* workspace,
                   size_t workspace_bytes);
int pd_plan_run(const pd_plan* plan, int32_t layer, const void* q, void* out, void* stream);

/* pd_plan_run_append -- `PagedKV.write(layer, k, v)` followed by `PagedKV.attend(layer, q)`
 * (model/paged.py:503-557) in ONE launch. Row b's new K and V rows, k_new / v_new
 * (B, H_kv, D) with element strides (k_sb, k_sh) / (v_sb, v_sh) in the plan's dtype and
 * 16-byte aligned rows, are stored at logical position pos[b] (int64) of the row -- pool
 * block block_table[b, pos / block_size], slot pos % block_size, exactly the slot
 * pd_kv_append_table writes -- and the decode of the same launch attends over them.
 * The result (out and the pools) equals pd_kv_append_table followed by pd_plan_run on the
 * same stream, provided no row reads a slot another row appends in this call (blocks are
 * not shared between rows for writing). A position outside the row's table or a block
 * outside the pool is skipped and recorded as PD_DEVERR_APPEND_RANGE, as in the append.
 */
int pd_plan_run_append(const pd_plan* plan, int32_t layer, const void* q, void* out,
                       const void* k_new, int64_t k_sb, int64_t k_sh, const void* v_new,
                       int64_t v_sb, int64_t v_sh, const int64_t* pos, void* stream);

/* pd_plan_run_append_rope -- pd_plan_run_append with the new K rows given BEFORE their
 * rotary embedding: the model's `k = apply_rotary_emb_partial(k, cos, sin, rotary_dim)`
 * (model/layers.py:59-117, called at layers.py:210-211 and qwen35.py:207-211) happens
 * inside the same launch. GPT-NeoX pairing (i, i + rotary_dim / 2) over the first
 * rotary_dim elements, the rest passing through; every product and sum is rounded to the
 * plan's dtype exactly as torch's elementwise ops round, so the stored rows are bit-identical
 * to rotating with torch and appending. rope_cos / rope_sin: row b's table at
 * rope_cos + b * rope_stride (elements), rotary_dim / 2 entries, the plan's dtype. */
int pd_plan_run_append_rope(const pd_plan* plan, int32_t layer, const void* q, void* out,
                            const void* k_new, int64_t k_sb, int64_t k_sh, const void* v_new,
                            int64_t v_sb, int64_t v_sh, const int64_t* pos, const void* rope_cos,
                            const void* rope_sin, int64_t rope_stride, int32_t rotary_dim,
                            void* stream);
/* pd_plan_set_overlap -- launches of this plan made afterwards (enable = 1) may start
 * before the previous kernel of their stream has finished (programmatic dependent launch):
 * the kernel reads seqlen, the append positions, the block table and the pools, computes
 * its work split and issues its first K/V copies, and only then waits for that kernel
 * before it reads q or the appended K/V rows, writes any output or touches the workspace.
 * Contract: the kernel launched just before on the stream writes none of seqlen, the
 * positions, the block table or this layer's pools (the previous layer's decode of a step,
 * a projection that produces q and the new rows: yes; a separate append into this layer's
 * pool, or the step's seqlen update: no). enable = 0 (the default) restores plain launches.
 * Needs a plan workspace of two halves (pd_plan_create): PD_ERR_WORKSPACE otherwise.
 * No reference counterpart (the reference launches one Triton kernel per call). */
int pd_plan_set_overlap(pd_plan* plan, int32_t enable);

/* pd_plan_set_static_table -- declares (fixed = 1) that the plan's block table keeps its
 * contents for the plan's lifetime (a decode container's table is built once and never
 * edited). Every plan caches its launches' work split in its workspace, keyed by a hash of the
 * clamped lengths and the plan's shape, so the layers of one decode step compute the split once
 * (model/paged.py:454-472 updates seqlen once per step); with a static table the cache also
 * keeps each warp's first block-table windows, so a layer's first K/V copies need no table
 * read. fixed = 0 (the default) re-reads the table, for callers that edit it in place between
 * launches. No reference counterpart. */
int pd_plan_set_static_table(pd_plan* plan, int32_t fixed);

void pd_plan_destroy(pd_plan* plan);

/* ---------------------------------------------------------------- split-KV partials
 *
 * The split-KV variant for long contexts and for context-parallel decode across GPUs.
 * No reference counterpart: split-K is "the documented next step" of the reference
 * (model/triton_decode.py:44-47). pd_decode_partials computes the same attention as
 * pd_decode but, instead of the normalised output, writes per (row, q head) the fp32 triple
 *   m[b, h]       running max of the log2-scaled scores (-inf for an empty range)
 *   l[b, h]       sum of exp2(score - m)
 *   acc[b, h, :]  sum of exp2(score - m) * v   (unnormalised)
 * for the tokens [0, seqlen[b]) of the given table. All three are contiguous: m and l are
 * (B, H), acc is (B, H, D). pd_lse_merge combines n_parts such triples -- part p's m and l
 * start at m_parts + p * ml_part_stride (resp. l_parts), its acc at acc_parts +
 * p * acc_part_stride, each (B, H[, D]) contiguous -- into out = sum_p 2^(m_p-M) acc_p /
 * max(sum_p 2^(m_p-M) l_p, 1) with M = max_p m_p, which is the reference's normalisation
 * acc / max(l, 1) (model/triton_decode.py:639) applied to the union of the parts.
 */
int pd_decode_partials(const void* q, int64_t q_sb, int64_t q_sh,
                       const void* k_cache, const void* v_cache, int64_t n_blocks,
                       int32_t block_size, const int64_t* k_strides, const int64_t* v_strides,
                       const int32_t* block_table, int64_t bt_stride, int32_t max_blocks,
                       const int32_t* seqlen, float* m_out, float* l_out, float* acc_out,
                       int32_t batch, int32_t n_head, int32_t n_kv_head, int32_t head_dim,
                       int32_t dtype, float scale_log2, void* workspace,
                       size_t workspace_bytes, void* stream);

int pd_lse_merge(const float* m_parts, const float* l_parts, const float* acc_parts,
                 int64_t ml_part_stride, int64_t acc_part_stride, int32_t n_parts,
                 int32_t batch, int32_t n_head, int32_t head_dim, void* out, int64_t o_sb,
                 int64_t o_sh, int32_t dtype, void* stream);

/* ---------------------------------------------------------------- paged-KV append
 *
 * pd_kv_append_slots replaces the body of `PagedPool.write_slots(layer, slot_ids, k, v)`
 * (model/paged.py:188-239): token i of k/v (n_tokens, H_kv, D) is copied into flat pool row
 * slot_ids[i] (= block_id * block_size + offset) of both pools, converting the source dtype
 * to the pool dtype with round-to-nearest-even (torch's Tensor.to). slot_dtype is PD_SLOT_I32
 * or PD_SLOT_I64. Slots outside [0, n_blocks * block_size) are skipped and flagged with
 * PD_DEVERR_APPEND_RANGE.
 *
 * pd_kv_append_table is the fused decode append behind `PagedKV.write(layer, k, v)`
 * (model/paged.py:503-520 with the slot map of _refresh_slots, 474-501): row b's token goes
 * to slot block_table[b, pos[b] / bs] * bs + pos[b] % bs, computed in the kernel from the
 * int32 block table and the int64 position vector, so no slot map is materialised.
 *
 * Source strides are element strides of (token/row, head, d) with unit d stride.
 */
#define PD_SLOT_I32 0
#define PD_SLOT_I64 1

int pd_kv_append_slots(void* k_pool, void* v_pool, int64_t n_blocks, int32_t block_size,
                       const int64_t* k_pool_strides, const int64_t* v_pool_strides,
                       int32_t pool_dtype, const void* slot_ids, int32_t slot_dtype,
                       const void* k, const int64_t* k_strides, const void* v,
                       const int64_t* v_strides, int32_t src_dtype, int64_t n_tokens,
                       int32_t n_kv_head, int32_t head_dim, void* stream);

int pd_kv_append_table(void* k_pool, void* v_pool, int64_t n_blocks, int32_t block_size,
                       const int64_t* k_pool_strides, const int64_t* v_pool_strides,
                       int32_t pool_dtype, const int32_t* block_table, int64_t bt_stride,
                       int32_t max_blocks, const int64_t* pos, const void* k,
                       const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       int32_t src_dtype, int32_t batch, int32_t n_kv_head, int32_t head_dim,
                       void* stream);

/* pd_kv_append_table_rope -- pd_kv_append_table with the K rows rotated first, exactly as
 * pd_plan_run_append_rope rotates them (source, pool and tables share one dtype; row b's
 * tables at rope_cos / rope_sin + b * rope_stride). */
int pd_kv_append_table_rope(void* k_pool, void* v_pool, int64_t n_blocks, int32_t block_size,
                            const int64_t* k_pool_strides, const int64_t* v_pool_strides,
                            int32_t pool_dtype, const int32_t* block_table, int64_t bt_stride,
                            int32_t max_blocks, const int64_t* pos, const void* k,
                            const int64_t* k_strides, const void* v, const int64_t* v_strides,
                            int32_t src_dtype, int32_t batch, int32_t n_kv_head, int32_t head_dim,
                            const void* rope_cos, const void* rope_sin, int64_t rope_stride,
                            int32_t rotary_dim, void* stream);

/* ---------------------------------------------------------------- tuning / introspection
 * Launch shape of the decode kernel: warps per CTA, pipeline stages per warp, CTAs per SM
 * and the minimum number of KV tiles a warp is given before fewer warps are used. Values
 * <= 0 keep the current setting. Changing them changes pd_decode_workspace_bytes. */
int pd_set_decode_tuning(int32_t warps_per_cta, int32_t stages, int32_t ctas_per_sm,
                         int32_t min_tiles_per_warp);
int pd_get_decode_tuning(int32_t* warps_per_cta, int32_t* stages, int32_t* ctas_per_sm,
                         int32_t* min_tiles_per_warp);

/* Decode kernel choice for calls and plans made afterwards. mode 0 (default): every warp
 * runs its own TMA pipeline; with bf16/fp16 pools, head_dim 64..256 and block_size >= 8 its
 * tile math runs on the tensor cores (mma.sync fed by ldmatrix from 128-byte-swizzled
 * stages), elsewhere on the CUDA cores. mode 2: per-warp pipelines with CUDA-core tile math
 * everywhere. mode 1: where a row has exactly 8 items (n_kv_head x q-head
 * chunks, e.g. 8 kv heads with 1-4 q heads each), bf16/fp16 and head_dim >= 64, the CTA
 * shares its pipeline stages -- a producer warp loads whole blocks of all kv heads and 8
 * consumer warps decode one item each; elsewhere mode 0 applies. shared_stages:
 * stage count of the shared-stage kernel (0 = as many as shared memory holds, at most 8).
 * row_cost (0..64, -1 = keep; default 3): when a row has one item per warp, the work is cut
 * into one range of (row, tile) columns per CTA, each row start counted as row_cost extra
 * columns, so that ranges crossing into a new row carry fewer tiles. Every kernel and every
 * row_cost compute the same function; results agree within rounding. Not thread-safe
 * against concurrent launches that size their workspace. No reference counterpart. */
int pd_set_decode_mode(int32_t mode, int32_t shared_stages, int32_t row_cost);
int pd_get_decode_mode(int32_t* mode, int32_t* shared_stages, int32_t* row_cost);

/* Prefill kernel for calls made afterwards: mode 0 (default) runs the tile math on the
 * 5th-generation tensor cores (tcgen05.mma with S and O accumulated in tensor memory, two
 * softmax threads per query row); mode 1 runs the warp-level mma.sync kernel. Both
 * compute pd_prefill's function; results agree within rounding. No reference counterpart. */
int pd_set_prefill_mode(int32_t mode);
int pd_get_prefill_mode(void);

/* Time limit, in nanoseconds, of the kernels' waits on a pipeline stage (mbarrier) or on a
 * split item's arrival counter, for launches made afterwards (default 1 s; 0 restores it;
 * at most 10 s). A wait that runs out records PD_DEVERR_WAIT_TIMEOUT in the device error word,
 * waits for its own copies still in flight (always with a fixed 0.1 s limit) and returns, so
 * the launch ends and the context stays usable; outputs of that launch are then unspecified.
 * Under a limit below 1000 ns every such wait gives up at once, complete or not: that is how a
 * test runs this error path deterministically, without a hang or a fault. No reference
 * counterpart (its kernel has no waits). */
int pd_set_wait_limit(uint64_t limit_ns);
uint64_t pd_get_wait_limit(void);

#ifdef __cplusplus
}
#endif
#endif /* PAGED_DECODE_H */
