// pd_tcgen05.cuh -- 5th-generation tensor-core (tcgen05 / UMMA) helpers for sm_100a.
//
// Inline-PTX wrappers for tensor-memory (TMEM) allocation, the single-thread tcgen05.mma of
// kind::f16 with both operands in shared memory (SS) or A in TMEM (TS), its commit to an
// mbarrier, TMEM loads and stores, the tcgen05 ordering fences, and the two 64-bit descriptors
// the MMA takes:
//
//  * shared-memory matrix descriptor: start address >> 4 in bits [0,14), leading-dimension
//    byte offset >> 4 in [16,30), stride-dimension byte offset >> 4 in [32,46), the constant 1
//    in [46,48) (the sm_100 descriptor version), base offset in [49,52) (0 here: every tile
//    starts on a 1024-byte boundary), and the layout type in [61,64) (2 = 128-byte swizzle);
//  * instruction descriptor (kind::f16): accumulator format in [4,6) (1 = f32), A and B formats
//    in [7,10) and [10,13) (0 = f16, 1 = bf16), A / B major-ness in bits 15 / 16 (0 = K-major,
//    1 = MN-major), N >> 3 in [17,23) and M >> 4 in [24,29).
//
// Operand layouts used with them (all 128-byte swizzled, the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B and the one the MMA reads with layout type 2):
//  * K-major (rows along M or N, 64 16-bit elements = 128 bytes of K per row): a "piece" of
//    64 K-elements holds the tile's rows at 128-byte pitch; 8-row groups are 1024 bytes apart
//    (stride byte offset 1024). One K=16 step is 32 bytes further along the row.
//  * MN-major (64 MN-elements = 128 bytes per K row): K rows at 128-byte pitch, 8-row groups
//    1024 bytes apart (stride byte offset), consecutive 64-element MN blocks `lbo` bytes apart
//    (leading byte offset). One K=16 step is 16 rows = 2048 bytes further.
#pragma once

#include <stdint.h>

namespace pd {
namespace tc {

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::f16 instruction descriptor: f32 accumulator, A and B both bf16 (or both f16).
__host__ __device__ constexpr uint32_t instr_desc_f16(bool bf16, int m, int n, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// ---- TMEM allocation (warp-collective; the allocated base address is written to smem)
__device__ __forceinline__ void tmem_alloc(uint32_t smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_dst), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---- ordering of tcgen05 operations around thread synchronisation
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- D[tmem] (+)= A[smem] * B[smem], issued by one thread
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

// ---- D[tmem] (+)= A[tmem] * B[smem], issued by one thread. A (M = 128 rows, K-major) sits in
// TMEM lanes 0..127, its K elements packed two 16-bit values per 32-bit column, the lower K
// index in the low half; one K = 16 step is 8 columns.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

// The mbarrier receives one arrival once every tcgen05.mma this thread issued before has
// completed (its TMEM results written, its shared-memory operands read).
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// ---- TMEM <-> registers, 32 lanes x 32 columns of 32 bits (warp-collective): thread t of the
// warp reads/writes lane (taddr.lane + t), columns taddr.col .. +31.
__device__ __forceinline__ void ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),
      "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 4 columns (thread t writes lane taddr.lane + t, columns taddr.col .. +3).
__device__ __forceinline__ void st_32x32b_x4(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace tc
}  // namespace pd
