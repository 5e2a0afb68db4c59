// tcgen05 (5th-generation tensor core) helpers for sm_100a: TMEM allocation,
// shared-memory matrix descriptors, the kind::f16 MMA, commit to an
// mbarrier and TMEM loads (each wrapper one PTX instruction, the loads with
// their completion wait).
#pragma once
#include "q35_dev.cuh"

namespace q35 {

// Shared-memory matrix descriptor, K-major with the 128-byte swizzle: 8-row
// atoms of 1024 bytes (row r of an atom at 128 r, its 16-byte chunk c at
// chunk c ^ r), atoms `sbo` bytes apart; the atom base must be 1024-byte
// aligned, and a K step of 16 elements advances the start by 32 bytes.
// Layout type 2 (SWIZZLE_128B) at bits [61,64).
Q35_DEV uint64_t tc_desc_sw128(uint32_t saddr, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3fffu) | (uint64_t(1) << 16) | (uint64_t((sbo >> 4) & 0x3fffu) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Shared-memory matrix descriptor, MN-major with the 128-byte swizzle: each
// 128-byte line holds 64 consecutive M/N elements of one K index, 8 lines (K
// indices) form a 1024-byte atom (chunk c of line r at chunk c ^ r), atoms of
// consecutive K groups `sbo` bytes apart and of consecutive 64-element M/N
// blocks `lbo` bytes apart; a K step of 16 advances the start by 2 atoms.
Q35_DEV uint64_t tc_desc_sw128_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3fffu) | (uint64_t((lbo >> 4) & 0x3fffu) << 16) |
         (uint64_t((sbo >> 4) & 0x3fffu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Byte offset of 16-byte chunk c (elements 8c..8c+7 of the 64-wide K block)
// of row r in a 128-byte-swizzled K-major tile.
__host__ __device__ inline uint32_t sw128_off(int r, int c) {
  return uint32_t((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Instruction descriptor of kind::f16 with bf16 A and B, f32 accumulator,
// both operands K-major: c_format [4,6) = 1, a_format [7,10) = 1, b_format
// [10,13) = 1, N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t tc_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// One warp (all lanes) allocates `cols` TMEM columns (power of two >= 32);
// the address lands in *dst (shared memory).
Q35_DEV void tc_alloc(uint32_t* dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
Q35_DEV void tc_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
Q35_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
Q35_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
Q35_DEV void tc_mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on *bar when every tcgen05 operation this thread issued so far
// has completed.
Q35_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// Warp-collective load of 8 consecutive f32 columns for the warp's 32 lanes
// (lane l of warp w reads TMEM lane 32 (w % 4) + l), with the completion wait
// in the same statement so no use of v can be scheduled before it.
Q35_DEV void tc_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// Warp-collective load of 32 consecutive f32 columns (same lane mapping);
// the completion wait sits in the same statement, so no use of v can be
// scheduled before it.
Q35_DEV void tc_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace q35
