// tcgen05 building blocks (sm_100a): shared-memory matrix descriptors, the instruction descriptor of a
// bf16 x bf16 -> fp32 MMA, TMEM allocation, MMA issue and commit, TMEM loads, mbarrier waits with an
// iteration limit, and the fences between the generic and async proxies.  Written from the PTX ISA's
// description of tcgen05 (the 5th-generation tensor core instructions); the descriptor bit layouts follow
// the ISA's "shared memory descriptor" and "instruction descriptor" tables.
#pragma once

#include <stdint.h>

namespace gl {

// Shared-memory matrix descriptor, 128-byte swizzle, for a tile stored as rows of 128 bytes in atoms of
// 8 rows (1024 bytes, 1024-aligned), chunk c of row r at byte 128 r + 16 (c ^ (r & 7)):
//   bits 0-13 start >> 4, 16-29 leading byte offset >> 4, 32-45 stride byte offset >> 4,
//   46-47 version (1 on sm_100), 61-63 layout (2 = 128-byte swizzle).
// K-major operand (rows = M or N, 64 bf16 of K per row): SBO = 1024 between 8-row groups, LBO unused (1).
// MN-major operand (rows = K, 64 bf16 of M or N per row): SBO = 1024 between 8-row K groups, LBO = the
// byte offset between 64-element blocks of M or N.
__device__ __forceinline__ uint64_t t5_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Byte offset of element (row, col) (col < 64, 2-byte elements) in a 128-byte-swizzled tile of 128-byte
// rows (the layout above).
__host__ __device__ __forceinline__ uint32_t t5_sw128_off(uint32_t row, uint32_t col) {
  return row * 128u + ((((col >> 3) ^ (row & 7u)) & 7u) << 4) + ((col & 7u) << 1);
}

// Instruction descriptor of kind::f16 with bf16 A and B, fp32 D: bits 4-5 D format (1 = f32), 7-9 A format
// (1 = bf16), 10-12 B format, 15 / 16 A / B major (0 = K, 1 = MN), 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t t5_idesc_bf16(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t t5_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// TMEM: one warp allocates `ncols` columns (a power of two >= 32) and writes the address to *dst (shared).
__device__ __forceinline__ void t5_tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}

__device__ __forceinline__ void t5_tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// D (TMEM) = A * B (+ D when accumulate != 0), A and B described in shared memory.  One thread issues.
__device__ __forceinline__ void t5_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// D (TMEM) = A * B (+ D), A read from TMEM (rows = the 128 lanes; column c of the A address holds K elements
// 2c and 2c + 1, the even one in the low half), B described in shared memory.  One thread issues.
__device__ __forceinline__ void t5_mma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive on the mbarrier once every MMA this thread issued before has completed.
__device__ __forceinline__ void t5_commit(uint32_t mbar_smem) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar_smem)
               : "memory");
}

__device__ __forceinline__ void t5_fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void t5_fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Generic-proxy shared-memory writes become visible to the tensor cores (async proxy).
__device__ __forceinline__ void t5_fence_smem_to_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void t5_mbar_init(uint32_t mbar_smem, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(mbar_smem), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Wait until the mbarrier's phase with this parity has completed; gives up after `limit` polls and
// returns false (the caller records the timeout and stops issuing work).
__device__ __forceinline__ bool t5_mbar_wait(uint32_t mbar_smem, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(mbar_smem), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (lane i of the warp gets lane base + i); the
// load and its completion wait are one statement, so no use of the registers can move between them.
__device__ __forceinline__ void t5_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
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

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes from registers (lane i of the warp writes lane
// base + i); completion is awaited with t5_wait_st.
__device__ __forceinline__ void t5_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void t5_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// One fp32 column of this warp's 32 TMEM lanes (load and completion wait in one statement, as t5_ld32).
__device__ __forceinline__ float t5_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r)
      : "r"(taddr)
      : "memory");
  return __uint_as_float(r);
}

// 16 fp32 values of this warp's 32 TMEM lanes at 16 columns given by address (taddr[i] = lanes | column),
// with one completion wait for all of them.
__device__ __forceinline__ void t5_ld16_cols(const uint32_t (&a)[16], float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%16];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%1}, [%17];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%2}, [%18];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%3}, [%19];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%4}, [%20];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%5}, [%21];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%6}, [%22];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%7}, [%23];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%8}, [%24];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%9}, [%25];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%10}, [%26];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%11}, [%27];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%12}, [%28];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%13}, [%29];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%14}, [%30];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%15}, [%31];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]), "r"(a[8]),
        "r"(a[9]), "r"(a[10]), "r"(a[11]), "r"(a[12]), "r"(a[13]), "r"(a[14]), "r"(a[15])
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace gl
