// Fifth-generation tensor-core (tcgen05) helpers for sm_100a: tensor-memory allocation,
// shared-memory matrix descriptors (128-byte-swizzled K-major, and the 32-byte-based
// swizzle for MN-major tf32), the single-
// thread MMA issue, its completion through an mbarrier (bounded wait), and the warp-wide
// tensor-memory load of an accumulator row.
//
// Layout conventions used by the callers:
//   * A (M x K) and B (N x K) operand tiles are fp32 (read as tf32), K-major: one row of
//     32 floats (128 bytes) per M / N index, 8-row atoms of 1024 bytes, the 16-byte chunk
//     c of row r stored at chunk position c ^ (r & 7). Tiles start on 1024-byte boundaries.
//     One MMA consumes 8 K values (32 bytes); K slice k starts 32 k bytes into the row.
//   * MN-major tf32 operands (the transposed reading: rows are K indices, 32 M / N values
//     per 128-byte row) use the 128-byte swizzle on a 32-byte base instead: the 32-byte
//     granule g of row r stored at granule position g ^ (r & 3), 4-row atoms of 512 bytes
//     (sw128_32b). One MMA consumes 8 rows (8 K values, 1024 bytes) per 32 M / N values.
//     This is the only shared-memory layout the tensor cores read MN-major for tf32.
//   * M = 64 accumulators (cta_group::1): row m lives in tensor-memory lane
//     (m % 16) + 32 (m / 16), column n in column n. Warp w may read lanes 32 w .. 32 w + 31,
//     so rows 16 w .. 16 w + 15 are read by lanes 0..15 of warp w.
#pragma once

#include <cstdint>

namespace semx {
namespace tc {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of the 16-byte chunk `c` (0..7) of row `r` in a 128-byte-swizzled tile.
__host__ __device__ __forceinline__ int sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Shared-memory descriptor of a K-major, 128-byte-swizzled operand starting at `addr`
// (the start of the K slice; the tile itself 1024-byte aligned): leading-byte offset 16
// (unused by swizzled K-major layouts), stride-byte offset 1024 (between 8-row atoms),
// descriptor version 1, swizzle mode 2 (128 bytes).
__device__ __forceinline__ uint64_t desc_sw128_kmajor(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Byte offset of column `c` (0..31, fp32) of row `r` in a tile of the 32-byte-based 128-byte
// swizzle (MN-major tf32 operands).
__host__ __device__ __forceinline__ int sw128_32b(int r, int c) {
  return r * 128 + (((c >> 3) ^ (r & 3)) << 5) + 4 * (c & 7);
}

// Shared-memory descriptor of an MN-major tf32 operand in the 32-byte-based 128-byte
// swizzle (layout type 1): `addr` is the start of its first 4-row K group (512-byte
// aligned), the next 32 M / N values start `mn_stride` bytes further (leading-byte offset),
// the next 4-row K group 512 bytes further (stride-byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t desc_sw128b32_mnmajor(uint32_t addr, uint32_t mn_stride) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((mn_stride >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)(512 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)1 << 61);
}

// Instruction descriptor of kind::tf32 with fp32 accumulation; both operands K-major, or
// both MN-major (`mn_major`).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool mn_major = false) {
  return (1u << 4)            // accumulator format: f32
         | (2u << 7)          // A format: tf32
         | (2u << 10)         // B format: tf32
         | (mn_major ? (1u << 15) | (1u << 16) : 0u)  // A, B major-ness
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Tensor-memory allocation of `ncols` columns (a power of two >= 32) by one whole warp;
// the address is written to the shared-memory word `slot`.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
// Makes this thread's generic-proxy shared-memory writes visible to the tensor cores.
__device__ __forceinline__ void fence_smem_to_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

// D (tensor memory) [+]= A (smem) x B (smem)^T, one instruction, issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}

// Arrives on `bar` once every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_addr(bar))
               : "memory");
}

// Waits for the completion of phase `parity` of `bar`, at most `limit` polls; false on
// timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit) {
  const uint32_t a = smem_addr(bar);
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// 32 consecutive fp32 columns of this thread's tensor-memory lane (whole warp). The load
// and its completion wait are one asm statement, so no use of the values can be scheduled
// before the wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace tc
}  // namespace semx
