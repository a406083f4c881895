// frc_umma.cuh - 5th-generation tensor core (tcgen05) building blocks for sm_100a.
//
// Operands live in shared memory in the K-major, no-swizzle canonical layout:
// a "core matrix" is 8 rows x 16 bytes stored as 128 contiguous bytes.  For
// an R x K int8 tile kept as [R/8][K/16] core matrices, element (r, k) is at
//
//   (r / 8) * sbo + (k / 16) * 128 + (r % 8) * 16 + k % 16,   sbo = 8 * K bytes,
//
// so one MMA step of K = 32 reads two core matrices 128 bytes apart (lbo) per
// 8-row group, and the next step starts 256 bytes further.  Accumulators are
// int32 in tensor memory: with M = 128, row m of D is TMEM lane m and column n
// of D is column base + n.
#pragma once
#include <stdint.h>

namespace frc {

// Byte offset of element (r, k) of an int8 tile of row length K in the layout above.
__host__ __device__ constexpr unsigned umma_off(unsigned r, unsigned k, unsigned K) {
  return (r >> 3) * (8 * K) + (k >> 4) * 128 + (r & 7) * 16 + (k & 15);
}

// Shared-memory matrix descriptor (sm_100 form: version 1 at bits 46-47,
// no swizzle, base offset 0): start address, leading-dimension byte offset
// (K direction) and stride-dimension byte offset (8-row groups), all >> 4.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16 |
         static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32 | 1ull << 46;
}

// Instruction descriptor of kind::i8: D int32 (bits 4-5 = 2), A and B signed
// int8 (bits 7-9 and 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t umma_idesc_i8(unsigned m, unsigned n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// D (+)= A * B^T for one K = 32 step; issued by one thread.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}
// Arrives once on `bar` when every MMA this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
               : "memory");
}

// Tensor-memory allocation (whole warp): the base address lands in *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, unsigned ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, unsigned ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 4 consecutive 32-bit columns of this thread's lane into r[0..3].
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
}

// 8 consecutive 32-bit columns of this thread's lane into r[0..7].
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

// 16 consecutive 32-bit columns of this thread's lane (warp w % 4 reads lanes
// 32 (w % 4) .. 32 (w % 4) + 31; taddr carries that lane base in bits 16-31).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

}  // namespace frc
