// Blackwell tensor-core plumbing for sm_100a: mbarriers, TMA tile loads,
// TMEM allocation and tcgen05.mma / tcgen05.ld, as thin inline-PTX wrappers.
#pragma once
#include <cuda.h>  // CUtensorMap

#include "common.cuh"

namespace q3t {

// Polls of an mbarrier before a wait gives up (each try_wait itself blocks
// for a hardware-defined slice); the caller records the timeout and carries on.
constexpr int kMbarPolls = 1 << 20;

Q3T_DEV void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
// make barrier initialisation visible to the async proxy (TMA, tensor cores)
Q3T_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// order this thread's generic-proxy shared-memory writes before later async-proxy reads
Q3T_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

Q3T_DEV void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

// true once the barrier completed phase `parity`; false after kMbarPolls polls
Q3T_DEV bool mbar_wait(uint64_t *bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  for (int i = 0; i < kMbarPolls; i++) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// 2-D TMA tile load (coordinates: x = innermost element index, y = row);
// completion is counted in bytes on `bar`.
Q3T_DEV void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// ---- tensor memory ----
// whole warp; writes the TMEM base address to *slot
Q3T_DEV void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
// whole warp (the allocating one)
Q3T_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
Q3T_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
Q3T_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 or bf16 inputs
// as the instruction descriptor says), f32 accumulate; one thread issues it.
Q3T_DEV void umma_kf16(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  const uint32_t mask = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask)
      : "memory");
}
// arrive on `bar` once every tcgen05.mma this thread issued has completed
Q3T_DEV void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// 3-D TMA tile load (x innermost); out-of-range coordinates read zeros
Q3T_DEV void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// 32 TMEM lanes x 16 consecutive f32 columns
Q3T_DEV void tmem_ld16(uint32_t taddr, float *v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// tcgen05.ld of 32 lanes x 8 columns without the wait; call tmem_wait_ld()
// before reading r
Q3T_DEV void tmem_ld8_async(uint32_t taddr, uint32_t *r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
Q3T_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 TMEM lanes (one per thread of the warp) x 8 consecutive f32 columns
Q3T_DEV void tmem_ld8(uint32_t taddr, float *v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor of a K-major SWIZZLE_128B operand: rows of
// 64 bf16 (128 bytes) with 16-byte chunk c of row r stored at chunk c ^ (r & 7),
// groups of 8 rows 1024 bytes apart; p = the first element of this K step
// (a 1024-byte-aligned atom base plus 32 bytes per K step of 16).
Q3T_DEV uint64_t sw128_desc(const void *p) {
  const uint64_t a = smem_addr(p);
  return ((a & 0x3FFFFull) >> 4)           // start address
         | (1ull << 16)                    // leading byte offset (unused by swizzled K-major)
         | ((uint64_t)(1024 >> 4) << 32)   // stride byte offset: 8 rows x 128 B
         | (1ull << 46)                    // descriptor version (Blackwell)
         | (2ull << 61);                   // SWIZZLE_128B
}

// The same for a K-major SWIZZLE_64B operand: rows of 32 16-bit elements
// (64 bytes), 8-row groups 512 bytes apart, 512-byte-aligned atoms.
Q3T_DEV uint64_t sw64_desc(const void *p) {
  const uint64_t a = smem_addr(p);
  return ((a & 0x3FFFFull) >> 4) | (1ull << 16) | ((uint64_t)(512 >> 4) << 32) | (1ull << 46) | (4ull << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16 with fp16 A and B (both
// K-major), f32 D, M x N.
constexpr uint32_t umma_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B (both
// K-major), f32 D, M x N.
constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4)                        // D format f32
         | (1u << 7)                      // A format bf16
         | (1u << 10)                     // B format bf16
         | ((uint32_t)(N >> 3) << 17)     // N / 8
         | ((uint32_t)(M >> 4) << 24);    // M / 16
}

}  // namespace q3t
