// ks_tmem.cuh -- Tensor Memory (TMEM) as per-thread accumulator storage.
//
// Each SM of sm_100a has 256 KB of TMEM (128 lanes x 512 columns of 32 bits),
// built for tcgen05.mma accumulators.  Kernels that keep many accumulators
// per thread park them there instead of in registers: warp w of a warpgroup
// may address lanes [32 (w % 4), 32 (w % 4) + 32), and with the 32x32b access
// shape thread `lane` of the warp reads or writes TMEM lane 32 (w % 4) + lane,
// consecutive columns.  The PTX used here (tcgen05.alloc / dealloc /
// relinquish_alloc_permit, tcgen05.ld / st .32x32b, tcgen05.wait::ld / ::st,
// tcgen05.fence) is the documented sm_100a interface.
#pragma once
#include <cstdint>

namespace ksb {
namespace tmem {

// Allocates n_cols columns (a power of two >= 32) for this CTA; executed by
// one whole warp; the TMEM address lands in *slot (shared memory).  The
// caller guarantees that all CTAs that can be resident on one SM together
// need at most 512 columns, so the allocation never waits.
__device__ __forceinline__ void alloc(uint32_t *slot, uint32_t n_cols) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(slot);
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s),
               "r"(n_cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
// Frees the columns; executed by the warp that allocated them, after every
// thread's last access (fence_before + __syncthreads + fence_after).
__device__ __forceinline__ void dealloc(uint32_t taddr, uint32_t n_cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(n_cols)
               : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// The ld / st / wait wrappers carry no memory clobber: TMEM is not generic
// memory, volatile asm keeps their order among themselves, and the compiler
// stays free to hoist global loads across them.
// 8 consecutive 32-bit columns of this thread's lane -> r (valid after wait_ld).
__device__ __forceinline__ void ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
// Waits for this thread's outstanding tcgen05.ld; the registers of the two
// loads are tied to the wait so no use of them is scheduled before it.
__device__ __forceinline__ void wait_ld(uint32_t (&a)[8], uint32_t (&b)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]),
                 "+r"(a[6]), "+r"(a[7]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]),
                 "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]));
}
// Waits for this thread's outstanding tcgen05.ld into one register block.
__device__ __forceinline__ void wait_ld(uint32_t (&a)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]),
                 "+r"(a[6]), "+r"(a[7]));
}
__device__ __forceinline__ void st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(
                   taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
               "r"(r[7]));
}
// Waits until this thread's tcgen05.st have completed.
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;"); }

__device__ __forceinline__ uint64_t pack(uint32_t lo, uint32_t hi) {
  return (uint64_t)lo | ((uint64_t)hi << 32);
}

}  // namespace tmem
}  // namespace ksb
