// eg_tc.cuh -- tcgen05 building blocks (sm_100a): tensor-memory allocation,
// shared-memory matrix descriptors, the kind::i8 MMA, its commit, and the
// tensor-memory loads of the epilogue.  Inline PTX only.
#pragma once
#include <stdint.h>

#include "eg_device.cuh"

namespace eg {

__device__ __forceinline__ unsigned long long tc_clock_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t)::"memory");
  return t;
}

constexpr uint32_t kTcWaitHintNs = 500;
// Bounded mbarrier phase wait with a short suspend-time hint: completions that
// come from the tensor core (tcgen05.commit) do not always wake a thread
// suspended with a hint, so these waits poll (try_wait's own short
// implementation-defined suspension).  false = gave up (error recorded or
// seen), after about as long as mbar_wait.
__device__ __forceinline__ bool mbar_try_nohint(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(a), "r"(parity), "r"(kTcWaitHintNs)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_test(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(a), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t a = smem_addr(bar);
  if (mbar_test(a, parity)) return true;  // already complete: no suspension
  const unsigned long long t0 = tc_clock_ns();
  for (long long i = 0;; i++) {
    if (mbar_try_nohint(a, parity)) return true;
    if ((i & 1023) == 1023) {
      if (err_set(err)) return false;
      if (tc_clock_ns() - t0 > 2000000000ull) {  // 2 s
        atomicExch(err, 1);
        return false;
      }
    }
  }
}
__device__ __forceinline__ bool tc_wait_bounded(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  const unsigned long long t0 = tc_clock_ns();
  while (!mbar_try_nohint(a, parity))
    if (tc_clock_ns() - t0 > 2000000000ull) return false;
  return true;
}

// Tensor memory: allocated by one whole warp, the base column address is
// written to shared memory; the allocating warp also frees it.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes made visible to the tensor core
// (async proxy) before the writer signals the MMA issuer.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes (rows 16 B apart); lbo = byte distance between core
// matrices adjacent along K, sbo = between core matrices adjacent along
// M / N.  Bits: start >> 4 [0,14), lbo >> 4 [16,30), sbo >> 4 [32,46),
// descriptor version 1 at [46,48), base offset 0, layout 0 (no swizzle).
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t lbo, uint32_t sbo) {
  const uint64_t a = (smem_addr(p) >> 4) & 0x3FFF;
  return a | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) | ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) |
         (1ull << 46);
}

// Instruction descriptor of tcgen05.mma kind::i8: D s32, A unsigned 8-bit,
// B signed 8-bit, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4)                          // D format s32
         | (0u << 7)                        // A: unsigned 8-bit
         | (1u << 10)                       // B: signed 8-bit
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// D[taddr] (+)= A(smem) * B(smem)^T, one instruction issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t taddr, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(taddr),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}
// The mbarrier completes once every MMA this thread issued so far is done.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace eg
