// sm_100a primitives used by the tcgen05 kernels: mbarriers with bounded
// waits, TMA tensor loads, tcgen05 TMEM allocation / MMA / commit / loads,
// and the shared-memory matrix descriptors of the 5th-generation tensor cores.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace spatten {
namespace sm100 {

// ---------------------------------------------------------------------------
// Device error word: a kernel whose wait runs out of time records where it gave
// up here (first writer wins) and returns instead of spinning forever. The
// word is static: each translation unit that includes this header
// (prog_attn_tc.cu, qkv_proj.cu, out_proj.cu) has its own and reads it back for
// spatten_device_error().
// ---------------------------------------------------------------------------
static __device__ unsigned int g_device_error = 0;

constexpr long long kWaitLimitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

SPATTEN_DEV void record_error(unsigned int code) { atomicCAS(&g_device_error, 0u, code); }

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
SPATTEN_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
SPATTEN_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
SPATTEN_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
SPATTEN_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
SPATTEN_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete. Returns false (and
// records `code`) if it did not within kWaitLimitCycles, or if `abort` is set.
SPATTEN_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int code,
                           volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    // try_wait suspends the thread for a while by itself; the abort flag and
    // the clock are checked once per batch of polls.
#pragma unroll 1
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      record_error(code);
      *abort = 1;
      return false;
    }
  }
}

// The same operations on an mbarrier named by its shared-memory address: a
// 32-bit handle that is a constant offset from the CTA's shared base, so a
// kernel holding many barriers keeps no 64-bit pointer per barrier live.
struct SBar {
  uint32_t a;
};
struct SBarArr {  // consecutive mbarriers
  uint32_t a;
  SPATTEN_DEV SBar operator[](int i) const { return SBar{a + 8u * (uint32_t)i}; }
};
SPATTEN_DEV void mbar_init(SBar bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar.a), "r"(count));
}
SPATTEN_DEV void mbar_arrive(SBar bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar.a) : "memory");
}
SPATTEN_DEV void mbar_arrive_expect_tx(SBar bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar.a), "r"(bytes)
               : "memory");
}
// One lane of a converged warp (elect.sync) arrives; predicated, so the warp
// takes no divergent branch.
SPATTEN_DEV void mbar_arrive_elect(SBar bar) {
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n"
      " @p mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n}\n" ::"r"(bar.a)
      : "memory");
}
SPATTEN_DEV bool mbar_try_wait(SBar bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar.a), "r"(parity)
      : "memory");
  return ok != 0;
}
SPATTEN_DEV bool mbar_wait(SBar bar, uint32_t parity, unsigned int code, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      record_error(code);
      *abort = 1;
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// proxies and fences
// ---------------------------------------------------------------------------
// generic-proxy shared-memory writes -> visible to the async proxy (MMA, TMA)
SPATTEN_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
SPATTEN_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SPATTEN_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// named barrier over `count` threads (id 1..15)
SPATTEN_DEV void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---------------------------------------------------------------------------
// TMA (no multicast): tiled tensor load into shared memory, completion on an
// mbarrier via complete_tx.
// ---------------------------------------------------------------------------
SPATTEN_DEV void tma_load_4d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}
SPATTEN_DEV void tma_load_4d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                             SBar bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar.a)
      : "memory");
}
SPATTEN_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}
SPATTEN_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation (whole warp), MMA (one thread), commit, loads
// ---------------------------------------------------------------------------
SPATTEN_DEV void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols));
}
SPATTEN_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
SPATTEN_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// D[tmem] (+)= A[smem] * B[smem]^T
SPATTEN_DEV void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
SPATTEN_DEV void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrive on `bar` once every tcgen05 operation issued so far by this thread completes.
SPATTEN_DEV void mma_commit(SBar bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar.a)
      : "memory");
}
SPATTEN_DEV void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t gets lane (base + t).
SPATTEN_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// The same load into fp32 registers (the bits as they are in tensor memory).
SPATTEN_DEV void tmem_ld32f(uint32_t taddr, float* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]),
        "=f"(r[7]), "=f"(r[8]), "=f"(r[9]), "=f"(r[10]), "=f"(r[11]), "=f"(r[12]), "=f"(r[13]),
        "=f"(r[14]), "=f"(r[15]), "=f"(r[16]), "=f"(r[17]), "=f"(r[18]), "=f"(r[19]),
        "=f"(r[20]), "=f"(r[21]), "=f"(r[22]), "=f"(r[23]), "=f"(r[24]), "=f"(r[25]),
        "=f"(r[26]), "=f"(r[27]), "=f"(r[28]), "=f"(r[29]), "=f"(r[30]), "=f"(r[31])
      : "r"(taddr));
}
// 32 lanes x 1 column
SPATTEN_DEV void tmem_ld1(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
}
SPATTEN_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), version 1.
//   K-major operand:  rows of 128 B, 8-row atoms of 1024 B: SBO = 1024, LBO unused.
//   MN-major operand: 128 B along MN per row, 8 rows along K per atom: SBO = stride
//                     between 8-row K groups, LBO = stride between 64-element MN blocks.
SPATTEN_DEV uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // version (sm_100)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::i8 / kind::f16 (dense, no negate, no shift).
//   c_fmt: 1 = F32, 2 = S32; ab_fmt: kind::i8 -> 1 = S8; kind::f16 -> 0 = F16, 1 = BF16
//   a_mn / b_mn: 1 = MN-major operand
__host__ __device__ constexpr uint32_t instr_desc(uint32_t c_fmt, uint32_t ab_fmt, uint32_t a_mn,
                                                  uint32_t b_mn, uint32_t M, uint32_t N) {
  return (c_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (a_mn << 15) | (b_mn << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

}  // namespace sm100
}  // namespace spatten
