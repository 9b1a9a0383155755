// tkb_common.cuh -- sm_100a building blocks shared by the tokamak_b200 kernels:
// mbarriers with bounded waits, TMA tensor loads, tcgen05 (UMMA + TMEM)
// wrappers, bf16 packing.  Everything here is inline PTX written for sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define TKB_DEVFN __device__ __forceinline__

namespace tkb {

// ---------------------------------------------------------------- errors
// Device-side error word.  Kernels OR a code into it when a bounded wait
// gives up; the host reads it with tkb_device_error().  Defined here: the
// library is one translation unit (tkb_all.cu).
__device__ unsigned int g_device_error = 0;

enum : unsigned int {
  ERR_WAIT_TIMEOUT = 1u << 0,   // an mbarrier wait ran past its time limit
  ERR_BAD_LAUNCH   = 1u << 1,   // a kernel saw inconsistent launch arguments
};

// Upper bound for any single mbarrier wait.  A correct pipeline never gets
// near it; a wrong one ends with an error code instead of a hung GPU.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

TKB_DEVFN uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

TKB_DEVFN unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
TKB_DEVFN void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

TKB_DEVFN void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

TKB_DEVFN void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

TKB_DEVFN void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

TKB_DEVFN bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed.  Gives up after
// kWaitLimitNs or when *abort becomes non-zero; returns false in that case
// after recording the code in g_device_error and raising *abort so that the
// other roles of the CTA stop waiting as well.
TKB_DEVFN bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(a, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitLimitNs) {
      atomicOr(&g_device_error, ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
  }
}

// The same for a whole warp, with one result for every lane: a wait that
// gives up in one lane gives up in all of them.  The tcgen05.ld / st that
// follow a wait in the compute warps are warp-collective (.sync.aligned) and
// must be executed by every lane of the warp or by none.
TKB_DEVFN bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
}

// The same with a caller-chosen limit (the self-test of the timeout path).
TKB_DEVFN bool mbar_wait_limit(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                               unsigned long long limit_ns) {
  const uint32_t a = smem_u32(bar);
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(a, parity)) {
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit_ns) {
      atomicOr(&g_device_error, ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- TMA
TKB_DEVFN void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 3-D tiled load (x innermost).  x * element size must be a multiple of 16 B.
TKB_DEVFN void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y, int z,
                           uint64_t cache_policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(cache_policy)
      : "memory");
}

// 2-D tiled load (x innermost).  x * element size must be a multiple of 16 B.
TKB_DEVFN void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Plain bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
TKB_DEVFN void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// The same with an L2 cache policy (createpolicy).
TKB_DEVFN void bulk_load_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t cache_policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(cache_policy)
      : "memory");
}

// 16-byte global store with an L2 cache policy.
TKB_DEVFN void st_global_hint(void* gaddr, uint4 v, uint64_t cache_policy) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(gaddr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w), "l"(cache_policy)
               : "memory");
}

// 16-byte streaming accesses: a load that does not allocate in L1 (read-only
// data), a store marked evict-first (written once, not read back soon).
TKB_DEVFN uint4 ld_stream_v4(const uint4* gaddr) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(gaddr));
  return r;
}
TKB_DEVFN void st_stream_v4(uint4* gaddr, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(gaddr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

TKB_DEVFN uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
TKB_DEVFN uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

TKB_DEVFN void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
TKB_DEVFN void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
TKB_DEVFN void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
TKB_DEVFN void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
TKB_DEVFN void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
TKB_DEVFN void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 "version 1").
//   bits  0-13 start address >> 4, 16-29 leading byte offset >> 4,
//   32-45 stride byte offset >> 4, 46-47 version = 1, 61-63 layout = 2 (SW128).
TKB_DEVFN uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Shared-memory matrix descriptor without swizzle: the operand is made of
// 8 x 16-byte core matrices (128 contiguous bytes each); lbo is the byte
// distance between core matrices adjacent along K, sbo along M/N.
TKB_DEVFN uint64_t sdesc_interleave(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  return d;
}

// Instruction descriptor for tcgen05.mma kind::f16 with an fp32 accumulator.
//   bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format (0 f16, 1 bf16),
//   15 A MN-major, 16 B MN-major, 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16kind(int M, int N, bool bf16, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// D(tmem) = A(smem) * B(smem) (+ D when accumulate != 0).  Issued by one thread.
TKB_DEVFN void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D(tmem) = A(tmem) * B(smem) (+ D).  A is M lanes x K columns, 2 elements per column.
TKB_DEVFN void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once every tcgen05 operation issued so far by this thread completes.
TKB_DEVFN void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
TKB_DEVFN void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
TKB_DEVFN void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
}
// 16 consecutive 32-bit columns of this warp's 32 lanes (r[0..15]).
TKB_DEVFN void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
TKB_DEVFN void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
TKB_DEVFN void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
TKB_DEVFN void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- CTA pairs (clusters of 2)
TKB_DEVFN uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
TKB_DEVFN uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
TKB_DEVFN void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (shared::cluster address).
TKB_DEVFN void mbar_arrive_remote(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
TKB_DEVFN bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// mbar_wait for a barrier that other CTAs of the cluster arrive on (acquire at cluster scope).
TKB_DEVFN bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait_cluster(a, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait_cluster(a, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitLimitNs) {
      atomicOr(&g_device_error, ERR_WAIT_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
  }
}
// 2-D tiled load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (bar: shared::cluster address).
TKB_DEVFN void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster_addr, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.cta_group::2"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar_cluster_addr)
      : "memory");
}
// TMEM allocation shared by a CTA pair: one warp of each CTA executes it.
TKB_DEVFN void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
TKB_DEVFN void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
TKB_DEVFN void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D(tmem of both CTAs) = A (rows split over the pair) * B (columns split over the pair).
TKB_DEVFN void umma_pair_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at this shared-memory offset in every CTA of `mask`
// once the pair's tcgen05 operations issued so far complete.
TKB_DEVFN void umma_pair_commit(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// ---------------------------------------------------------------- math
TKB_DEVFN float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
TKB_DEVFN float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Three-input maximum (one instruction on sm_100).
TKB_DEVFN float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two fp32 lanes in one 64-bit register pair (lo in bits 0-31), operated on by
// the packed f32x2 instructions of sm_100: one issue slot for two results.
TKB_DEVFN uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
TKB_DEVFN void f2_split(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
TKB_DEVFN uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
TKB_DEVFN uint64_t add_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
TKB_DEVFN uint64_t mul_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
TKB_DEVFN uint64_t sub_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x of two lanes on the FMA pipe (no MUFU): x = n + f with n = rint(x) taken
// from the low mantissa bits of x + 1.5*2^23, f in [-1/2, 1/2]; 2^f by a
// degree-3 polynomial with p(0) = 1 fitted here (Lawson-reweighted least
// squares on Chebyshev nodes) to a relative error of 1.02e-4, below half an
// ulp of bf16 (2^-9) and of f16 (2^-11); the result is p with n added to its
// exponent field.  Inputs are clamped at -125 so that the exponent stays
// normal: 2^-125 in place of a smaller value or of 0 (a masked -inf) is
// below 1e-37 in a sum whose largest term is at least 1.
TKB_DEVFN void ex2_poly_f2(float x0, float x1, float& y0, float& y1) {
  const uint64_t x = f2(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t magic = f2(12582912.f, 12582912.f);
  const uint64_t t = add_f2(x, magic);
  const uint64_t f = sub_f2(x, sub_f2(t, magic));
  uint64_t p = fma_f2(f2(0.05500893f, 0.05500893f), f, f2(0.24221095f, 0.24221095f));
  p = fma_f2(p, f, f2(0.6932829f, 0.6932829f));
  p = fma_f2(p, f, f2(1.f, 1.f));
  float p0, p1, t0, t1;
  f2_split(p, p0, p1);
  f2_split(t, t0, t1);
  y0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  y1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// Pack two floats into one 32-bit word of 16-bit values, lo in bits 0-15.
template <bool BF16>
TKB_DEVFN uint32_t pack2(float lo, float hi) {
  uint32_t r;
  if constexpr (BF16) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  } else {
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  }
  return r;
}

// The same pack kept off the XU pipe.  The f32 -> bf16x2 conversion issues
// on the XU pipe, as ex2 does, and the attention forward's softmax phase
// keeps that pipe 86 % busy (ncu); packing P on the integer pipes made the
// forward 3-7 % faster (same-box A/B), while the dK/dV kernel, whose integer
// pipe is busier, ran 2-5 % slower with it and keeps cvt.  For bf16 this
// rounds on the integer pipes: add half of the dropped
// range (0x8000) to each float's bits and keep the high halves (one byte
// permute per pair).  That is round-to-nearest with ties away from zero in
// magnitude; it differs from cvt.rn only when the dropped 16 bits are
// exactly 0x8000 and the kept part is even (1 in 65536 of arbitrary values),
// by one bf16 ulp.  Finite inputs only (P in [0, 1]).  f16 keeps cvt.rn.
template <bool BF16>
TKB_DEVFN uint32_t pack2_int(float lo, float hi) {
  if constexpr (BF16) {
    const uint32_t a = __float_as_uint(lo) + 0x8000u, b = __float_as_uint(hi) + 0x8000u;
    return __byte_perm(a, b, 0x7632);
  } else {
    return pack2<false>(lo, hi);
  }
}
template <bool BF16>
TKB_DEVFN float2 unpack2(uint32_t v) {
  if constexpr (BF16) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
  } else {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
  }
}

TKB_DEVFN void red_add_v4(float* gaddr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(gaddr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

TKB_DEVFN int warp_id() { return threadIdx.x >> 5; }
TKB_DEVFN int lane_id() { return threadIdx.x & 31; }

}  // namespace tkb
