// Hand-written inline-PTX wrappers for sm_100a (B200).
//
// Every wrapper here is written from the PTX ISA's published syntax for the
// instruction it emits; none depends on <cuda/ptx>, whose coverage of the
// tcgen05 family differs between CUDA releases (CUDA 12.9 has no
// elect_sync wrapper, for instance).
//
// Waits are bounded: bb_wait() spins on mbarrier.try_wait.parity and gives
// up after kWaitBudgetNs of %globaltimer time, recording a status code in a
// device word that the host reads after the launch. A kernel whose wait gave
// up drains its own copies (bounded), frees its TMEM and returns, so the
// context stays usable; nothing here traps.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace bb {

// Status codes shared by every kernel's device status word and by the C ABI.
enum : int {
  kDevOk = 0,
  kDevTimeoutProducer = 0x101,
  kDevTimeoutMma = 0x102,
  kDevTimeoutEpilogue = 0x103,
  kDevTimeoutConsumer = 0x104,
  kDevTimeoutProbe = 0x105,
  kDevTimeoutTest = 0x106,
  kDevBadLaunch = 0x200,
};

// Two seconds of wall time per individual wait. A healthy wait in any kernel
// of this library lasts microseconds; a wait this long means a lost arrival.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;
// A waiting thread reads the shared abort word (a global load) at most once
// per kAbortPollNs of waiting. Every waiting warp of every CTA polls the same
// word, so frequent reads keep one L2 slice busy with them, and that slice
// also serves its share of the operand tiles the kernels stream.
constexpr uint64_t kAbortPollNs = 20000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint64_t clock64_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(t)::"memory");
  return t;
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(r));
  return r;
}

// elect.sync over the full warp: true in exactly one lane.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- cluster
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Map a shared::cta address of this CTA to the same offset in CTA `rank`
// of the cluster (a shared::cluster address).
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t addr, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(addr), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_inval(uint32_t addr) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(addr) : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init_cluster() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Orders this thread's earlier generic-proxy view of global memory (e.g.
// data published by other CTAs and acquired here) before its later
// async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t addr) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(addr) : "memory");
}
// Arrive on an mbarrier given by a shared::cluster address (own or peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// Relaxed variant: for hand-offs whose only payload was already completed by
// the arriving thread (TMEM reads finished by tcgen05.wait::ld); a
// cluster-scope release arrive measured ~1300 clocks per hand-off here.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(addr), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Same, with a suspend-time hint: a thread whose phase is not complete yet
// may sleep in the instruction (up to `hint_ns`) instead of spinning, and
// wakes when the phase completes.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t addr, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait_cluster_hint(uint32_t addr, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Cluster-scope acquire variant, for barriers that peer CTAs arrive on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with parity `parity` to complete. Returns false
// (and records `code` in *status unless a code is already there) when the
// budget runs out. Once *abort_flag is set by another role, waits give up
// immediately so the whole CTA reaches its teardown quickly.
template <bool kClusterScope = false>
__device__ __forceinline__ bool bb_wait(uint32_t addr, uint32_t parity, int* status, int code,
                                        bool honor_abort = true, uint64_t budget_ns = kWaitBudgetNs) {
  auto probe = [&]() {
    return kClusterScope ? mbar_try_wait_cluster(addr, parity) : mbar_try_wait(addr, parity);
  };
  if (probe()) return true;
  const uint64_t t0 = globaltimer_ns();
  uint64_t next_abort_check = t0 + kAbortPollNs;
  uint32_t spins = 0;
  while (true) {
    if (probe()) return true;
    if ((++spins & 31u) == 0) {
      const uint64_t now = globaltimer_ns();
      if (now - t0 > budget_ns) {
        if (status) atomicCAS(status, 0, code);
        return false;
      }
      if (honor_abort && status && now >= next_abort_check) {
        if (*reinterpret_cast<volatile int*>(status) != 0) return false;
        next_abort_check = now + kAbortPollNs;
      }
    }
  }
}

// Warp-wide bounded wait: every lane of the (converged) warp polls with a
// 1 ms suspend hint; lane 0's outcome is returned to all lanes, so loops
// around it stay warp-uniform. Issue loops built this way (whole warp waits,
// one elect.sync lane issues) keep tcgen05 issue well ahead of execution; a
// lone lane looping inside a divergent branch issues markedly slower.
// kHint = false polls without the suspend hint (lowest wake-up latency, for
// waits on the critical path of a tight hand-off).
template <bool kClusterScope = false, bool kHint = true>
__device__ __forceinline__ bool bb_wait_warp(uint32_t addr, uint32_t parity, int* status, int code,
                                             bool honor_abort = true, uint64_t budget_ns = kWaitBudgetNs) {
  constexpr uint32_t kHintNs = 1000000u;
  auto probe = [&]() {
    if constexpr (kHint) {
      return kClusterScope ? mbar_try_wait_cluster_hint(addr, parity, kHintNs) : mbar_try_wait_hint(addr, parity, kHintNs);
    } else {
      return kClusterScope ? mbar_try_wait_cluster(addr, parity) : mbar_try_wait(addr, parity);
    }
  };
  bool ok = probe();
  if (!ok) {
    // The budget and the abort word (a global load) are checked every 8th
    // probe only: a phase that completes during those checks is seen late.
    const uint64_t t0 = globaltimer_ns();
    uint64_t next_abort_check = t0 + kAbortPollNs;
    uint32_t spins = 0;
    while (true) {
      if (probe()) {
        ok = true;
        break;
      }
      if ((++spins & 7u) == 0) {
        const uint64_t now = globaltimer_ns();
        if (now - t0 > budget_ns) {
          if (status && (threadIdx.x % 32) == 0) atomicCAS(status, 0, code);
          break;
        }
        if (honor_abort && status && now >= next_abort_check) {
          if (*reinterpret_cast<volatile int*>(status) != 0) break;
          next_abort_check = now + kAbortPollNs;
        }
      }
    }
  }
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// Sleep for about `ns` nanoseconds (bounded drain for copies in flight).
__device__ __forceinline__ void bounded_sleep_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < ns) __nanosleep(1000);
}

// ---------------------------------------------------------------- cp.async (LDGSTS)
// Untiled bulk copy of `bytes` (a multiple of 16, both addresses 16-byte
// aligned) from global memory into this CTA's shared memory, completing on
// the mbarrier `mbar` of this CTA (this CTA only).
__device__ __forceinline__ void bulk_load_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(mbar)
               : "memory");
}
__device__ __forceinline__ void cp_async_16(uint32_t smem_addr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- TMA
// Rank-2 and rank-3 tiled loads into this CTA's shared memory, completing
// on an mbarrier of this CTA.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t mbar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(mbar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t mbar, int32_t x,
                                            int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(mbar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// CTA-pair form: data lands in this CTA's shared memory, completion is
// signalled on an mbarrier that may live in the peer CTA of the pair
// (`mbar_cluster` is a shared::cluster address). The data goes to this CTA only.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void* tmap, uint32_t mbar_cluster,
                                                 int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(mbar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_store_3d(const void* tmap, uint32_t src, int32_t x, int32_t y,
                                             int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          tmap),
      "r"(src), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// L2 cache policies for the cache-hinted TMA forms below.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_store_2d_hint(const void* tmap, uint32_t src, int32_t x, int32_t y,
                                                  uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
          tmap),
      "r"(src), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------- tcgen05
template <int kCtaGroup>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  if constexpr (kCtaGroup == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
  } else {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
  }
}
template <int kCtaGroup>
__device__ __forceinline__ void tmem_relinquish() {
  if constexpr (kCtaGroup == 1) {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  } else {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
}
template <int kCtaGroup>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  if constexpr (kCtaGroup == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
  } else {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
  }
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (BF16/F16 inputs).
template <int kCtaGroup>
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  if constexpr (kCtaGroup == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Make the mbarrier at `mbar` (shared::cluster address: this CTA's or the
// peer's) track completion of every tcgen05 op this thread issued so far.
// The same MMA keeping A in the tensor core's collector buffer: kFill = true
// reads A from shared memory and keeps it, kFill = false reuses the kept A
// (its descriptor must name the same A) and releases it. Two N = 256 MMAs
// that share A per K step then read A from shared memory once.
template <int kCtaGroup, bool kFill>
__device__ __forceinline__ void umma_f16_keep_a(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  if constexpr (kCtaGroup == 1 && kFill) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16.collector::a::fill [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (kCtaGroup == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16.collector::a::lastuse [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (kFill) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16.collector::a::fill [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16.collector::a::lastuse [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

template <int kCtaGroup>
__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  if constexpr (kCtaGroup == 1) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     mbar)
                 : "memory");
  } else {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     mbar)
                 : "memory");
  }
}

// 32 lanes x 32 columns of 32-bit TMEM cells; lane i of the warp gets row
// (taddr.lane + i), registers r[j] = column (taddr.col + j).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor for tcgen05.mma (sm_100 format):
//   [0,14)  start address >> 4
//   [16,30) leading-dimension byte offset >> 4
//   [32,46) stride-dimension byte offset >> 4
//   [46,48) version = 1
//   [49,52) base offset (0: every tile here is 1024-byte aligned)
//   [52]    LBO mode (0)
//   [61,64) layout: 0 none, 2 swizzle-128B, 4 swizzle-64B, 6 swizzle-32B
enum : uint32_t { kLayoutNone = 0, kLayoutSw128 = 2 };

__host__ __device__ constexpr uint64_t make_smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                      uint32_t layout) {
  return (static_cast<uint64_t>((addr >> 4) & 0x3FFFu)) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
         (static_cast<uint64_t>(layout & 0x7u) << 61);
}

// K-major operand staged by TMA with 128-byte swizzle: rows of 64 BF16
// (128 B), 8-row swizzle atoms of 1024 B stacked along M/N (SBO = 1024).
// LBO is unused for swizzled K-major layouts; 16 B is the customary value.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t addr) {
  return make_smem_desc(addr, 16, 1024, kLayoutSw128);
}

// Instruction descriptor, kind::f16:
//   [4,6) D format (1 = F32); [7,10) A format (1 = BF16); [10,13) B format;
//   [15] A major (0 = K); [16] B major (0 = K); [17,23) N >> 3; [24,29) M >> 4.
__host__ __device__ constexpr uint32_t make_idesc_bf16_f32(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((static_cast<uint32_t>(n) >> 3) << 17) |
         ((static_cast<uint32_t>(m) >> 4) << 24);
}
static_assert(make_idesc_bf16_f32(128, 256) == 0x08400490u, "idesc M=128 N=256");
static_assert(make_idesc_bf16_f32(256, 256) == 0x10400490u, "idesc M=256 N=256");
static_assert(make_idesc_bf16_f32(128, 64) == 0x08100490u, "idesc M=128 N=64");

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ float4 ld_shared_v4f(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

}  // namespace bb
