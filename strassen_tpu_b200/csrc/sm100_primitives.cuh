// sm100_primitives.cuh -- thin inline-PTX wrappers for the Blackwell (sm_100a)
// features the Strassen kernel uses: mbarriers, TMA tile loads, tcgen05
// (TMEM allocation, UMMA issue, commit, TMEM loads) and bf16x2 arithmetic.
//
// Every wait here is bounded: it polls with mbarrier.try_wait and gives up
// after kWaitTimeoutNs of %globaltimer, recording an error code for the host
// instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace sb {

constexpr uint64_t kWaitTimeoutNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (after
// raising *abort_flag and recording `code` in *err) on timeout, or when another
// thread of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int code) {
  uint64_t start = 0;
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort_flag) return false;
      const uint64_t now = global_timer_ns();
      if (start == 0) {
        start = now;
      } else if (now - start > kWaitTimeoutNs) {
        *abort_flag = 1;
        atomicExch(err, code);
        return false;
      }
    }
  }
}

// try_wait with an explicit suspend-time hint (ns): a thread whose phase is not
// yet complete sleeps until it completes or the hint expires, instead of the
// system default, which measured slower on B200 for waits that usually succeed
// within a few hundred cycles.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}

// Bounded wait built on mbar_try_wait_hint; same give-up rule as mbar_wait (the
// clock is read every 8 tries because each try may sleep up to 20 us).
__device__ __forceinline__ bool mbar_wait_hint(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                               int* err, int code) {
  if (mbar_try_wait_hint(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_hint(bar, parity)) return true;
    if ((it & 7u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - start > kWaitTimeoutNs) {
        *abort_flag = 1;
        atomicExch(err, code);
        return false;
      }
    }
  }
}

// Named barrier `id` over `count` threads (whole warps) that also ORs a
// predicate across them.  Used to hand a step from a waiting warp to the MMA
// warp: a tcgen05.mma issuer that itself polls an mbarrier (or any shared
// memory word) stalls until its queued MMAs have been accepted, which idles the
// tensor pipe for ~350 cycles per wait on B200; a named barrier does not.
__device__ __forceinline__ bool named_bar_red_or(uint32_t id, uint32_t count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}\n"
      : "=r"(out)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

// Warp-uniform bounded wait: lane 0 polls, the verdict is broadcast, and on
// success every lane observes the completed phase itself (so each lane's later
// reads are ordered after the barrier).  The phase cannot advance in between
// because the caller's own arrival gates the next one.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int code) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) {
    for (uint32_t it = 0; it < (1u << 20) && !mbar_try_wait(bar, parity); ++it) {
    }
  }
  return ok != 0;
}

// Bounded wait that ignores the abort flag (used to drain in-flight async work
// before teardown).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
  uint64_t start = 0;
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      const uint64_t now = global_timer_ns();
      if (start == 0) start = now;
      else if (now - start > kWaitTimeoutNs) return false;
    }
  }
}

// ---------------------------------------------------------------- fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- TMA loads
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3,
                                            int32_t c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
template <uint32_t kCols>
__device__ __forceinline__ void tmem_alloc(uint32_t holder_smem) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder_smem),
               "r"(kCols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

template <uint32_t kCols>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(kCols)
               : "memory");
}

// UMMA shared-memory matrix descriptor (tcgen05 "matrix descriptor" format):
// start address (>>4) in bits [0,14), leading byte offset (>>4) in [16,30),
// stride byte offset (>>4) in [32,46), version 1 in [46,48), base offset 0,
// LBO mode 0, swizzle/layout type in [61,64).
enum : uint32_t {
  kLayoutSwizzleNone = 0,
  kLayoutSwizzle128B = 2,
  kLayoutSwizzle64B = 4,
  kLayoutSwizzle32B = 6,
};

__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t saddr, uint32_t lbo_bytes,
                                                   uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and an f32 accumulator.
// Bits: D format [4,6)=1 (f32); A format [7,10)=1 (bf16); B format [10,13)=1
// (bf16); A major bit 15; B major bit 16 (1 = MN-major); N>>3 in [17,23);
// M>>4 in [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(uint32_t m, uint32_t n, bool a_mn_major,
                                                           bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem], issued by one thread.
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (+)= A * B with A read from TMEM (128 lanes = rows, K/2 32-bit columns of
// packed bf16 pairs, even k in the low half) and B from shared memory.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Each thread writes 8 consecutive 32-bit TMEM columns of its lane (the warp's
// lane quarter); tmem_store_wait() waits for this thread's stores to land.
__device__ __forceinline__ void tmem_store_8(uint32_t taddr, uint4 lo, uint4 hi) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(lo.x), "r"(lo.y), "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
      : "memory");
}
__device__ __forceinline__ void tmem_store_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrive (once) on an mbarrier when all previously issued tcgen05.mma of this
// thread have completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// Load 8 consecutive fp32 TMEM columns of this warp's 32-lane quarter (one lane
// per thread) and wait for completion inside the same asm statement, so no
// consumer of the registers can be scheduled before the data has landed.
__device__ __forceinline__ void tmem_load_8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- bf16x2 math
// Exact sum / difference rounded once to bf16 (round-to-nearest-even), the
// same rounding as the reference's bf16 pre-adds (x.astype(bf16) + y.astype(bf16)).
__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// x * 0.5 and x * 0.25 on bf16x2 (exact: the power-of-two formula's scalings).
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint4 half4(uint4 a) {
  const uint32_t h = 0x3F003F00u;  // (0.5, 0.5)
  return make_uint4(bf16x2_mul(a.x, h), bf16x2_mul(a.y, h), bf16x2_mul(a.z, h), bf16x2_mul(a.w, h));
}
__device__ __forceinline__ uint4 quarter4(uint4 a) {
  const uint32_t q = 0x3E803E80u;  // (0.25, 0.25)
  return make_uint4(bf16x2_mul(a.x, q), bf16x2_mul(a.y, q), bf16x2_mul(a.z, q), bf16x2_mul(a.w, q));
}
__device__ __forceinline__ uint4 add4(uint4 a, uint4 b) {
  return make_uint4(bf16x2_add(a.x, b.x), bf16x2_add(a.y, b.y), bf16x2_add(a.z, b.z),
                    bf16x2_add(a.w, b.w));
}
__device__ __forceinline__ uint4 sub4(uint4 a, uint4 b) {
  return make_uint4(bf16x2_sub(a.x, b.x), bf16x2_sub(a.y, b.y), bf16x2_sub(a.z, b.z),
                    bf16x2_sub(a.w, b.w));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------- clusters
// Distributed shared memory between the CTAs of a thread-block cluster: plain
// remote stores, remote mbarrier arrivals and shared-to-shared bulk copies.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of `local` (a shared::cta address) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

// Every thread of every CTA of the cluster: release own writes, wait for all.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

// Arrive on an mbarrier in another CTA of the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_remote_arrive(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait with cluster-scope acquire, for phases completed by arrivals
// from another CTA whose prior writes (into this CTA's shared memory) must be
// visible afterwards.  Same give-up rule as mbar_wait.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                  int* err, int code) {
  uint64_t start = 0;
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort_flag) return false;
      const uint64_t now = global_timer_ns();
      if (start == 0) {
        start = now;
      } else if (now - start > kWaitTimeoutNs) {
        *abort_flag = 1;
        atomicExch(err, code);
        return false;
      }
    }
  }
}

// Copy `bytes` (a multiple of 16, both addresses 16-byte aligned) from this
// CTA's shared memory into another CTA's; completion is signalled as
// transaction bytes on the destination CTA's mbarrier `mbar_cluster`.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                  uint32_t mbar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(mbar_cluster)
      : "memory");
}

__device__ __forceinline__ void st_cluster_f32x4(uint32_t cluster_addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__device__ __forceinline__ float4 lds_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace sb
