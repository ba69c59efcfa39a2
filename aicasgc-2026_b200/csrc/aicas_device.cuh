// Device-side primitives for sm_100a: mbarriers, bulk async copies
// (global -> shared, completed on an mbarrier), bounded waits and a bounded
// software grid barrier.  Every wait here gives up after a time limit or when
// another CTA raised the scratch `abort` word, so a fault never hangs the GPU.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "aicas_phase_program.h"

namespace aicas {

// Error codes written to AicasScratch::error (also returned by the C ABI).
enum : int {
  kErrNone = 0,
  kErrBarrierTimeout = 10,   // grid barrier did not complete in time
  kErrFullTimeout = 11,      // a stage's bulk copy did not land in time
  kErrEmptyTimeout = 12,     // consumers did not release a stage in time
  kErrDrainTimeout = 13,     // in-flight copies did not land before exit
  kErrBadPhase = 14,         // unknown phase kind / bad descriptor
  kErrBadInput = 15,         // token id or cache position out of range
  kErrInputTimeout = 16,     // an LL input vector did not arrive in time
  kErrTmemTimeout = 17,      // a tensor-memory slot hand-off did not complete in time
};

// Wait limit: two seconds of %globaltimer.  Far above any legal phase time
// (a full 28-layer step is ~0.5 ms) and far below a watchdog.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

// Arrive `count` times at once.
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Variants addressed by 32-bit shared-window addresses (kept in registers by
// the hot loops, so a memory clobber never forces them to be reloaded).
__device__ __forceinline__ bool mbar_try_wait_s(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void mbar_arrive_s(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds_u2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// Order this thread's generic-proxy shared-memory writes before later
// async-proxy (bulk copy) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bulk async copy global -> this CTA's shared memory; completes `bytes` of
// transaction count on `bar`.  dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bulk prefetch of [src, src + bytes) into L2 (16-byte aligned, bytes % 16 ==
// 0) with an L2 eviction-priority hint for the prefetched lines.
__device__ __forceinline__ void bulk_prefetch_l2_hint(const void* src, uint32_t bytes, uint64_t policy) {
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(src), "r"(bytes), "l"(policy)
               : "memory");
}

// One 128-byte line into L2 (a hint; no register result).
__device__ __forceinline__ void prefetch_l2_line(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ int ld_volatile_int(const int32_t* p) {
  return *reinterpret_cast<const volatile int32_t*>(p);
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Record the first error and tell every other wait to give up.
__device__ __forceinline__ void raise_error(AicasScratch* s, int code) {
  atomicCAS(&s->error, 0, code);
  atomicExch(&s->abort, 1);
}

// Bounded wait for phase `parity` of `bar`; false on timeout or abort.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, AicasScratch* s, int err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (ld_volatile_int(&s->abort)) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_error(s, err);
        return false;
      }
    }
  }
}

// Bounded wait for a bulk copy this CTA issued from valid memory: the abort
// word does not end it (the copy lands in microseconds either way), so the
// barrier's phases stay in step and no copy is still writing shared memory
// when the CTA moves on or exits.  False only on the time limit.
__device__ __forceinline__ bool mbar_wait_copy(uint64_t* bar, uint32_t parity, AicasScratch* s, int err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_error(s, err);
      return false;
    }
  }
}

// Bounded wait on the mbarrier at shared address `bar` (see mbar_wait_bounded).
__device__ __forceinline__ bool mbar_wait_bounded_s(uint32_t bar, uint32_t parity, AicasScratch* s, int err) {
  if (mbar_try_wait_s(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_s(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (ld_volatile_int(&s->abort)) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_error(s, err);
        return false;
      }
    }
  }
}

// ---- tensor memory (tcgen05) ----------------------------------------------
// TMEM address: lane in bits 31..16, column in bits 15..0.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (K-major, no swizzle: core matrices of 8
// rows x 16 bytes, rows 16 bytes apart; 8-row groups `sbo` bytes apart, the
// two 16-byte halves of a 256-bit row `lbo` bytes apart; version 1).
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// 128 TMEM lanes x 256 bits from shared memory (asynchronous; completion via
// tcgen05_commit).
__device__ __forceinline__ void tcgen05_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// Arrive once on the mbarrier when every tcgen05 operation this thread issued
// before has completed.
__device__ __forceinline__ void tcgen05_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// 32 lanes x 32 columns (the warp's lane quarter): r[i] = column col + i of
// this thread's lane.  Completed by tmem_wait_ld.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// The same straight into 8 uint4 (w[i] = columns 4i..4i+3).
__device__ __forceinline__ void tmem_ld_32x32b_x32_u4(uint32_t taddr, uint4 (&w)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(w[0].x), "=r"(w[0].y), "=r"(w[0].z), "=r"(w[0].w), "=r"(w[1].x), "=r"(w[1].y), "=r"(w[1].z),
        "=r"(w[1].w), "=r"(w[2].x), "=r"(w[2].y), "=r"(w[2].z), "=r"(w[2].w), "=r"(w[3].x), "=r"(w[3].y),
        "=r"(w[3].z), "=r"(w[3].w), "=r"(w[4].x), "=r"(w[4].y), "=r"(w[4].z), "=r"(w[4].w), "=r"(w[5].x),
        "=r"(w[5].y), "=r"(w[5].z), "=r"(w[5].w), "=r"(w[6].x), "=r"(w[6].y), "=r"(w[6].z), "=r"(w[6].w),
        "=r"(w[7].x), "=r"(w[7].y), "=r"(w[7].z), "=r"(w[7].w)
      : "r"(taddr)
      : "memory");
}
// 32 lanes x 2 columns: a = column col, b = column col + 1 of this thread's lane.
__device__ __forceinline__ void tmem_ld_32x32b_x2(uint32_t taddr, uint32_t& a, uint32_t& b) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Software grid barrier over `nct` co-resident CTAs, split into arrive and
// wait so a CTA can do independent work in between.  One thread per CTA
// calls both.  The 64-bit arrival counter only grows (it never wraps and is
// never reset), so barrier k of a launch completes when the counter reaches
// base + (k + 1) * nct, where base = counter at launch start rounded down to
// a multiple of nct (a CTA that reads the counter late can only see fewer than
// nct extra arrivals: barrier 0 cannot complete without it).
__device__ __forceinline__ void red_release_add_u64(uint64_t* p, uint64_t v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Arrival: a release reduction, called by one thread after a CTA-wide
// barrier, so every write the CTA made before the barrier is visible to a
// thread that observes the new count (release is cumulative over the
// writes ordered before it by bar.sync).
__device__ __forceinline__ void grid_arrive(AicasScratch* s) { red_release_add_u64(&s->bar_count, 1ull); }

__device__ __forceinline__ void fence_acquire_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Bounded wait until `target` arrivals (relaxed polling, one acquire fence
// on success); false on timeout or abort.
__device__ __forceinline__ bool grid_wait(AicasScratch* s, uint64_t target) {
  if ((int64_t)(ld_relaxed_u64(&s->bar_count) - target) >= 0) {
    fence_acquire_gpu();
    return true;
  }
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if ((int64_t)(ld_relaxed_u64(&s->bar_count) - target) >= 0) {
      fence_acquire_gpu();
      return true;
    }
    if ((it & 31u) == 0) {
      if (ld_volatile_int(&s->abort)) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_error(s, kErrBarrierTimeout);
        return false;
      }
    }
  }
}

// LL vectors (aicas_phase_program.h): 32-bit words {fp16 value (low), uint16 epoch (high)}.
__device__ __forceinline__ uint4 ll_load4w(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ll_load1w(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void ll_store(uint32_t* p, float value, uint32_t epoch16) {
  const uint32_t v = (epoch16 << 16) | (uint32_t)__half_as_ushort(__float2half_rn(value));
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 64-bit LL words {fp32 value (low), uint32 epoch (high)} (split-KV partials):
// one aligned 64-bit store is single-copy atomic, so a reader that sees the
// epoch also sees the value, with no fence on either side.
__device__ __forceinline__ void ll64_store(uint64_t* p, float value, uint32_t epoch) {
  const uint64_t v = ((uint64_t)epoch << 32) | (uint64_t)__float_as_uint(value);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ll64_load(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ll64_epoch(uint64_t v) { return (uint32_t)(v >> 32); }
__device__ __forceinline__ float ll64_value(uint64_t v) { return __uint_as_float((uint32_t)v); }

__device__ __forceinline__ bool ll_ok(uint4 v, uint32_t e) {
  return (v.x >> 16) == e && (v.y >> 16) == e && (v.z >> 16) == e && (v.w >> 16) == e;
}

// two LL words -> one half2 word (low halves)
__device__ __forceinline__ uint32_t ll_pack(uint32_t lo, uint32_t hi) { return (lo & 0xffffu) | (hi << 16); }

// Bounded poll of the 8 LL words holding values [col, col + 8) (col % 4 == 0
// and the word array 16-byte aligned); returns the 8 fp16 values packed.  On
// timeout or abort the error is recorded and the last read is returned.
__device__ __forceinline__ uint4 ll_poll8(const uint32_t* words, int col, uint32_t epoch16, AicasScratch* s) {
  const uint32_t* p = words + col;
  uint4 a, b;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    a = ll_load4w(p);
    b = ll_load4w(p + 4);
    if (ll_ok(a, epoch16) && ll_ok(b, epoch16)) break;
    if (it == 0) t0 = globaltimer_ns();
    if ((it & 31u) == 31u) {
      if (ld_volatile_int(&s->abort)) break;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_error(s, kErrInputTimeout);
        break;
      }
    }
  }
  return make_uint4(ll_pack(a.x, a.y), ll_pack(a.z, a.w), ll_pack(b.x, b.y), ll_pack(b.z, b.w));
}

// Bounded poll of N groups of 8 LL words at once (group i starts at value
// index cols[i]; a negative index skips the group and yields zeros).  Every
// round issues the loads of all groups with no branch between them and packs
// each group into `out` as it lands, so data that has already arrived costs
// one round trip in total rather than one per group, and a group's raw words
// die as soon as they are packed.
template <int N>
__device__ __forceinline__ void ll_poll8_n(const uint32_t* words, const int (&cols)[N], uint32_t epoch16,
                                           AicasScratch* s, uint4 (&out)[N]) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    bool ok = true;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      if (cols[i] >= 0) {
        const uint4 a = ll_load4w(words + cols[i]);
        const uint4 b = ll_load4w(words + cols[i] + 4);
        ok = ok && ll_ok(a, epoch16) && ll_ok(b, epoch16);
        out[i] = make_uint4(ll_pack(a.x, a.y), ll_pack(a.z, a.w), ll_pack(b.x, b.y), ll_pack(b.z, b.w));
      } else {
        out[i] = make_uint4(0, 0, 0, 0);
      }
    }
    if (ok) break;
    if (it == 0) t0 = globaltimer_ns();
    if ((it & 31u) == 31u) {
      if (ld_volatile_int(&s->abort)) break;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_error(s, kErrInputTimeout);
        break;
      }
    }
  }
}

// Same for the 4 words holding values [col, col + 4).
__device__ __forceinline__ uint2 ll_poll4(const uint32_t* words, int col, uint32_t epoch16, AicasScratch* s) {
  const uint32_t* p = words + col;
  uint4 a;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    a = ll_load4w(p);
    if (ll_ok(a, epoch16)) break;
    if (it == 0) t0 = globaltimer_ns();
    if ((it & 31u) == 31u) {
      if (ld_volatile_int(&s->abort)) break;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_error(s, kErrInputTimeout);
        break;
      }
    }
  }
  return make_uint2(ll_pack(a.x, a.y), ll_pack(a.z, a.w));
}

// fp16 helpers -------------------------------------------------------------
__device__ __forceinline__ float r16(float x) { return __half2float(__float2half_rn(x)); }

// acc += w * x for the two fp16 lanes of each 32-bit word (exact fp16
// products, fp32 accumulation: PTX mixed-precision fma, sm_100+).
__device__ __forceinline__ float fma2_f16_f32(uint32_t w, uint32_t x, float acc) {
  asm("{\n .reg .f16 wl, wh, xl, xh;\n"
      " mov.b32 {wl, wh}, %1;\n"
      " mov.b32 {xl, xh}, %2;\n"
      " fma.rn.f32.f16 %0, wl, xl, %0;\n"
      " fma.rn.f32.f16 %0, wh, xh, %0;\n}\n"
      : "+f"(acc)
      : "r"(w), "r"(x));
  return acc;
}

__device__ __forceinline__ float dot8_f16(const uint4 w, const uint4 x, float acc) {
  acc = fma2_f16_f32(w.x, x.x, acc);
  acc = fma2_f16_f32(w.y, x.y, acc);
  acc = fma2_f16_f32(w.z, x.z, acc);
  acc = fma2_f16_f32(w.w, x.w, acc);
  return acc;
}

__device__ __forceinline__ uint4 ldcg_u4(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ float ldcg_half(const __half* p) {
  unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(p));
  return __half2float(__ushort_as_half(u));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Named barrier over the consumer warps only (the producer warp never joins).
__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

}  // namespace aicas
