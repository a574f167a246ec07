// Shared device helpers for the W4A8 MoE kernels (sm_100a only).
//
// Contents:
//   * status word + bounded mbarrier waits (every spin has an iteration/clock
//     limit; on expiry the kernel records an error code and unwinds),
//   * thin inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor, no
//     multicast anywhere), and tcgen05 (alloc / mma.kind::i8 / commit / ld),
//   * the device-side expert tile scheduler used by every grouped GEMM: it turns
//     `expert_offsets` (int32 [E+1], device memory) into a prefix table of
//     tiles in shared memory, so no host synchronisation is ever needed
//     (the reference host-syncs with `.item()` at
//     Task1/v1.6/task1-codex5.5-all-v1.6.py:62-64).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#if defined(__CUDA_ARCH__) && !defined(__CUDA_ARCH_FEAT_SM100_ALL)
#error "this library targets sm_100a only (build with -gencode arch=compute_100a,code=sm_100a)"
#endif

namespace w4a8 {

// ----------------------------------------------------------------------------
// device status word (error codes written by kernels, read by the host)
// ----------------------------------------------------------------------------
enum DeviceStatus : int {
  kDevOk = 0,
  kDevTimeoutLoadFull = 101,
  kDevTimeoutLoadEmpty = 102,
  kDevTimeoutAFull = 103,
  kDevTimeoutAEmpty = 104,
  kDevTimeoutTmemFull = 105,
  kDevTimeoutTmemEmpty = 106,
  kDevTimeoutTileDone = 107,   // the epilogue never reported a tile's rows (row-address store)
  kDevBadShape = 110,
  kDevTimeoutSelfTest = 120,
  kDevTimeoutPeer = 130,     // a peer rank's signal did not arrive (expert-parallel exchange / barrier)
  kDevEpOverflow = 131,      // a rank would receive more rows than its receive buffer holds
};

// Roughly one second at B200 clocks.  A correct pipeline never waits this
// long; an expired wait means a protocol bug, and the kernel unwinds instead
// of hanging the GPU.
#ifndef W4A8_WAIT_LIMIT_CYCLES
#define W4A8_WAIT_LIMIT_CYCLES (2000000000LL)
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

// ----------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(tx)
               : "memory");
}
// try_wait with the system's default suspend limit (a 10 ms suspendTimeHint
// measured no faster on B200).  Every waiter in this library uses it, the MMA
// issuer included: a waiting try_wait hands off in ~125 cycles on B200 against
// ~170 for a test_wait polling loop.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false (after recording `code` in *status and raising
// the CTA-local abort flag) when the wait has run `limit` cycles or another
// role of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, int* status, int code,
                                                volatile int* abort_flag, long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      atomicCAS(status, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                                          volatile int* abort_flag) {
  return mbar_wait_limit(bar, parity, status, code, abort_flag, W4A8_WAIT_LIMIT_CYCLES);
}

// ----------------------------------------------------------------------------
// TMA (tiled, 2-D, no multicast)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------------
// tcgen05 (1-CTA group)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, s8 x s8 -> s32.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on `bar` when every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns per thread, with the wait in the
// same asm statement (the registers are defined only once the load lands).
__device__ __forceinline__ void tmem_ld_x16_wait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor (tcgen05 format): K-major operand stored in
// the canonical 128-byte-swizzled layout (8-row x 128-byte atoms, atoms 1024
// bytes apart along M/N).  `addr` must sit inside a 1024-byte-aligned atom
// row; advancing along K inside the 128-byte row is done by adding bytes to
// the start address (the swizzle is applied on absolute address bits).
__device__ __forceinline__ uint64_t make_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFF) >> 4);         // start address, bits [0,14)
  d |= static_cast<uint64_t>(1) << 16;                       // LBO (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;               // SBO = 1024 B between 8-row atoms
  d |= static_cast<uint64_t>(1) << 46;                       // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                       // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::i8: s8 x s8 -> s32, both operands K-major.
__host__ __device__ constexpr uint32_t make_idesc_i8(int m, int n) {
  return (2u << 4)                                 // D format: S32
         | (1u << 7)                               // A: signed 8-bit
         | (1u << 10)                              // B: signed 8-bit
         | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

// ----------------------------------------------------------------------------
// Device-side expert tile scheduler
// ----------------------------------------------------------------------------
// A "tile" is (expert e, weight block nb of `BW` output channels, token block
// tb of up to `bt` rows of that expert's segment).  Tiles are numbered expert
// by expert; inside an expert nb is the slow index and tb the fast one, so
// tiles that share a weight block run on neighbouring CTAs at the same time
// and the second read of the weight block hits L2 (tb_slow flips the order,
// for a kernel that keeps the token block resident instead).
//
// Segment semantics follow the reference loop (docs/Task1.md:88-96): rows
// [off[e], off[e+1]) belong to expert e; empty or inverted segments are
// skipped; rows outside every segment are never touched.  Offsets are clamped
// to [0, M_total], which matches Python slicing of x_q for in-range values.
struct TileSched {
  int* prefix;  // [E+1] tile prefix (smem)
  int* seg;     // [E+1] clamped segment starts; seg[E] unused (smem)
  int* cnt;     // [E] rows per expert (smem)
  int E, bt, NB;
  int min_rows = 1;           // experts with fewer rows are left to another kernel
  int max_rows = 0x7fffffff;  // experts with more rows are left to another kernel
  bool tb_slow = false;       // token block as the slow index inside an expert
};

// Must be called by all threads of the CTA (contains __syncthreads()).
__device__ __forceinline__ int sched_build(TileSched& s, const int32_t* __restrict__ offsets,
                                           int M_total) {
  // rows per expert
  for (int e = threadIdx.x; e < s.E; e += blockDim.x) {
    int a = offsets[e], b = offsets[e + 1];
    a = a < 0 ? 0 : (a > M_total ? M_total : a);
    b = b < 0 ? 0 : (b > M_total ? M_total : b);
    int c = b > a ? b - a : 0;
    if (c < s.min_rows || c > s.max_rows) c = 0;  // not this kernel's expert
    s.seg[e] = a;
    s.cnt[e] = c;
  }
  __syncthreads();
  // inclusive scan of tiles-per-expert by warp 0 (E is small: <= a few hundred)
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int per = (s.E + 31) / 32;
    const int lo = lane * per;
    int local = 0;
    for (int i = 0; i < per; ++i) {
      const int e = lo + i;
      if (e < s.E) local += ((s.cnt[e] + s.bt - 1) / s.bt) * s.NB;
    }
    int incl = local;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    int run = incl - local;
    for (int i = 0; i < per; ++i) {
      const int e = lo + i;
      if (e < s.E) {
        s.prefix[e] = run;
        run += ((s.cnt[e] + s.bt - 1) / s.bt) * s.NB;
      }
    }
    if (lane == 31) s.prefix[s.E] = incl;
  }
  __syncthreads();
  return s.prefix[s.E];
}

struct Tile {
  int e;     // expert
  int m0;    // first row of the token block (absolute row in x_q / out)
  int rows;  // rows of the block that belong to expert e (1..bt)
  int nb;    // weight block index
};

__device__ __forceinline__ Tile sched_tile(const TileSched& s, int t) {
  // largest e with prefix[e] <= t (prefix is non-decreasing; empty experts repeat values)
  int lo = 0, hi = s.E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s.prefix[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int e = lo;
  const int local = t - s.prefix[e];
  const int tbs = (s.cnt[e] + s.bt - 1) / s.bt;
  Tile r;
  r.e = e;
  int tb;
  if (s.tb_slow) {
    tb = local / s.NB;
    r.nb = local - tb * s.NB;
  } else {
    r.nb = local / tbs;
    tb = local - r.nb * tbs;
  }
  r.m0 = s.seg[e] + tb * s.bt;
  const int left = s.cnt[e] - tb * s.bt;
  r.rows = left < s.bt ? left : s.bt;
  return r;
}

// Walks consecutive tiles t, t+1, ... without a search per tile: tiles are
// numbered expert by expert, weight block (slow) by token block (fast).
struct TileWalk {
  const TileSched* s;
  Tile cur;
  int tb, tbs;
  __device__ __forceinline__ void start(const TileSched& sch, int t) {
    s = &sch;
    cur = sched_tile(sch, t);
    tbs = (sch.cnt[cur.e] + sch.bt - 1) / sch.bt;
    tb = (cur.m0 - sch.seg[cur.e]) / sch.bt;
  }
  // Advance to the next tile (the caller keeps it below the tile total).
  __device__ __forceinline__ void next() {
    if (s->tb_slow) {
      if (++cur.nb < s->NB) {
        // same token block
      } else if (cur.nb = 0, ++tb < tbs) {
        cur.m0 += s->bt;
      } else {
        tb = 0;
        do { ++cur.e; } while (cur.e < s->E - 1 && s->prefix[cur.e + 1] == s->prefix[cur.e]);
        tbs = (s->cnt[cur.e] + s->bt - 1) / s->bt;
        cur.m0 = s->seg[cur.e];
      }
    } else if (++tb < tbs) {
      cur.m0 += s->bt;
    } else if (tb = 0, ++cur.nb < s->NB) {
      cur.m0 = s->seg[cur.e];
    } else {
      cur.nb = 0;
      do { ++cur.e; } while (cur.e < s->E - 1 && s->prefix[cur.e + 1] == s->prefix[cur.e]);
      tbs = (s->cnt[cur.e] + s->bt - 1) / s->bt;
      cur.m0 = s->seg[cur.e];
    }
    const int left = s->cnt[cur.e] - tb * s->bt;
    cur.rows = left < s->bt ? left : s->bt;
  }
};

}  // namespace w4a8
