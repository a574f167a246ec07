// Grouped W4A8 GEMM on the 5th-generation tensor cores (sm_100a):
// TMA -> int4 unpack in shared memory -> tcgen05.mma.kind::i8 (int32 in TMEM,
// one accumulator per K-group) -> fp32 group-scale epilogue -> bf16.
//
// Semantics are those of the reference entry point (docs/Task1.md:53-114):
//   out[m,n] = bf16( x_scale[m] * sum_g w_scale[e,n,g] * P[m,n,g] ),
//   P[m,n,g] = sum_{k in g} x_q[m,k] * int8(nibble(e,n,k) - w_zero[e,n,g])   (int32, exact)
// for every row m of expert e's segment [off[e], off[e+1]).
//
// Design (swap-AB): the MMA's M dimension is 128 weight rows (output
// channels) and its N dimension is the token block (16..256 rows of the
// expert's segment, rounded up to 16 per tile at run time).  With weights on
// the M side every epilogue thread owns one output channel, so the per-group
// weight scale is one register per thread.
//
// Per K-group accumulators, seeded by the tensor core: each group starts with
// one bf16 MMA (enable-input-d off) whose operands are constant atoms in
// shared memory and whose fp32 result is 1.5 * 2^23 in every element; the
// int8 MMAs then add the integer partial P to those bits.  For |P| < 2^22
// (|P| <= 2^21 here) the sum read as fp32 is exactly 1.5 * 2^23 + P, so one
// exact FSUB recovers float(P) - no quarter-rate I2F, no TMEM stores and no
// integer add in the epilogue.  Scale accumulation then uses packed fp32x2
// FSUB/FFMA, which round exactly like the scalar fmaf of the CUDA-core kernel
// (both kernels produce identical bits).
//
// Warp roles (512 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer of token tiles [rows x 128 B] (128-byte swizzle)
//   warps 1, 3  MMA issuers, one thread each, alternating K-groups between
//               them (warp 1 also allocates TMEM)
//   warp 2      TMA producer of packed weight tiles [128 rows x 64 B] (64-byte
//               swizzle), running ahead on its own deeper ring
//   transform   one warpgroup (warps 4-7) or, with 64-token tiles, two
//               taking K blocks in turn (warps 4-11): thread r unpacks weight
//               row r (nibble order of docs/Task1.md:78-81, zero fold with the
//               int8 wrap of :84-85) into the canonical 128B-swizzled K-major
//               layout the MMA reads
//   epilogue    the remaining warpgroups (warps 8-15 as two column halves,
//               or warps 12-15); an accumulator is handed back to the MMA as
//               soon as its last columns are in registers, before their fp32
//               math
//
// The packed-weight ring is read with ordinary shared loads and refilled by
// TMA (async proxy): a stage is released only after the unpacked bytes that
// depend on every loaded value have been stored, so no refill can overtake
// an outstanding read.
//
// Register split (setmaxnreg), per tile configuration: the producer/issuer
// and transform warpgroups drop, the epilogue warpgroups rise, within the
// launch's 512 x 128 (see TcSmall / TcMid / TcWide).
#include "common.cuh"
#include "w4a8_internal.h"

#include <cudaTypedefs.h>
#include <mutex>

namespace w4a8 {

namespace {
// Epilogue variants of the kernel (separate instances, so the plain one
// carries none of the others' code or registers):
constexpr int kModePlain = 0;      // bf16 rows (the reference's store)
constexpr int kModeCombine = 1;    // fused top-k combine into fp32 token rows
constexpr int kModePartials = 2;   // int32 per-group partials only, no scale math, no bf16 store
constexpr int kModeRows = 3;       // bf16 rows stored through a row-address table (peer memory too)

constexpr int kBW = 128;         // weight rows per tile (MMA M)
constexpr int kBK = 128;         // K bytes per pipeline stage
constexpr int kWStages = 8;      // packed weight ring
constexpr int kABytes = kBW * kBK;          // 16 KB
constexpr int kWBytes = kBW * (kBK / 2);    // 8 KB
constexpr int kTmemCols = 512;   // all of TMEM: kBufs accumulators x kBT columns
constexpr int kMaxExperts = 1024;

constexpr int kTransformWarp0 = 4;
constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagic = 12582912.0f;

constexpr int kSeedBytes = 2048;   // two 1 KB swizzle atoms holding the accumulator-seed operands
constexpr long long kDrainCycles = 20000000LL;   // ~10 ms: bounded drain after an aborted wait

// Tile configurations.  kBT: token rows per tile (MMA N, rounded up to 16 per
// tile at run time); kStages: depth of the token-tile and unpacked-weight
// rings (one stage of each per K block, released together by one MMA commit
// per group); kBufs: TMEM accumulators, alternating between the
// two MMA issuers; kTransformWGs / kEpilogueWGs: warpgroups 1-3 split
// between the int4 -> int8 transform (taking K blocks in turn) and the
// epilogue (splitting the tile's columns).  With few tokens per tile the
// epilogue has little to do and the per-K-group period is set by the
// transform and by round trips through the rings, so narrower tiles trade
// token-tile width for ring depth (and, at 64 tokens, a second transform
// warpgroup).
template <int BT, int S, int NB, int TW, int EW, int CR, int TR, int ER>
struct TcConfig {
  static constexpr int kBT = BT;
  static constexpr int kStages = S;
  static constexpr int kBufs = NB;
  static constexpr int kTransformWGs = TW;
  static constexpr int kEpilogueWGs = EW;
  static constexpr int kThreads = 128 * (1 + TW + EW);
  // registers per thread at launch (one CTA per SM): the pool setmaxnreg redistributes
  static constexpr int kLaunchRegs = (65536 / kThreads) & ~7;
  static constexpr int kEpiWarp0 = kTransformWarp0 + 4 * TW;
  static constexpr int kEpiWarps = 4 * kEpilogueWGs;
  static constexpr int kXBytes = BT * kBK;
  // Token rows per TMA box: a tile loads its full 64-row boxes with one copy
  // each and its ragged tail in 16-row boxes (so at most 15 rows of the next
  // expert are over-fetched).  Copies of 2 KB could not keep the tensor core
  // fed (measured on B200: 12 x 2 KB bulk copies per K-group took 2.1x the
  // MMA time, 3 x 8 KB kept pace).
  static constexpr int kXBoxRows = BT < 64 ? BT : 64;
  static constexpr int kXTailRows = 16;
  static constexpr int kEpiCols = BT / kEpilogueWGs;   // columns per epilogue warpgroup
  static constexpr int kControlRegs = CR;          // setmaxnreg of the producer / issuer warpgroup
  static constexpr int kTransformRegs = TR;        // setmaxnreg of the transform warpgroups
  static constexpr int kEpilogueRegs = ER;         // setmaxnreg of the epilogue warpgroups
  static constexpr size_t kSmemTiles =
      size_t(kSeedBytes) + size_t(S) * kXBytes + size_t(S) * kABytes + size_t(kWStages) * kWBytes;
  static constexpr int kNumBars = 3 * S + 2 * kWStages + 2 * NB + 2 + 2;   // + 2 abort-drain, 2 tile-done barriers
  static constexpr size_t smem_bytes(int E) {
    return 1024 /*alignment slack*/ + kSmemTiles + kNumBars * 8 + 16 + sizeof(int) * 3 * (E + 1);
  }
  static_assert(NB % 2 == 0 && NB * BT <= kTmemCols && TW >= 1 && TW <= 3 && EW >= 1 && kEpiCols % 32 == 0 &&
                    BT % kXBoxRows == 0 && kXBoxRows % kXTailRows == 0 && S >= 2,
                "tile configuration");
  // the register split must fit the launch's 512 x 128 registers, or a
  // setmaxnreg.inc waits forever
  static_assert(128 * (CR + TW * TR + EW * ER) <= kThreads * (kLaunchRegs > 128 ? 128 : kLaunchRegs) &&
                    CR % 8 == 0 && TR % 8 == 0 && ER % 8 == 0,
                "register split");
};
// Three tile widths, chosen per launch by the average rows per expert
// (measured on B200, 256 experts, N 4096, K 7168): at <= 32 rows per expert
// the 64-token tiles with a second transform warpgroup run 1.66 ms against
// 2.18 ms for 256-token tiles; at 128 rows the 128-token tiles run 2.27 ms
// against 3.41 ms; from ~200 rows on the 256-token tiles are fastest.
using TcSmall = TcConfig<64, 6, 8, 2, 1, 56, 64, 200>;     // up to 64 tokens per tile, two transform warpgroups
using TcMid = TcConfig<128, 4, 4, 1, 2, 56, 56, 200>;      // up to 128 tokens per tile
// 256-token tiles: the int4 -> int8 transform of a weight block is paid once
// per token tile, so the widest MMA (N = 256) gives it the fewest tiles
// (192-token tiles with a double-buffered epilogue measured 31 % slower on
// 256 experts x 512 rows).
using TcWide = TcConfig<256, 3, 2, 1, 2, 56, 56, 200>;     // up to 256 tokens per tile
constexpr int kSmallTileAvgRows = 48;    // average rows per expert up to which TcSmall runs
constexpr int kMidTileAvgRows = 160;     // ... and TcMid
static_assert(TcSmall::smem_bytes(kMaxExperts) <= 227 * 1024, "small configuration exceeds shared memory");
static_assert(TcMid::smem_bytes(kMaxExperts) <= 227 * 1024, "mid configuration exceeds shared memory");
static_assert(TcWide::smem_bytes(kMaxExperts) <= 227 * 1024, "wide configuration exceeds shared memory");

// signed byte b (0..7) of an 8-byte window
__device__ __forceinline__ int window_byte(uint2 w, int b) {
  const uint32_t v = b < 4 ? w.x : w.y;
  return static_cast<int>(static_cast<int8_t>(static_cast<uint8_t>(v >> ((b & 3) * 8))));
}

__device__ __forceinline__ uint32_t pack_fold(uint32_t nib4, uint32_t c7, uint32_t c8) {
  // byte-wise (nib - z) mod 256 for nib in [0,15]: nib + (c & 0x7f) never
  // carries out of a byte, and adding the top bit mod 256 is an XOR.
  return (nib4 + c7) ^ c8;
}

// 32 lanes x 32 columns as 16 packed column pairs for the fp32x2 math.  The
// wait sits in the same asm statement as the load (the registers are only
// written when the load lands, so nothing may read them before the wait),
// and so do the pairing moves, which lets the register allocator place the
// loaded columns as aligned pairs.
__device__ __forceinline__ void tmem_ld_x32_pairs(uint32_t taddr, uint64_t (&d)[16]) {
  asm volatile(
      "{\n\t.reg .b32 t<32>;\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{t0,t1,t2,t3,t4,t5,t6,t7,t8,t9,t10,t11,t12,t13,t14,t15,"
      "t16,t17,t18,t19,t20,t21,t22,t23,t24,t25,t26,t27,t28,t29,t30,t31}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n\t"
      "mov.b64 %0, {t0, t1};\n\tmov.b64 %1, {t2, t3};\n\tmov.b64 %2, {t4, t5};\n\tmov.b64 %3, {t6, t7};\n\t"
      "mov.b64 %4, {t8, t9};\n\tmov.b64 %5, {t10, t11};\n\tmov.b64 %6, {t12, t13};\n\tmov.b64 %7, {t14, t15};\n\t"
      "mov.b64 %8, {t16, t17};\n\tmov.b64 %9, {t18, t19};\n\tmov.b64 %10, {t20, t21};\n\tmov.b64 %11, {t22, t23};\n\t"
      "mov.b64 %12, {t24, t25};\n\tmov.b64 %13, {t26, t27};\n\tmov.b64 %14, {t28, t29};\n\tmov.b64 %15, {t30, t31};\n\t}"
      : "=l"(d[0]), "=l"(d[1]), "=l"(d[2]), "=l"(d[3]), "=l"(d[4]), "=l"(d[5]), "=l"(d[6]), "=l"(d[7]),
        "=l"(d[8]), "=l"(d[9]), "=l"(d[10]), "=l"(d[11]), "=l"(d[12]), "=l"(d[13]), "=l"(d[14]), "=l"(d[15])
      : "r"(taddr)
      : "memory");
}

// D[tmem] = A * B^T with bf16 operands and an fp32 result (enable-input-d off).
__device__ __forceinline__ void mma_bf16_ss_overwrite(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc)
      : "memory");
}
// Instruction descriptor for kind::f16: bf16 x bf16 -> f32, both operands K-major.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return static_cast<uint64_t>(__float_as_uint(lo)) | (static_cast<uint64_t>(__float_as_uint(hi)) << 32);
}

// Row-address store: copies a finished tile's bf16 rows from the staging
// output to their destination addresses (possibly another GPU's memory),
// 16 threads per row with 16 bytes each (the weight block's 128 channels),
// nthreads / 16 rows at a time.  (Batching several rows per thread, out of
// line, measured slower: 6.19 against 5.96 ms for the 2-GPU down GEMM.)
__device__ __forceinline__ void copy_tile_rows(const uint64_t* __restrict__ out_rows, const __nv_bfloat16* out,
                                               int64_t out_stride0, int N, int m0, int rows, int nb, int tid,
                                               int nthreads) {
  const int n0 = nb * kBW + (tid & 15) * 8;
  if (n0 >= N) return;
  for (int rr = tid >> 4; rr < rows; rr += nthreads >> 4) {
    const int m = m0 + rr;
    const uint64_t dst = __ldg(out_rows + m);
    if (dst == 0) continue;
    const __nv_bfloat16* src = out + static_cast<int64_t>(m) * out_stride0;
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(dst);
    if (n0 + 8 <= N)
      *reinterpret_cast<uint4*>(d + n0) = __ldcg(reinterpret_cast<const uint4*>(src + n0));
    else
      for (int c = n0; c < N; ++c) d[c] = __ldcg(src + c);
  }
}

template <class C, int kMode>
__global__ void __launch_bounds__(C::kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_xt,
               const __grid_constant__ CUtensorMap tm_w, const GemmArgs a) {
  constexpr int kBT = C::kBT, kStages = C::kStages, kBufs = C::kBufs;
  constexpr int kXBytes = C::kXBytes, kEpiCols = C::kEpiCols, kEpiWarp0 = C::kEpiWarp0;
  constexpr int kXBoxRows = C::kXBoxRows, kXTailRows = C::kXTailRows;
  constexpr int kTransformWGs = C::kTransformWGs;
  extern __shared__ unsigned char smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sX = base;
  uint8_t* sA = sX + kStages * kXBytes;
  uint8_t* sW = sA + kStages * kABytes;
  uint8_t* sSeed = sW + kWStages * kWBytes;   // [A atom | B atom], 1024-aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSeed + kSeedBytes);
  uint64_t* x_full = bars;
  uint64_t* op_empty = x_full + kStages;   // token stage s and unpacked-weight stage s are free again
  uint64_t* w_full = op_empty + kStages;
  uint64_t* w_empty = w_full + kWStages;
  uint64_t* a_full = w_empty + kWStages;
  uint64_t* tmem_full = a_full + kStages;
  uint64_t* tmem_empty = tmem_full + kBufs;
  uint64_t* drain_bar = tmem_empty + kBufs;   // [2]: one per MMA issuer, used only after an abort
  uint64_t* tile_done = drain_bar + 2;        // [2]: a tile's rows are in the staging output (row-address mode)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* sched_mem = reinterpret_cast<int*>(tmem_slot + 4);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    const int groups_per_block = kBK / a.gs;   // MMA issuers (one per group) that read a K block
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&op_empty[s], groups_per_block);   // one MMA commit per group of the block
      mbar_init(&a_full[s], 4);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 4);   // 4 transform warps
    }
    for (int b = 0; b < kBufs; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], C::kEpiWarps);
    }
    mbar_init(&drain_bar[0], 1);
    mbar_init(&drain_bar[1], 1);
    mbar_init(&tile_done[0], C::kEpiWarps);
    mbar_init(&tile_done[1], C::kEpiWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_xt);
    prefetch_tmap(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }

  // Seed operands: every 16-byte chunk of the A atom holds bf16 (1, 0 x 7) and
  // of the B atom bf16 (0.75 * 2^23, 0 x 7); a K = 16 product of them is
  // 2 * 0.75 * 2^23 = 1.5 * 2^23, written to every accumulator element by one
  // MMA whose row-group stride is 0 (all row groups read the same atom).
  for (int i = threadIdx.x; i < kSeedBytes / 16; i += C::kThreads)
    reinterpret_cast<uint4*>(sSeed)[i] = make_uint4(i < 64 ? 0x3F80u : 0x4AC0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  TileSched sch{sched_mem, sched_mem + (a.E + 1), sched_mem + 2 * (a.E + 1), a.E, kBT,
                (a.N + kBW - 1) / kBW, a.min_rows, a.max_rows};
  const int total = sched_build(sch, a.offsets, a.M_total);  // contains __syncthreads
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;


  const int G = a.K / a.gs;
  const int KB = (a.K + kBK - 1) / kBK;
  const int gpk = kBK / a.gs;  // groups per K block: 1 (gs=128) or 2 (gs=64)
  const int kpg = a.gs / 32;   // MMA K-steps (32 bytes each) per group

  // Each warpgroup's branch starts with its own setmaxnreg, so the compiler
  // allocates the code that follows within that budget.
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::kControlRegs));
   // The producer and issuer warps run their loops with all 32 lanes (the
   // waits too), and only the TMA / MMA / commit instructions sit in a short
   // lane-0 block: a loop run by one lane of a diverged warp pays a
   // branch-resolution stall on every branch, which measured ~20-30 cycles
   // per instruction here and set the K-group period of small tiles.
   if (warp == 0) {
    // ------------------------------------------------------------ TMA producer: token tiles
    const uint64_t pol_x = policy_evict_last();
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const Tile tile = sched_tile(sch, t);
      const int nbig = tile.rows / kXBoxRows;                                        // full boxes
      const int ntail = (tile.rows - nbig * kXBoxRows + kXTailRows - 1) / kXTailRows;   // 16-row boxes
      const uint32_t bytes = (nbig * kXBoxRows + ntail * kXTailRows) * kBK;
      for (int kb = 0; kb < KB; ++kb) {
        if (!mbar_wait(&op_empty[stage], phase ^ 1, a.status, kDevTimeoutLoadEmpty, abort_flag))
          goto x_done;
        if (lane == 0) {
          mbar_arrive_expect_tx(&x_full[stage], bytes);
          uint8_t* dst = sX + stage * kXBytes;
          for (int j = 0; j < nbig; ++j)
            tma_load_2d(dst + j * kXBoxRows * kBK, &tm_x, &x_full[stage], kb * kBK, tile.m0 + j * kXBoxRows, pol_x);
          for (int j = 0; j < ntail; ++j)
            tma_load_2d(dst + (nbig * kXBoxRows + j * kXTailRows) * kBK, &tm_xt, &x_full[stage], kb * kBK,
                        tile.m0 + nbig * kXBoxRows + j * kXTailRows, pol_x);
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
  x_done:;
  } else if (warp == 2) {
    // ------------------------------------------------------------ TMA producer: packed weights
    const uint64_t pol_keep = policy_evict_last(), pol_drop = policy_evict_first();
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const Tile tile = sched_tile(sch, t);
      const int wrow = tile.e * a.N + tile.nb * kBW;
      // The token blocks of one weight block run as neighbouring tiles: the
      // earlier ones keep the weight block in L2 for the later ones, the
      // last one lets it go.
      const bool last_tb = tile.m0 + tile.rows >= sch.seg[tile.e] + sch.cnt[tile.e];
      const uint64_t pol_w = last_tb ? pol_drop : pol_keep;
      for (int kb = 0; kb < KB; ++kb) {
        if (!mbar_wait(&w_empty[stage], phase ^ 1, a.status, kDevTimeoutLoadEmpty, abort_flag))
          goto w_done;
        if (lane == 0) {
          mbar_arrive_expect_tx(&w_full[stage], kWBytes);
          tma_load_2d(sW + stage * kWBytes, &tm_w, &w_full[stage], kb * (kBK / 2), wrow, pol_w);
        }
        __syncwarp();
        if (++stage == kWStages) { stage = 0; phase ^= 1; }
      }
    }
  w_done:;
  } else if (warp == 1 || warp == 3) {
    // ------------------------------------------------------------ MMA issuers
    // Two issuing threads: thread p issues the groups c with c % 2 == p (c
    // counts this CTA's groups) into TMEM accumulator c % kBufs, so one
    // thread's waits and commits overlap the other's MMAs.  Each group's MMAs read one
    // K block; its issuer commits the block's release once per group (a block
    // of two gs = 64 groups is released by both issuers; a trailing block
    // with one group is committed twice by its issuer).
    {
      const int p = warp == 1 ? 0 : 1;
      const uint64_t desc_x0 = make_desc_sw128(smem_u32(sX));
      const uint64_t desc_a0 = make_desc_sw128(smem_u32(sA));
      constexpr uint64_t kSboMask = ~(static_cast<uint64_t>(0x3FFF) << 32);
      const uint64_t seed_a = make_desc_sw128(smem_u32(sSeed)) & kSboMask;          // row-group stride 0
      const uint64_t seed_b = make_desc_sw128(smem_u32(sSeed + 1024)) & kSboMask;
      int stage = 0, c = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const Tile tile = sched_tile(sch, t);
        const int n_mma = (tile.rows + 15) & ~15;
        const uint32_t idesc = make_idesc_i8(kBW, n_mma);
        const uint32_t idesc_seed = make_idesc_bf16(kBW, n_mma);
        int sub = 0;   // group within the K block (gs = 64: two groups per block)
        for (int g = 0; g < G; ++g, ++c) {
          const bool block_end = (sub + 1 == gpk) || g == G - 1;
          if ((c & 1) == p) {
            if (!mbar_wait(&x_full[stage], phase, a.status, kDevTimeoutLoadFull, abort_flag)) goto mma_done;
            if (!mbar_wait(&a_full[stage], phase, a.status, kDevTimeoutAFull, abort_flag)) goto mma_done;
            const int buf = c % kBufs;
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kBT);
            if (!mbar_wait(&tmem_empty[buf], ((c / kBufs) & 1) ^ 1, a.status, kDevTimeoutTmemEmpty, abort_flag))
              goto mma_done;
            // descriptors advance by (byte offset >> 4) in their start-address field
            const uint64_t adesc = desc_a0 + static_cast<uint64_t>((stage * kABytes + sub * kpg * 32) >> 4);
            const uint64_t bdesc = desc_x0 + static_cast<uint64_t>((stage * kXBytes + sub * kpg * 32) >> 4);
            const bool trailing = block_end && sub + 1 < gpk;   // a trailing block with fewer groups than its count
            if (lane == 0) {
              tc_fence_after();
              // seed: every accumulator element = bits of 1.5 * 2^23; the int8 MMAs then add P
              mma_bf16_ss_overwrite(d_tmem, seed_a, seed_b, idesc_seed);
#pragma unroll 4
              for (int ks = 0; ks < kpg; ++ks)
                mma_i8_ss(d_tmem, adesc + 2 * ks, bdesc + 2 * ks, idesc, 1u);
              mma_commit(&tmem_full[buf]);
              mma_commit(&op_empty[stage]);
              if (trailing) mma_commit(&op_empty[stage]);
            }
            __syncwarp();
          }
          if (block_end) {
            sub = 0;
            if (++stage == kStages) { stage = 0; phase ^= 1; }
          } else {
            ++sub;
          }
        }
      }
    mma_done:;
    }
   }
  } else if (warp < kEpiWarp0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::kTransformRegs));
    // ------------------------------------------------------------ int4 -> int8 transform
    const int tg = (warp - kTransformWarp0) >> 2;              // transform warpgroup: K blocks kb % kTransformWGs == tg
    const int r = ((warp - kTransformWarp0) & 3) * 32 + lane;  // weight row within the tile
    const int sw = (r >> 1) & 3;                         // 64-byte swizzle of the packed tile
    // Zero points arrive in windows of 8 groups (one 8-byte load), the next
    // window in flight while the current one is used: a global load's latency
    // (the tile's zero points and scales do not stay in L1 beside this
    // kernel's shared memory) is spread over 8 K-groups instead of stalling
    // every one.  Rows with G % 8 != 0 load each K block's bytes when used.
    const bool zvec = (G % 8) == 0 && (reinterpret_cast<uintptr_t>(a.w_zero) % 8) == 0;
    int stage = 0, astage = 0;
    uint32_t phase = 0, aphase = 0;
    // Row-address mode: this warpgroup, which has slack beside the epilogue,
    // streams each finished tile's rows to their destinations one tile
    // later, so those (peer) stores overlap the next tiles' MMAs.
    const int copy_tid = threadIdx.x - kTransformWarp0 * 32;
    Tile prev{};
    int ti = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const Tile tile = sched_tile(sch, t);
      const int n = tile.nb * kBW + r;
      const bool valid = n < a.N;
      const int8_t* zrow = a.w_zero + (static_cast<int64_t>(tile.e) * a.N + (valid ? n : 0)) * G;
      uint2 zw = make_uint2(0u, 0u), zw_next = make_uint2(0u, 0u);
      int zwi = 0;   // window held in zw
      if (zvec && valid) {
        zw = __ldg(reinterpret_cast<const uint2*>(zrow));
        if (G > 8) zw_next = __ldg(reinterpret_cast<const uint2*>(zrow + 8));
      }
      for (int kb = 0; kb < KB; ++kb) {
        if constexpr (kTransformWGs > 1) {
          if (kb % kTransformWGs != tg) {   // the other warpgroup's block: advance the rings only
            if (++stage == kWStages) { stage = 0; phase ^= 1; }
            if (++astage == kStages) { astage = 0; aphase ^= 1; }
            continue;
          }
        }
        const int g0 = kb * gpk;
        int z0 = 0, z1 = 0;
        if (zvec) {
          const int b = g0 & 7;
          if ((g0 >> 3) != zwi) {   // blocks step by at most 6 groups: windows advance one at a time
            zw = zw_next;
            ++zwi;
            const int next = 8 * (zwi + 1);   // first group of the following window (8-byte aligned)
            if (valid && next < G) zw_next = __ldg(reinterpret_cast<const uint2*>(zrow + next));
          }
          z0 = window_byte(zw, b);
          z1 = gpk == 2 ? window_byte(zw, b + 1) : z0;   // gs = 64: b is even, b + 1 in the same window
        } else if (valid) {
          z0 = zrow[g0];
          z1 = (gpk == 2 && g0 + 1 < G) ? zrow[g0 + 1] : z0;
        }
        if (!mbar_wait(&w_full[stage], phase, a.status, kDevTimeoutLoadFull, abort_flag)) goto tr_done;
        uint4 pk[4];
        {
          const uint8_t* src = sW + stage * kWBytes + r * (kBK / 2);
#pragma unroll
          for (int c = 0; c < 4; ++c) pk[c] = *reinterpret_cast<const uint4*>(src + ((c ^ sw) << 4));
        }
        // The packed stage is released only after its bytes have been consumed
        // (below): the release is a generic-proxy arrive while the refill is an
        // async-proxy TMA write, so an arrive issued right after the shared
        // loads does not order them before the refill.
        const int wstage = stage;
        if (++stage == kWStages) { stage = 0; phase ^= 1; }

        if (!mbar_wait(&op_empty[astage], aphase ^ 1, a.status, kDevTimeoutAEmpty, abort_flag)) goto tr_done;
        uint8_t* dst_row = sA + astage * kABytes + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          // packed chunk c (16 B) -> K offsets [32c, 32c+32) -> output chunks 2c, 2c+1
          const int zc = (c < 2) ? z0 : z1;   // gs=64: chunks 0-1 are group 2kb, 2-3 group 2kb+1
          const uint32_t cb = static_cast<uint32_t>(-zc) & 0xFFu;
          const uint32_t c7 = (cb & 0x7Fu) * 0x01010101u;
          const uint32_t c8 = (cb & 0x80u) * 0x01010101u;
          const uint32_t wv[4] = {pk[c].x, pk[c].y, pk[c].z, pk[c].w};
          uint32_t o[8];
          if (a.layout == 0) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t lo = wv[q] & 0x0F0F0F0Fu;          // k = 8q + 0, 2, 4, 6
              const uint32_t hi = (wv[q] >> 4) & 0x0F0F0F0Fu;   // k = 8q + 1, 3, 5, 7
              o[2 * q] = pack_fold(__byte_perm(lo, hi, 0x5140), c7, c8);
              o[2 * q + 1] = pack_fold(__byte_perm(lo, hi, 0x7362), c7, c8);
            }
          } else {   // prepacked: the low nibbles are k = 8q..8q+3, the high ones 8q+4..8q+7
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              o[2 * q] = pack_fold(wv[q] & 0x0F0F0F0Fu, c7, c8);
              o[2 * q + 1] = pack_fold((wv[q] >> 4) & 0x0F0F0F0Fu, c7, c8);
            }
          }
          const int j0 = 2 * c, j1 = 2 * c + 1;
          *reinterpret_cast<uint4*>(dst_row + ((j0 ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(dst_row + ((j1 ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&w_empty[wstage]);   // the stores above depend on every byte read from it
          mbar_arrive(&a_full[astage]);
        }
        if (++astage == kStages) { astage = 0; aphase ^= 1; }
      }
      if constexpr (kMode == kModeRows) {
        if (ti > 0) {
          if (!mbar_wait(&tile_done[(ti - 1) & 1], ((ti - 1) >> 1) & 1, a.status, kDevTimeoutTileDone, abort_flag))
            goto tr_done;
          copy_tile_rows(a.out_rows, a.out, a.out_stride0, a.N, prev.m0, prev.rows, prev.nb, copy_tid,
                         128 * kTransformWGs);
        }
        prev = tile;
        ++ti;
      }
    }
    if constexpr (kMode == kModeRows) {
      if (ti > 0) {
        if (!mbar_wait(&tile_done[(ti - 1) & 1], ((ti - 1) >> 1) & 1, a.status, kDevTimeoutTileDone, abort_flag))
          goto tr_done;
        copy_tile_rows(a.out_rows, a.out, a.out_stride0, a.N, prev.m0, prev.rows, prev.nb, copy_tid,
                       128 * kTransformWGs);
      }
    }
  tr_done:;
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::kEpilogueRegs));
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;                     // TMEM lane quarter this warp may access
    const int wg = (warp - kEpiWarp0) >> 2;           // column range of this warpgroup
    const int r = quarter * 32 + lane;                // weight row within the tile
    const uint64_t magic2 = f2_pack(kMagic, kMagic);
    constexpr int kChunks = kEpiCols / 32;
    int buf = 0, tile_i = 0;   // tile_i: this CTA's tiles so far (row-address mode)
    uint32_t bphase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const Tile tile = sched_tile(sch, t);
      const int n = tile.nb * kBW + r;
      const bool valid = n < a.N;
      const int n_mma = (tile.rows + 15) & ~15;
      const int my_cols = n_mma - wg * kEpiCols;      // columns of this warpgroup holding tokens (may be <= 0)
      const float* wsrow = a.w_scale + (static_cast<int64_t>(tile.e) * a.N + (valid ? n : 0)) * G;
      if constexpr (kMode == kModePartials) {
        // Partials export: each group's accumulator is drained and written as
        // int32, [G, M_total, N] (consecutive lanes hold consecutive output
        // channels, so every store is one 128-byte line).
        for (int g = 0; g < G; ++g) {
          if (!mbar_wait(&tmem_full[buf], bphase, a.status, kDevTimeoutTmemFull, abort_flag)) goto epi_done;
          tc_fence_after();
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                 static_cast<uint32_t>(buf * kBT + wg * kEpiCols);
#pragma unroll 1
          for (int c32 = 0; c32 < kChunks; ++c32) {
            const bool have = c32 * 32 < my_cols;   // warp-uniform
            uint64_t d[16];
            __syncwarp();
            if (have) tmem_ld_x32_pairs(taddr + c32 * 32, d);
            if (c32 == kChunks - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&tmem_empty[buf]);
            }
            if (have && valid) {
              int32_t* prow = a.partials + (static_cast<int64_t>(g) * a.M_total + tile.m0) * a.N + n;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int col = wg * kEpiCols + c32 * 32 + j;
                if (col < tile.rows)
                  prow[static_cast<int64_t>(col) * a.N] =
                      static_cast<int>(static_cast<uint32_t>(d[j >> 1] >> (32 * (j & 1))) - kMagicBits);
              }
            }
          }
          if (++buf == kBufs) { buf = 0; bphase ^= 1; }
        }
        continue;
      }
      uint64_t acc[kEpiCols / 2];
#pragma unroll
      for (int c = 0; c < kEpiCols / 2; ++c) acc[c] = 0;
      float ws_next = valid ? __ldg(wsrow) : 0.f;
      for (int g = 0; g < G; ++g) {
        const float ws = ws_next;
        if (valid && g + 1 < G) ws_next = __ldg(wsrow + g + 1);
        const uint64_t ws2 = f2_pack(ws, ws);
        if (!mbar_wait(&tmem_full[buf], bphase, a.status, kDevTimeoutTmemFull, abort_flag)) goto epi_done;
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(buf * kBT + wg * kEpiCols);
        // Drain 32 columns per load; the accumulator goes back to the MMA as
        // soon as the last chunk is in registers, before its math.  (Loading
        // the next chunk while this one's math runs needs a second 32-column
        // buffer, which does not fit the 256-token tile's registers.)
#pragma unroll
        for (int c32 = 0; c32 < kChunks; ++c32) {
          const bool have = c32 * 32 < my_cols;   // warp-uniform
          uint64_t d[16];
          __syncwarp();
          if (have) tmem_ld_x32_pairs(taddr + c32 * 32, d);
          if (c32 == kChunks - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[buf]);
          }
          if (have) {
#pragma unroll
            for (int j = 0; j < 16; ++j)   // P + 1.5 * 2^23 read as fp32, minus 1.5 * 2^23 = float(P)
              acc[c32 * 16 + j] = f2_fma(f2_sub(d[j], magic2), ws2, acc[c32 * 16 + j]);
          }
        }
        if (++buf == kBufs) { buf = 0; bphase ^= 1; }
      }
      if (valid) {
#pragma unroll
        for (int c = 0; c < kEpiCols / 2; ++c) {
          const int col = wg * kEpiCols + 2 * c;
          if (col < tile.rows) {
            const int m = tile.m0 + col;
            const float lo = __uint_as_float(static_cast<uint32_t>(acc[c]));
            const float hi = __uint_as_float(static_cast<uint32_t>(acc[c] >> 32));
            if constexpr (kMode == kModeCombine) {
              // fused top-k combine: the weighted bf16 row result goes to its token's fp32 row
              store_output(a, m, n, lo);
              if (col + 1 < tile.rows) store_output(a, m + 1, n, hi);
            } else {
              __nv_bfloat16* o = a.out + static_cast<int64_t>(m) * a.out_stride0 + static_cast<int64_t>(n) * a.out_stride1;
              *o = __float2bfloat16_rn(lo * __ldg(a.x_scale + m));
              if (col + 1 < tile.rows) o[a.out_stride0] = __float2bfloat16_rn(hi * __ldg(a.x_scale + m + 1));
            }
          }
        }
      }
      if constexpr (kMode == kModeRows) {
        // the tile's rows are in the staging output: the transform warpgroup
        // copies them on (release: the stores above before the arrive)
        __syncwarp();
        if (lane == 0) mbar_arrive(&tile_done[tile_i & 1]);
        ++tile_i;
      }
    }
  epi_done:;
  }

  // A wait that gave up left the pipeline mid-flight: before TMEM is freed,
  // each MMA issuer waits (bounded) for its own MMAs through one more commit,
  // and every thread then idles a bounded while so TMA copies in flight land
  // in shared memory before the CTA exits.
  if (*abort_flag) {
    if ((warp == 1 || warp == 3) && lane == 0) {
      mma_commit(&drain_bar[warp == 1 ? 0 : 1]);
      const long long t0 = clock64();
      while (!mbar_try_wait(&drain_bar[warp == 1 ? 0 : 1], 0) && clock64() - t0 < kDrainCycles) {
      }
    }
    const long long t0 = clock64();
    while (clock64() - t0 < kDrainCycles) {
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

bool encode_2d_u8(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                  uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <class C, int kMode>
cudaError_t launch_tc_kernel(const CUtensorMap& tm_x, const CUtensorMap& tm_xt, const CUtensorMap& tm_w,
                             const GemmArgs& a, cudaStream_t stream) {
  static_assert(kMode == kModePlain || kMode == kModeCombine || kMode == kModePartials || kMode == kModeRows,
                "epilogue mode");
  // The setmaxnreg split relies on the launch's 512 x 128 registers; with
  // fewer, the epilogue's setmaxnreg.inc could wait forever, so refuse to
  // launch.
  static int regs_checked = 0;
  if (!regs_checked) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, gemm_tc_kernel<C, kMode>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != C::kLaunchRegs) return cudaErrorInvalidConfiguration;
    regs_checked = 1;
  }
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = C::smem_bytes(a.E);
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<C, kMode>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  gemm_tc_kernel<C, kMode><<<sms, C::kThreads, smem, stream>>>(tm_x, tm_xt, tm_w, a);
  return cudaGetLastError();
}

template <class C>
cudaError_t launch_tc_config(const CUtensorMap& tm_w, const GemmArgs& a, cudaStream_t stream) {
  CUtensorMap tm_x, tm_xt;
  if (!encode_2d_u8(&tm_x, a.x_q, static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.M_total),
                    static_cast<uint64_t>(a.x_stride0), kBK, C::kXBoxRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d_u8(&tm_xt, a.x_q, static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.M_total),
                    static_cast<uint64_t>(a.x_stride0), kBK, C::kXTailRows, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  // The fused combine and the int32 partials export are separate instances:
  // the plain epilogue carries none of their code or registers (the
  // combine's store path alone, compiled into the plain kernel, made it
  // 1.4-1.9x slower).  With a partials export the plain kernel writes the
  // bf16 rows and a second launch of the same pipeline writes the partials.
  if (a.comb_out != nullptr) return launch_tc_kernel<C, kModeCombine>(tm_x, tm_xt, tm_w, a, stream);
  if (a.out_rows != nullptr) return launch_tc_kernel<C, kModeRows>(tm_x, tm_xt, tm_w, a, stream);
  GemmArgs plain = a;
  plain.partials = nullptr;
  cudaError_t e = launch_tc_kernel<C, kModePlain>(tm_x, tm_xt, tm_w, plain, stream);
  if (e == cudaSuccess && a.partials != nullptr) e = launch_tc_kernel<C, kModePartials>(tm_x, tm_xt, tm_w, a, stream);
  return e;
}

}  // namespace

cudaError_t launch_gemm_tc(const GemmArgs& a, cudaStream_t stream) {
  if (a.M_total <= 0) return cudaSuccess;
  if (a.K < kBK || (a.K % 64) != 0 || (a.gs != 64 && a.gs != 128) || a.E > kMaxExperts)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.x_q) & 15) || (a.x_stride0 % 16) ||
      (reinterpret_cast<uintptr_t>(a.w_packed) & 15))
    return cudaErrorInvalidValue;
  CUtensorMap tm_w;
  if (!encode_2d_u8(&tm_w, a.w_packed, static_cast<uint64_t>(a.K / 2),
                    static_cast<uint64_t>(a.E) * static_cast<uint64_t>(a.N), static_cast<uint64_t>(a.K / 2),
                    kBK / 2, kBW, CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;

  // Tile width by the average rows per expert (the launch's configuration is
  // fixed on the host, without a device synchronisation).
  const int64_t rows = a.rows_hint > 0 ? a.rows_hint : a.M_total, experts = a.E;
  if (rows <= kSmallTileAvgRows * experts) return launch_tc_config<TcSmall>(tm_w, a, stream);
  if (rows <= kMidTileAvgRows * experts) return launch_tc_config<TcMid>(tm_w, a, stream);
  return launch_tc_config<TcWide>(tm_w, a, stream);
}

bool gemm_tc_supports(int K, int gs, int E) { return K >= kBK && K % 64 == 0 && (gs == 64 || gs == 128) && E <= kMaxExperts; }

}  // namespace w4a8
