// Streaming W4A8 grouped GEMM for experts with few rows (decode): the weights
// are read from HBM exactly once by the TMA engine, CUDA cores do the math.
//
// At 1-4 tokens per expert the layer is bound by reading the packed weights.
// A 128-row tensor-core tile with N = 16 pays a fixed per-group cost (MMA
// issue, TMEM round trip, barrier hand-offs) longer than its 8 KB of weights
// take to arrive, so this path keeps the tensor cores out of it:
//   * one producer warp streams a block of RB contiguous weight rows of one
//     expert (RB * K/2 bytes, about 32 KB) into a shared-memory ring with a
//     single cp.async.bulk per stage (no multicast), plus the block's
//     w_scale / w_zero rows (bulk copies when 16-byte aligned, else loaded by
//     the consumers directly);
//   * the token rows of the current expert (at most kGvRows) are staged once
//     in shared memory, split per 8-byte K block into the even-k and odd-k
//     bytes, i.e. the order in which the low and high nibbles of a packed
//     word come out of a mask and a shift, together with the sum of every
//     32-value chunk of each row;
//   * eight consumer warps each take rows of the block: a lane handles 32 K
//     values (16 packed bytes) per 1024-wide K step.  The exact int32 partial
//     of docs/Task1.md:100-104 is
//         sum_k int8(nib - z) * x  =  sum_k nib * x  -  z * sum_k x
//     whenever nib - z cannot leave int8 (z >= -112), so the raw nibbles go
//     straight into dp4a (unsigned x signed; the odd-k nibbles are left in
//     the high half of their bytes and the 16x sum is shifted back) and the
//     zero point costs one multiply per chunk;
//     groups whose zero point can wrap (z < -112) fold each nibble with the
//     reference's int8 wrap instead (docs/Task1.md:78-85);
//   * the 4 (gs = 128) or 2 (gs = 64) lanes of a K-group are summed with
//     shuffles -> the exact int32 partial; the group's first lane applies
//     w_scale, a warp reduction and x_scale give the bf16 output
//     (docs/Task1.md:107-112).
// fp32 summation order differs from the tile kernels (per lane, then across
// lanes): outputs agree with them within bf16 rounding; int32 partials are
// identical.
#include "common.cuh"
#include "w4a8_internal.h"

namespace w4a8 {

namespace {

constexpr int kGvConsumers = 8;
constexpr int kGvThreads = (kGvConsumers + 1) * 32;   // + producer warp
constexpr int kGvRows = kGemvMaxTokens;                // tokens per pass
static_assert(kGvRows <= 4, "the token-scale slot in shared memory holds 4 floats");
constexpr int kGvMaxStages = 4;   // ring depth per CTA
constexpr int kGvTargetW = 32 * 1024;                  // preferred weight bytes per stage
constexpr int kGvMaxRB = 32;                           // rows per block
constexpr int kGvSmemBudget = 110 * 1024;   // two CTAs per SM when it fits
constexpr int kGvPlain = 0;      // epilogue modes: bf16 rows
constexpr int kGvCombine = 1;    // fused top-k combine into fp32 token rows
constexpr int kGvPartials = 2;   // bf16 rows and the int32 per-group partials
constexpr int kGvRowAddr = 3;    // bf16 rows stored through a row-address table
constexpr int kWrapZero = -112;   // z >= kWrapZero: nib - z stays inside int8 for every nibble

struct GvParams {
  int stages;      // ring depth (1..4)
  int stage_w;     // weight bytes per stage (RB * row_bytes)
  int RB;          // weight rows per block (a multiple of the consumer warp count)
  int row_bytes;   // K/2
  int meta_bulk;   // 1: scales / zero points travel with the block (16-byte aligned)
  int ws_bytes;    // per-stage bytes reserved for scales (RB*G*4, 16-aligned)
  int z_bytes;     // per-stage bytes reserved for zero points (RB*G, 16-aligned)
  int x_bytes;     // token tile: kGvRows rows x K bytes (even half + odd half)
  int sx_bytes;    // group sums: kGvRows rows x G int32
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Named barrier over the consumer warps only (the producer keeps streaming).
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kGvConsumers * 32) : "memory");
}

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

struct TokenTile {
  const uint8_t* xe;   // [kGvRows][K/2] even-k bytes, 16 per 32-value chunk
  const uint8_t* xo;   // [kGvRows][K/2] odd-k bytes
  const int* sx;       // [kGvRows][G] group sums
  const float* xsc;    // [kGvRows] token scales of the rows
};

struct RowJob {
  const uint8_t* w;      // packed weight row in shared memory
  const int8_t* z;       // zero points of the row in shared memory (nullptr: read global)
  const float* ws;       // scales of the row in shared memory (nullptr: read global)
  int m0, n;             // first token row, output channel
  int64_t grow;          // e * N + n
};

// Exact int32 partials of NG K-groups (one lane's) whose zero points cannot
// wrap: sum nib * x - z * sum x.  lo holds the even-k nibbles as bytes
// 0..15, hi16 the odd-k nibbles in the high half of each byte (16 * nib,
// unsigned), so their sum is 16x and one arithmetic shift restores it.  The
// NG groups are independent chains the scheduler interleaves.
template <int R, int GS, int NG>
__device__ __forceinline__ void partials_nowrap(const uint8_t* const (&wg)[NG], const uint8_t* const (&xeg)[NG],
                                                const uint8_t* const (&xog)[NG], int rot, int half_k,
                                                int (&p)[NG][R], const int (&z)[NG], const int (&sxv)[NG][R]) {
  constexpr int kCpg = GS / 32;
  int se[NG][R], so[NG][R];
#pragma unroll
  for (int n = 0; n < NG; ++n)
#pragma unroll
    for (int r = 0; r < R; ++r) { se[n][r] = -z[n] * sxv[n][r]; so[n][r] = 0; }
#pragma unroll
  for (int i = 0; i < kCpg; ++i) {
    const int ch = 16 * ((i + rot) & (kCpg - 1));
#pragma unroll
    for (int n = 0; n < NG; ++n) {
      const uint4 w = *reinterpret_cast<const uint4*>(wg[n] + ch);
      const uint32_t l0 = w.x & 0x0F0F0F0Fu, l1 = w.y & 0x0F0F0F0Fu, l2 = w.z & 0x0F0F0F0Fu, l3 = w.w & 0x0F0F0F0Fu;
      const uint32_t h0 = w.x & 0xF0F0F0F0u, h1 = w.y & 0xF0F0F0F0u, h2 = w.z & 0xF0F0F0F0u, h3 = w.w & 0xF0F0F0F0u;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint4 xe = *reinterpret_cast<const uint4*>(xeg[n] + r * half_k + ch);
        const uint4 xo = *reinterpret_cast<const uint4*>(xog[n] + r * half_k + ch);
        se[n][r] = dp4a_us(l0, xe.x, se[n][r]);
        so[n][r] = dp4a_us(h0, xo.x, so[n][r]);
        se[n][r] = dp4a_us(l1, xe.y, se[n][r]);
        so[n][r] = dp4a_us(h1, xo.y, so[n][r]);
        se[n][r] = dp4a_us(l2, xe.z, se[n][r]);
        so[n][r] = dp4a_us(h2, xo.z, so[n][r]);
        se[n][r] = dp4a_us(l3, xe.w, se[n][r]);
        so[n][r] = dp4a_us(h3, xo.w, so[n][r]);
      }
    }
  }
#pragma unroll
  for (int n = 0; n < NG; ++n)
#pragma unroll
    for (int r = 0; r < R; ++r) p[n][r] = se[n][r] + (so[n][r] >> 4);
}

// Exact int32 partial of one K-group whose zero point can wrap: every
// nibble is folded to int8(nib - z) as the reference does (nib + (c & 0x7f)
// never carries; the top bit is an XOR).
template <int R, int GS>
__device__ __forceinline__ void partials_wrap(const uint8_t* wg, const uint8_t* xeg, const uint8_t* xog, int rot,
                                              int half_k, int z, int (&p)[R]) {
  constexpr int kCpg = GS / 32;
  const uint32_t cb = static_cast<uint32_t>(-z) & 0xFFu;
  const uint32_t c7 = (cb & 0x7Fu) * 0x01010101u;
  const uint32_t c8 = (cb & 0x80u) * 0x01010101u;
#pragma unroll
  for (int r = 0; r < R; ++r) p[r] = 0;
#pragma unroll
  for (int i = 0; i < kCpg; ++i) {
    const int ch = 16 * ((i + rot) & (kCpg - 1));
    const uint4 w = *reinterpret_cast<const uint4*>(wg + ch);
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      lo[q] = ((wv[q] & 0x0F0F0F0Fu) + c7) ^ c8;          // k = 8q + 0, 2, 4, 6 of the chunk
      hi[q] = (((wv[q] >> 4) & 0x0F0F0F0Fu) + c7) ^ c8;   // k = 8q + 1, 3, 5, 7
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint4 xe = *reinterpret_cast<const uint4*>(xeg + r * half_k + ch);
      const uint4 xo = *reinterpret_cast<const uint4*>(xog + r * half_k + ch);
      int s = p[r];
      s = __dp4a(static_cast<int>(lo[0]), static_cast<int>(xe.x), s);
      s = __dp4a(static_cast<int>(hi[0]), static_cast<int>(xo.x), s);
      s = __dp4a(static_cast<int>(lo[1]), static_cast<int>(xe.y), s);
      s = __dp4a(static_cast<int>(hi[1]), static_cast<int>(xo.y), s);
      s = __dp4a(static_cast<int>(lo[2]), static_cast<int>(xe.z), s);
      s = __dp4a(static_cast<int>(hi[2]), static_cast<int>(xo.z), s);
      s = __dp4a(static_cast<int>(lo[3]), static_cast<int>(xe.w), s);
      s = __dp4a(static_cast<int>(hi[3]), static_cast<int>(xo.w), s);
      p[r] = s;
    }
  }
}

// One weight row against R token rows (R = the tile's token count).  Lane l
// owns K-groups l, l + 32, ...: it reads each group's GS/2 packed bytes as
// GS/32 16-byte chunks (visited in a lane-rotated order, so the 16-byte
// shared loads of a quarter warp hit distinct banks), forms the exact int32
// partials on its own and applies w_scale; one warp reduction per token row
// finishes the output.  NG groups of a lane are in flight at once.  HALF:
// rows with at most 16 K-groups are taken two per warp, one per half-warp
// (`write` is false for a half-warp without a row of its own).
template <int R, int GS, int NG, bool HALF, int kMode>
__device__ __forceinline__ void gv_row(const GemmArgs& a, const RowJob& j, const TokenTile& tt, int G, int lane,
                                       bool write) {
  constexpr int kRot = GS == 128 ? 1 : 2;       // lane -> chunk rotation (conflict-free quarter warps)
  constexpr int kSpan = HALF ? 16 : 32;         // lanes sharing one weight row
  const int l = HALF ? (lane & 15) : lane;
  const int half_k = a.K >> 1;
  const int rot = l >> kRot;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  for (int g0 = l; g0 < G; g0 += kSpan * NG) {
    int g[NG], z[NG], sxv[NG][R];
    bool valid[NG];
    const uint8_t* wg[NG];
    const uint8_t* xeg[NG];
    const uint8_t* xog[NG];
    bool any_wrap = false;
#pragma unroll
    for (int n = 0; n < NG; ++n) {
      valid[n] = g0 + kSpan * n < G;
      g[n] = valid[n] ? g0 + kSpan * n : g0;   // an idle slot repeats the first group (result unused)
      z[n] = j.z != nullptr ? j.z[g[n]] : a.w_zero[j.grow * G + g[n]];
      any_wrap |= z[n] < kWrapZero;
      wg[n] = j.w + g[n] * (GS / 2);
      xeg[n] = tt.xe + g[n] * (GS / 2);
      xog[n] = tt.xo + g[n] * (GS / 2);
#pragma unroll
      for (int r = 0; r < R; ++r) sxv[n][r] = tt.sx[r * G + g[n]];
    }
    int p[NG][R];
    if (!any_wrap) {
      partials_nowrap<R, GS, NG>(wg, xeg, xog, rot, half_k, p, z, sxv);
    } else {
#pragma unroll
      for (int n = 0; n < NG; ++n) {
        if (z[n] < kWrapZero) {
          partials_wrap<R, GS>(wg[n], xeg[n], xog[n], rot, half_k, z[n], p[n]);
        } else {
          const uint8_t* const w1[1] = {wg[n]};
          const uint8_t* const e1[1] = {xeg[n]};
          const uint8_t* const o1[1] = {xog[n]};
          int p1[1][R], z1[1] = {z[n]}, s1[1][R];
#pragma unroll
          for (int r = 0; r < R; ++r) s1[0][r] = sxv[n][r];
          partials_nowrap<R, GS, 1>(w1, e1, o1, rot, half_k, p1, z1, s1);
#pragma unroll
          for (int r = 0; r < R; ++r) p[n][r] = p1[0][r];
        }
      }
    }
#pragma unroll
    for (int n = 0; n < NG; ++n) {
      if (!valid[n]) continue;
      const float ws = j.ws != nullptr ? j.ws[g[n]] : __ldg(a.w_scale + j.grow * G + g[n]);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        acc[r] = fmaf(static_cast<float>(p[n][r]), ws, acc[r]);
        if constexpr (kMode == kGvPartials)
          if (write) a.partials[(static_cast<int64_t>(g[n]) * a.M_total + j.m0 + r) * a.N + j.n] = p[n][r];
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float v = acc[r];
#pragma unroll
    for (int d = kSpan / 2; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    if (l == 0 && write) {
      const int m = j.m0 + r;
      if constexpr (kMode == kGvCombine) {
        store_output(a, m, j.n, v);   // fused top-k combine into the token's fp32 row
      } else if constexpr (kMode == kGvRowAddr) {
        const uint64_t row = __ldg(a.out_rows + m);
        if (row != 0) reinterpret_cast<__nv_bfloat16*>(row)[j.n] = __float2bfloat16_rn(v * tt.xsc[r]);
      } else {
        a.out[static_cast<int64_t>(m) * a.out_stride0 + static_cast<int64_t>(j.n) * a.out_stride1] =
            __float2bfloat16_rn(v * tt.xsc[r]);
      }
    }
  }
}

// Exact int32 partials of one K-group (one lane's) for two weight rows
// against the same R token rows, zero points that cannot wrap (the sums of
// partials_nowrap); each token chunk is read from shared memory once for
// both rows.
template <int R, int GS>
__device__ __forceinline__ void partials_nowrap_pair(const uint8_t* const (&wg)[2], const uint8_t* xeg,
                                                     const uint8_t* xog, int rot, int half_k, int (&p)[2][R],
                                                     const int (&z)[2], const int (&sxv)[R]) {
  constexpr int kCpg = GS / 32;
  int se[2][R], so[2][R];
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int r = 0; r < R; ++r) { se[n][r] = -z[n] * sxv[r]; so[n][r] = 0; }
#pragma unroll
  for (int i = 0; i < kCpg; ++i) {
    const int ch = 16 * ((i + rot) & (kCpg - 1));
    uint32_t lo[2][4], hi[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const uint4 w = *reinterpret_cast<const uint4*>(wg[n] + ch);
      lo[n][0] = w.x & 0x0F0F0F0Fu; lo[n][1] = w.y & 0x0F0F0F0Fu;
      lo[n][2] = w.z & 0x0F0F0F0Fu; lo[n][3] = w.w & 0x0F0F0F0Fu;
      hi[n][0] = w.x & 0xF0F0F0F0u; hi[n][1] = w.y & 0xF0F0F0F0u;
      hi[n][2] = w.z & 0xF0F0F0F0u; hi[n][3] = w.w & 0xF0F0F0F0u;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint4 xe = *reinterpret_cast<const uint4*>(xeg + r * half_k + ch);
      const uint4 xo = *reinterpret_cast<const uint4*>(xog + r * half_k + ch);
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        se[n][r] = dp4a_us(lo[n][0], xe.x, se[n][r]);
        so[n][r] = dp4a_us(hi[n][0], xo.x, so[n][r]);
        se[n][r] = dp4a_us(lo[n][1], xe.y, se[n][r]);
        so[n][r] = dp4a_us(hi[n][1], xo.y, so[n][r]);
        se[n][r] = dp4a_us(lo[n][2], xe.z, se[n][r]);
        so[n][r] = dp4a_us(hi[n][2], xo.z, so[n][r]);
        se[n][r] = dp4a_us(lo[n][3], xe.w, se[n][r]);
        so[n][r] = dp4a_us(hi[n][3], xo.w, so[n][r]);
      }
    }
  }
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int r = 0; r < R; ++r) p[n][r] = se[n][r] + (so[n][r] >> 4);
}

// Short rows (at most 16 K-groups) at one token row per expert: a half-warp
// takes two weight rows (j[0], j[1]) and each lane reads its K-group's token
// chunks once for both, so the shared-memory reads per weight byte fall from
// three to two (weights, even-k and odd-k token bytes for one row against
// weights of two rows and one set of token bytes).  Each row's sum is formed
// as in gv_row (same lane order, same reduction), so the outputs equal
// gv_row's bit for bit.  write[n] is false for a row the caller has not got
// (computed on a duplicate index, not stored).
template <int R, int GS, int kMode>
__device__ __forceinline__ void gv_pair_half(const GemmArgs& a, const RowJob (&j)[2], const bool (&write)[2],
                                             const TokenTile& tt, int G, int lane) {
  constexpr int kRot = GS == 128 ? 1 : 2;
  const int l = lane & 15;
  const int half_k = a.K >> 1;
  const int rot = l >> kRot;
  float acc[2][R];
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int r = 0; r < R; ++r) acc[n][r] = 0.f;
  for (int g = l; g < G; g += 16) {
    int z[2], sxv[R];
    const uint8_t* wg[2];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      z[n] = j[n].z != nullptr ? j[n].z[g] : a.w_zero[j[n].grow * G + g];
      wg[n] = j[n].w + g * (GS / 2);
    }
    const uint8_t* xeg = tt.xe + g * (GS / 2);
    const uint8_t* xog = tt.xo + g * (GS / 2);
#pragma unroll
    for (int r = 0; r < R; ++r) sxv[r] = tt.sx[r * G + g];
    int p[2][R];
    if (z[0] >= kWrapZero && z[1] >= kWrapZero) {
      partials_nowrap_pair<R, GS>(wg, xeg, xog, rot, half_k, p, z, sxv);
    } else {
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        if (z[n] < kWrapZero) {
          partials_wrap<R, GS>(wg[n], xeg, xog, rot, half_k, z[n], p[n]);
        } else {
          const uint8_t* const w1[1] = {wg[n]};
          const uint8_t* const e1[1] = {xeg};
          const uint8_t* const o1[1] = {xog};
          int p1[1][R], z1[1] = {z[n]}, s1[1][R];
#pragma unroll
          for (int r = 0; r < R; ++r) s1[0][r] = sxv[r];
          partials_nowrap<R, GS, 1>(w1, e1, o1, rot, half_k, p1, z1, s1);
#pragma unroll
          for (int r = 0; r < R; ++r) p[n][r] = p1[0][r];
        }
      }
    }
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const float ws = j[n].ws != nullptr ? j[n].ws[g] : __ldg(a.w_scale + j[n].grow * G + g);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        acc[n][r] = fmaf(static_cast<float>(p[n][r]), ws, acc[n][r]);
        if constexpr (kMode == kGvPartials)
          if (write[n]) a.partials[(static_cast<int64_t>(g) * a.M_total + j[n].m0 + r) * a.N + j[n].n] = p[n][r];
      }
    }
  }
#pragma unroll
  for (int n = 0; n < 2; ++n) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float v = acc[n][r];
#pragma unroll
      for (int d = 8; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
      if (l == 0 && write[n]) {
        const int m = j[n].m0 + r;
        if constexpr (kMode == kGvCombine) {
          store_output(a, m, j[n].n, v);
        } else if constexpr (kMode == kGvRowAddr) {
          const uint64_t row = __ldg(a.out_rows + m);
          if (row != 0) reinterpret_cast<__nv_bfloat16*>(row)[j[n].n] = __float2bfloat16_rn(v * tt.xsc[r]);
        } else {
          a.out[static_cast<int64_t>(m) * a.out_stride0 + static_cast<int64_t>(j[n].n) * a.out_stride1] =
              __float2bfloat16_rn(v * tt.xsc[r]);
        }
      }
    }
  }
}

// One ring stage of short rows (at most 16 K-groups; rows [0, rows) of the
// block at n0) against the tile's R token rows.  R = 1: a pair of weight
// rows per half-warp, four per warp (gv_pair_half); R >= 2: one row per
// half-warp, two per warp (the second row's chains would not fit the
// register budget).
template <int R, int GS, int kMode>
__device__ __forceinline__ void gv_short_stage(const GemmArgs& a, const GvParams& gp, const Tile& tile, int n0,
                                               int rows, const uint8_t* st, const float* s_ws, const int8_t* s_z,
                                               const TokenTile& tt, int G, int warp, int lane) {
  auto job = [&](int ri) {
    return RowJob{st + ri * gp.row_bytes, gp.meta_bulk ? s_z + ri * G : nullptr,
                  gp.meta_bulk ? s_ws + ri * G : nullptr, tile.m0, n0 + ri,
                  static_cast<int64_t>(tile.e) * a.N + n0 + ri};
  };
  if constexpr (R == 1) {
    for (int rr = 4 * warp; rr < rows; rr += 4 * kGvConsumers) {
      const int r0 = rr + 2 * (lane >> 4);
      const bool write[2] = {r0 < rows, r0 + 1 < rows};
      const int i0 = write[0] ? r0 : rr;
      const RowJob jb[2] = {job(i0), job(write[1] ? r0 + 1 : i0)};
      gv_pair_half<1, GS, kMode>(a, jb, write, tt, G, lane);
    }
  } else {
    for (int rr = 2 * warp; rr < rows; rr += 2 * kGvConsumers) {
      const int mine = rr + (lane >> 4);
      const bool write = mine < rows;
      gv_row<R, GS, 1, true, kMode>(a, job(write ? mine : rr), tt, G, lane, write);
    }
  }
}

// Stages the token rows [m0, m0 + rows) of x_q: per 32-value chunk the 16
// even-k bytes and the 16 odd-k bytes, and per K-group the sum of its
// values.  Called by all consumer threads between two consumer barriers.
__device__ __forceinline__ void stage_tokens(const GemmArgs& a, int m0, int rows, uint8_t* xe, uint8_t* xo, int* sx,
                                             float* xsc) {
  // token scales: read once per token block here instead of by every row's
  // store (a global load at the end of each row's chain)
  if (threadIdx.x < rows) xsc[threadIdx.x] = __ldg(a.x_scale + m0 + threadIdx.x);
  const int half_k = a.K >> 1;
  const int G = a.K / a.gs;
  const int cpg = a.gs / 32;
  for (int i = threadIdx.x; i < rows * G; i += kGvConsumers * 32) {
    const int r = i / G, g = i - r * G;
    int s = 0;
    for (int cc = 0; cc < cpg; ++cc) {
      const int c = g * cpg + cc;
      const uint4* src = reinterpret_cast<const uint4*>(a.x_q + static_cast<int64_t>(m0 + r) * a.x_stride0 + 32 * c);
      const uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
      const uint32_t wv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      uint32_t e[4], o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        // reference layout: 8 bytes x0..x7 -> (x0, x2, x4, x6) and (x1, x3, x5, x7);
        // prepacked weights: (x0, x1, x2, x3) and (x4, x5, x6, x7), the k order of
        // a weight word's low and high nibbles
        e[q] = a.layout == 0 ? __byte_perm(wv[2 * q], wv[2 * q + 1], 0x6420) : wv[2 * q];
        o[q] = a.layout == 0 ? __byte_perm(wv[2 * q], wv[2 * q + 1], 0x7531) : wv[2 * q + 1];
        s = __dp4a(static_cast<int>(wv[2 * q]), 0x01010101, s);
        s = __dp4a(static_cast<int>(wv[2 * q + 1]), 0x01010101, s);
      }
      *reinterpret_cast<uint4*>(xe + r * half_k + 16 * c) = make_uint4(e[0], e[1], e[2], e[3]);
      *reinterpret_cast<uint4*>(xo + r * half_k + 16 * c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    sx[r * G + g] = s;
  }
}

// Splits the tiles into gridDim.x contiguous ranges of equal cost and
// writes this CTA's range to range[0..1].  A block of R token rows costs
// R + 2 units (measured streaming rates at 1, 2 and 4 rows per expert are in
// the ratio 1 : 1.34 : 2.03), so CTAs that meet multi-row experts get fewer
// blocks and finish with the others.  Out of line, so its registers do not
// weigh on the streaming loop.  Called by all threads (contains
// __syncthreads); cprefix is [E+1] shared scratch.
__device__ __noinline__ void cost_balanced_range(int E, int NB, const int* cnt, const int* prefix, int total,
                                                  long long* cprefix, int* range) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int per = (E + 31) / 32;
    const int lo = lane * per;
    long long local = 0;
    for (int i = 0; i < per; ++i) {
      const int e = lo + i;
      if (e < E) {
        const int c = cnt[e];
        local += static_cast<long long>(NB) * (c + 2 * ((c + kGvRows - 1) / kGvRows));
      }
    }
    long long incl = local;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const long long v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    long long run = incl - local;
    for (int i = 0; i < per; ++i) {
      const int e = lo + i;
      if (e < E) {
        cprefix[e] = run;
        const int c = cnt[e];
        run += static_cast<long long>(NB) * (c + 2 * ((c + kGvRows - 1) / kGvRows));
      }
    }
    if (lane == 31) cprefix[E] = incl;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long total_cost = cprefix[E];
    for (int side = 0; side < 2; ++side) {
      const unsigned b = blockIdx.x + side;
      int t;
      if (b == 0) {
        t = 0;
      } else if (b == gridDim.x) {
        t = total;
      } else {   // first tile whose cost start is at or past the window edge
        const long long target = total_cost * b / gridDim.x;
        int lo = 0, hi = E - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (cprefix[mid] <= target) lo = mid; else hi = mid - 1;
        }
        const int tiles_e = prefix[lo + 1] - prefix[lo];
        const long long cost_e = cprefix[lo + 1] - cprefix[lo];
        long long local = cost_e > 0 ? ((target - cprefix[lo]) * tiles_e + cost_e - 1) / cost_e : 0;
        if (local > tiles_e) local = tiles_e;
        t = prefix[lo] + static_cast<int>(local);
      }
      range[side] = t;
    }
  }
  __syncthreads();
}

// kShort: every row has at most 16 K-groups and a warp takes two rows, one
// per half-warp (a separate instantiation, so neither mode's register
// allocation pays for the other's code).  kMode: plain bf16 rows, the fused
// top-k combine store, or bf16 rows plus the int32 partials export (each its
// own instantiation, so the plain kernel carries neither).
template <bool kShort, int kMode>
__global__ void __launch_bounds__(kGvThreads, 2)
gemm_gemv_kernel(const GemmArgs a, const GvParams gp) {
  extern __shared__ unsigned char smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int stage_bytes = gp.stage_w + gp.ws_bytes + gp.z_bytes;
  uint8_t* s_xe = base + gp.stages * stage_bytes;
  uint8_t* s_xo = s_xe + gp.x_bytes / 2;
  int* s_sx = reinterpret_cast<int*>(s_xe + gp.x_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(s_sx) + gp.sx_bytes);
  uint64_t* empty = full + kGvMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kGvMaxStages);
  float* s_xsc = const_cast<float*>(reinterpret_cast<volatile float*>(abort_flag + 4));   // [kGvRows]
  int* sched_mem = const_cast<int*>(reinterpret_cast<volatile int*>(abort_flag)) + 8;

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < gp.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGvConsumers);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  // token block as the slow index: a CTA stages each block's token rows once
  TileSched sch{sched_mem, sched_mem + (a.E + 1), sched_mem + 2 * (a.E + 1), a.E, kGvRows,
                (a.N + gp.RB - 1) / gp.RB, a.min_rows, a.max_rows, true};
  const int total = sched_build(sch, a.offsets, a.M_total);   // contains __syncthreads
  const int G = a.K / a.gs;
  // Each CTA takes a contiguous range of blocks (consecutive blocks belong to
  // the same expert, so its token rows are staged once for many blocks),
  // sized by cost rather than by count (see cost_balanced_range).
  __shared__ int s_range[2];
  cost_balanced_range(a.E, sch.NB, sch.cnt, sch.prefix, total,
                      reinterpret_cast<long long*>(sched_mem + ((3 * (a.E + 1) + 1) & ~1)), s_range);
  const int t_begin = s_range[0], t_end = s_range[1];

  if (warp == kGvConsumers) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      TileWalk walk;
      if (t_begin < t_end) walk.start(sch, t_begin);
      for (int t = t_begin; t < t_end; ++t) {
        if (t > t_begin) walk.next();
        const Tile tile = walk.cur;
        const int n0 = tile.nb * gp.RB;
        const int rows = min(gp.RB, a.N - n0);
        const int64_t row0 = static_cast<int64_t>(tile.e) * a.N + n0;
        if (!mbar_wait(&empty[stage], phase ^ 1, a.status, kDevTimeoutLoadEmpty, abort_flag)) break;
        uint8_t* st = base + stage * stage_bytes;
        const uint32_t wbytes = static_cast<uint32_t>(rows) * gp.row_bytes;
        const uint32_t mbytes = gp.meta_bulk ? static_cast<uint32_t>(rows * G * 5) : 0u;
        mbar_arrive_expect_tx(&full[stage], wbytes + mbytes);
        bulk_g2s(st, a.w_packed + row0 * gp.row_bytes, wbytes, &full[stage], pol);
        if (gp.meta_bulk) {
          bulk_g2s(st + gp.stage_w, a.w_scale + row0 * G, static_cast<uint32_t>(rows * G * 4), &full[stage], pol);
          bulk_g2s(st + gp.stage_w + gp.ws_bytes, a.w_zero + row0 * G, static_cast<uint32_t>(rows * G),
                   &full[stage], pol);
        }
        if (++stage == gp.stages) { stage = 0; phase ^= 1; }
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const TokenTile tt{s_xe, s_xo, s_sx, s_xsc};
    int cur_m0 = -1, cur_rows = 0;
    int stage = 0;
    uint32_t phase = 0;
    bool failed = false;   // after a timed-out wait, keep walking the tiles (no work) so the
                           // consumer barriers below still see every consumer warp
    TileWalk walk;
    if (t_begin < t_end) walk.start(sch, t_begin);
    for (int t = t_begin; t < t_end; ++t) {
      if (t > t_begin) walk.next();
      const Tile tile = walk.cur;
      if (tile.m0 != cur_m0 || tile.rows != cur_rows) {   // uniform over the consumers
        consumers_sync();                                 // nobody still reads the old rows
        stage_tokens(a, tile.m0, tile.rows, s_xe, s_xo, s_sx, s_xsc);
        consumers_sync();
        cur_m0 = tile.m0;
        cur_rows = tile.rows;
      }
      if (failed) continue;
      const int n0 = tile.nb * gp.RB;
      const int rows = min(gp.RB, a.N - n0);
      if (!mbar_wait(&full[stage], phase, a.status, kDevTimeoutLoadFull, abort_flag)) {
        failed = true;
        continue;
      }
      const uint8_t* st = base + stage * stage_bytes;
      const float* s_ws = reinterpret_cast<const float*>(st + gp.stage_w);
      const int8_t* s_z = reinterpret_cast<const int8_t*>(st + gp.stage_w + gp.ws_bytes);
      if constexpr (kShort) {
        // the token count is switched on once per stage, outside the row loop
        if (a.gs == 128) {
          switch (tile.rows) {   // warp-uniform: the tile's token count
            case 1: gv_short_stage<1, 128, kMode>(a, gp, tile, n0, rows, st, s_ws, s_z, tt, G, warp, lane); break;
            case 2: gv_short_stage<2, 128, kMode>(a, gp, tile, n0, rows, st, s_ws, s_z, tt, G, warp, lane); break;
            case 3: gv_short_stage<3, 128, kMode>(a, gp, tile, n0, rows, st, s_ws, s_z, tt, G, warp, lane); break;
            default: gv_short_stage<4, 128, kMode>(a, gp, tile, n0, rows, st, s_ws, s_z, tt, G, warp, lane); break;
          }
        } else {
          switch (tile.rows) {
            case 1: gv_short_stage<1, 64, kMode>(a, gp, tile, n0, rows, st, s_ws, s_z, tt, G, warp, lane); break;
            case 2: gv_short_stage<2, 64, kMode>(a, gp, tile, n0, rows, st, s_ws, s_z, tt, G, warp, lane); break;
            case 3: gv_short_stage<3, 64, kMode>(a, gp, tile, n0, rows, st, s_ws, s_z, tt, G, warp, lane); break;
            default: gv_short_stage<4, 64, kMode>(a, gp, tile, n0, rows, st, s_ws, s_z, tt, G, warp, lane); break;
          }
        }
      } else {
        for (int rr = warp; rr < rows; rr += kGvConsumers) {
          const RowJob job{st + rr * gp.row_bytes, gp.meta_bulk ? s_z + rr * G : nullptr,
                           gp.meta_bulk ? s_ws + rr * G : nullptr, tile.m0, n0 + rr,
                           static_cast<int64_t>(tile.e) * a.N + n0 + rr};
          if (a.gs == 128) {
            switch (tile.rows) {   // warp-uniform: the tile's token count
              // two groups in flight per lane only when every lane has a second
              // group (G > 32); with G <= 32 the second slot would repeat the first
              case 1:
                if (G > 32) gv_row<1, 128, 2, false, kMode>(a, job, tt, G, lane, true);
                else gv_row<1, 128, 1, false, kMode>(a, job, tt, G, lane, true);
                break;
              case 2:
                if (G > 32) gv_row<2, 128, 2, false, kMode>(a, job, tt, G, lane, true);
                else gv_row<2, 128, 1, false, kMode>(a, job, tt, G, lane, true);
                break;
              case 3: gv_row<3, 128, 1, false, kMode>(a, job, tt, G, lane, true); break;
              default: gv_row<4, 128, 1, false, kMode>(a, job, tt, G, lane, true); break;
            }
          } else {
            switch (tile.rows) {
              case 1:
                if (G > 32) gv_row<1, 64, 2, false, kMode>(a, job, tt, G, lane, true);
                else gv_row<1, 64, 1, false, kMode>(a, job, tt, G, lane, true);
                break;
              case 2:
                if (G > 32) gv_row<2, 64, 2, false, kMode>(a, job, tt, G, lane, true);
                else gv_row<2, 64, 1, false, kMode>(a, job, tt, G, lane, true);
                break;
              case 3: gv_row<3, 64, 1, false, kMode>(a, job, tt, G, lane, true); break;
              default: gv_row<4, 64, 1, false, kMode>(a, job, tt, G, lane, true); break;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == gp.stages) { stage = 0; phase ^= 1; }
    }
  }
}

}  // namespace

cudaError_t launch_gemm_gemv(const GemmArgs& a, cudaStream_t stream) {
  if (a.M_total <= 0) return cudaSuccess;
  const int row_bytes = a.K / 2;
  const int G = a.K / a.gs;
  if ((a.gs != 64 && a.gs != 128) || (a.K % 64) != 0 || (reinterpret_cast<uintptr_t>(a.x_q) & 15) ||
      (a.x_stride0 % 16) || (reinterpret_cast<uintptr_t>(a.w_packed) & 15))
    return cudaErrorInvalidValue;
  GvParams gp;
  gp.row_bytes = row_bytes;
  // rows per block: a multiple of the consumer warps, about kGvTargetW bytes
  gp.RB = (kGvTargetW / row_bytes) / kGvConsumers * kGvConsumers;
  if (gp.RB < kGvConsumers) gp.RB = kGvConsumers;
  if (gp.RB > kGvMaxRB) gp.RB = kGvMaxRB;
  gp.stage_w = gp.RB * row_bytes;
  // scales / zero points ride with the block when every block's slice of
  // them is 16-byte aligned in start and size
  auto al16 = [](int64_t v) { return (v % 16) == 0; };
  const int tail = a.N % gp.RB;
  gp.meta_bulk = al16(static_cast<int64_t>(a.N) * G) && al16(static_cast<int64_t>(gp.RB) * G) &&
                 al16(static_cast<int64_t>(tail) * G) && (reinterpret_cast<uintptr_t>(a.w_scale) % 16 == 0) &&
                 (reinterpret_cast<uintptr_t>(a.w_zero) % 16 == 0);
  gp.ws_bytes = gp.meta_bulk ? gp.RB * G * 4 : 0;
  gp.z_bytes = gp.meta_bulk ? ((gp.RB * G + 15) / 16) * 16 : 0;
  gp.x_bytes = kGvRows * a.K;                    // K is a multiple of 64: both halves stay 16-byte aligned
  gp.sx_bytes = ((kGvRows * G * 4 + 15) / 16) * 16;
  const size_t stage_bytes = gp.stage_w + gp.ws_bytes + gp.z_bytes;
  const size_t fixed = 128 + gp.x_bytes + gp.sx_bytes + 2 * kGvMaxStages * 8 + 32 + sizeof(int) * 3 * (a.E + 1) + 8 +
                       sizeof(long long) * (a.E + 1);
  // deepest ring that keeps two CTAs per SM, else the deepest that fits one
  gp.stages = kGvMaxStages;
  while (gp.stages > 2 && fixed + gp.stages * stage_bytes > kGvSmemBudget) --gp.stages;
  if (fixed + gp.stages * stage_bytes > kGvSmemBudget) {
    gp.stages = kGvMaxStages;
    while (gp.stages > 1 && fixed + gp.stages * stage_bytes > 227 * 1024) --gp.stages;
  }
  const size_t smem = fixed + gp.stages * stage_bytes;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  auto kernel = a.comb_out != nullptr
                     ? (G <= 16 ? gemm_gemv_kernel<true, kGvCombine> : gemm_gemv_kernel<false, kGvCombine>)
                 : a.out_rows != nullptr
                     ? (G <= 16 ? gemm_gemv_kernel<true, kGvRowAddr> : gemm_gemv_kernel<false, kGvRowAddr>)
                 : a.partials != nullptr
                     ? (G <= 16 ? gemm_gemv_kernel<true, kGvPartials> : gemm_gemv_kernel<false, kGvPartials>)
                     : (G <= 16 ? gemm_gemv_kernel<true, kGvPlain> : gemm_gemv_kernel<false, kGvPlain>);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kGvThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  kernel<<<sms * per_sm, kGvThreads, smem, stream>>>(a, gp);   // persistent: resident CTAs only
  return cudaGetLastError();
}

}  // namespace w4a8
