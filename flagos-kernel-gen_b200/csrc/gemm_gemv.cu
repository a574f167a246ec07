// Streaming W4A8 grouped GEMM for experts with few rows (decode): the weights
// are read from HBM exactly once by the TMA engine, CUDA cores do the math.
//
// At 1-4 tokens per expert the layer is bound by reading the packed weights.
// A 128-row tensor-core tile with N = 16 pays a fixed ~64-cycle MMA floor per
// 32-byte K step plus TMEM round trips per K-group, longer than its 8 KB of
// weights take to arrive, so this path keeps the tensor cores out of it:
//   * one producer warp streams a block of RB contiguous weight rows of one
//     expert (RB * K/2 bytes, <= 32 KB) into a 4-stage shared-memory ring with
//     a single cp.async.bulk per stage (no multicast), plus the block's
//     w_scale / w_zero rows (bulk copies when 16-byte aligned, else loaded by
//     the consumers directly);
//   * eight consumer warps each take rows of the block: lanes read 16 packed
//     bytes (32 K values) per 1024-wide K step from shared memory, unpack the
//     nibbles and fold the zero point with the reference's int8 wrap
//     (docs/Task1.md:78-85), dp4a against up to kGvRows token rows (read from
//     L1: every row of the expert uses them);
//   * the 4 (gs = 128) or 2 (gs = 64) lanes of a K-group are summed with
//     shuffles -> the exact int32 partial of docs/Task1.md:100-104; the group's
//     first lane applies w_scale, a warp reduction and x_scale give the bf16
//     output (docs/Task1.md:107-112).
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
constexpr int kGvMaxStages = 4;   // ring depth per CTA (two CTAs per SM)
constexpr int kGvTargetW = 32 * 1024;                  // preferred weight bytes per stage
constexpr int kGvMaxRB = 32;                           // rows per block
constexpr int kGvSmemBudget = 110 * 1024;   // two CTAs per SM

struct GvParams {
  int stages;      // ring depth (2..4)
  int stage_w;     // weight bytes per stage (RB * row_bytes)
  int RB;          // weight rows per block (a multiple of the consumer warp count)
  int row_bytes;   // K/2
  int meta_bulk;   // 1: scales / zero points travel with the block (16-byte aligned)
  int ws_bytes;    // per-stage bytes reserved for scales (RB*G*4, 16-aligned)
  int z_bytes;     // per-stage bytes reserved for zero points (RB*G, 16-aligned)
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void unpack_fold(uint4 w, int z, uint32_t (&o)[8]) {
  const uint32_t cb = static_cast<uint32_t>(-z) & 0xFFu;
  const uint32_t c7 = (cb & 0x7Fu) * 0x01010101u;
  const uint32_t c8 = (cb & 0x80u) * 0x01010101u;
  const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t lo = wv[q] & 0x0F0F0F0Fu;
    const uint32_t hi = (wv[q] >> 4) & 0x0F0F0F0Fu;
    o[2 * q] = (__byte_perm(lo, hi, 0x5140) + c7) ^ c8;
    o[2 * q + 1] = (__byte_perm(lo, hi, 0x7362) + c7) ^ c8;
  }
}

struct RowJob {
  const uint8_t* w;      // packed weight row in shared memory
  const int8_t* z;       // zero points of the row in shared memory (nullptr: read global)
  const float* ws;       // scales of the row in shared memory (nullptr: read global)
  const int8_t* x;       // first token row of the tile (global)
  int m0, n;             // first token row, output channel
  int64_t grow;          // e * N + n
};

// One weight row against R token rows (R = the tile's token count).
template <int R>
__device__ __forceinline__ void gv_row(const GemmArgs& a, const RowJob& j, int G, int lane) {
  const int lpg = a.gs / 32;   // lanes per K-group (4 or 2)
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
#pragma unroll 2
  for (int kstep = 0; kstep < a.K; kstep += 1024) {
    const int k0 = kstep + lane * 32;
    const bool active = k0 < a.K;
    const int g = active ? k0 / a.gs : 0;
    int p[R];
#pragma unroll
    for (int r = 0; r < R; ++r) p[r] = 0;
    if (active) {
      const int z = j.z != nullptr ? j.z[g] : a.w_zero[j.grow * G + g];
      uint32_t o[8];
      unpack_fold(*reinterpret_cast<const uint4*>(j.w + k0 / 2), z, o);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint4* xr = reinterpret_cast<const uint4*>(j.x + static_cast<int64_t>(r) * a.x_stride0 + k0);
        const uint4 x0 = __ldg(xr), x1 = __ldg(xr + 1);
        int s = 0;
        s = __dp4a(static_cast<int>(o[0]), static_cast<int>(x0.x), s);
        s = __dp4a(static_cast<int>(o[1]), static_cast<int>(x0.y), s);
        s = __dp4a(static_cast<int>(o[2]), static_cast<int>(x0.z), s);
        s = __dp4a(static_cast<int>(o[3]), static_cast<int>(x0.w), s);
        s = __dp4a(static_cast<int>(o[4]), static_cast<int>(x1.x), s);
        s = __dp4a(static_cast<int>(o[5]), static_cast<int>(x1.y), s);
        s = __dp4a(static_cast<int>(o[6]), static_cast<int>(x1.z), s);
        s = __dp4a(static_cast<int>(o[7]), static_cast<int>(x1.w), s);
        p[r] = s;
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      p[r] += __shfl_xor_sync(0xffffffffu, p[r], 1);
      if (lpg == 4) p[r] += __shfl_xor_sync(0xffffffffu, p[r], 2);
    }
    if (active && (lane % lpg) == 0) {
      const float ws = j.ws != nullptr ? j.ws[g] : __ldg(a.w_scale + j.grow * G + g);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        acc[r] = fmaf(static_cast<float>(p[r]), ws, acc[r]);
        if (a.partials != nullptr) a.partials[(static_cast<int64_t>(j.m0 + r) * a.N + j.n) * G + g] = p[r];
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float v = acc[r];
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    if (lane == 0) {
      const int m = j.m0 + r;
      a.out[static_cast<int64_t>(m) * a.out_stride0 + static_cast<int64_t>(j.n) * a.out_stride1] =
          __float2bfloat16_rn(v * __ldg(a.x_scale + m));
    }
  }
}

__global__ void __launch_bounds__(kGvThreads, 2)
gemm_gemv_kernel(const GemmArgs a, const GvParams gp) {
  extern __shared__ unsigned char smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int stage_bytes = gp.stage_w + gp.ws_bytes + gp.z_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + gp.stages * stage_bytes);
  uint64_t* empty = full + kGvMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kGvMaxStages);
  int* sched_mem = const_cast<int*>(reinterpret_cast<volatile int*>(abort_flag)) + 4;

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < gp.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGvConsumers);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  TileSched sch{sched_mem, sched_mem + (a.E + 1), sched_mem + 2 * (a.E + 1), a.E, kGvRows,
                (a.N + gp.RB - 1) / gp.RB, a.min_rows, a.max_rows};
  const int total = sched_build(sch, a.offsets, a.M_total);   // contains __syncthreads
  const int G = a.K / a.gs;
  // Each CTA takes a contiguous range of blocks: consecutive blocks belong to
  // the same expert, so its token rows stay resident in this SM's L1.
  const int per_cta = (total + gridDim.x - 1) / gridDim.x;
  const int t_begin = min(total, static_cast<int>(blockIdx.x) * per_cta);
  const int t_end = min(total, t_begin + per_cta);

  if (warp == kGvConsumers) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      for (int t = t_begin; t < t_end; ++t) {
        const Tile tile = sched_tile(sch, t);
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
    int stage = 0;
    uint32_t phase = 0;
    for (int t = t_begin; t < t_end; ++t) {
      const Tile tile = sched_tile(sch, t);
      const int n0 = tile.nb * gp.RB;
      const int rows = min(gp.RB, a.N - n0);
      if (!mbar_wait(&full[stage], phase, a.status, kDevTimeoutLoadFull, abort_flag)) break;
      const uint8_t* st = base + stage * stage_bytes;
      const float* s_ws = reinterpret_cast<const float*>(st + gp.stage_w);
      const int8_t* s_z = reinterpret_cast<const int8_t*>(st + gp.stage_w + gp.ws_bytes);
      const int8_t* xbase = a.x_q + static_cast<int64_t>(tile.m0) * a.x_stride0;
      for (int rr = warp; rr < rows; rr += kGvConsumers) {
        const RowJob job{st + rr * gp.row_bytes, gp.meta_bulk ? s_z + rr * G : nullptr,
                         gp.meta_bulk ? s_ws + rr * G : nullptr, xbase, tile.m0, n0 + rr,
                         static_cast<int64_t>(tile.e) * a.N + n0 + rr};
        switch (tile.rows) {   // warp-uniform: the tile's token count
          case 1: gv_row<1>(a, job, G, lane); break;
          case 2: gv_row<2>(a, job, G, lane); break;
          case 3: gv_row<3>(a, job, G, lane); break;
          default: gv_row<4>(a, job, G, lane); break;
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
  const size_t stage_bytes = gp.stage_w + gp.ws_bytes + gp.z_bytes;
  const size_t fixed = 128 + 2 * kGvMaxStages * 8 + 16 + sizeof(int) * 3 * (a.E + 1);
  gp.stages = kGvMaxStages;
  while (gp.stages > 2 && fixed + gp.stages * stage_bytes > kGvSmemBudget) --gp.stages;
  const size_t smem = fixed + gp.stages * stage_bytes;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(gemm_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_gemv_kernel, kGvThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  gemm_gemv_kernel<<<sms * per_sm, kGvThreads, smem, stream>>>(a, gp);   // persistent: resident CTAs only
  return cudaGetLastError();
}

}  // namespace w4a8
