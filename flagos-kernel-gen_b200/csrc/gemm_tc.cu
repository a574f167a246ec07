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
// channels) and its N dimension is the token block (16..128 rows of the
// expert's segment, rounded up to 16 per tile at run time).  With weights on
// the M side, every epilogue thread owns one output channel, so the per-group
// weight scale is a single register per thread and the int32 -> fp32 scale
// step is one FMA per element.
//
// Warp roles (448 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer: packed weight tile [128 rows x 64 B] and the
//               token tile [rows x 128 B] (128-byte swizzle) per 128-wide K block
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2-5   transform: thread r unpacks weight row r (nibble order of
//               docs/Task1.md:78-81, zero fold with int8 wrap of :84-85) into the
//               canonical 128B-swizzled K-major layout the MMA reads
//   warps 6-13  epilogue: two warpgroups, each reads 64 token columns of the
//               per-group int32 accumulator from TMEM, applies w_scale, and
//               finally x_scale and the bf16 store
// TMEM holds two 128-column int32 accumulators so that group g+1's MMAs run
// while the epilogue drains group g.
#include "common.cuh"
#include "w4a8_internal.h"

#include <cudaTypedefs.h>
#include <mutex>

namespace w4a8 {

namespace {

constexpr int kBW = 128;         // weight rows per tile (MMA M)
constexpr int kBT = 128;         // max token rows per tile (MMA N)
constexpr int kBK = 128;         // K bytes per pipeline stage
constexpr int kStages = 4;       // TMA stages (packed weights + tokens)
constexpr int kAStages = 2;      // unpacked weight stages
constexpr int kXBytes = kBT * kBK;          // 16 KB
constexpr int kABytes = kBW * kBK;          // 16 KB
constexpr int kWBytes = kBW * (kBK / 2);    // 8 KB
constexpr int kThreads = 448;
constexpr int kTmemCols = 256;   // 2 accumulators x 128 columns
constexpr int kXBoxRows = 16;

constexpr int kTransformWarp0 = 2;
constexpr int kEpilogueWarp0 = 6;
constexpr int kNumEpilogueWarps = 8;
constexpr int kEpiCols = kBT / 2;           // columns per epilogue warpgroup

constexpr size_t kSmemTiles = size_t(kStages) * kXBytes + size_t(kAStages) * kABytes +
                              size_t(kStages) * kWBytes;
constexpr int kNumBars = 2 * kStages + 2 * kAStages + 4;

__host__ __device__ constexpr size_t tc_smem_bytes(int E) {
  return 1024 /*alignment slack*/ + kSmemTiles + kNumBars * 8 + 16 + sizeof(int) * 3 * (E + 1);
}

__device__ __forceinline__ uint32_t pack_fold(uint32_t nib4, uint32_t c7, uint32_t c8) {
  // byte-wise (nib - z) mod 256 for nib in [0,15]: nib + (c & 0x7f) never
  // carries out of a byte, and adding the top bit mod 256 is an XOR.
  return (nib4 + c7) ^ c8;
}

__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
               const GemmArgs a) {
  extern __shared__ unsigned char smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sX = base;
  uint8_t* sA = sX + kStages * kXBytes;
  uint8_t* sW = sA + kAStages * kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + kStages * kWBytes);
  uint64_t* load_full = bars;
  uint64_t* load_empty = load_full + kStages;
  uint64_t* a_full = load_empty + kStages;
  uint64_t* a_empty = a_full + kAStages;
  uint64_t* tmem_full = a_empty + kAStages;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* sched_mem = reinterpret_cast<int*>(tmem_slot + 4);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&load_full[s], 1);
      mbar_init(&load_empty[s], 4 + 1);  // 4 transform warps + 1 MMA commit
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&a_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], kNumEpilogueWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }

  TileSched sch{sched_mem, sched_mem + (a.E + 1), sched_mem + 2 * (a.E + 1), a.E, kBT,
                (a.N + kBW - 1) / kBW};
  const int total = sched_build(sch, a.offsets, a.M_total);  // contains __syncthreads
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int G = a.K / a.gs;
  const int KB = (a.K + kBK - 1) / kBK;
  const int gpk = kBK / a.gs;  // groups per K block: 1 (gs=128) or 2 (gs=64)
  const int kpg = a.gs / 32;   // MMA K-steps (32 bytes each) per group

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const Tile tile = sched_tile(sch, t);
        const int nx = (tile.rows + kXBoxRows - 1) / kXBoxRows;
        const uint32_t bytes = kWBytes + nx * kXBoxRows * kBK;
        const int wrow = tile.e * a.N + tile.nb * kBW;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&load_empty[stage], phase ^ 1, a.status, kDevTimeoutLoadEmpty, abort_flag))
            goto producer_done;
          mbar_arrive_expect_tx(&load_full[stage], bytes);
          tma_load_2d(sW + stage * kWBytes, &tm_w, &load_full[stage], kb * (kBK / 2), wrow, pol_w);
          for (int j = 0; j < nx; ++j)
            tma_load_2d(sX + stage * kXBytes + j * kXBoxRows * kBK, &tm_x, &load_full[stage],
                        kb * kBK, tile.m0 + j * kXBoxRows, pol_x);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, astage = 0, buf = 0;
      uint32_t phase = 0, aphase = 0, bphase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const Tile tile = sched_tile(sch, t);
        int n_mma = (tile.rows + 15) & ~15;
        const uint32_t idesc = make_idesc_i8(kBW, n_mma);
        for (int g = 0; g < G; ++g) {
          const int sub = g % gpk;
          if (sub == 0) {
            if (!mbar_wait(&load_full[stage], phase, a.status, kDevTimeoutLoadFull, abort_flag))
              goto mma_done;
            if (!mbar_wait(&a_full[astage], aphase, a.status, kDevTimeoutAFull, abort_flag))
              goto mma_done;
            tc_fence_after();
          }
          if (!mbar_wait(&tmem_empty[buf], bphase ^ 1, a.status, kDevTimeoutTmemEmpty, abort_flag))
            goto mma_done;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kBT);
          const uint32_t a_addr = smem_u32(sA + astage * kABytes);
          const uint32_t b_addr = smem_u32(sX + stage * kXBytes);
          for (int ks = 0; ks < kpg; ++ks) {
            const uint32_t koff = static_cast<uint32_t>((sub * kpg + ks) * 32);
            mma_i8_ss(d_tmem, make_desc_sw128(a_addr + koff), make_desc_sw128(b_addr + koff), idesc,
                      ks > 0 ? 1u : 0u);
          }
          mma_commit(&tmem_full[buf]);
          buf ^= 1;
          if (buf == 0) bphase ^= 1;
          if (sub == gpk - 1 || g == G - 1) {
            mma_commit(&load_empty[stage]);
            mma_commit(&a_empty[astage]);
            if (++stage == kStages) { stage = 0; phase ^= 1; }
            if (++astage == kAStages) { astage = 0; aphase ^= 1; }
          }
        }
      }
    mma_done:;
    }
  } else if (warp >= kTransformWarp0 && warp < kTransformWarp0 + 4) {
    // ------------------------------------------------------------ int4 -> int8 transform
    const int r = (warp - kTransformWarp0) * 32 + lane;  // weight row within the tile
    int stage = 0, astage = 0;
    uint32_t phase = 0, aphase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const Tile tile = sched_tile(sch, t);
      const int n = tile.nb * kBW + r;
      const bool valid = n < a.N;
      const int8_t* zrow = a.w_zero + (static_cast<int64_t>(tile.e) * a.N + (valid ? n : 0)) * G;
      for (int kb = 0; kb < KB; ++kb) {
        const int g0 = kb * gpk;
        const int z0 = valid ? zrow[g0] : 0;
        const int z1 = (gpk == 2 && valid && g0 + 1 < G) ? zrow[g0 + 1] : z0;
        if (!mbar_wait(&load_full[stage], phase, a.status, kDevTimeoutLoadFull, abort_flag)) goto tr_done;
        // Packed row r (64 B) is read as four 16-byte chunks.  Register slot c
        // holds chunk (c + rot) & 3: rotating by row pair puts the 8 lanes of a
        // quarter-warp on 8 distinct 16-byte bank groups.
        const int rot = (r >> 1) & 3;
        uint4 pk[4];
        {
          const uint8_t* src = sW + stage * kWBytes + r * (kBK / 2);
#pragma unroll
          for (int c = 0; c < 4; ++c) pk[c] = *reinterpret_cast<const uint4*>(src + ((c + rot) & 3) * 16);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&load_empty[stage]);
        if (++stage == kStages) { stage = 0; phase ^= 1; }

        if (!mbar_wait(&a_empty[astage], aphase ^ 1, a.status, kDevTimeoutAEmpty, abort_flag)) goto tr_done;
        uint8_t* dst_row = sA + astage * kABytes + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          // packed chunk cc (16 B) -> K offsets [32cc, 32cc+32) -> output chunks 2cc, 2cc+1
          const int cc = (c + rot) & 3;
          const int zc = (cc < 2) ? z0 : z1;   // gs=64: chunks 0-1 are group 2kb, 2-3 group 2kb+1
          const uint32_t cb = static_cast<uint32_t>(-zc) & 0xFFu;
          const uint32_t c7 = (cb & 0x7Fu) * 0x01010101u;
          const uint32_t c8 = (cb & 0x80u) * 0x01010101u;
          uint32_t o[8];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t wq = q == 0 ? pk[c].x : q == 1 ? pk[c].y : q == 2 ? pk[c].z : pk[c].w;
            const uint32_t lo = wq & 0x0F0F0F0Fu;
            const uint32_t hi = (wq >> 4) & 0x0F0F0F0Fu;
            o[2 * q] = pack_fold(__byte_perm(lo, hi, 0x5140), c7, c8);
            o[2 * q + 1] = pack_fold(__byte_perm(lo, hi, 0x7362), c7, c8);
          }
          const int j0 = 2 * cc, j1 = 2 * cc + 1;
          *reinterpret_cast<uint4*>(dst_row + ((j0 ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(dst_row + ((j1 ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[astage]);
        if (++astage == kAStages) { astage = 0; aphase ^= 1; }
      }
    }
  tr_done:;
  } else if (warp >= kEpilogueWarp0 && warp < kEpilogueWarp0 + kNumEpilogueWarps) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;                     // TMEM lane quarter this warp may access
    const int wg = (warp - kEpilogueWarp0) >> 2;      // column half
    const int r = quarter * 32 + lane;                // weight row within the tile
    int buf = 0;
    uint32_t bphase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const Tile tile = sched_tile(sch, t);
      const int n = tile.nb * kBW + r;
      const bool valid = n < a.N;
      const float* wsrow = a.w_scale + (static_cast<int64_t>(tile.e) * a.N + (valid ? n : 0)) * G;
      float acc[kEpiCols];
#pragma unroll
      for (int c = 0; c < kEpiCols; ++c) acc[c] = 0.f;
      float ws_next = valid ? __ldg(wsrow) : 0.f;
      for (int g = 0; g < G; ++g) {
        const float ws = ws_next;
        if (valid && g + 1 < G) ws_next = __ldg(wsrow + g + 1);
        if (!mbar_wait(&tmem_full[buf], bphase, a.status, kDevTimeoutTmemFull, abort_flag)) goto epi_done;
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(buf * kBT + wg * kEpiCols);
#pragma unroll
        for (int c16 = 0; c16 < kEpiCols / 16; ++c16) {
          uint32_t v[16];
          __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp must be converged
          tmem_ld_x16(taddr + c16 * 16, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            acc[c16 * 16 + j] = fmaf(static_cast<float>(static_cast<int>(v[j])), ws, acc[c16 * 16 + j]);
          }
          if (a.partials != nullptr && valid) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = wg * kEpiCols + c16 * 16 + j;
              if (col < tile.rows)
                a.partials[(static_cast<int64_t>(tile.m0 + col) * a.N + n) * G + g] = static_cast<int>(v[j]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[buf]);
        buf ^= 1;
        if (buf == 0) bphase ^= 1;
      }
      if (valid) {
#pragma unroll
        for (int c = 0; c < kEpiCols; ++c) {
          const int col = wg * kEpiCols + c;
          if (col < tile.rows) {
            const int m = tile.m0 + col;
            const float y = acc[c] * __ldg(a.x_scale + m);
            a.out[static_cast<int64_t>(m) * a.out_stride0 + static_cast<int64_t>(n) * a.out_stride1] =
                __float2bfloat16_rn(y);
          }
        }
      }
    }
  epi_done:;
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

}  // namespace

cudaError_t launch_gemm_tc(const GemmArgs& a, cudaStream_t stream) {
  if (a.M_total <= 0) return cudaSuccess;
  if (a.K < kBK || (a.K % 64) != 0 || (a.gs != 64 && a.gs != 128)) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.x_q) & 15) || (a.x_stride0 % 16) ||
      (reinterpret_cast<uintptr_t>(a.w_packed) & 15))
    return cudaErrorInvalidValue;
  CUtensorMap tm_x, tm_w;
  if (!encode_2d_u8(&tm_x, a.x_q, static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.M_total),
                    static_cast<uint64_t>(a.x_stride0), kBK, kXBoxRows, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!encode_2d_u8(&tm_w, a.w_packed, static_cast<uint64_t>(a.K / 2),
                    static_cast<uint64_t>(a.E) * static_cast<uint64_t>(a.N), static_cast<uint64_t>(a.K / 2),
                    kBK / 2, kBW, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;

  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = tc_smem_bytes(a.E);
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  gemm_tc_kernel<<<sms, kThreads, smem, stream>>>(tm_x, tm_w, a);
  return cudaGetLastError();
}

}  // namespace w4a8
