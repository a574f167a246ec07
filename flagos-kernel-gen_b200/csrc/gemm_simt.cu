// Grouped W4A8 GEMM on CUDA cores (dp4a).  This is the simple, obviously
// correct GPU path: every output is an int32 dot product per K-group followed
// by the fp32 group-scale / token-scale epilogue, exactly the reference
// semantics of docs/Task1.md:78-112:
//
//   w[e,n,k]      = int8( nibble(e,n,k) - w_zero[e,n,k/gs] )        (:78-85)
//   partial[m,n,g]= sum_{k in g} x_q[m,k] * w[e,n,k]   (int32)       (:100-104)
//   out[m,n]      = bf16( x_scale[m] * sum_g partial[m,n,g]*w_scale[e,n,g] ) (:107-112)
//
// It is used as the GPU cross-check of the tensor-core kernel and as the path
// that can export the int32 per-group partials at any shape.  It shares the
// device-side tile scheduler (no host synchronisation).
#include "common.cuh"
#include "w4a8_internal.h"

namespace w4a8 {

namespace {

constexpr int kSimtBM = 32;   // rows per tile
constexpr int kSimtBN = 64;   // output channels per tile
constexpr int kSimtThreads = 256;
constexpr int kMaxGs = 128;

__global__ void __launch_bounds__(kSimtThreads)
gemm_simt_kernel(GemmArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int* s_prefix = reinterpret_cast<int*>(smem_raw);
  int* s_seg = s_prefix + (a.E + 1);
  int* s_cnt = s_seg + (a.E + 1);
  // x tile [BM][gs] and w tile [BN][gs+4] (row padding keeps the per-lane
  // 4-byte reads of different rows in different banks)
  int8_t* s_x = reinterpret_cast<int8_t*>(s_cnt + a.E + 4);
  s_x = reinterpret_cast<int8_t*>((reinterpret_cast<uintptr_t>(s_x) + 15) & ~uintptr_t(15));
  const int wstride = a.gs + 4;
  int8_t* s_w = s_x + kSimtBM * a.gs;

  TileSched s{s_prefix, s_seg, s_cnt, a.E, kSimtBM, (a.N + kSimtBN - 1) / kSimtBN, a.min_rows, a.max_rows};
  const int total = sched_build(s, a.offsets, a.M_total);
  const int G = a.K / a.gs;
  const int tid = threadIdx.x;
  const int tn = tid % kSimtBN;     // output channel within the tile
  const int tm = tid / kSimtBN;     // 0..3, rows tm, tm+4, ...

  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    const Tile tile = sched_tile(s, t);
    const int n0 = tile.nb * kSimtBN;
    const int n = n0 + tn;
    float acc[kSimtBM / 4];
#pragma unroll
    for (int i = 0; i < kSimtBM / 4; ++i) acc[i] = 0.f;

    for (int g = 0; g < G; ++g) {
      const int k0 = g * a.gs;
      __syncthreads();
      // activations: rows of this token block, columns of group g
      for (int idx = tid; idx < kSimtBM * (a.gs / 4); idx += kSimtThreads) {
        const int r = idx / (a.gs / 4), c4 = idx % (a.gs / 4);
        int v = 0;
        if (r < tile.rows) {
          const int8_t* src = a.x_q + static_cast<int64_t>(tile.m0 + r) * a.x_stride0 + k0 + 4 * c4;
          v = *reinterpret_cast<const int*>(src);  // x rows are 4-byte aligned (checked on host)
        }
        reinterpret_cast<int*>(s_x + r * a.gs)[c4] = v;
      }
      // weights: unpack nibbles of group g, fold the zero point with int8 wrap
      for (int idx = tid; idx < kSimtBN * (a.gs / 2); idx += kSimtThreads) {
        const int r = idx / (a.gs / 2), b = idx % (a.gs / 2);
        const int nn = n0 + r;
        int8_t lo = 0, hi = 0;
        if (nn < a.N) {
          const int64_t row = static_cast<int64_t>(tile.e) * a.N + nn;
          const uint8_t p = a.w_packed[row * (a.K / 2) + k0 / 2 + b];
          const int z = a.w_zero[row * G + g];
          lo = static_cast<int8_t>(static_cast<int16_t>(p & 0x0F) - z);
          hi = static_cast<int8_t>(static_cast<int16_t>(p >> 4) - z);
        }
        // byte b holds k = 2b, 2b+1 (reference) or 8(b/4) + b%4, + 4 (prepacked)
        const int pl = a.layout == 0 ? 2 * b : 8 * (b >> 2) + (b & 3);
        s_w[r * wstride + pl] = lo;
        s_w[r * wstride + pl + (a.layout == 0 ? 1 : 4)] = hi;
      }
      __syncthreads();
      if (n < a.N) {
        const float ws = a.w_scale[(static_cast<int64_t>(tile.e) * a.N + n) * G + g];
        const int* wrow = reinterpret_cast<const int*>(s_w + tn * wstride);
#pragma unroll
        for (int i = 0; i < kSimtBM / 4; ++i) {
          const int r = tm + 4 * i;
          const int* xrow = reinterpret_cast<const int*>(s_x + r * a.gs);
          int p = 0;
          for (int c = 0; c < a.gs / 4; ++c) p = __dp4a(xrow[c], wrow[c], p);
          acc[i] = fmaf(static_cast<float>(p), ws, acc[i]);
          if (a.partials != nullptr && r < tile.rows) {
            a.partials[(static_cast<int64_t>(g) * a.M_total + tile.m0 + r) * a.N + n] = p;
          }
        }
      }
    }
    if (n < a.N) {
#pragma unroll
      for (int i = 0; i < kSimtBM / 4; ++i) {
        const int r = tm + 4 * i;
        if (r < tile.rows) store_output(a, tile.m0 + r, n, acc[i]);
      }
    }
  }
}

}  // namespace

cudaError_t launch_gemm_simt(const GemmArgs& a, cudaStream_t stream) {
  if (a.gs > kMaxGs) return cudaErrorInvalidValue;
  const size_t smem = sizeof(int) * (3 * (a.E + 1) + 8) + 16 + kSimtBM * a.gs + kSimtBN * (a.gs + 4);
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(gemm_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  gemm_simt_kernel<<<sms * 4, kSimtThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace w4a8
