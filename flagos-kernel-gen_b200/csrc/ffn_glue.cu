// Routed-MoE glue kernels around the grouped GEMM.
//
// silu_mul_requant: h bf16 [R, 2I] (gate = h[:, :I], up = h[:, I:], the split
//   of docs/Task3.md:99-100) -> y = silu(gate) * up in fp32 (forward formula of
//   docs/Task3.md:107-110) -> per-row symmetric int8 with the quantiser of
//   docs/Task3.md:58-67 (scale = max(amax/127, 1e-10), truncating cast).
// moe_combine: out[t, :] = bf16( sum_{j ascending} topk_w[t, j] * y[inv_pos[t*k+j], :] )
//   with each product and each sum rounded to fp32 (no FMA contraction), so
//   the result is bit-exact against the same loop on the CPU.
#include <algorithm>

#include "common.cuh"
#include "w4a8_internal.h"

namespace w4a8 {

namespace {

constexpr int kGThreads = 256;

__device__ __forceinline__ float block_max256(float v, float* red) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < kGThreads / 32) ? red[l] : 0.f;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// 1 / (1 + e^-g) with a correctly rounded reciprocal: the same bits as the
// IEEE division 1.0f / (1.0f + expf(-g)), for fewer instructions.
__device__ __forceinline__ float silu_mul(float g, float u) {
  const float sig = __frcp_rn(1.0f + expf(-g));
  return __fmul_rn(__fmul_rn(g, sig), u);
}

constexpr int kSVec = 4;   // 16-byte vectors (8 columns) per thread on the register path: I <= 8192

__device__ __forceinline__ uint32_t quant4(float a, float b, float c, float d, float s) {
  auto q = [s](float v) {
    float r = __fdiv_rn(v, s);
    r = fminf(fmaxf(r, -127.f), 127.f);
    return static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(__float2int_rz(r))));
  };
  return q(a) | (q(b) << 8) | (q(c) << 16) | (q(d) << 24);
}

// Register path: each thread owns 8 consecutive columns per vector (16-byte
// loads of gate and up, 8-byte stores of the quantised row).
__global__ void __launch_bounds__(kGThreads)
silu_mul_requant_vec_kernel(const __nv_bfloat16* __restrict__ h, int64_t h_stride0, int I,
                            int8_t* __restrict__ q, int64_t q_stride0, float* __restrict__ s_out,
                            const int32_t* __restrict__ valid_rows) {
  __shared__ float red[32];
  // one row per CTA, or (valid_rows: a row count read on the device) a
  // grid-stride loop over the rows below it
  const int64_t lim = valid_rows != nullptr ? *valid_rows : gridDim.x;
  for (int64_t row = blockIdx.x; row < lim; row += gridDim.x) {
  const __nv_bfloat16* hr = h + row * h_stride0;
  const int nv = I / 8;
  float y[kSVec][8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kSVec; ++i) {
    const int v = threadIdx.x + i * kGThreads;
    if (v < nv) {
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(hr) + v);
      const uint4 uv = __ldg(reinterpret_cast<const uint4*>(hr + I) + v);
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
      const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 g = __bfloat1622float2(g2[j]);
        const float2 u = __bfloat1622float2(u2[j]);
        y[i][2 * j] = silu_mul(g.x, u.x);
        y[i][2 * j + 1] = silu_mul(g.y, u.y);
        amax = fmaxf(amax, fmaxf(fabsf(y[i][2 * j]), fabsf(y[i][2 * j + 1])));
      }
    }
  }
  amax = block_max256(amax, red);
  const float s = fmaxf(__fdiv_rn(amax, 127.f), 1e-10f);
  if (threadIdx.x == 0) s_out[row] = s;
  int8_t* qr = q + row * q_stride0;
#pragma unroll
  for (int i = 0; i < kSVec; ++i) {
    const int v = threadIdx.x + i * kGThreads;
    if (v < nv)
      reinterpret_cast<uint2*>(qr)[v] = make_uint2(quant4(y[i][0], y[i][1], y[i][2], y[i][3], s),
                                                   quant4(y[i][4], y[i][5], y[i][6], y[i][7], s));
  }
  }
}

// One warp per row for I <= 32 * 8 * kWVec (Qwen3's I = 768): each lane owns
// kV 16-byte vectors of gate and up, the row maximum is a warp reduction, and
// a CTA of 8 warps serves 8 rows.  The arithmetic is that of the
// CTA-per-row kernel, element by element (the same bits).  Measured on B200:
// 32768 rows x 768 in 66 us against 132 us for a CTA per row; at I = 2048
// the lane's 64 values need more registers than two CTAs per SM leave
// (665 us, spilling, against 605 us), so wider rows keep a CTA per row.
constexpr int kWVec = 4;
template <int kV>
__global__ void __launch_bounds__(kGThreads, 2)
silu_mul_requant_warp_kernel(const __nv_bfloat16* __restrict__ h, int64_t h_stride0, int I, int R,
                             int8_t* __restrict__ q, int64_t q_stride0, float* __restrict__ s_out,
                             const int32_t* __restrict__ valid_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t lim = valid_rows != nullptr ? *valid_rows : R;
  const int nv = I / 8;
  for (int64_t row = blockIdx.x * static_cast<int64_t>(kGThreads / 32) + (threadIdx.x >> 5); row < lim;
       row += static_cast<int64_t>(gridDim.x) * (kGThreads / 32)) {
    const __nv_bfloat16* hr = h + row * h_stride0;
    uint4 gv[kV], uv[kV];
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int v = lane + 32 * i;
      if (v < nv) {
        gv[i] = __ldg(reinterpret_cast<const uint4*>(hr) + v);
        uv[i] = __ldg(reinterpret_cast<const uint4*>(hr + I) + v);
      }
    }
    float y[kV][8];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      if (lane + 32 * i < nv) {
        const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv[i]);
        const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 g = __bfloat1622float2(g2[j]);
          const float2 u = __bfloat1622float2(u2[j]);
          y[i][2 * j] = silu_mul(g.x, u.x);
          y[i][2 * j + 1] = silu_mul(g.y, u.y);
          amax = fmaxf(amax, fmaxf(fabsf(y[i][2 * j]), fabsf(y[i][2 * j + 1])));
        }
      }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
    const float s = fmaxf(__fdiv_rn(amax, 127.f), 1e-10f);
    if (lane == 0) s_out[row] = s;
    int8_t* qr = q + row * q_stride0;
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int v = lane + 32 * i;
      if (v < nv)
        reinterpret_cast<uint2*>(qr)[v] = make_uint2(quant4(y[i][0], y[i][1], y[i][2], y[i][3], s),
                                                     quant4(y[i][4], y[i][5], y[i][6], y[i][7], s));
    }
  }
}

// One CTA per row.  The fp32 products are staged in shared memory (I <= 16384).
__global__ void __launch_bounds__(kGThreads)
silu_mul_requant_kernel(const __nv_bfloat16* __restrict__ h, int64_t h_stride0, int I,
                        int8_t* __restrict__ q, int64_t q_stride0, float* __restrict__ s_out,
                        const int32_t* __restrict__ valid_rows) {
  extern __shared__ float s_y[];
  __shared__ float red[32];
  const int64_t lim = valid_rows != nullptr ? *valid_rows : gridDim.x;
  for (int64_t row = blockIdx.x; row < lim; row += gridDim.x) {
  const __nv_bfloat16* hr = h + row * h_stride0;
  float amax = 0.f;
  const bool vec = ((I & 1) == 0) && ((reinterpret_cast<uintptr_t>(hr) & 3) == 0);
  if (vec) {
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(hr);
    const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(hr + I);
    for (int i = threadIdx.x; i < I / 2; i += kGThreads) {
      const float2 g = __bfloat1622float2(g2[i]);
      const float2 u = __bfloat1622float2(u2[i]);
      const float y0 = silu_mul(g.x, u.x), y1 = silu_mul(g.y, u.y);
      s_y[2 * i] = y0;
      s_y[2 * i + 1] = y1;
      amax = fmaxf(amax, fmaxf(fabsf(y0), fabsf(y1)));
    }
  } else {
    for (int i = threadIdx.x; i < I; i += kGThreads) {
      const float y = silu_mul(__bfloat162float(hr[i]), __bfloat162float(hr[I + i]));
      s_y[i] = y;
      amax = fmaxf(amax, fabsf(y));
    }
  }
  amax = block_max256(amax, red);
  const float s = fmaxf(__fdiv_rn(amax, 127.f), 1e-10f);
  if (threadIdx.x == 0) s_out[row] = s;
  int8_t* qr = q + row * q_stride0;
  for (int i = threadIdx.x; i < I; i += kGThreads) {
    float v = __fdiv_rn(s_y[i], s);
    v = fminf(fmaxf(v, -127.f), 127.f);
    qr[i] = static_cast<int8_t>(__float2int_rz(v));
  }
  __syncthreads();   // s_y is rewritten by the next row
  }
}

// Vector path with the token's kK slots unrolled: all kK 16-byte loads are in
// flight before the first add (a loop over a run-time top-k issued them one
// after another, each after the previous one's adds), and the adds still run
// j ascending with every product and sum rounded to fp32 (the same bits).
template <int kK>
__global__ void __launch_bounds__(kGThreads)
moe_combine_unrolled_kernel(const __nv_bfloat16* __restrict__ y, int64_t y_stride0, const int32_t* __restrict__ inv_pos,
                            const float* __restrict__ topk_w, int H, __nv_bfloat16* __restrict__ out,
                            int64_t out_stride0) {
  const int t = blockIdx.x;
  const int32_t* pos = inv_pos + static_cast<int64_t>(t) * kK;
  const float* wt = topk_w + static_cast<int64_t>(t) * kK;
  __nv_bfloat16* o = out + static_cast<int64_t>(t) * out_stride0;
  int p[kK];
  float w[kK];
#pragma unroll
  for (int j = 0; j < kK; ++j) {
    p[j] = __ldg(pos + j);
    w[j] = __ldg(wt + j);
  }
  for (int c = blockIdx.y * kGThreads + threadIdx.x; c < H / 8; c += kGThreads * gridDim.y) {
    uint4 v[kK];
#pragma unroll
    for (int j = 0; j < kK; ++j)
      if (p[j] >= 0) v[j] = __ldg(reinterpret_cast<const uint4*>(y + static_cast<int64_t>(p[j]) * y_stride0) + c);
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kK; ++j) {
      if (p[j] < 0) continue;
      const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&v[j]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(v2[i]);
        acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(w[j], f.x));
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(w[j], f.y));
      }
    }
    uint4 r;
    __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) r2[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
    reinterpret_cast<uint4*>(o)[c] = r;
  }
}

// One CTA per (token, column slice); each thread owns 8 consecutive columns
// (16-byte vectors).  The column slices (gridDim.y) give a decode-sized batch
// enough CTAs to fill the GPU.
__global__ void __launch_bounds__(kGThreads)
moe_combine_kernel(const __nv_bfloat16* __restrict__ y, int64_t y_stride0, const int32_t* __restrict__ inv_pos,
                   const float* __restrict__ topk_w, int topk, int H, __nv_bfloat16* __restrict__ out,
                   int64_t out_stride0) {
  const int t = blockIdx.x;
  const int32_t* pos = inv_pos + static_cast<int64_t>(t) * topk;
  const float* wt = topk_w + static_cast<int64_t>(t) * topk;
  __nv_bfloat16* o = out + static_cast<int64_t>(t) * out_stride0;
  const bool vec = ((H & 7) == 0) && ((y_stride0 & 7) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(o) & 15) == 0);
  if (vec) {
    for (int c = blockIdx.y * kGThreads + threadIdx.x; c < H / 8; c += kGThreads * gridDim.y) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int j = 0; j < topk; ++j) {
        const int p = pos[j];
        if (p < 0) continue;
        const float w = wt[j];
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(y + static_cast<int64_t>(p) * y_stride0) + c);
        const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(v2[i]);
          acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(w, f.x));
          acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(w, f.y));
        }
      }
      uint4 r;
      __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
      for (int i = 0; i < 4; ++i) r2[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      reinterpret_cast<uint4*>(o)[c] = r;
    }
  } else {
    for (int c = blockIdx.y * kGThreads + threadIdx.x; c < H; c += kGThreads * gridDim.y) {
      float acc = 0.f;
      for (int j = 0; j < topk; ++j) {
        const int p = pos[j];
        if (p < 0) continue;
        acc = __fadd_rn(acc, __fmul_rn(wt[j], __bfloat162float(y[static_cast<int64_t>(p) * y_stride0 + c])));
      }
      o[c] = __float2bfloat16_rn(acc);
    }
  }
}

// Last step of the fused combine: out[t, :] = bf16(acc[t, :]) and acc[t, :]
// = 0, so the accumulator is ready for the next batch without a memset.  One
// CTA per (token, column slice); 16-byte vectors when the rows allow.
__global__ void __launch_bounds__(kGThreads)
combine_finish_kernel(float* __restrict__ acc, int64_t acc_stride0, int H, __nv_bfloat16* __restrict__ out,
                      int64_t out_stride0) {
  float* a = acc + static_cast<int64_t>(blockIdx.x) * acc_stride0;
  __nv_bfloat16* o = out + static_cast<int64_t>(blockIdx.x) * out_stride0;
  const bool vec = ((H & 7) == 0) && ((reinterpret_cast<uintptr_t>(a) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(o) & 15) == 0);
  if (vec) {
    for (int c = blockIdx.y * kGThreads + threadIdx.x; c < H / 8; c += kGThreads * gridDim.y) {
      float4* p = reinterpret_cast<float4*>(a) + 2 * c;
      const float4 v0 = p[0], v1 = p[1];
      p[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      p[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      uint4 r;
      __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&r);
      r2[0] = __floats2bfloat162_rn(v0.x, v0.y);
      r2[1] = __floats2bfloat162_rn(v0.z, v0.w);
      r2[2] = __floats2bfloat162_rn(v1.x, v1.y);
      r2[3] = __floats2bfloat162_rn(v1.z, v1.w);
      reinterpret_cast<uint4*>(o)[c] = r;
    }
  } else {
    for (int c = blockIdx.y * kGThreads + threadIdx.x; c < H; c += kGThreads * gridDim.y) {
      o[c] = __float2bfloat16_rn(a[c]);
      a[c] = 0.f;
    }
  }
}

// dst row i = src row index[i] (row_bytes bytes each); index < 0 leaves dst row i untouched.
__global__ void __launch_bounds__(kGThreads)
gather_rows_kernel(const uint8_t* __restrict__ src, int64_t src_stride, const int32_t* __restrict__ index,
                   int64_t row_bytes, uint8_t* __restrict__ dst, int64_t dst_stride, bool vec16) {
  const int64_t i = blockIdx.x;
  const int j = index[i];
  if (j < 0) return;
  const uint8_t* s = src + static_cast<int64_t>(j) * src_stride;
  uint8_t* d = dst + i * dst_stride;
  if (vec16) {
    const int64_t n = row_bytes / 16;
    for (int64_t c = threadIdx.x; c < n; c += kGThreads)
      reinterpret_cast<uint4*>(d)[c] = __ldg(reinterpret_cast<const uint4*>(s) + c);
  } else {
    for (int64_t c = threadIdx.x; c < row_bytes; c += kGThreads) d[c] = s[c];
  }
}

}  // namespace

cudaError_t launch_gather_rows(const void* src, int64_t src_stride, const int32_t* index, int64_t rows,
                               int64_t row_bytes, void* dst, int64_t dst_stride, cudaStream_t stream) {
  if (rows <= 0 || row_bytes <= 0) return cudaSuccess;
  const bool vec16 = (row_bytes % 16 == 0) && (src_stride % 16 == 0) && (dst_stride % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (reinterpret_cast<uintptr_t>(dst) % 16 == 0);
  gather_rows_kernel<<<static_cast<unsigned>(rows), kGThreads, 0, stream>>>(
      static_cast<const uint8_t*>(src), src_stride, index, row_bytes, static_cast<uint8_t*>(dst), dst_stride, vec16);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul_requant(const __nv_bfloat16* h, int64_t h_stride0, int R, int I, int8_t* q,
                                    int64_t q_stride0, float* s, const int32_t* valid_rows,
                                    cudaStream_t stream) {
  if (R <= 0) return cudaSuccess;
  const bool wvec = (I % 8) == 0 && I / 8 <= 32 * kWVec && (h_stride0 % 8) == 0 &&
                    (reinterpret_cast<uintptr_t>(h) % 16) == 0 && (q_stride0 % 8) == 0 &&
                    (reinterpret_cast<uintptr_t>(q) % 8) == 0;
  if (wvec) {   // one warp per row, 8 rows per CTA; with valid_rows a resident grid strides over them
    int grid = (R + kGThreads / 32 - 1) / (kGThreads / 32);
    if (valid_rows != nullptr) {
      int dev = 0, sms = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      grid = grid < sms * 8 ? grid : sms * 8;
    }
    const int kv = (I / 8 + 31) / 32;
    if (kv <= 2)
      silu_mul_requant_warp_kernel<2><<<grid, kGThreads, 0, stream>>>(h, h_stride0, I, R, q, q_stride0, s, valid_rows);
    else
      silu_mul_requant_warp_kernel<4><<<grid, kGThreads, 0, stream>>>(h, h_stride0, I, R, q, q_stride0, s, valid_rows);
    return cudaGetLastError();
  }
  if (valid_rows != nullptr) {   // rows counted on the device: a resident grid strides over them
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    R = R < sms * 8 ? R : sms * 8;
  }
  const bool vec = (I % 8) == 0 && I / 8 <= kGThreads * kSVec && (h_stride0 % 8) == 0 &&
                   (reinterpret_cast<uintptr_t>(h) % 16) == 0 && (q_stride0 % 8) == 0 &&
                   (reinterpret_cast<uintptr_t>(q) % 8) == 0;
  if (vec) {
    silu_mul_requant_vec_kernel<<<R, kGThreads, 0, stream>>>(h, h_stride0, I, q, q_stride0, s, valid_rows);
    return cudaGetLastError();
  }
  const size_t smem = sizeof(float) * static_cast<size_t>(I);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(silu_mul_requant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  silu_mul_requant_kernel<<<R, kGThreads, smem, stream>>>(h, h_stride0, I, q, q_stride0, s, valid_rows);
  return cudaGetLastError();
}

cudaError_t launch_moe_combine(const __nv_bfloat16* y, int64_t y_stride0, const int32_t* inv_pos,
                               const float* topk_w, int T, int topk, int H, __nv_bfloat16* out,
                               int64_t out_stride0, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  const int slices = std::max(1, std::min(8, (H / 8 + kGThreads - 1) / kGThreads));   // column slices per token
  const bool vec = (H & 7) == 0 && (y_stride0 & 7) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15) == 0 && (out_stride0 & 7) == 0;
  const dim3 grid(T, slices);
  if (vec && topk == 8) {
    moe_combine_unrolled_kernel<8><<<grid, kGThreads, 0, stream>>>(y, y_stride0, inv_pos, topk_w, H, out, out_stride0);
  } else if (vec && topk == 2) {
    moe_combine_unrolled_kernel<2><<<grid, kGThreads, 0, stream>>>(y, y_stride0, inv_pos, topk_w, H, out, out_stride0);
  } else if (vec && topk == 4) {
    moe_combine_unrolled_kernel<4><<<grid, kGThreads, 0, stream>>>(y, y_stride0, inv_pos, topk_w, H, out, out_stride0);
  } else {
    moe_combine_kernel<<<grid, kGThreads, 0, stream>>>(y, y_stride0, inv_pos, topk_w, topk, H, out, out_stride0);
  }
  return cudaGetLastError();
}

cudaError_t launch_combine_finish(float* acc, int64_t acc_stride0, int T, int H, __nv_bfloat16* out,
                                  int64_t out_stride0, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  const int slices = std::max(1, std::min(8, (H / 8 + kGThreads - 1) / kGThreads));
  combine_finish_kernel<<<dim3(T, slices), kGThreads, 0, stream>>>(acc, acc_stride0, H, out, out_stride0);
  return cudaGetLastError();
}

}  // namespace w4a8
