// Per-token symmetric int8 activation quantisation, and its fused variant that
// writes each quantised token row straight to its top-k slots in expert-sorted
// order (the dispatch step of the routed MoE layer).
//
// Convention (the repository's only int8 quantiser, docs/Task3.md:58-67):
//   scale = max(amax / 127, 1e-10)         (IEEE fp32 division)
//   q     = int8(trunc(clamp(x / scale, -127, 127)))   (.to(int8) truncates)
// Every step is an exactly rounded fp32 operation, so the result is bit-exact
// against any IEEE restatement of the same formula.
#include "common.cuh"
#include "w4a8_internal.h"
#include "ep_p2p.cuh"

namespace w4a8 {

namespace {

constexpr int kQThreads = 256;
constexpr int kQMaxVec = 8;  // 8 x 8 bf16 per thread -> H <= 16384 on the register path

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.f;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ int8_t quant1(float x, float s) {
  float q = __fdiv_rn(x, s);
  q = fminf(fmaxf(q, -127.f), 127.f);
  return static_cast<int8_t>(__float2int_rz(q));
}

}  // namespace

// Destinations of a quantised token row: row t of one local array, or (with
// rows_out) rows rows_out[t*topk + j] of it, j < topk.
struct LocalRows {
  int8_t* q;
  int64_t q_stride0;
  float* s;
  const int32_t* rows_out;
  int topk;
  __device__ __forceinline__ int count() const { return rows_out ? topk : 1; }
  // row pointer of destination d (nullptr: none); the thread with
  // threadIdx.x == d also stores the scale
  __device__ __forceinline__ int8_t* row(int t, int d, float scale, bool meta) const {
    const int64_t r = rows_out ? rows_out[static_cast<int64_t>(t) * topk + d] : t;
    if (r < 0) return nullptr;   // slot routed to no local expert
    if (meta) s[r] = scale;
    return q + r * q_stride0;
  }
};

namespace {

// One CTA per token row.  On the vector path each element is quantised once,
// into registers, and the packed row is then stored to every destination
// (Dest: LocalRows here, the peer receive buffers of ep_p2p.cu for the
// expert-parallel dispatch).
template <class Dest>
__device__ __forceinline__ void quant_row(const __nv_bfloat16* __restrict__ x, int64_t x_stride0, int H,
                                          const Dest& dest, int t, float* red) {
  const __nv_bfloat16* xr = x + static_cast<int64_t>(t) * x_stride0;
  const bool vec = ((H & 7) == 0) && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0) &&
                   (H / 8 <= kQThreads * kQMaxVec);
  float amax = 0.f;
  uint4 buf[kQMaxVec];
  const int nv = H / 8;
  if (vec) {
#pragma unroll
    for (int i = 0; i < kQMaxVec; ++i) {
      const int v = threadIdx.x + i * kQThreads;
      if (v < nv) {
        buf[i] = __ldg(reinterpret_cast<const uint4*>(xr) + v);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&buf[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h2[j]);
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    }
  } else {
    for (int k = threadIdx.x; k < H; k += kQThreads) amax = fmaxf(amax, fabsf(__bfloat162float(xr[k])));
  }
  amax = block_max(amax, red);
  const float s = fmaxf(__fdiv_rn(amax, 127.f), 1e-10f);
  const int ndst = dest.count();
  if (threadIdx.x < ndst) dest.row(t, threadIdx.x, s, true);   // scale and routing metadata
  // packed int8 row in registers (vector path): 8 values per uint2
  uint2 qv[kQMaxVec];
  if (vec) {
#pragma unroll
    for (int i = 0; i < kQMaxVec; ++i) {
      const int v = threadIdx.x + i * kQThreads;
      if (v < nv) {
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&buf[i]);
        uint32_t w[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float2 f0 = __bfloat1622float2(h2[2 * j]);
          const float2 f1 = __bfloat1622float2(h2[2 * j + 1]);
          const uint32_t b0 = static_cast<uint8_t>(quant1(f0.x, s));
          const uint32_t b1 = static_cast<uint8_t>(quant1(f0.y, s));
          const uint32_t b2 = static_cast<uint8_t>(quant1(f1.x, s));
          const uint32_t b3 = static_cast<uint8_t>(quant1(f1.y, s));
          w[j] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
        qv[i] = make_uint2(w[0], w[1]);
      }
    }
  }
  for (int d = 0; d < ndst; ++d) {
    int8_t* qr = dest.row(t, d, s, false);
    if (qr == nullptr) continue;
    if (vec && ((reinterpret_cast<uintptr_t>(qr) & 7) == 0)) {
#pragma unroll
      for (int i = 0; i < kQMaxVec; ++i) {
        const int v = threadIdx.x + i * kQThreads;
        if (v < nv) reinterpret_cast<uint2*>(qr)[v] = qv[i];
      }
    } else {
      for (int k = threadIdx.x; k < H; k += kQThreads) qr[k] = quant1(__bfloat162float(xr[k]), s);
    }
  }
}

template <class Dest>
__global__ void __launch_bounds__(kQThreads)
act_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride0, int H, const Dest dest) {
  __shared__ float red[32];
  quant_row(x, x_stride0, H, dest, blockIdx.x, red);
}

// Router of one token, run by one warp: scores (softmax or sigmoid of the E
// logits), the top-k experts by score in descending order, their weights
// renormalised to sum to 1.  Follows the routing of the benchmark inputs
// (softmax | sigmoid -> torch.topk -> w / w.sum()).  Experts are ranked by
// logit, which orders them exactly as their scores do (both maps are
// increasing), with ties going to the lower expert index, so the selection
// does not depend on how the scores round.  Lane l holds logits l, l + 32, ...
template <int kPerLane>
__device__ __forceinline__ void route_token(const RouterArgs& r, int t, int lane) {
  const float* lg = r.logits + static_cast<int64_t>(t) * r.logits_stride0;
  float v[kPerLane];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPerLane; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < r.E ? __ldg(lg + e) : -INFINITY;
    mx = fmaxf(mx, v[j]);
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, d));
  float denom = 1.f;   // softmax: sum of exp(logit - max) over all experts
  if (r.scoring == 0) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j)
      if (lane + 32 * j < r.E) s = __fadd_rn(s, expf(v[j] - mx));
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, d));
    denom = s;
  }
  uint32_t taken = 0;   // bit j: this lane's logit j already selected
  float my_w = 0.f, wsum = 0.f;
  int my_id = 0;
  for (int k = 0; k < r.topk; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int e = lane + 32 * j;
      if (e < r.E && !((taken >> j) & 1u) && (v[j] > best || bi == 0x7fffffff)) { best = v[j]; bi = e; }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, d);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, d);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    const float score = r.scoring == 0 ? __fdiv_rn(expf(best - mx), denom) : __fdiv_rn(1.f, 1.f + expf(-best));
    wsum = __fadd_rn(wsum, score);
    if (lane == k) { my_w = score; my_id = bi; }
  }
  if (lane < r.topk) {
    const int64_t o = static_cast<int64_t>(t) * r.topk + lane;
    r.ids[o] = my_id;
    r.weights[o] = r.renormalize ? __fdiv_rn(my_w, wsum) : my_w;
  }
}

// Router + quantisation of kRouterTokens tokens per CTA: each warp routes
// one of them (a CTA per token routed by one warp was bound by CTA launches
// and the serial top-k: 110 us for 16384 tokens), then the CTA quantises
// their hidden rows one after another (when x is given) into rows t of x_q.
constexpr int kRouterTokens = kQThreads / 32;
template <int kPerLane>
__global__ void __launch_bounds__(kQThreads)
router_quant_kernel(const RouterArgs r, int T, const __nv_bfloat16* __restrict__ x, int64_t x_stride0, int H,
                    const LocalRows dest) {
  __shared__ float red[32];
  const int t0 = blockIdx.x * kRouterTokens;
  const int mine = t0 + (threadIdx.x >> 5);
  if (mine < T) route_token<kPerLane>(r, mine, threadIdx.x & 31);
  if (x != nullptr)
    for (int t = t0; t < T && t < t0 + kRouterTokens; ++t) quant_row(x, x_stride0, H, dest, t, red);
}

}  // namespace

cudaError_t launch_router(const RouterArgs& r, int T, const __nv_bfloat16* x, int64_t x_stride0, int H, int8_t* q,
                          int64_t q_stride0, float* s, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  const LocalRows dest{q, q_stride0, s, nullptr, 1};
  const int grid = (T + kRouterTokens - 1) / kRouterTokens;
  if (r.E <= 256)
    router_quant_kernel<8><<<grid, kQThreads, 0, stream>>>(r, T, x, x_stride0, H, dest);
  else
    router_quant_kernel<32><<<grid, kQThreads, 0, stream>>>(r, T, x, x_stride0, H, dest);
  return cudaGetLastError();
}

cudaError_t launch_act_quant(const __nv_bfloat16* x, int64_t x_stride0, int T, int H, int8_t* q,
                             int64_t q_stride0, float* s, const int32_t* rows_out, int topk,
                             cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  act_quant_kernel<LocalRows><<<T, kQThreads, 0, stream>>>(x, x_stride0, H, LocalRows{q, q_stride0, s, rows_out, topk});
  return cudaGetLastError();
}

cudaError_t launch_ep_dispatch(const __nv_bfloat16* x, int64_t x_stride0, int T, int H, const PeerRows& dest,
                               cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  act_quant_kernel<PeerRows><<<T, kQThreads, 0, stream>>>(x, x_stride0, H, dest);
  return cudaGetLastError();
}

}  // namespace w4a8
