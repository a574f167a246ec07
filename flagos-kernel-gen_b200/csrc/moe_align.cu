// Token -> expert sort / align (counting sort, deterministic, no host sync).
//
// Input: topk_ids int32 [T, topk] (flat index f = t*topk + j, R = T*topk).
// Outputs (all int32, device):
//   expert_offsets [E+1]  unpadded segment starts (the `expert_offsets`
//                         argument of the reference entry point, docs/Task1.md:15)
//   sorted_ids     [R]    flat index at each sorted position; inside an
//                         expert the order is ascending f (stable)
//   inv_pos        [R]    sorted position of flat index f
//   padded form (moe_align_block_size style, block size bs):
//   padded_ids     [R + E*(bs-1)]  flat index per padded slot, sentinel R for padding
//   block_expert   [ceil((R + E*(bs-1))/bs)]  expert of each bs-row block, -1 past the end
//   num_post_pad   [1]    total padded rows (sum_e roundup(count_e, bs))
// Expert ids outside [0, E) are not routed anywhere: they are counted in no
// segment, get inv_pos = -1 and appear in neither sorted list.
//
// Three launches: (1) per-chunk histograms and in-chunk stable ranks,
// (2) one CTA scans chunks and experts, (3) scatter.  Scratch: chunk
// histograms [num_chunks, E] int32 (caller-provided workspace).
#include "common.cuh"
#include "w4a8_internal.h"

namespace w4a8 {

namespace {

constexpr int kAlignThreads = 256;
constexpr int kAlignWarps = kAlignThreads / 32;
constexpr int kChunk = 2048;                 // flat entries per chunk (8 per thread)
constexpr int kPerWarp = kChunk / kAlignWarps;  // 256 consecutive entries per warp

// (1) chunk histogram + stable rank of each entry inside its chunk.
// s_hist[w][e] counts expert e among warp w's entries; the rank of an entry is
// (entries of the same expert in earlier warps) + (earlier entries in its warp).
__global__ void __launch_bounds__(kAlignThreads)
align_rank_kernel(const int32_t* __restrict__ ids, int R, int E, int32_t* __restrict__ rank_out,
                  int32_t* __restrict__ chunk_hist) {
  extern __shared__ int s_hist[];  // [kAlignWarps][E]
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kAlignWarps * E; i += kAlignThreads) s_hist[i] = 0;
  __syncthreads();
  const int base = blockIdx.x * kChunk + w * kPerWarp;
  int* h = s_hist + w * E;
  for (int r = 0; r < kPerWarp / 32; ++r) {
    const int f = base + r * 32 + l;
    int e = (f < R) ? ids[f] : -1;
    if (e >= E) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int before = __popc(peers & ((1u << l) - 1u));
    int cur = 0;
    if (e >= 0) cur = h[e];
    __syncwarp();
    if (e >= 0) {
      if (f < R) rank_out[f] = cur + before;
      if (before == 0) h[e] = cur + __popc(peers);  // one writer per expert
    } else if (f < R) {
      rank_out[f] = -1;
    }
    __syncwarp();
  }
  __syncthreads();
  // exclusive scan over warps per expert; chunk total to global
  for (int e = threadIdx.x; e < E; e += kAlignThreads) {
    int run = 0;
    for (int ww = 0; ww < kAlignWarps; ++ww) {
      const int c = s_hist[ww * E + e];
      s_hist[ww * E + e] = run;
      run += c;
    }
    chunk_hist[static_cast<int64_t>(blockIdx.x) * E + e] = run;
  }
  __syncthreads();
  for (int r = 0; r < kPerWarp / 32; ++r) {
    const int f = base + r * 32 + l;
    if (f < R) {
      const int e = ids[f];
      if (e >= 0 && e < E) rank_out[f] += s_hist[w * E + e];
    }
  }
}

// (2) one CTA: chunk prefix per expert (in place), expert offsets, padded
// offsets, block map, padding sentinels.
__global__ void __launch_bounds__(1024)
align_scan_kernel(int R, int E, int bs, int num_chunks, int32_t* __restrict__ chunk_hist,
                  int32_t* __restrict__ expert_offsets, int32_t* __restrict__ padded_offsets_ws,
                  int32_t* __restrict__ padded_ids, int32_t* __restrict__ block_expert,
                  int32_t* __restrict__ num_post_pad) {
  extern __shared__ int sm[];
  int* s_cnt = sm;            // [E]
  int* s_off = sm + E;        // [E+1]
  int* s_poff = s_off + E + 1;  // [E+1]
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int c = 0; c < num_chunks; ++c) {
      const int64_t i = static_cast<int64_t>(c) * E + e;
      const int v = chunk_hist[i];
      chunk_hist[i] = run;
      run += v;
    }
    s_cnt[e] = run;
  }
  __syncthreads();
  if (E <= static_cast<int>(blockDim.x)) {
    // block-wide exclusive scan of (count, padded count), one expert per thread
    __shared__ int s_wc[32], s_wp[32];
    const int e = threadIdx.x, lane = e & 31, wid = e >> 5;
    const int c = e < E ? s_cnt[e] : 0;
    const int pc = (c + bs - 1) / bs * bs;
    int ic = c, ip = pc;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int uc = __shfl_up_sync(0xffffffffu, ic, d), up = __shfl_up_sync(0xffffffffu, ip, d);
      if (lane >= d) { ic += uc; ip += up; }
    }
    if (lane == 31) { s_wc[wid] = ic; s_wp[wid] = ip; }
    __syncthreads();
    if (wid == 0) {
      const int nw = static_cast<int>(blockDim.x) >> 5;
      int vc = lane < nw ? s_wc[lane] : 0, vp = lane < nw ? s_wp[lane] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int uc = __shfl_up_sync(0xffffffffu, vc, d), up = __shfl_up_sync(0xffffffffu, vp, d);
        if (lane >= d) { vc += uc; vp += up; }
      }
      if (lane < nw) { s_wc[lane] = vc; s_wp[lane] = vp; }   // inclusive warp totals
    }
    __syncthreads();
    const int bc = wid > 0 ? s_wc[wid - 1] : 0, bp = wid > 0 ? s_wp[wid - 1] : 0;
    if (e < E) {
      s_off[e] = bc + ic - c;
      s_poff[e] = bp + ip - pc;
    }
    if (e == E - 1) {
      s_off[E] = bc + ic;
      s_poff[E] = bp + ip;
      if (num_post_pad != nullptr) *num_post_pad = bp + ip;
    }
  } else if (threadIdx.x == 0) {
    int o = 0, p = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = o;
      s_poff[e] = p;
      o += s_cnt[e];
      p += (s_cnt[e] + bs - 1) / bs * bs;
    }
    s_off[E] = o;
    s_poff[E] = p;
    if (num_post_pad != nullptr) *num_post_pad = p;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    expert_offsets[e] = s_off[e];
    padded_offsets_ws[e] = s_poff[e];
  }
  const int cap = R + E * (bs - 1);
  const int nblocks = (cap + bs - 1) / bs;
  for (int b = threadIdx.x; block_expert != nullptr && b < nblocks; b += blockDim.x) {
    const int row = b * bs;
    int ex = -1;
    if (row < s_poff[E]) {
      int lo = 0, hi = E - 1;  // largest e with poff[e] <= row
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_poff[mid] <= row) lo = mid; else hi = mid - 1;
      }
      ex = lo;
    }
    block_expert[b] = ex;
  }
  // sentinels: per-expert padding tails and everything past num_post_pad
  if (padded_ids != nullptr) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      for (int p = s_poff[e] + s_cnt[e]; p < s_poff[e + 1]; ++p) padded_ids[p] = R;
    }
    for (int p = s_poff[E] + threadIdx.x; p < cap; p += blockDim.x) padded_ids[p] = R;
  }
}

// (3) scatter
__global__ void __launch_bounds__(kAlignThreads)
align_scatter_kernel(const int32_t* __restrict__ ids, int R, int E, const int32_t* __restrict__ rank,
                     const int32_t* __restrict__ chunk_base, const int32_t* __restrict__ expert_offsets,
                     const int32_t* __restrict__ padded_offsets, int32_t* __restrict__ sorted_ids,
                     int32_t* __restrict__ inv_pos, int32_t* __restrict__ padded_ids) {
  const int f = blockIdx.x * kAlignThreads + threadIdx.x;
  if (f >= R) return;
  const int e = ids[f];
  if (e < 0 || e >= E) {
    inv_pos[f] = -1;
    return;
  }
  const int within = chunk_base[static_cast<int64_t>(f / kChunk) * E + e] + rank[f];
  const int p = expert_offsets[e] + within;
  sorted_ids[p] = f;
  inv_pos[f] = p;
  if (padded_ids != nullptr) padded_ids[padded_offsets[e] + within] = f;
}

}  // namespace

size_t align_workspace_bytes(int R, int E) {
  const int chunks = (R + kChunk - 1) / kChunk;
  // chunk histograms + in-chunk ranks + padded offsets
  return sizeof(int32_t) * (static_cast<size_t>(chunks > 0 ? chunks : 1) * E + R + (E + 1));
}

cudaError_t launch_moe_align(const int32_t* ids, int R, int E, int bs, int32_t* expert_offsets,
                             int32_t* sorted_ids, int32_t* inv_pos, int32_t* padded_ids,
                             int32_t* block_expert, int32_t* num_post_pad, void* workspace,
                             cudaStream_t stream) {
  const int chunks = R > 0 ? (R + kChunk - 1) / kChunk : 0;
  int32_t* hist = static_cast<int32_t*>(workspace);
  int32_t* rank = hist + static_cast<size_t>(chunks > 0 ? chunks : 1) * E;
  int32_t* poff = rank + R;
  if (chunks > 0) {
    const size_t sm1 = sizeof(int) * kAlignWarps * E;
    if (sm1 > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(align_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(sm1));
      if (e != cudaSuccess) return e;
    }
    align_rank_kernel<<<chunks, kAlignThreads, sm1, stream>>>(ids, R, E, rank, hist);
  }
  const size_t sm2 = sizeof(int) * (3 * E + 2);
  if (sm2 > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(align_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(sm2));
    if (e != cudaSuccess) return e;
  }
  align_scan_kernel<<<1, 1024, sm2, stream>>>(R, E, bs, chunks, hist, expert_offsets, poff, padded_ids,
                                              block_expert, num_post_pad);
  if (R > 0) {
    align_scatter_kernel<<<(R + kAlignThreads - 1) / kAlignThreads, kAlignThreads, 0, stream>>>(
        ids, R, E, rank, hist, expert_offsets, poff, sorted_ids, inv_pos, padded_ids);
  }
  return cudaGetLastError();
}

}  // namespace w4a8
