// Expert parallelism over peer memory (NVLink P2P): counts exchange,
// barrier and the return of result rows to their home ranks.  The fused
// quantise + dispatch kernel is the quantiser of act_quant.cu with the
// PeerRows destinations of ep_p2p.cuh.
//
// One forward on every rank (world ranks, E experts, epr = E / world each):
//   align by global expert (w4a8_moe_align) -> exchange (counts to every
//   peer, one signal, the receive-row bases) -> dispatch (each token
//   quantised once, its rows stored into the owners' receive buffers) ->
//   barrier -> local grouped GEMMs on the receive buffer -> return (result
//   rows stored into the home ranks' slot buffers) -> barrier -> combine.
// No host synchronisation, no NCCL on the data path.  Waits on peers are
// bounded: on expiry the kernel records kDevTimeoutPeer in the status word
// and returns (the host reads it with w4a8_device_status).
#include "../../include/w4a8moe.h"
#include "common.cuh"
#include "ep_p2p.cuh"
#include "w4a8_internal.h"

#include <cstdio>

namespace w4a8 {
void set_last_error(const char* msg);

namespace {

constexpr int kEpMaxWorld = 64;
constexpr long long kPeerWaitCycles = 4000000000LL;   // ~2 s: a peer that has not signalled by then is gone

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Signals `epoch` to every rank and waits (bounded) until every rank has
// signalled it here.  Called by the whole CTA; returns false on expiry.
__device__ bool signal_and_wait(uint8_t* const* peers, int64_t flags_off, int world, int rank, int epoch,
                                int* status, int* s_abort) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();   // this CTA's (and, through the kernel boundary, earlier kernels') stores first
    for (int d = 0; d < world; ++d) st_release_sys(reinterpret_cast<int32_t*>(peers[d] + flags_off) + rank, epoch);
    *s_abort = 0;
  }
  __syncthreads();
  if (threadIdx.x < world) {
    const int32_t* f = reinterpret_cast<const int32_t*>(peers[rank] + flags_off) + threadIdx.x;
    const long long t0 = clock64();
    while (ld_acquire_sys(f) < epoch) {
      if (clock64() - t0 > kPeerWaitCycles) {
        atomicCAS(status, 0, kDevTimeoutPeer);
        atomicExch(s_abort, 1);
        break;
      }
    }
  }
  __syncthreads();
  return *s_abort == 0;
}

__global__ void ep_barrier_kernel(uint8_t* const* peers, int64_t flags_off, int world, int rank, int epoch,
                                  int* status) {
  __shared__ int s_abort;
  signal_and_wait(peers, flags_off, world, rank, epoch, status, &s_abort);
}

// One CTA: publish this rank's routed rows per expert into every peer's
// counts matrix, wait for every peer's, then derive the receive-row bases.
//   dest_base[e]      first row of this rank's slots of expert e in e's owner's buffer
//                     (-1 when the owner would overflow its cap rows)
//   local_offsets[j]  segment starts of this rank's experts in its own buffer, j <= epr
__global__ void __launch_bounds__(1024)
ep_exchange_kernel(const int32_t* __restrict__ offsets, int E, int world, int rank, uint8_t* const* peers,
                   int64_t counts_off, int64_t flags_off, int epoch, int cap, int32_t* __restrict__ dest_base,
                   int32_t* __restrict__ local_offsets, int* status) {
  extern __shared__ int sm[];
  int* tot = sm;              // [E] rows of expert e over all senders
  int* before = sm + E;       // [E] rows of expert e from senders < rank
  int* seg = sm + 2 * E;      // [E] start of expert e's segment in its owner's buffer
  int* shard = sm + 3 * E;    // [world] rows each rank receives
  __shared__ int s_abort;
  const int epr = E / world;
  for (int i = threadIdx.x; i < world * E; i += blockDim.x) {
    const int d = i / E, e = i - d * E;
    reinterpret_cast<int32_t*>(peers[d] + counts_off)[rank * E + e] = offsets[e + 1] - offsets[e];
  }
  if (!signal_and_wait(peers, flags_off, world, rank, epoch, status, &s_abort)) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) dest_base[e] = -1;
    for (int j = threadIdx.x; j <= epr; j += blockDim.x) local_offsets[j] = 0;
    return;
  }
  const int32_t* M = reinterpret_cast<const int32_t*>(peers[rank] + counts_off);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t = 0, b = 0;
    for (int s = 0; s < world; ++s) {
      const int c = __ldcv(M + s * E + e);
      t += c;
      if (s < rank) b += c;
    }
    tot[e] = t;
    before[e] = b;
  }
  __syncthreads();
  if (threadIdx.x < world) {   // serial prefix inside each owner's shard (epr <= a few hundred)
    const int d = threadIdx.x;
    int run = 0;
    for (int j = 0; j < epr; ++j) {
      seg[d * epr + j] = run;
      run += tot[d * epr + j];
    }
    shard[d] = run;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int d = e / epr;
    dest_base[e] = shard[d] > cap ? -1 : seg[e] + before[e];
  }
  if (threadIdx.x < world && shard[threadIdx.x] > cap) atomicCAS(status, 0, kDevEpOverflow);
  for (int j = threadIdx.x; j <= epr; j += blockDim.x) {
    const int v = j < epr ? seg[rank * epr + j] : shard[rank];
    local_offsets[j] = shard[rank] > cap ? 0 : v;   // an overflowing rank computes nothing
  }
}

// Result rows back to their home ranks: row r of y (this rank's receive
// order) goes to row f of its sender's slot buffer, from src[r] = sender *
// tk_max + f.  Grid-stride over the rows this rank received.
__global__ void __launch_bounds__(256)
ep_return_kernel(const __nv_bfloat16* __restrict__ y, int64_t y_stride0, int H, const int32_t* __restrict__ src,
                 const int32_t* __restrict__ total_rows, int64_t tk_max, uint8_t* const* peers, int64_t yhome_off) {
  const int rows = *total_rows;
  const bool vec = (H % 8) == 0 && (y_stride0 % 8) == 0 && (reinterpret_cast<uintptr_t>(y) % 16) == 0;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t code = src[r];
    const int s = static_cast<int>(code / tk_max);
    const int64_t f = code - s * tk_max;
    const __nv_bfloat16* yr = y + static_cast<int64_t>(r) * y_stride0;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peers[s] + yhome_off) + f * H;
    if (vec) {
      for (int v = threadIdx.x; v < H / 8; v += blockDim.x)
        reinterpret_cast<uint4*>(dst)[v] = __ldg(reinterpret_cast<const uint4*>(yr) + v);
    } else {
      for (int c = threadIdx.x; c < H; c += blockDim.x) dst[c] = yr[c];
    }
  }
}

// Return addresses of the received rows: row r < *total_rows of this rank's
// receive order goes to row f of its sender's yhome (src[r] = sender * tk_max
// + f); rows past the count get 0.  A grouped GEMM given this table
// (w4a8_group_gemm_moe_rows) stores its results straight into the senders'
// buffers, so no separate return pass runs.
__global__ void ep_row_addr_kernel(const int32_t* __restrict__ src, const int32_t* __restrict__ total_rows, int cap,
                                   int64_t tk_max, int64_t row_bytes, uint8_t* const* peers, int64_t yhome_off,
                                   uint64_t* __restrict__ out_rows) {
  const int rows = *total_rows;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < cap; r += gridDim.x * blockDim.x) {
    uint64_t a = 0;
    if (r < rows) {
      const int64_t code = src[r];
      const int snd = static_cast<int>(code / tk_max);
      a = reinterpret_cast<uint64_t>(peers[snd] + yhome_off + (code - snd * tk_max) * row_bytes);
    }
    out_rows[r] = a;
  }
}

// Deduplicated dispatch, receiver side: row r < *total_rows whose dup entry
// names an earlier row of the same token takes that row's bytes (the sender
// crossed NVLink once per destination rank, not once per slot).
__global__ void ep_replicate_kernel(int8_t* __restrict__ xq, int H, const int32_t* __restrict__ dup,
                                    const int32_t* __restrict__ total_rows) {
  const int rows = *total_rows;
  const bool vec = (H % 16) == 0 && (reinterpret_cast<uintptr_t>(xq) % 16) == 0;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int p = dup[r];
    if (p < 0 || p >= rows) continue;   // a first row is always one of this forward's rows
    const int8_t* src = xq + static_cast<int64_t>(p) * H;
    int8_t* dst = xq + static_cast<int64_t>(r) * H;
    if (vec) {
      for (int v = threadIdx.x; v < H / 16; v += blockDim.x)
        reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(src)[v];
    } else {
      for (int c = threadIdx.x; c < H; c += blockDim.x) dst[c] = src[c];
    }
  }
}

int ep_fail(int code, const char* msg) {
  set_last_error(msg);
  return code;
}

}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" {

int w4a8_ep_exchange(const int32_t* expert_offsets, int64_t E, int64_t world, int64_t rank, void* const* peers,
                     int64_t counts_off, int64_t flags_off, int32_t epoch, int64_t cap_rows, int32_t* dest_base,
                     int32_t* local_offsets, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(be));
  if (world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world || E <= 0 || E > 1024 || E % world ||
      cap_rows < 0 || cap_rows > INT32_MAX || epoch <= 0)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_exchange: bad sizes (world <= 64, E <= 1024 divisible by world, epoch > 0)");
  if (expert_offsets == nullptr || peers == nullptr || dest_base == nullptr || local_offsets == nullptr)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_exchange: null pointer");
  int* st = device_status_ptr();
  if (st == nullptr) return ep_fail(W4A8_ERR_CUDA, "cannot resolve the device status word");
  const size_t smem = sizeof(int) * (3 * E + world);
  ep_exchange_kernel<<<1, 1024, smem, static_cast<cudaStream_t>(stream)>>>(
      expert_offsets, (int)E, (int)world, (int)rank, reinterpret_cast<uint8_t* const*>(peers), counts_off, flags_off,
      epoch, (int)cap_rows, dest_base, local_offsets, st);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? W4A8_OK : ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(e));
}

int w4a8_ep_dispatch(const void* x, int64_t x_stride0, int64_t T, int64_t H, const int32_t* topk_ids, int64_t topk,
                     int64_t E, int64_t world, int64_t rank, int64_t tk_max, const int32_t* expert_offsets,
                     const int32_t* inv_pos, const int32_t* dest_base, void* const* peers, int64_t xq_off,
                     int64_t xs_off, int64_t src_off, int32_t* home_pos, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(be));
  if (T < 0 || H <= 0 || H > 16384 || topk <= 0 || topk > 256 || world < 1 || world > kEpMaxWorld || rank < 0 ||
      rank >= world || E <= 0 || E % world || T * topk > tk_max || world * tk_max > INT32_MAX)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_dispatch: bad sizes (H <= 16384, T*topk <= tk_max, world*tk_max < 2^31)");
  if (T == 0) return W4A8_OK;
  if (x == nullptr || topk_ids == nullptr || expert_offsets == nullptr || inv_pos == nullptr || dest_base == nullptr ||
      peers == nullptr || home_pos == nullptr)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_dispatch: null pointer");
  PeerRows d{topk_ids, (int)topk, (int)E, (int)(E / world), (int)rank, tk_max, (int)H, expert_offsets, inv_pos,
             dest_base, reinterpret_cast<uint8_t* const*>(peers), xq_off, xs_off, src_off, home_pos};
  const cudaError_t e = launch_ep_dispatch(static_cast<const __nv_bfloat16*>(x), x_stride0, (int)T, (int)H, d,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(e));
}

int w4a8_ep_dispatch_dedup(const void* x, int64_t x_stride0, int64_t T, int64_t H, const int32_t* topk_ids,
                           int64_t topk, int64_t E, int64_t world, int64_t rank, int64_t tk_max,
                           const int32_t* expert_offsets, const int32_t* inv_pos, const int32_t* dest_base,
                           void* const* peers, int64_t xq_off, int64_t xs_off, int64_t src_off, int64_t dup_off,
                           int32_t* home_pos, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(be));
  if (T < 0 || H <= 0 || H > 16384 || topk <= 0 || topk > 256 || world < 1 || world > kEpMaxWorld || rank < 0 ||
      rank >= world || E <= 0 || E % world || T * topk > tk_max || world * tk_max > INT32_MAX || dup_off < 0)
    return ep_fail(W4A8_ERR_INVALID,
                   "w4a8_ep_dispatch_dedup: bad sizes (H <= 16384, T*topk <= tk_max, world*tk_max < 2^31, dup_off >= 0)");
  if (T == 0) return W4A8_OK;
  if (x == nullptr || topk_ids == nullptr || expert_offsets == nullptr || inv_pos == nullptr || dest_base == nullptr ||
      peers == nullptr || home_pos == nullptr)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_dispatch_dedup: null pointer");
  PeerRows d{topk_ids, (int)topk, (int)E, (int)(E / world), (int)rank, tk_max, (int)H, expert_offsets, inv_pos,
             dest_base, reinterpret_cast<uint8_t* const*>(peers), xq_off, xs_off, src_off, home_pos, dup_off};
  const cudaError_t e = launch_ep_dispatch(static_cast<const __nv_bfloat16*>(x), x_stride0, (int)T, (int)H, d,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(e));
}

int w4a8_ep_replicate(void* buf, int64_t xq_off, int64_t dup_off, int64_t H, const int32_t* total_rows,
                      int64_t rows_hint, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(be));
  if (H <= 0 || rows_hint < 0 || xq_off < 0 || dup_off < 0) return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_replicate: bad sizes");
  if (buf == nullptr || total_rows == nullptr) return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_replicate: null pointer");
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = rows_hint > 0 ? rows_hint : 1;
  const int grid = static_cast<int>(want < sms * 8 ? want : sms * 8);
  uint8_t* b = static_cast<uint8_t*>(buf);
  ep_replicate_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<int8_t*>(b + xq_off), (int)H, reinterpret_cast<const int32_t*>(b + dup_off), total_rows);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? W4A8_OK : ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(e));
}

int w4a8_ep_barrier(void* const* peers, int64_t flags_off, int64_t world, int64_t rank, int32_t epoch, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(be));
  if (world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world || epoch <= 0 || peers == nullptr)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_barrier: bad arguments");
  int* st = device_status_ptr();
  if (st == nullptr) return ep_fail(W4A8_ERR_CUDA, "cannot resolve the device status word");
  ep_barrier_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<uint8_t* const*>(peers),
                                                                      flags_off, (int)world, (int)rank, epoch, st);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? W4A8_OK : ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(e));
}

int w4a8_ep_return(const void* y, int64_t y_stride0, int64_t H, const int32_t* src, const int32_t* total_rows,
                   int64_t rows_hint, int64_t tk_max, void* const* peers, int64_t yhome_off, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(be));
  if (H <= 0 || y_stride0 < H || rows_hint < 0 || tk_max <= 0)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_return: bad sizes");
  if (y == nullptr || src == nullptr || total_rows == nullptr || peers == nullptr)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_return: null pointer");
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = rows_hint > 0 ? rows_hint : 1;
  const int grid = static_cast<int>(want < sms * 8 ? want : sms * 8);
  ep_return_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), y_stride0, (int)H, src, total_rows, tk_max,
      reinterpret_cast<uint8_t* const*>(peers), yhome_off);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? W4A8_OK : ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(e));
}

int w4a8_ep_row_addresses(const int32_t* src, const int32_t* total_rows, int64_t cap_rows, int64_t H,
                          int64_t tk_max, void* const* peers, int64_t yhome_off, uint64_t* out_rows, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(be));
  if (cap_rows < 0 || cap_rows > INT32_MAX || H <= 0 || tk_max <= 0)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_row_addresses: bad sizes");
  if (cap_rows == 0) return W4A8_OK;
  if (src == nullptr || total_rows == nullptr || peers == nullptr || out_rows == nullptr)
    return ep_fail(W4A8_ERR_INVALID, "w4a8_ep_row_addresses: null pointer");
  const int64_t blocks = (cap_rows + 255) / 256;
  ep_row_addr_kernel<<<static_cast<int>(blocks < 1184 ? blocks : 1184), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src, total_rows, static_cast<int>(cap_rows), tk_max, H * 2, reinterpret_cast<uint8_t* const*>(peers),
      yhome_off, out_rows);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? W4A8_OK : ep_fail(W4A8_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
