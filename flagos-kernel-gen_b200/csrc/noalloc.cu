// w4a8_moe_align_noalloc: the token -> expert align for callers that cannot
// allocate device memory.
//
// Some callers can't call cudaMalloc: an inference server that has handed all
// free device memory to its own pool (KV cache, activations) and exposes no
// way to borrow a scratch buffer from it, or a plain C caller that owns no
// allocator at all.  w4a8_moe_align needs a caller-provided workspace; this
// variant keeps its scratch in a fixed-size array in the library's own device
// memory instead, so the caller passes only inputs and outputs.
//
// The array lives for the lifetime of the process on every GPU that loads the
// library (kNoAllocScratchBytes each).  All calls share it and it keeps the
// previous call's contents; the align kernels overwrite every scratch word they
// read, so nothing needs clearing.  Two calls that overlap on the GPU (on
// different streams, or from different threads) race on the array: serialise
// them.  The first call on a device resolves the array's device address
// (cudaGetSymbolAddress, with that device current); make that first call
// before capturing a stream.
#include "../../include/w4a8moe.h"
#include "common.cuh"
#include "w4a8_internal.h"

#include <cstdio>
#include <mutex>

namespace w4a8 {
void set_last_error(const char* msg);   // capi.cu: message returned by w4a8_last_error()
size_t align_workspace_bytes(int R, int E);
cudaError_t launch_moe_align(const int32_t* ids, int R, int E, int bs, int32_t* expert_offsets,
                             int32_t* sorted_ids, int32_t* inv_pos, int32_t* padded_ids,
                             int32_t* block_expert, int32_t* num_post_pad, void* workspace,
                             cudaStream_t stream);
}  // namespace w4a8

namespace {

// Limits of the scratch array: T * topk <= 131072 routed slots, E <= 512
// experts.  align scratch = chunk histograms (64 chunks x 512 experts) +
// per-slot ranks (131072) + padded offsets (513), all int32 = 641 KB.
constexpr int64_t kNoAllocMaxSlots = 131072;
constexpr int64_t kNoAllocMaxExperts = 512;
constexpr size_t kNoAllocScratchBytes = 660 * 1024;

__device__ __align__(256) unsigned char g_align_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the scratch array on the stream's device (the symbol's
// host-side name is not a device address).  For the NULL stream the device is
// that of the driver context current on the calling thread (as for every
// entry point of the library).
cudaError_t scratch_for(void* stream, void** out) {
  cudaError_t e = w4a8::bind_stream_device(stream);
  if (e != cudaSuccess) return e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_align_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

int noalloc_fail(const char* msg) {
  w4a8::set_last_error(msg);
  return W4A8_ERR_INVALID;
}

}  // namespace

extern "C" {

int w4a8_moe_align_noalloc(const int32_t* topk_ids, int64_t T, int64_t topk, int64_t E, int64_t block_size,
                           int32_t* expert_offsets, int32_t* sorted_ids, int32_t* inv_pos,
                           int32_t* padded_ids, int32_t* block_expert, int32_t* num_post_pad, void* stream) {
  if (T < 0 || topk <= 0 || E <= 0 || block_size <= 0 || block_size > w4a8::kMaxAlignBlock)
    return noalloc_fail("w4a8_moe_align_noalloc: bad sizes (block_size must be in [1, 4096])");
  if (T * topk > kNoAllocMaxSlots || E > kNoAllocMaxExperts)
    return noalloc_fail("w4a8_moe_align_noalloc: T*topk must be <= 131072 and E <= 512 (fixed scratch size); "
                        "use w4a8_moe_align with a caller workspace for larger problems");
  if (expert_offsets == nullptr || (T > 0 && (topk_ids == nullptr || sorted_ids == nullptr || inv_pos == nullptr)))
    return noalloc_fail("w4a8_moe_align_noalloc: null pointer");
  const size_t need = w4a8::align_workspace_bytes(static_cast<int>(T * topk), static_cast<int>(E));
  if (need > kNoAllocScratchBytes) return noalloc_fail("w4a8_moe_align_noalloc: scratch too small");
  void* scratch = nullptr;
  cudaError_t e = scratch_for(stream, &scratch);
  if (e == cudaSuccess)
    e = w4a8::launch_moe_align(topk_ids, static_cast<int>(T * topk), static_cast<int>(E),
                               static_cast<int>(block_size), expert_offsets, sorted_ids, inv_pos, padded_ids,
                               block_expert, num_post_pad, scratch, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "w4a8_moe_align_noalloc: %s", cudaGetErrorString(e));
    w4a8::set_last_error(buf);
    return W4A8_ERR_CUDA;
  }
  return W4A8_OK;
}

}  // extern "C"
