// Offline weight prepack: the word-interleaved nibble layout.
//
// Reference layout (docs/Task1.md:78-81): byte j of a packed row holds
// k = 2j in its low nibble and k = 2j + 1 in its high nibble, so the eight
// nibbles of a 32-bit word q come out of the two nibble masks as
// (k0, k2, k4, k6) and (k1, k3, k5, k7) and every unpack to int8 needs two
// byte permutes to restore k order.  Prepacked layout: byte b (0..3) of word
// q holds k = 8q + b low and k = 8q + 4 + b high, so the masks give
// (k0..k3) and (k4..k7) directly.  Same size, same rows, same scales and zero
// points; the grouped GEMMs read it with w4a8_group_gemm_moe_prepacked.
#include "../../include/w4a8moe.h"
#include "common.cuh"
#include "w4a8_internal.h"

namespace w4a8 {
void set_last_error(const char* msg);

namespace {

__device__ __forceinline__ uint32_t prepack_word(uint32_t w) {
  const uint32_t ev = w & 0x0F0F0F0Fu;          // k0, k2, k4, k6
  const uint32_t od = (w >> 4) & 0x0F0F0F0Fu;   // k1, k3, k5, k7
  const uint32_t lo = __byte_perm(ev, od, 0x5140);   // k0, k1, k2, k3
  const uint32_t hi = __byte_perm(ev, od, 0x7362);   // k4, k5, k6, k7
  return lo | (hi << 4);
}

// (each 16-byte piece is read and written by the same thread, so in place is fine)
__global__ void prepack_kernel(const uint4* in, uint4* out, int64_t n16) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint4 v = in[i];
    v.x = prepack_word(v.x);
    v.y = prepack_word(v.y);
    v.z = prepack_word(v.z);
    v.w = prepack_word(v.w);
    out[i] = v;
  }
}

}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" int w4a8_prepack_weights(const uint8_t* w_q4_packed, uint8_t* out, int64_t rows, int64_t K,
                                    void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) {
    set_last_error(cudaGetErrorString(be));
    return W4A8_ERR_CUDA;
  }
  if (rows < 0 || K <= 0 || (K % 64) != 0) {
    set_last_error("w4a8_prepack_weights: rows >= 0 and K a multiple of 64 required");
    return W4A8_ERR_INVALID;
  }
  if (rows == 0) return W4A8_OK;
  if (w_q4_packed == nullptr || out == nullptr ||
      (reinterpret_cast<uintptr_t>(w_q4_packed) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) {
    set_last_error("w4a8_prepack_weights: 16-byte aligned input and output required");
    return W4A8_ERR_INVALID;
  }
  const int64_t n16 = rows * (K / 2) / 16;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n16 + 255) / 256;
  const int grid = static_cast<int>(want < sms * 16 ? want : sms * 16);
  prepack_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(w_q4_packed), reinterpret_cast<uint4*>(out), n16);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return W4A8_ERR_CUDA;
  }
  return W4A8_OK;
}
