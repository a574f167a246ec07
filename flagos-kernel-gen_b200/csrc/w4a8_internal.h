// Internal launch interfaces shared by the .cu files of the library.  The
// public C ABI lives in include/w4a8moe.h; nothing here is exported.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace w4a8 {

// One grouped GEMM call: the arguments of the reference entry point
// (docs/Task1.md:8-17) flattened to pointers, sizes and strides.
struct GemmArgs {
  const int8_t* x_q;          // [M_total, K], row stride x_stride0 (elements == bytes)
  const float* x_scale;       // [M_total]
  const uint8_t* w_packed;    // [E, N, K/2] contiguous
  const float* w_scale;       // [E, N, G] contiguous
  const int8_t* w_zero;       // [E, N, G] contiguous
  const int32_t* offsets;     // [E+1]
  __nv_bfloat16* out;         // [M_total, N] with strides (out_stride0, out_stride1) in elements
  int32_t* partials;          // optional [M_total, N, G] int32 (debug / parity export)
  int* status;                // device status word
  int64_t x_stride0, out_stride0, out_stride1;
  int M_total, E, N, K, gs;
  // expert row-count window this launch handles (the others are left to the
  // other kernel of a split launch); default: every expert
  int min_rows = 1;
  int max_rows = 0x7fffffff;
};

cudaError_t launch_gemm_simt(const GemmArgs& a, cudaStream_t stream);
cudaError_t launch_gemm_gemv(const GemmArgs& a, cudaStream_t stream);
constexpr int kGemvMaxTokens = 4;  // tokens per pass of the streaming kernel
constexpr int kGemvAutoRows = 4;   // AUTO dispatch: experts with at most this many rows stream
cudaError_t launch_gemm_tc(const GemmArgs& a, cudaStream_t stream);
bool gemm_tc_supports(int K, int gs, int E);

int* device_status_ptr();  // per-device status word (static __device__ storage)

// Makes the device of `stream` (for NULL: of the driver context current on
// the calling thread) current in the library's own runtime.
cudaError_t bind_stream_device(void* stream);

// Largest padded-block size the align entry points accept: the padded
// outputs hold T*topk + E*(block_size-1) entries, which must stay well inside
// the kernels' 32-bit index range.
constexpr int kMaxAlignBlock = 4096;

}  // namespace w4a8
