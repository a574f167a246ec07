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
  int32_t* partials;          // optional [G, M_total, N] int32 (debug / parity export)
  int* status;                // device status word
  int64_t x_stride0, out_stride0, out_stride1;
  int M_total, E, N, K, gs;
  // expert row-count window this launch handles (the others are left to the
  // other kernel of a split launch); default: every expert
  int min_rows = 1;
  int max_rows = 0x7fffffff;
  // expected rows when M_total is only a capacity (the rows are counted on the
  // device from the offsets): picks kernels and tile widths; 0 = M_total
  int rows_hint = 0;
  // Fused top-k combine (comb_out != nullptr): instead of storing row m's
  // bf16 result y to `out`, add topk_w[f] * y (fp32, y rounded to bf16 first,
  // as the unfused combine reads it) into comb_out[f / comb_topk, n], where
  // f = comb_ids[m] is the row's flat (token, slot) index.
  float* comb_out = nullptr;
  const int32_t* comb_ids = nullptr;
  const float* comb_w = nullptr;
  int comb_topk = 1;
  int64_t comb_stride = 0;
  // Row-address store (out_rows != nullptr): row m's bf16 results go to the
  // N contiguous elements at address out_rows[m] (0: row not stored) — e.g.
  // straight into another GPU's buffer over NVLink peer memory.
  const uint64_t* out_rows = nullptr;
  // Weight nibble layout: 0 = the reference's (byte j of a row holds k = 2j
  // low, 2j + 1 high); 1 = the word-interleaved prepack of w4a8_prepack_weights
  // (byte b of 32-bit word q holds k = 8q + b low, 8q + 4 + b high).
  int layout = 0;
};

#ifdef __CUDACC__
// Output of row m, column n of a grouped GEMM: v is the fp32 group-scale sum,
// the row's token scale is applied and the result rounded to bf16 (the
// reference's store, docs/Task1.md:110-112); with the fused combine the
// weighted bf16 value is added to the token's fp32 output row instead, and
// with a row-address table it goes to that row's address.
__device__ __forceinline__ void store_row_addr(const GemmArgs& a, int m, int n, float v) {
  const uint64_t row = __ldg(a.out_rows + m);
  if (row != 0) reinterpret_cast<__nv_bfloat16*>(row)[n] = __float2bfloat16_rn(v * __ldg(a.x_scale + m));
}
__device__ __forceinline__ void store_output(const GemmArgs& a, int m, int n, float v) {
  if (a.out_rows != nullptr) {
    store_row_addr(a, m, n, v);
    return;
  }
  const __nv_bfloat16 y = __float2bfloat16_rn(v * __ldg(a.x_scale + m));
  if (a.comb_out == nullptr) {
    a.out[static_cast<int64_t>(m) * a.out_stride0 + static_cast<int64_t>(n) * a.out_stride1] = y;
  } else {
    const int f = __ldg(a.comb_ids + m);
    const float w = __ldg(a.comb_w + f);
    atomicAdd(a.comb_out + static_cast<int64_t>(f / a.comb_topk) * a.comb_stride + n, __fmul_rn(w, __bfloat162float(y)));
  }
}
#endif

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

// Router of a token batch (scores, top-k, renormalisation) on the device.
struct RouterArgs {
  const float* logits;      // [T, E], row stride logits_stride0
  int64_t logits_stride0;
  int E, topk;
  int scoring;              // 0 softmax, 1 sigmoid
  int renormalize;          // weights divided by their sum over the k selected
  int32_t* ids;             // [T, topk]
  float* weights;           // [T, topk]
};
constexpr int kRouterMaxExperts = 1024;
constexpr int kRouterMaxTopk = 32;
// Routes T tokens and, with x given, quantises each token's hidden row into
// row t of q (the act-quant convention) in the same launch.
cudaError_t launch_router(const RouterArgs& r, int T, const __nv_bfloat16* x, int64_t x_stride0, int H, int8_t* q,
                          int64_t q_stride0, float* s, cudaStream_t stream);

// Largest padded-block size the align entry points accept: the padded
// outputs hold T*topk + E*(block_size-1) entries, which must stay well inside
// the kernels' 32-bit index range.
constexpr int kMaxAlignBlock = 4096;

}  // namespace w4a8
