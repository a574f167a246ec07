// extern "C" entry points (include/w4a8moe.h): argument validation, device
// status handling and kernel dispatch.  Validation mirrors the reference's
// asserts (docs/Task1.md:74-75: K_half*2 == K, K % group_size == 0) and its
// group-size rule (Task1/各平台最高/task1-海光-26.44.py:226: 64 or 128).
#include "../../include/w4a8moe.h"
#include "common.cuh"
#include "w4a8_internal.h"

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

namespace w4a8 {
cudaError_t launch_act_quant(const __nv_bfloat16* x, int64_t x_stride0, int T, int H, int8_t* q,
                             int64_t q_stride0, float* s, const int32_t* rows_out, int topk,
                             cudaStream_t stream);
size_t align_workspace_bytes(int R, int E);
cudaError_t launch_moe_align(const int32_t* ids, int R, int E, int bs, int32_t* expert_offsets,
                             int32_t* sorted_ids, int32_t* inv_pos, int32_t* padded_ids,
                             int32_t* block_expert, int32_t* num_post_pad, void* workspace,
                             cudaStream_t stream);
cudaError_t launch_silu_mul_requant(const __nv_bfloat16* h, int64_t h_stride0, int R, int I, int8_t* q,
                                    int64_t q_stride0, float* s, const int32_t* valid_rows,
                                    cudaStream_t stream);
cudaError_t launch_gather_rows(const void* src, int64_t src_stride, const int32_t* index, int64_t rows,
                               int64_t row_bytes, void* dst, int64_t dst_stride, cudaStream_t stream);
cudaError_t launch_moe_combine(const __nv_bfloat16* y, int64_t y_stride0, const int32_t* inv_pos,
                               const float* topk_w, int T, int topk, int H, __nv_bfloat16* out,
                               int64_t out_stride0, cudaStream_t stream);
cudaError_t launch_combine_finish(float* acc, int64_t acc_stride0, int T, int H, __nv_bfloat16* out,
                                  int64_t out_stride0, cudaStream_t stream);

namespace {
__device__ int g_status_word;

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(W4A8_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {};
std::mutex g_status_mu;

// cuCtxGetDevice of the driver, resolved through the runtime (the library
// does not link libcuda).
using CtxGetDeviceFn = CUresult (*)(CUdevice*);
CtxGetDeviceFn ctx_get_device_fn() {
  static CtxGetDeviceFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetDevice", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetDeviceFn>(p);
  });
  return fn;
}
}  // namespace

// Makes the caller's device current in this library's runtime.  The library
// links its own (static) CUDA runtime, whose "current device" is separate
// from the caller's runtime (torch's, for example).  A stream names its
// device; for the NULL stream the device is that of the driver context
// current on the calling thread, which is the context the caller's runtime
// made current with cudaSetDevice / torch.cuda.set_device and its first CUDA
// call.  With no current context the library's own current device is kept.
cudaError_t bind_stream_device(void* stream) {
  int want = -1, cur = 0;
  if (stream != nullptr) {
    cudaError_t e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &want);
    if (e != cudaSuccess) return e;
  } else if (CtxGetDeviceFn fn = ctx_get_device_fn(); fn != nullptr) {
    CUdevice d = 0;
    if (fn(&d) == CUDA_SUCCESS) want = static_cast<int>(d);
  }
  if (want < 0) return cudaSuccess;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return e;
  return want == cur ? cudaSuccess : cudaSetDevice(want);
}

void set_last_error(const char* msg) { g_last_error = msg; }

int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

}  // namespace w4a8

using namespace w4a8;

namespace {
// Validation shared by the grouped-GEMM entry points and the argument block;
// returns W4A8_OK with *a filled in, or an error code.
int gemm_setup(GemmArgs* a, const int8_t* x_q, int64_t x_stride0, const float* x_scale, const uint8_t* w_q4_packed,
               const float* w_scale, const int8_t* w_zero, const int32_t* expert_offsets, int64_t M_total,
               int64_t E, int64_t N, int64_t K, int64_t group_size, int32_t kernel, bool need_out, void* out) {
  if (group_size != 64 && group_size != 128)
    return fail(W4A8_ERR_INVALID, "group_size must be 64 or 128 (got %lld)", (long long)group_size);
  if (K <= 0 || K % group_size != 0)
    return fail(W4A8_ERR_INVALID, "K %% group_size != 0 (K=%lld, group_size=%lld)", (long long)K,
                (long long)group_size);
  if (M_total < 0 || E <= 0 || N <= 0)
    return fail(W4A8_ERR_INVALID, "bad sizes M_total=%lld E=%lld N=%lld", (long long)M_total, (long long)E,
                (long long)N);
  if (M_total > INT32_MAX || E * N > INT32_MAX || K > INT32_MAX || E > 4096)
    return fail(W4A8_ERR_INVALID, "sizes exceed the 32-bit index range of the kernels");
  if (M_total > 0 && (x_q == nullptr || x_scale == nullptr || (need_out && out == nullptr)))
    return fail(W4A8_ERR_INVALID, "null activation / output pointer");
  if (w_q4_packed == nullptr || w_scale == nullptr || w_zero == nullptr || expert_offsets == nullptr)
    return fail(W4A8_ERR_INVALID, "null weight / offset pointer");
  if (x_stride0 < K) return fail(W4A8_ERR_INVALID, "x_q row stride %lld < K", (long long)x_stride0);
  if (kernel != W4A8_KERNEL_AUTO && kernel != W4A8_KERNEL_TC && kernel != W4A8_KERNEL_SIMT &&
      kernel != W4A8_KERNEL_GEMV)
    return fail(W4A8_ERR_INVALID, "unknown kernel selector %d", kernel);
  a->x_q = x_q;
  a->x_scale = x_scale;
  a->w_packed = w_q4_packed;
  a->w_scale = w_scale;
  a->w_zero = w_zero;
  a->offsets = expert_offsets;
  a->out = static_cast<__nv_bfloat16*>(out);
  a->x_stride0 = x_stride0;
  a->M_total = static_cast<int>(M_total);
  a->E = static_cast<int>(E);
  a->N = static_cast<int>(N);
  a->K = static_cast<int>(K);
  a->gs = static_cast<int>(group_size);
  return W4A8_OK;
}

// Kernel choice and launch(es) of one grouped GEMM (the AUTO rule is
// documented at W4A8_KERNEL_AUTO in the header).
int gemm_dispatch(GemmArgs& a, int32_t kernel, void* stream) {
  a.status = device_status_ptr();
  if (a.status == nullptr) return fail(W4A8_ERR_CUDA, "cannot resolve the device status word");
  const bool aligned16 = (reinterpret_cast<uintptr_t>(a.x_q) % 16 == 0) && (a.x_stride0 % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(a.w_packed) % 16 == 0);
  const bool tc_ok = gemm_tc_supports(a.K, a.gs, a.E) && aligned16;
  const bool gemv_ok = aligned16;
  const bool simt_ok = (reinterpret_cast<uintptr_t>(a.x_q) % 4 == 0) && (a.x_stride0 % 4 == 0);
  const int64_t M_total = a.rows_hint > 0 ? a.rows_hint : a.M_total, E = a.E;   // rows the kernel choice assumes
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  switch (kernel) {
    case W4A8_KERNEL_TC:
      if (!tc_ok)
        return fail(W4A8_ERR_INVALID,
                    "tensor-core kernel needs K >= 128, E <= 1024 and 16-byte aligned x_q rows / weights");
      e = launch_gemm_tc(a, st);
      break;
    case W4A8_KERNEL_GEMV:
      if (!gemv_ok) return fail(W4A8_ERR_INVALID, "streaming kernel needs 16-byte aligned x_q rows / weights");
      e = launch_gemm_gemv(a, st);
      break;
    case W4A8_KERNEL_SIMT:
      if (!simt_ok) return fail(W4A8_ERR_INVALID, "CUDA-core kernel needs 4-byte aligned x_q rows");
      e = launch_gemm_simt(a, st);
      break;
    default: {  // W4A8_KERNEL_AUTO
      // Experts with at most kGemvAutoRows rows are weight-streaming bound and
      // go to the streaming kernel, the others to the tensor-core kernel
      // (measured on B200: at 5-8 rows per expert a second streaming pass costs
      // more than the tensor-core tiles).  The split is applied on
      // the device by each kernel's scheduler (row-count window), so no host
      // synchronisation is needed; a launch whose window holds no expert exits
      // after its prologue.
      if (!tc_ok) {
        if (gemv_ok && M_total <= kGemvAutoRows) e = launch_gemm_gemv(a, st);
        else if (simt_ok) e = launch_gemm_simt(a, st);
        else return fail(W4A8_ERR_INVALID, "x_q rows must be at least 4-byte aligned");
      } else if (M_total <= kGemvAutoRows || M_total <= 2 * E) {
        // at most two rows per expert on average (decode): every expert streams,
        // one with more than kGemvMaxTokens rows in several passes, which costs
        // less than the tensor-core launch's fixed per-K-group work
        e = launch_gemm_gemv(a, st);
      } else if (M_total >= 64 * E) {
        e = launch_gemm_tc(a, st);
      } else {
        GemmArgs small = a, big = a;
        small.max_rows = kGemvAutoRows;
        big.min_rows = kGemvAutoRows + 1;
        e = launch_gemm_gemv(small, st);
        if (e == cudaSuccess) e = launch_gemm_tc(big, st);
      }
    }
  }
  if (e != cudaSuccess) return cuda_fail(e, "grouped GEMM launch");
  return W4A8_OK;
}
}  // namespace

extern "C" {

int w4a8_abi_version(void) { return 1; }

const char* w4a8_last_error(void) { return g_last_error.c_str(); }

int w4a8_group_gemm_moe_ex(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                           const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                           const int32_t* expert_offsets, void* out, int64_t out_stride0,
                           int64_t out_stride1, int64_t M_total, int64_t E, int64_t N, int64_t K,
                           int64_t group_size, int32_t kernel, int32_t* partials, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  GemmArgs a{};
  int rc = gemm_setup(&a, x_q, x_stride0, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, M_total, E, N, K,
                      group_size, kernel, true, out);
  if (rc != W4A8_OK || M_total == 0) return rc;
  a.partials = partials;
  a.out_stride0 = out_stride0;
  a.out_stride1 = out_stride1;
  return gemm_dispatch(a, kernel, stream);
}

int w4a8_group_gemm_moe_prepacked(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                                  const uint8_t* w_prepacked, const float* w_scale, const int8_t* w_zero,
                                  const int32_t* expert_offsets, void* out, int64_t out_stride0,
                                  int64_t out_stride1, int64_t M_total, int64_t E, int64_t N, int64_t K,
                                  int64_t group_size, int32_t kernel, int32_t* partials, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  GemmArgs a{};
  int rc = gemm_setup(&a, x_q, x_stride0, x_scale, w_prepacked, w_scale, w_zero, expert_offsets, M_total, E, N, K,
                      group_size, kernel, true, out);
  if (rc != W4A8_OK || M_total == 0) return rc;
  a.partials = partials;
  a.out_stride0 = out_stride0;
  a.out_stride1 = out_stride1;
  a.layout = 1;
  return gemm_dispatch(a, kernel, stream);
}

int w4a8_group_gemm_moe_hint(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                             const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                             const int32_t* expert_offsets, void* out, int64_t out_stride0, int64_t out_stride1,
                             int64_t M_total, int64_t E, int64_t N, int64_t K, int64_t group_size,
                             int64_t rows_hint, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  GemmArgs a{};
  int rc = gemm_setup(&a, x_q, x_stride0, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, M_total, E, N, K,
                      group_size, W4A8_KERNEL_AUTO, true, out);
  if (rc != W4A8_OK || M_total == 0) return rc;
  if (rows_hint < 0 || rows_hint > M_total)
    return fail(W4A8_ERR_INVALID, "rows_hint %lld outside [0, M_total=%lld]", (long long)rows_hint, (long long)M_total);
  a.out_stride0 = out_stride0;
  a.out_stride1 = out_stride1;
  a.rows_hint = static_cast<int>(rows_hint);
  return gemm_dispatch(a, W4A8_KERNEL_AUTO, stream);
}

int w4a8_group_gemm_moe_rows(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                             const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                             const int32_t* expert_offsets, void* out_stage, const uint64_t* out_rows,
                             int64_t M_total, int64_t E, int64_t N, int64_t K, int64_t group_size, int64_t rows_hint,
                             void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  GemmArgs a{};
  int rc = gemm_setup(&a, x_q, x_stride0, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, M_total, E, N, K,
                      group_size, W4A8_KERNEL_AUTO, true, out_stage);
  if (rc != W4A8_OK || M_total == 0) return rc;
  if (out_rows == nullptr) return fail(W4A8_ERR_INVALID, "null row-address table");
  if ((reinterpret_cast<uintptr_t>(out_stage) & 15) || (N % 8) != 0)
    return fail(W4A8_ERR_INVALID, "row-address store needs a 16-byte aligned staging output and N %% 8 == 0");
  a.out_stride0 = N;
  a.out_stride1 = 1;
  if (rows_hint < 0 || rows_hint > M_total)
    return fail(W4A8_ERR_INVALID, "rows_hint %lld outside [0, M_total=%lld]", (long long)rows_hint, (long long)M_total);
  a.out_rows = out_rows;
  a.rows_hint = static_cast<int>(rows_hint);
  return gemm_dispatch(a, W4A8_KERNEL_AUTO, stream);
}

int w4a8_group_gemm_moe_combine(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                                const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                                const int32_t* expert_offsets, const int32_t* sorted_ids, const float* topk_w,
                                int64_t topk, float* acc_out, int64_t acc_stride0, int64_t M_total, int64_t E,
                                int64_t N, int64_t K, int64_t group_size, int32_t kernel, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  GemmArgs a{};
  int rc = gemm_setup(&a, x_q, x_stride0, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, M_total, E, N, K,
                      group_size, kernel, false, nullptr);
  if (rc != W4A8_OK) return rc;
  if (topk <= 0 || topk > 256 || acc_stride0 < N)
    return fail(W4A8_ERR_INVALID, "bad combine arguments topk=%lld acc_stride0=%lld (N=%lld)", (long long)topk,
                (long long)acc_stride0, (long long)N);
  if (M_total == 0) return W4A8_OK;
  if (sorted_ids == nullptr || topk_w == nullptr || acc_out == nullptr)
    return fail(W4A8_ERR_INVALID, "null combine pointer");
  a.comb_out = acc_out;
  a.comb_ids = sorted_ids;
  a.comb_w = topk_w;
  a.comb_topk = static_cast<int>(topk);
  a.comb_stride = acc_stride0;
  return gemm_dispatch(a, kernel, stream);
}

int w4a8_group_gemm_moe(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                        const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                        const int32_t* expert_offsets, void* out, int64_t out_stride0,
                        int64_t out_stride1, int64_t M_total, int64_t E, int64_t N, int64_t K,
                        int64_t group_size, void* stream) {
  return w4a8_group_gemm_moe_ex(x_q, x_stride0, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, out,
                                out_stride0, out_stride1, M_total, E, N, K, group_size, W4A8_KERNEL_AUTO,
                                nullptr, stream);
}

int w4a8_act_quant(const void* x, int64_t x_stride0, int64_t T, int64_t H, int8_t* x_q, int64_t q_stride0,
                   float* x_scale, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  if (T < 0 || H <= 0 || T > INT32_MAX || H > INT32_MAX)
    return fail(W4A8_ERR_INVALID, "bad sizes T=%lld H=%lld", (long long)T, (long long)H);
  if (T == 0) return W4A8_OK;
  if (x == nullptr || x_q == nullptr || x_scale == nullptr) return fail(W4A8_ERR_INVALID, "null pointer");
  cudaError_t e = launch_act_quant(static_cast<const __nv_bfloat16*>(x), x_stride0, (int)T, (int)H, x_q,
                                   q_stride0, x_scale, nullptr, 1, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : cuda_fail(e, "act_quant launch");
}

int w4a8_router_topk(const float* logits, int64_t logits_stride0, int64_t T, int64_t E, int64_t topk,
                     int32_t scoring, int32_t renormalize, int32_t* topk_ids, float* topk_weights,
                     const void* x, int64_t x_stride0, int64_t H, int8_t* x_q, int64_t q_stride0,
                     float* x_scale, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  if (T < 0 || T > INT32_MAX || E <= 0 || E > kRouterMaxExperts || topk <= 0 || topk > E ||
      topk > kRouterMaxTopk || (scoring != 0 && scoring != 1) || logits_stride0 < E)
    return fail(W4A8_ERR_INVALID, "bad router arguments T=%lld E=%lld topk=%lld scoring=%d", (long long)T,
                (long long)E, (long long)topk, (int)scoring);
  if (x != nullptr && (H <= 0 || H > INT32_MAX || x_stride0 < H || q_stride0 < H || x_q == nullptr ||
                       x_scale == nullptr))
    return fail(W4A8_ERR_INVALID, "bad quantisation arguments H=%lld", (long long)H);
  if (T == 0) return W4A8_OK;
  if (logits == nullptr || topk_ids == nullptr || topk_weights == nullptr) return fail(W4A8_ERR_INVALID, "null pointer");
  const RouterArgs r{logits, logits_stride0, (int)E, (int)topk, (int)scoring, renormalize != 0 ? 1 : 0,
                     topk_ids, topk_weights};
  cudaError_t e = launch_router(r, (int)T, static_cast<const __nv_bfloat16*>(x), x_stride0, (int)H, x_q, q_stride0,
                                x_scale, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : cuda_fail(e, "router launch");
}

int w4a8_quant_scatter(const void* x, int64_t x_stride0, int64_t T, int64_t H, const int32_t* inv_pos,
                       int64_t topk, int8_t* x_sorted, float* xs_sorted, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  if (T < 0 || H <= 0 || topk <= 0 || topk > 256 || T * topk > INT32_MAX || H > INT32_MAX)
    return fail(W4A8_ERR_INVALID, "bad sizes T=%lld H=%lld topk=%lld", (long long)T, (long long)H,
                (long long)topk);
  if (T == 0) return W4A8_OK;
  if (x == nullptr || inv_pos == nullptr || x_sorted == nullptr || xs_sorted == nullptr)
    return fail(W4A8_ERR_INVALID, "null pointer");
  cudaError_t e = launch_act_quant(static_cast<const __nv_bfloat16*>(x), x_stride0, (int)T, (int)H, x_sorted,
                                   H, xs_sorted, inv_pos, (int)topk, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : cuda_fail(e, "quant_scatter launch");
}

size_t w4a8_moe_align_workspace_size(int64_t T, int64_t topk, int64_t E) {
  if (T < 0 || topk <= 0 || E <= 0 || T * topk > INT32_MAX) return 0;
  return align_workspace_bytes((int)(T * topk), (int)E);
}

int w4a8_moe_align(const int32_t* topk_ids, int64_t T, int64_t topk, int64_t E, int64_t block_size,
                   int32_t* expert_offsets, int32_t* sorted_ids, int32_t* inv_pos, int32_t* padded_ids,
                   int32_t* block_expert, int32_t* num_post_pad, void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  if (T < 0 || topk <= 0 || E <= 0 || E > 8192 || block_size <= 0 || block_size > kMaxAlignBlock ||
      T * topk > INT32_MAX / 2 || T * topk + E * (block_size - 1) > INT32_MAX / 2)
    return fail(W4A8_ERR_INVALID,
                "bad sizes T=%lld topk=%lld E=%lld block_size=%lld (block_size <= %d, T*topk + E*(block_size-1) "
                "must fit the 32-bit padded index range)",
                (long long)T, (long long)topk, (long long)E, (long long)block_size, kMaxAlignBlock);
  if (expert_offsets == nullptr || (T > 0 && (topk_ids == nullptr || sorted_ids == nullptr || inv_pos == nullptr)))
    return fail(W4A8_ERR_INVALID, "null pointer");
  const size_t need = w4a8_moe_align_workspace_size(T, topk, E);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(W4A8_ERR_INVALID, "workspace too small (%zu < %zu bytes)", workspace_bytes, need);
  cudaError_t e = launch_moe_align(topk_ids, (int)(T * topk), (int)E, (int)block_size, expert_offsets,
                                   sorted_ids, inv_pos, padded_ids, block_expert, num_post_pad, workspace,
                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : cuda_fail(e, "moe_align launch");
}

int w4a8_silu_mul_requant(const void* h, int64_t h_stride0, int64_t R, int64_t I, int8_t* q, float* s,
                          void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  if (R < 0 || I <= 0 || I > 16384 || R > INT32_MAX || h_stride0 < 2 * I)
    return fail(W4A8_ERR_INVALID, "bad sizes R=%lld I=%lld (I <= 16384)", (long long)R, (long long)I);
  if (R == 0) return W4A8_OK;
  if (h == nullptr || q == nullptr || s == nullptr) return fail(W4A8_ERR_INVALID, "null pointer");
  cudaError_t e = launch_silu_mul_requant(static_cast<const __nv_bfloat16*>(h), h_stride0, (int)R, (int)I, q, I,
                                          s, nullptr, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : cuda_fail(e, "silu_mul_requant launch");
}

int w4a8_silu_mul_requant_rows(const void* h, int64_t h_stride0, int64_t R, int64_t I, int8_t* q, float* s,
                               const int32_t* valid_rows, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  if (R < 0 || I <= 0 || I > 16384 || R > INT32_MAX || h_stride0 < 2 * I)
    return fail(W4A8_ERR_INVALID, "bad sizes R=%lld I=%lld (I <= 16384)", (long long)R, (long long)I);
  if (R == 0) return W4A8_OK;
  if (h == nullptr || q == nullptr || s == nullptr || valid_rows == nullptr)
    return fail(W4A8_ERR_INVALID, "null pointer");
  cudaError_t e = launch_silu_mul_requant(static_cast<const __nv_bfloat16*>(h), h_stride0, (int)R, (int)I, q, I,
                                          s, valid_rows, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : cuda_fail(e, "silu_mul_requant launch");
}

int w4a8_moe_combine(const void* y, int64_t y_stride0, const int32_t* inv_pos, const float* topk_w, int64_t T,
                     int64_t topk, int64_t H, void* out, int64_t out_stride0, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  if (T < 0 || topk <= 0 || H <= 0 || T > INT32_MAX || H > INT32_MAX)
    return fail(W4A8_ERR_INVALID, "bad sizes T=%lld topk=%lld H=%lld", (long long)T, (long long)topk,
                (long long)H);
  if (T == 0) return W4A8_OK;
  if (y == nullptr || inv_pos == nullptr || topk_w == nullptr || out == nullptr)
    return fail(W4A8_ERR_INVALID, "null pointer");
  cudaError_t e = launch_moe_combine(static_cast<const __nv_bfloat16*>(y), y_stride0, inv_pos, topk_w, (int)T,
                                     (int)topk, (int)H, static_cast<__nv_bfloat16*>(out), out_stride0,
                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : cuda_fail(e, "moe_combine launch");
}

int w4a8_combine_finish(float* acc, int64_t acc_stride0, int64_t T, int64_t H, void* out, int64_t out_stride0,
                        void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  if (T < 0 || H <= 0 || T > INT32_MAX || H > INT32_MAX || acc_stride0 < H || out_stride0 < H)
    return fail(W4A8_ERR_INVALID, "bad sizes T=%lld H=%lld", (long long)T, (long long)H);
  if (T == 0) return W4A8_OK;
  if (acc == nullptr || out == nullptr) return fail(W4A8_ERR_INVALID, "null pointer");
  cudaError_t e = launch_combine_finish(acc, acc_stride0, (int)T, (int)H, static_cast<__nv_bfloat16*>(out),
                                        out_stride0, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : cuda_fail(e, "combine_finish launch");
}

int w4a8_gather_rows(const void* src, int64_t src_stride_bytes, const int32_t* index, int64_t rows,
                     int64_t row_bytes, void* dst, int64_t dst_stride_bytes, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  if (rows < 0 || rows > INT32_MAX || row_bytes < 0 || src_stride_bytes < row_bytes || dst_stride_bytes < row_bytes)
    return fail(W4A8_ERR_INVALID, "bad sizes rows=%lld row_bytes=%lld", (long long)rows, (long long)row_bytes);
  if (rows == 0 || row_bytes == 0) return W4A8_OK;
  if (src == nullptr || index == nullptr || dst == nullptr) return fail(W4A8_ERR_INVALID, "null pointer");
  cudaError_t e = launch_gather_rows(src, src_stride_bytes, index, rows, row_bytes, dst, dst_stride_bytes,
                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? W4A8_OK : cuda_fail(e, "gather_rows launch");
}

int w4a8_device_status(int32_t* status_out, int32_t reset, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) return cuda_fail(be, "stream device");
  int* p = device_status_ptr();
  if (p == nullptr) return fail(W4A8_ERR_CUDA, "cannot resolve the device status word");
  int v = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "device status read");
  if (reset && v != 0) {
    e = cudaMemsetAsync(p, 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "device status reset");
  }
  if (status_out) *status_out = v;
  return W4A8_OK;
}

}  // extern "C"
