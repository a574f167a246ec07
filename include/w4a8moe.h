/*
 * w4a8moe.h -- C ABI of the B200 (sm_100a) W4A8 Mixture-of-Experts library.
 *
 * Plain pointers, sizes and strides; every pointer is CUDA device memory on
 * the stream's device unless stated otherwise; `stream` is a cudaStream_t.
 * The library links its own CUDA runtime: it runs each call on the device of
 * `stream`, and for a NULL stream (the legacy default stream) on the device
 * of the driver context current on the calling thread, i.e. the device the
 * caller selected with cudaSetDevice (torch.cuda.set_device) and has used
 * since.  Nothing here allocates device memory:
 * scratch space is passed in by the caller.  No call synchronises the host
 * except w4a8_device_status().
 *
 * Return value: W4A8_OK, or an error code; w4a8_last_error() then returns a
 * message for the calling thread.
 *
 * The reference ("CaiJichang212/flagos-kernel-gen", Task 1) is a Python/Triton
 * operator; each entry point below names the reference interface it replaces.
 */
#ifndef W4A8MOE_H_
#define W4A8MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define W4A8_OK 0
#define W4A8_ERR_INVALID 1 /* bad shape, stride, alignment or argument */
#define W4A8_ERR_CUDA 2    /* CUDA runtime / launch error */
#define W4A8_ERR_DEVICE 3  /* a kernel reported an error in the device status word */

/* Kernel selector for w4a8_group_gemm_moe_ex. */
#define W4A8_KERNEL_AUTO 0 /* experts with <= 4 rows: streaming kernel; others: tensor-core kernel
                              (CUDA-core kernel where the tensor-core shape rules fail) */
#define W4A8_KERNEL_TC 1   /* TMA + tcgen05.mma.kind::i8 kernel (K >= 128, E <= 1024, 16-byte aligned x_q rows) */
#define W4A8_KERNEL_SIMT 2 /* dp4a CUDA-core tile kernel (any shape; 4-byte aligned x_q rows) */
#define W4A8_KERNEL_GEMV 3 /* weight-streaming CUDA-core kernel for few rows per expert
                              (16-byte aligned x_q rows / weights) */

int w4a8_abi_version(void);
const char* w4a8_last_error(void);

/*
 * Grouped W4A8 GEMM over expert segments.
 * Replaces: w4a8_group_gemm_moe(x_q, x_scale, w_q4_packed, w_scale, w_zero,
 *           expert_offsets, out, group_size)   docs/Task1.md:8-17 (reference
 *           implementation docs/Task1.md:53-114; Triton launcher
 *           Task1/v1.6/task1-codex5.5-all-v1.6.py:986-1030).
 *   x_q            int8  [M_total, K], row stride x_stride0 (elements), unit column stride
 *   x_scale        fp32  [M_total]
 *   w_q4_packed    uint8 [E, N, K/2] contiguous; low nibble = even k, high = odd k
 *   w_scale        fp32  [E, N, K/group_size] contiguous
 *   w_zero         int8  [E, N, K/group_size] contiguous
 *   expert_offsets int32 [E+1]: rows [off[e], off[e+1]) belong to expert e
 *   out            bf16  [M_total, N] with strides (out_stride0, out_stride1) in elements;
 *                  rows outside every segment are not written
 *   group_size     64 or 128; K % group_size == 0
 */
int w4a8_group_gemm_moe(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                        const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                        const int32_t* expert_offsets, void* out, int64_t out_stride0,
                        int64_t out_stride1, int64_t M_total, int64_t E, int64_t N, int64_t K,
                        int64_t group_size, void* stream);

/*
 * Same as w4a8_group_gemm_moe with an explicit kernel choice and an optional
 * export of the exact int32 per-group partial sums
 *   partials[g, m, n] = sum_{k in group g} x_q[m,k] * int8(nibble - zero)
 * (int32 [K/group_size, M_total, N], group-major so that the export is
 * written in full lines; entries of rows inside a segment are written; NULL
 * to skip).  Replaces the per-group einsum of docs/Task1.md:100-104, which
 * the reference keeps internal (there as [m, n, g]).
 */
int w4a8_group_gemm_moe_ex(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                           const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                           const int32_t* expert_offsets, void* out, int64_t out_stride0,
                           int64_t out_stride1, int64_t M_total, int64_t E, int64_t N, int64_t K,
                           int64_t group_size, int32_t kernel, int32_t* partials, void* stream);

/*
 * w4a8_group_gemm_moe (AUTO kernel choice) for a caller whose x_q / out hold
 * M_total rows of capacity while the rows actually routed are known only on
 * the device (expert_offsets[E] <= M_total, e.g. the receive buffer of the
 * expert-parallel mode).  rows_hint (1..M_total, 0 = M_total) is the row
 * count the kernel and tile-width choice assumes; results do not depend on
 * it.  No reference counterpart (the reference reads the offsets on the
 * host, Task1/v1.6/task1-codex5.5-all-v1.6.py:62-64).
 */
int w4a8_group_gemm_moe_hint(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                             const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                             const int32_t* expert_offsets, void* out, int64_t out_stride0,
                             int64_t out_stride1, int64_t M_total, int64_t E, int64_t N, int64_t K,
                             int64_t group_size, int64_t rows_hint, void* stream);

/*
 * Offline weight prepack (no reference counterpart; the reference unpacks the
 * packed bytes on every call, docs/Task1.md:78-81).  Writes the same int4
 * weights in the word-interleaved nibble layout: for each 32-bit word q of a
 * row (k = 8q .. 8q + 7), byte b (0..3) holds k = 8q + b in its low nibble
 * and k = 8q + 4 + b in its high nibble (the reference layout has k = 2j and
 * 2j + 1 in byte j).  Same size; scales and zero points are unchanged.  With
 * this layout the int4 -> int8 unpack needs no byte permutes.  out may equal
 * w_q4_packed (in place).
 *   w_q4_packed, out  uint8 [rows, K/2] contiguous, 16-byte aligned; K % 64 == 0
 */
int w4a8_prepack_weights(const uint8_t* w_q4_packed, uint8_t* out, int64_t rows, int64_t K, void* stream);

/*
 * w4a8_group_gemm_moe_ex on weights prepacked by w4a8_prepack_weights (all
 * kernels; results identical to the reference layout's).
 */
int w4a8_group_gemm_moe_prepacked(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                                  const uint8_t* w_prepacked, const float* w_scale, const int8_t* w_zero,
                                  const int32_t* expert_offsets, void* out, int64_t out_stride0,
                                  int64_t out_stride1, int64_t M_total, int64_t E, int64_t N, int64_t K,
                                  int64_t group_size, int32_t kernel, int32_t* partials, void* stream);

/*
 * Grouped W4A8 GEMM with the weighted top-k combine fused into its epilogue.
 * Replaces the bf16 store of docs/Task1.md:110-112 (the reference's operator
 * ends there) followed by a separate combine: each row m's result is still
 * rounded to bf16 exactly as w4a8_group_gemm_moe stores it, then multiplied
 * by its top-k weight in fp32 and added (fp32 atomics) into the token's row
 *   acc_out[f / topk, n] += topk_w[f] * y[m, n],   f = sorted_ids[m]
 * (f = t*topk + j, as written by w4a8_moe_align).  acc_out fp32 [T, N] (row
 * stride acc_stride0) must hold zeros before the first GEMM of a batch;
 * w4a8_combine_finish then writes the bf16 output and clears it again.  The
 * order of the fp32 additions is not fixed, so results may differ from the
 * unfused path (w4a8_moe_combine, j ascending) in the last fp32 bit.
 * Other arguments as w4a8_group_gemm_moe_ex (no partials export).
 */
int w4a8_group_gemm_moe_combine(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                                const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                                const int32_t* expert_offsets, const int32_t* sorted_ids, const float* topk_w,
                                int64_t topk, float* acc_out, int64_t acc_stride0, int64_t M_total, int64_t E,
                                int64_t N, int64_t K, int64_t group_size, int32_t kernel, void* stream);

/*
 * w4a8_group_gemm_moe_hint with the bf16 rows also stored through a
 * row-address table (no reference counterpart): row m's N results go to the
 * contiguous bf16 elements at address out_rows[m] (0: the row is not
 * stored).  The addresses may lie in another GPU's memory mapped into this
 * one (NVLink peer memory), so a grouped GEMM can return expert results
 * straight to the ranks that own the tokens.  The tensor-core kernel writes
 * each tile's rows to out_stage first and copies them on in 16-byte pieces;
 * out_stage's contents afterwards are unspecified.
 *   out_stage bf16 [M_total, N] contiguous, 16-byte aligned; N % 8 == 0
 *   out_rows  uint64 [M_total]
 */
int w4a8_group_gemm_moe_rows(const int8_t* x_q, int64_t x_stride0, const float* x_scale,
                             const uint8_t* w_q4_packed, const float* w_scale, const int8_t* w_zero,
                             const int32_t* expert_offsets, void* out_stage, const uint64_t* out_rows,
                             int64_t M_total, int64_t E, int64_t N, int64_t K, int64_t group_size, int64_t rows_hint,
                             void* stream);

/*
 * Finishes a fused combine (no reference counterpart):
 *   out[t, :] = bf16(acc[t, :]);  acc[t, :] = 0      for t < T
 *   acc fp32 [T, H] (row stride acc_stride0), out bf16 [T, H] (row stride out_stride0)
 */
int w4a8_combine_finish(float* acc, int64_t acc_stride0, int64_t T, int64_t H, void* out,
                        int64_t out_stride0, void* stream);

/*
 * Per-token symmetric int8 quantisation of bf16 activations.
 * No counterpart kernel in the reference (its entry point takes x_q/x_scale
 * already quantised, docs/Task1.md:9-10); the convention is the repository's
 * int8 quantiser, docs/Task3.md:58-67:
 *   x_scale[t] = max(max_k |x[t,k]| / 127, 1e-10);  x_q = trunc(clamp(x / x_scale, -127, 127))
 *   x bf16 [T, H] (row stride x_stride0), x_q int8 [T, H] (row stride q_stride0), x_scale fp32 [T]
 */
int w4a8_act_quant(const void* x, int64_t x_stride0, int64_t T, int64_t H, int8_t* x_q,
                   int64_t q_stride0, float* x_scale, void* stream);

/*
 * Router + top-k, optionally fused with the activation quantisation.  The
 * reference takes routing as given (its entry point receives expert_offsets,
 * docs/Task1.md:13); this is the routing its benchmark inputs use: scores =
 * softmax (scoring 0) or sigmoid (scoring 1) of the logits, the topk experts
 * by score in descending order (torch.topk), weights renormalised to sum to 1
 * (renormalize != 0).  Experts are ranked by logit (the same order as their
 * scores), ties to the lower expert index.
 *   logits fp32 [T, E] (row stride logits_stride0), E <= 1024, topk <= min(E, 32)
 *   topk_ids int32 [T, topk], topk_weights fp32 [T, topk] (contiguous)
 *   x bf16 [T, H] (row stride x_stride0) or NULL: with x, also x_q int8 [T, H]
 *   (row stride q_stride0) and x_scale fp32 [T] exactly as w4a8_act_quant.
 */
int w4a8_router_topk(const float* logits, int64_t logits_stride0, int64_t T, int64_t E, int64_t topk,
                     int32_t scoring, int32_t renormalize, int32_t* topk_ids, float* topk_weights,
                     const void* x, int64_t x_stride0, int64_t H, int8_t* x_q, int64_t q_stride0,
                     float* x_scale, void* stream);

/*
 * Fused quantise + dispatch: quantises token t once (as w4a8_act_quant) and
 * writes it to rows inv_pos[t*topk + j] (j < topk) of x_sorted / xs_sorted,
 * i.e. straight into expert-sorted order.  inv_pos comes from w4a8_moe_align;
 * entries < 0 are skipped.  No reference counterpart.
 *   x_sorted int8 [T*topk, H] contiguous, xs_sorted fp32 [T*topk]
 */
int w4a8_quant_scatter(const void* x, int64_t x_stride0, int64_t T, int64_t H,
                       const int32_t* inv_pos, int64_t topk, int8_t* x_sorted, float* xs_sorted,
                       void* stream);

/* Bytes of scratch device memory w4a8_moe_align needs. */
size_t w4a8_moe_align_workspace_size(int64_t T, int64_t topk, int64_t E);

/*
 * Token-to-expert sort and block alignment (counting sort, deterministic).
 * No reference counterpart (the reference takes expert_offsets as input,
 * docs/Task1.md:15); the padded outputs follow the moe_align_block_size
 * convention (sentinel = T*topk for padding).
 *   topk_ids       int32 [T, topk]  expert of each (token, slot); ids outside [0,E) are dropped
 *   expert_offsets int32 [E+1]      unpadded segment starts
 *   sorted_ids     int32 [T*topk]   flat index t*topk+j per sorted row; ascending inside an expert
 *   inv_pos        int32 [T*topk]   sorted row of each flat index (-1 if dropped)
 *   padded_ids     int32 [T*topk + E*(block_size-1)] or NULL
 *   block_expert   int32 [ceil((T*topk + E*(block_size-1)) / block_size)] or NULL (-1 past the end)
 *   num_post_pad   int32 [1] or NULL
 *   workspace      >= w4a8_moe_align_workspace_size(T, topk, E) bytes
 * block_size is 1..4096 and T*topk + E*(block_size-1) must be below 2^30;
 * other values return W4A8_ERR_INVALID.
 */
int w4a8_moe_align(const int32_t* topk_ids, int64_t T, int64_t topk, int64_t E, int64_t block_size,
                   int32_t* expert_offsets, int32_t* sorted_ids, int32_t* inv_pos,
                   int32_t* padded_ids, int32_t* block_expert, int32_t* num_post_pad,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * SiLU-mul + per-row int8 requantisation between the gate/up and down GEMMs.
 * No reference kernel; formula of docs/Task3.md:99-110 (gate = h[:, :I],
 * up = h[:, I:], y = silu(gate) * up in fp32) and the quantiser of
 * docs/Task3.md:58-67.
 *   h bf16 [R, 2I] (row stride h_stride0) -> q int8 [R, I] contiguous, s fp32 [R]
 */
int w4a8_silu_mul_requant(const void* h, int64_t h_stride0, int64_t R, int64_t I, int8_t* q,
                          float* s, void* stream);

/*
 * w4a8_silu_mul_requant over the first *valid_rows rows (a count read on the
 * device, at most R; R is the capacity of h / q / s).  No reference
 * counterpart; used on the expert-parallel receive buffer.
 */
int w4a8_silu_mul_requant_rows(const void* h, int64_t h_stride0, int64_t R, int64_t I, int8_t* q,
                               float* s, const int32_t* valid_rows, void* stream);

/*
 * Weighted top-k combine back to token order (no reference counterpart):
 *   out[t, :] = bf16( sum_{j=0..topk-1} topk_w[t,j] * y[inv_pos[t*topk+j], :] )  (fp32, j ascending)
 *   y bf16 [*, H] (row stride y_stride0), topk_w fp32 [T, topk], out bf16 [T, H] (row stride out_stride0)
 */
int w4a8_moe_combine(const void* y, int64_t y_stride0, const int32_t* inv_pos, const float* topk_w,
                     int64_t T, int64_t topk, int64_t H, void* out, int64_t out_stride0,
                     void* stream);

/*
 * Row permutation: dst row i = src row index[i] (row_bytes bytes per row;
 * strides in bytes; rows with index[i] < 0 are left untouched).  Used by the
 * expert-parallel path to move received token rows into local expert order
 * and back.  No reference counterpart.
 */
int w4a8_gather_rows(const void* src, int64_t src_stride_bytes, const int32_t* index, int64_t rows,
                     int64_t row_bytes, void* dst, int64_t dst_stride_bytes, void* stream);

/*
 * w4a8_moe_align without a caller workspace, for callers that cannot
 * allocate device memory (a server whose pool already owns all free device
 * memory and lends none, or a plain C caller with no allocator).  No
 * counterpart in the reference.  Same outputs as w4a8_moe_align (bit for
 * bit); its scratch is a fixed 660 KB array in the library's device memory,
 * held by every GPU that loads the library until the process exits.
 * Limits: T*topk <= 131072, E <= 512 and block_size <= 4096, else
 * W4A8_ERR_INVALID with a message.
 * Allocates nothing.  All calls share the array: calls that overlap on the GPU
 * race, so serialise them.  The first call on a device resolves the array's
 * device address; make it before capturing a stream.
 */
int w4a8_moe_align_noalloc(const int32_t* topk_ids, int64_t T, int64_t topk, int64_t E,
                           int64_t block_size, int32_t* expert_offsets, int32_t* sorted_ids,
                           int32_t* inv_pos, int32_t* padded_ids, int32_t* block_expert,
                           int32_t* num_post_pad, void* stream);

/*
 * Expert parallelism over peer memory (no reference counterpart: the
 * reference has no multi-GPU mode).  Every rank owns a receive buffer of one
 * layout, mapped into every peer (peers: device array [world] of the buffers'
 * base addresses as seen from this GPU, e.g. torch symmetric memory).  Byte
 * offsets (identical on all ranks): flags int32 [world] (zero before the
 * first epoch), counts int32 [world, E], xq int8 [cap_rows, H], xs fp32
 * [cap_rows], src int32 [cap_rows], yhome bf16 [tk_max, H]; tk_max = the
 * most slots (tokens x topk) one rank routes.  All ranks make the same calls
 * in the same order with increasing epochs.  Waits on peers are bounded
 * (~2 s): on expiry the kernel records code 130 in the device status word
 * and returns; a rank that would receive more than cap_rows rows records 131
 * and nothing is sent to it.
 *
 * w4a8_ep_exchange: this rank's rows per global expert (from its
 *   w4a8_moe_align expert_offsets [E+1]) into every peer's counts row
 *   `rank`, one signal of `epoch`, then dest_base int32 [E] (first receive
 *   row of this rank's slots of expert e on its owner, -1 if none) and
 *   local_offsets int32 [E/world + 1] (segments of this rank's experts in its
 *   own xq; local_offsets[E/world] = rows received).
 * w4a8_ep_dispatch: quantises each token once (as w4a8_act_quant) and stores
 *   its row, scale and return address into the owners' receive buffers;
 *   home_pos int32 [T*topk] = the slot's index, or -1 for dropped slots.
 * w4a8_ep_dispatch_dedup: as w4a8_ep_dispatch, but a token's int8 row
 *   crosses to each remote rank once: a later slot of the same token on the
 *   same remote rank stores only its scale, return address and, in the dup
 *   int32 [cap_rows] region at dup_off, the receive row of that first slot
 *   (-1 for rows whose bytes were sent).  The owner then runs
 *   w4a8_ep_replicate after the barrier.
 * w4a8_ep_replicate: on the receiving rank, row r < *total_rows of xq whose
 *   dup entry is p >= 0 takes the bytes of row p.
 * w4a8_ep_barrier: every rank signals `epoch` and waits for all.
 * w4a8_ep_return: row r of y (this rank's receive order, r < *total_rows)
 *   into row f of its sender's yhome (src[r] = sender * tk_max + f).
 * w4a8_ep_row_addresses: the same destinations as a row-address table
 *   out_rows uint64 [cap_rows] (rows r >= *total_rows get 0), for
 *   w4a8_group_gemm_moe_rows, whose epilogue then stores the results into
 *   the senders' yhome directly (no return pass).
 */
int w4a8_ep_exchange(const int32_t* expert_offsets, int64_t E, int64_t world, int64_t rank,
                     void* const* peers, int64_t counts_off, int64_t flags_off, int32_t epoch,
                     int64_t cap_rows, int32_t* dest_base, int32_t* local_offsets, void* stream);
int w4a8_ep_dispatch(const void* x, int64_t x_stride0, int64_t T, int64_t H, const int32_t* topk_ids,
                     int64_t topk, int64_t E, int64_t world, int64_t rank, int64_t tk_max,
                     const int32_t* expert_offsets, const int32_t* inv_pos, const int32_t* dest_base,
                     void* const* peers, int64_t xq_off, int64_t xs_off, int64_t src_off,
                     int32_t* home_pos, void* stream);
int w4a8_ep_dispatch_dedup(const void* x, int64_t x_stride0, int64_t T, int64_t H, const int32_t* topk_ids,
                           int64_t topk, int64_t E, int64_t world, int64_t rank, int64_t tk_max,
                           const int32_t* expert_offsets, const int32_t* inv_pos, const int32_t* dest_base,
                           void* const* peers, int64_t xq_off, int64_t xs_off, int64_t src_off, int64_t dup_off,
                           int32_t* home_pos, void* stream);
int w4a8_ep_replicate(void* buf, int64_t xq_off, int64_t dup_off, int64_t H, const int32_t* total_rows,
                      int64_t rows_hint, void* stream);
int w4a8_ep_barrier(void* const* peers, int64_t flags_off, int64_t world, int64_t rank, int32_t epoch,
                    void* stream);
int w4a8_ep_return(const void* y, int64_t y_stride0, int64_t H, const int32_t* src,
                   const int32_t* total_rows, int64_t rows_hint, int64_t tk_max, void* const* peers,
                   int64_t yhome_off, void* stream);
int w4a8_ep_row_addresses(const int32_t* src, const int32_t* total_rows, int64_t cap_rows, int64_t H,
                          int64_t tk_max, void* const* peers, int64_t yhome_off, uint64_t* out_rows, void* stream);

/*
 * Health check of the failure-detection path (no reference counterpart; the
 * reference kernels have no bounded waits).  Launches one small kernel in
 * which a thread waits on an mbarrier that is never completed, with a limit
 * of limit_cycles (0 < limit_cycles <= the production limit of ~2e9
 * cycles), while a second warp waits on another such barrier with the
 * production limit.  The first wait runs out and records status code 120 in
 * the device status word; the second leaves through the kernel's abort flag;
 * the kernel returns.  No TMA, MMA or other asynchronous work is issued.
 * report: int32 [3] device memory: [0] = first wait succeeded (expect 0),
 * [1] = second wait succeeded (expect 0), [2] = kilocycles the second waited.
 * Read the status with w4a8_device_status afterwards.
 */
int w4a8_selftest_wait_timeout(int64_t limit_cycles, int32_t* report, void* stream);

/*
 * Reads (and, if reset != 0, clears) the device status word that the kernels
 * set when a bounded wait expires.  Synchronises `stream`.  0 = healthy.
 */
int w4a8_device_status(int32_t* status_out, int32_t reset, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* W4A8MOE_H_ */
