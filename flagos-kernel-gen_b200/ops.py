"""Host-side mirror of the reference operator, over the C ABI.

``w4a8_group_gemm_moe`` keeps the reference entry point exactly
(docs/Task1.md:8-17): same name, argument order, dtypes, shapes, in-place
``out`` that is also returned, and the same ``AssertionError`` for the two
shape rules the reference asserts (docs/Task1.md:74-75).  Unlike the
reference it never synchronises the host (no ``.item()``,
Task1/v1.6/task1-codex5.5-all-v1.6.py:62-64): expert segments are read on the
device.

The remaining functions are the routed-MoE stages that the reference does not
have (activation quantisation, align, SiLU-mul requant, combine); each is one
C-ABI call on the current CUDA stream.
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple

import torch

from . import _lib


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise RuntimeError("w4a8moe ops run on CUDA tensors only (there is no CPU path)")
    for t in tensors[1:]:
        if t.device != dev:
            raise RuntimeError(f"all tensors must be on {dev}, got {t.device}")
    return dev


def _contig(t: torch.Tensor, dtype: torch.dtype, name: str) -> torch.Tensor:
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    return t if t.is_contiguous() else t.contiguous()


def _gemm_operands(x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, out, group_size):
    M_total, K = x_q.shape
    E, N, K_half = w_q4_packed.shape
    # the reference's own shape rules (docs/Task1.md:74-75)
    assert K_half * 2 == K
    assert K % group_size == 0
    G = K // group_size
    dev = _require_cuda(x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, *([] if out is None else [out]))
    if x_q.dtype != torch.int8:
        raise TypeError(f"x_q must be int8, got {x_q.dtype}")
    if out is not None and out.dtype != torch.bfloat16:
        raise TypeError(f"out must be bfloat16, got {out.dtype}")
    if out is not None and tuple(out.shape) != (M_total, N):
        raise ValueError(f"out must have shape {(M_total, N)}, got {tuple(out.shape)}")
    if tuple(w_scale.shape) != (E, N, G) or tuple(w_zero.shape) != (E, N, G):
        raise ValueError(f"w_scale / w_zero must have shape {(E, N, G)}")
    if tuple(x_scale.shape) != (M_total,) or expert_offsets.numel() != E + 1:
        raise ValueError("x_scale must be [M_total] and expert_offsets [E+1]")
    # rows with unit column stride; the C ABI takes the row stride
    if x_q.stride(1) != 1 or (M_total > 1 and x_q.stride(0) < K) or x_q.data_ptr() % 4 or x_q.stride(0) % 4:
        x_q = x_q.contiguous()
    x_scale = _contig(x_scale, torch.float32, "x_scale")
    w_q4_packed = _contig(w_q4_packed, torch.uint8, "w_q4_packed")
    w_scale = _contig(w_scale, torch.float32, "w_scale")
    w_zero = _contig(w_zero, torch.int8, "w_zero")
    if expert_offsets.dtype != torch.int32:
        expert_offsets = expert_offsets.to(torch.int32)
    expert_offsets = expert_offsets.contiguous()
    return dev, x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, M_total, E, N, K


GEMV_AUTO_ROWS = 4   # AUTO: experts with at most this many rows take the streaming kernel


def gemm_auto_kernels(m_total: int, num_experts: int) -> tuple[str, ...]:
    """Kernels the AUTO dispatch of the library launches for a grouped GEMM of
    ``m_total`` rows over ``num_experts`` experts (the host-side rule of
    ``w4a8_group_gemm_moe_ex``; the per-expert split is then made on the
    device).  Used for launch accounting and roofline labels."""
    if m_total <= GEMV_AUTO_ROWS or m_total <= 2 * num_experts:
        return ("gemm_gemv_kernel",)
    if m_total >= 64 * num_experts:
        return ("gemm_tc_kernel",)
    return ("gemm_gemv_kernel", "gemm_tc_kernel")


def w4a8_group_gemm_moe(
    x_q: torch.Tensor,
    x_scale: torch.Tensor,
    w_q4_packed: torch.Tensor,
    w_scale: torch.Tensor,
    w_zero: torch.Tensor,
    expert_offsets: torch.Tensor,
    out: torch.Tensor,
    group_size: int,
) -> torch.Tensor:
    """W4A8 grouped GEMM over expert segments (drop-in for docs/Task1.md:8-17).

    out[m, n] = bf16(x_scale[m] * sum_g w_scale[e,n,g] * sum_{k in g} x_q[m,k] * int8(nib(e,n,k) - w_zero[e,n,g]))
    for every row m in expert e's segment [expert_offsets[e], expert_offsets[e+1]);
    rows outside every segment are left untouched.  Returns ``out``.
    """
    return w4a8_group_gemm_moe_ex(x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, out,
                                  group_size)


def w4a8_group_gemm_moe_ex(x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, out, group_size,
                           kernel: int = _lib.KERNEL_AUTO, partials: torch.Tensor | None = None,
                           prepacked: bool = False):
    """``w4a8_group_gemm_moe`` with a kernel selector and the optional int32
    per-group partial-sum export ``partials`` (int32 [M_total, N, K/group_size],
    the layout of the reference's einsum; the library writes it group-major,
    [G, M_total, N], and it is transposed into ``partials`` here).
    ``prepacked``: ``w_q4_packed`` is in the layout of ``prepack_weights``."""
    dev, x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, M_total, E, N, K = _gemm_operands(
        x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, out, group_size)
    staging = None
    if partials is not None:
        G = K // group_size
        if partials.dtype != torch.int32 or tuple(partials.shape) != (M_total, N, G) or not partials.is_contiguous():
            raise ValueError(f"partials must be a contiguous int32 tensor of shape {(M_total, N, G)}")
        staging = torch.zeros((G, M_total, N), dtype=torch.int32, device=dev)
    lib = _lib.load()
    fn = lib.w4a8_group_gemm_moe_prepacked if prepacked else lib.w4a8_group_gemm_moe_ex
    rc = fn(
        x_q.data_ptr(), x_q.stride(0) if M_total > 0 else K, x_scale.data_ptr(), w_q4_packed.data_ptr(),
        w_scale.data_ptr(), w_zero.data_ptr(), expert_offsets.data_ptr(), out.data_ptr(), out.stride(0),
        out.stride(1), M_total, E, N, K, group_size, kernel, _ptr(staging), _stream(dev))
    _lib.check(rc, "w4a8_group_gemm_moe")
    if staging is not None:
        partials.copy_(staging.permute(1, 2, 0))
    return out


def prepack_weights(w_q4_packed: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Offline prepack of packed int4 weights (uint8 [..., K/2], contiguous):
    the same nibbles in the word-interleaved layout the grouped GEMMs read
    without byte permutes (``prepacked=True``).  ``out`` may be the input
    (in place)."""
    dev = _require_cuda(w_q4_packed)
    if w_q4_packed.dtype != torch.uint8 or not w_q4_packed.is_contiguous():
        raise TypeError("w_q4_packed must be a contiguous uint8 tensor")
    if out is None:
        out = torch.empty_like(w_q4_packed)
    if out.shape != w_q4_packed.shape or out.dtype != torch.uint8 or not out.is_contiguous():
        raise ValueError("out must be a contiguous uint8 tensor of the input's shape")
    K = w_q4_packed.shape[-1] * 2
    rows = w_q4_packed.numel() // max(w_q4_packed.shape[-1], 1)
    rc = _lib.load().w4a8_prepack_weights(w_q4_packed.data_ptr(), out.data_ptr(), rows, K, _stream(dev))
    _lib.check(rc, "prepack_weights")
    return out


def w4a8_group_gemm_moe_combine(x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, sorted_ids,
                                topk_weights, acc_out, group_size, kernel: int = _lib.KERNEL_AUTO):
    """Grouped GEMM whose epilogue adds ``topk_weights[t, j] * y`` (y the bf16
    row result of ``w4a8_group_gemm_moe``) into ``acc_out[t]`` (fp32 [T, N],
    zero before the batch's first GEMM), t, j from ``sorted_ids`` (flat
    t*topk + j per sorted row, as ``moe_align`` writes it).  Finish with
    ``combine_finish``.  The fp32 additions run in no fixed order."""
    dev, x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, M_total, E, N, K = _gemm_operands(
        x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, None, group_size)
    _require_cuda(x_q, sorted_ids, topk_weights, acc_out)
    T, k = topk_weights.shape
    tw = _contig(topk_weights, torch.float32, "topk_weights")
    if sorted_ids.dtype != torch.int32 or sorted_ids.numel() < M_total:
        raise ValueError("sorted_ids must be int32 with at least one entry per row")
    if acc_out.dtype != torch.float32 or acc_out.dim() != 2 or acc_out.shape[1] != N or acc_out.shape[0] < T \
            or acc_out.stride(1) != 1:
        raise ValueError(f"acc_out must be fp32 [>= {T}, {N}] with unit column stride")
    rc = _lib.load().w4a8_group_gemm_moe_combine(
        x_q.data_ptr(), x_q.stride(0) if M_total > 0 else K, x_scale.data_ptr(), w_q4_packed.data_ptr(),
        w_scale.data_ptr(), w_zero.data_ptr(), expert_offsets.data_ptr(), sorted_ids.data_ptr(), tw.data_ptr(), k,
        acc_out.data_ptr(), acc_out.stride(0), M_total, E, N, K, group_size, kernel, _stream(dev))
    _lib.check(rc, "w4a8_group_gemm_moe_combine")
    return acc_out


def combine_finish(acc: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[t] = bf16(acc[t]) and acc[t] = 0 for t < out.shape[0]."""
    dev = _require_cuda(acc, out)
    T, H = out.shape
    if acc.dtype != torch.float32 or acc.stride(1) != 1 or acc.shape[1] != H or acc.shape[0] < T:
        raise ValueError("acc must be fp32 [>= T, H] with unit column stride")
    if out.dtype != torch.bfloat16 or out.stride(1) != 1:
        raise ValueError("out must be bf16 with unit column stride")
    rc = _lib.load().w4a8_combine_finish(acc.data_ptr(), acc.stride(0), T, H, out.data_ptr(), out.stride(0),
                                         _stream(dev))
    _lib.check(rc, "combine_finish")
    return out


def act_quant(x: torch.Tensor, x_q: torch.Tensor | None = None, x_scale: torch.Tensor | None = None):
    """Per-token int8 quantisation of bf16 ``x`` [T, H] -> (x_q int8 [T, H], x_scale fp32 [T])."""
    dev = _require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be a 2-D bfloat16 tensor")
    if x.stride(1) != 1:
        x = x.contiguous()
    T, H = x.shape
    if x_q is None:
        x_q = torch.empty((T, H), dtype=torch.int8, device=dev)
    if x_scale is None:
        x_scale = torch.empty((T,), dtype=torch.float32, device=dev)
    if x_q.stride(1) != 1 or x_scale.dtype != torch.float32 or not x_scale.is_contiguous():
        raise ValueError("x_q needs unit column stride and x_scale must be contiguous fp32")
    rc = _lib.load().w4a8_act_quant(x.data_ptr(), x.stride(0), T, H, x_q.data_ptr(), x_q.stride(0),
                                    x_scale.data_ptr(), _stream(dev))
    _lib.check(rc, "act_quant")
    return x_q, x_scale


def router_topk(logits: torch.Tensor, topk: int, scoring: str = "softmax", renormalize: bool = True,
                x: torch.Tensor | None = None):
    """Router on the device: scores (``"softmax"`` or ``"sigmoid"`` of fp32
    ``logits`` [T, E]), the ``topk`` experts by score in descending order,
    weights renormalised to sum to 1 -> (ids int32 [T, k], weights fp32 [T, k]).
    With bf16 ``x`` [T, H] the same launch also quantises every token row as
    ``act_quant`` does and returns (ids, weights, x_q, x_scale).  Ranking is
    by logit (the scores' order), ties to the lower expert index."""
    dev = _require_cuda(logits)
    if logits.dtype != torch.float32 or logits.dim() != 2:
        raise TypeError("logits must be a 2-D float32 tensor")
    if scoring not in ("softmax", "sigmoid"):
        raise ValueError("scoring must be 'softmax' or 'sigmoid'")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    T, E = logits.shape
    ids = torch.empty((T, topk), dtype=torch.int32, device=dev)
    w = torch.empty((T, topk), dtype=torch.float32, device=dev)
    xq = xs = None
    xp, xstride, H, qp, qstride, sp = None, 0, 0, None, 0, None
    if x is not None:
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[0] != T or x.device != dev:
            raise TypeError("x must be a bfloat16 [T, H] tensor on the logits' device")
        if x.stride(1) != 1:
            x = x.contiguous()
        H = x.shape[1]
        xq = torch.empty((T, H), dtype=torch.int8, device=dev)
        xs = torch.empty((T,), dtype=torch.float32, device=dev)
        xp, xstride, qp, qstride, sp = x.data_ptr(), x.stride(0), xq.data_ptr(), xq.stride(0), xs.data_ptr()
    rc = _lib.load().w4a8_router_topk(logits.data_ptr(), logits.stride(0), T, E, topk,
                                      0 if scoring == "softmax" else 1, 1 if renormalize else 0,
                                      ids.data_ptr(), w.data_ptr(), xp, xstride, H, qp, qstride, sp, _stream(dev))
    _lib.check(rc, "router_topk")
    return (ids, w) if x is None else (ids, w, xq, xs)


class AlignResult(NamedTuple):
    expert_offsets: torch.Tensor   # int32 [E+1]
    sorted_ids: torch.Tensor       # int32 [R]
    inv_pos: torch.Tensor          # int32 [R]
    padded_ids: torch.Tensor       # int32 [R + E*(bs-1)]
    block_expert: torch.Tensor     # int32 [ceil(cap/bs)]
    num_post_pad: torch.Tensor     # int32 [1]


def align_capacity(R: int, E: int, block_size: int) -> tuple[int, int]:
    cap = R + E * (block_size - 1)
    return cap, (cap + block_size - 1) // block_size


def moe_align(topk_ids: torch.Tensor, num_experts: int, block_size: int = 128,
              workspace: torch.Tensor | None = None) -> AlignResult:
    """Counting-sort of (token, slot) pairs by expert; see include/w4a8moe.h."""
    dev = _require_cuda(topk_ids)
    if topk_ids.dim() != 2:
        raise ValueError("topk_ids must be [T, topk]")
    if topk_ids.dtype != torch.int32:
        topk_ids = topk_ids.to(torch.int32)
    topk_ids = topk_ids.contiguous()
    T, k = topk_ids.shape
    R = T * k
    E = int(num_experts)
    lib = _lib.load()
    need = lib.w4a8_moe_align_workspace_size(T, k, E)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty((max(need, 4),), dtype=torch.uint8, device=dev)
    cap, nblk = align_capacity(R, E, block_size)
    off = torch.empty((E + 1,), dtype=torch.int32, device=dev)
    sorted_ids = torch.empty((R,), dtype=torch.int32, device=dev)
    inv_pos = torch.empty((R,), dtype=torch.int32, device=dev)
    padded = torch.empty((cap,), dtype=torch.int32, device=dev)
    blk = torch.empty((nblk,), dtype=torch.int32, device=dev)
    npp = torch.empty((1,), dtype=torch.int32, device=dev)
    rc = lib.w4a8_moe_align(topk_ids.data_ptr(), T, k, E, block_size, off.data_ptr(), sorted_ids.data_ptr(),
                            inv_pos.data_ptr(), padded.data_ptr(), blk.data_ptr(), npp.data_ptr(),
                            workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream(dev))
    _lib.check(rc, "moe_align")
    return AlignResult(off, sorted_ids, inv_pos, padded, blk, npp)


def quant_scatter(x: torch.Tensor, inv_pos: torch.Tensor, topk: int, x_sorted: torch.Tensor | None = None,
                  xs_sorted: torch.Tensor | None = None):
    """Quantise each token once and write it to its ``topk`` expert-sorted rows."""
    dev = _require_cuda(x, inv_pos)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be a 2-D bfloat16 tensor")
    if x.stride(1) != 1:
        x = x.contiguous()
    T, H = x.shape
    R = T * topk
    if x_sorted is None:
        x_sorted = torch.empty((R, H), dtype=torch.int8, device=dev)
    if xs_sorted is None:
        xs_sorted = torch.empty((R,), dtype=torch.float32, device=dev)
    if not x_sorted.is_contiguous() or tuple(x_sorted.shape[1:]) != (H,) or x_sorted.shape[0] < R:
        raise ValueError("x_sorted must be a contiguous int8 tensor [>= T*topk, H]")
    rc = _lib.load().w4a8_quant_scatter(x.data_ptr(), x.stride(0), T, H, inv_pos.data_ptr(), topk,
                                        x_sorted.data_ptr(), xs_sorted.data_ptr(), _stream(dev))
    _lib.check(rc, "quant_scatter")
    return x_sorted, xs_sorted


def silu_mul_requant(h: torch.Tensor, q: torch.Tensor | None = None, s: torch.Tensor | None = None):
    """h bf16 [R, 2I] -> (int8 [R, I], fp32 [R]) with y = silu(h[:, :I]) * h[:, I:]."""
    dev = _require_cuda(h)
    if h.dtype != torch.bfloat16 or h.dim() != 2 or h.shape[1] % 2:
        raise TypeError("h must be a 2-D bfloat16 tensor with an even number of columns")
    if h.stride(1) != 1:
        h = h.contiguous()
    R, I2 = h.shape
    I = I2 // 2
    if q is None:
        q = torch.empty((R, I), dtype=torch.int8, device=dev)
    if s is None:
        s = torch.empty((R,), dtype=torch.float32, device=dev)
    rc = _lib.load().w4a8_silu_mul_requant(h.data_ptr(), h.stride(0), R, I, q.data_ptr(), s.data_ptr(),
                                           _stream(dev))
    _lib.check(rc, "silu_mul_requant")
    return q, s


def moe_combine(y: torch.Tensor, inv_pos: torch.Tensor, topk_weights: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = bf16(sum_j topk_weights[t, j] * y[inv_pos[t*topk + j]])  (fp32, j ascending)."""
    dev = _require_cuda(y, inv_pos, topk_weights)
    T, k = topk_weights.shape
    H = y.shape[1]
    if y.stride(1) != 1:
        y = y.contiguous()
    tw = _contig(topk_weights, torch.float32, "topk_weights")
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    if out.stride(1) != 1:
        raise ValueError("out needs unit column stride")
    rc = _lib.load().w4a8_moe_combine(y.data_ptr(), y.stride(0), inv_pos.data_ptr(), tw.data_ptr(), T, k, H,
                                      out.data_ptr(), out.stride(0), _stream(dev))
    _lib.check(rc, "moe_combine")
    return out


def gather_rows(src: torch.Tensor, index: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[i] = src[index[i]] for a 1-D or 2-D tensor (rows with index < 0 untouched)."""
    dev = _require_cuda(src, index)
    if index.dtype != torch.int32:
        raise TypeError("index must be int32")
    index = index.contiguous()
    s2 = src if src.dim() == 2 else src.view(-1, 1)
    if s2.stride(1) != 1:
        s2 = s2.contiguous()
    rows = index.numel()
    if out is None:
        out = torch.empty((rows,) + tuple(src.shape[1:]), dtype=src.dtype, device=dev)
    o2 = out if out.dim() == 2 else out.view(-1, 1)
    if o2.stride(1) != 1 or o2.dtype != src.dtype or o2.shape[1] != s2.shape[1]:
        raise ValueError("out must match src's row layout")
    es = src.element_size()
    rc = _lib.load().w4a8_gather_rows(s2.data_ptr(), s2.stride(0) * es, index.data_ptr(), rows, s2.shape[1] * es,
                                      o2.data_ptr(), o2.stride(0) * es, _stream(dev))
    _lib.check(rc, "gather_rows")
    return out


def device_status(reset: bool = True, device: torch.device | None = None) -> int:
    """Reads (and clears) the device status word; synchronises the current stream."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    v = ctypes.c_int32(0)
    rc = _lib.load().w4a8_device_status(ctypes.byref(v), 1 if reset else 0, _stream(dev))
    _lib.check(rc, "device_status")
    return int(v.value)
