"""Routed W4A8 MoE layer built on the reference operator.

The reference has only the grouped GEMM over pre-grouped rows
(docs/Task1.md:8-17).  A routed layer adds the stages around it; every stage
is one CUDA kernel of this library, and nothing synchronises the host:

  1. moe_align        topk_ids [T, k] -> expert_offsets, sorted order, inverse
  2. quant_scatter    x bf16 [T, H] -> int8 rows in expert-sorted order + scales
  3. grouped GEMM     gate/up:  [R, H] x W13[E, 2I, H] -> h bf16 [R, 2I]
  4. silu_mul_requant h -> int8 [R, I] + per-row scale
  5. grouped GEMM     down:     [R, I] x W2[E, H, I] -> y bf16 [R, H]
  6. moe_combine      out[t] = bf16(sum_j w[t, j] * y[pos(t, j)])

(R = T * k.)  For the single-GEMM form (no down projection) steps 4-5 are
skipped and the combine runs on the gate/up output.

``MoELayer`` keeps all intermediates in preallocated buffers sized for a
maximum token count, so a step allocates nothing and can be replayed from a
CUDA graph.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from . import ops


@dataclass
class W4A8Weights:
    """One projection: packed int4 [E, N, K/2] + scale / zero [E, N, K/gs]."""
    packed: torch.Tensor
    scale: torch.Tensor
    zero: torch.Tensor

    @property
    def shape(self):
        E, N, Kh = self.packed.shape
        return E, N, 2 * Kh


class _Ev:
    """Optional CUDA-event bracketing of a stage (no-op when events is None)."""

    def __init__(self, events):
        self.events = events
        self.cur = None

    def start(self, name):
        if self.events is not None:
            s = torch.cuda.Event(enable_timing=True)
            s.record()
            self.cur = (name, s)

    def stop(self):
        if self.events is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.events.append((self.cur[0], self.cur[1], e))


class MoELayer:
    """Routed W4A8 MoE (gate/up -> SiLU-mul -> down, or a single up GEMM)."""

    def __init__(self, w13: W4A8Weights, w2: W4A8Weights | None, group_size: int, topk: int,
                 max_tokens: int, align_block: int = 128, fused_combine: bool = False,
                 prepack: bool = False):
        """``fused_combine``: the last grouped GEMM adds its weighted rows into
        an fp32 token accumulator in its epilogue (``w4a8_group_gemm_moe_combine``)
        instead of writing [R, H] bf16 rows for a separate combine; the fp32
        additions then run in no fixed order (results may differ from the
        unfused, j-ascending combine in the last fp32 bit).
        ``prepack``: the layer keeps a copy of the weights in the prepacked
        nibble layout (``ops.prepack_weights``) and runs its GEMMs on it
        (same results)."""
        if prepack and fused_combine:
            raise ValueError("prepack and fused_combine are not combined")
        self.fused_combine = fused_combine
        self.prepacked = prepack
        if prepack:
            w13 = W4A8Weights(ops.prepack_weights(w13.packed), w13.scale, w13.zero)
            if w2 is not None:
                w2 = W4A8Weights(ops.prepack_weights(w2.packed), w2.scale, w2.zero)
        self.w13, self.w2 = w13, w2
        self.gs, self.topk = group_size, topk
        E, N13, H = w13.shape
        self.E, self.H = E, H
        self.ffn = w2 is not None
        self.I = N13 // 2 if self.ffn else N13
        if self.ffn:
            E2, H2, I2 = w2.shape
            if E2 != E or H2 != H or I2 != self.I:
                raise ValueError("w2 must be [E, H, I] for w13 [E, 2I, H]")
        self.align_block = align_block
        self.device = w13.packed.device
        self._alloc(max_tokens)

    def _alloc(self, max_tokens: int):
        dev, E, H, I, k = self.device, self.E, self.H, self.I, self.topk
        self.max_tokens = max_tokens
        R = max_tokens * k
        lib = _lib.load()
        ws_bytes = max(int(lib.w4a8_moe_align_workspace_size(max_tokens, k, E)), 4)
        self.ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.offsets = torch.empty((E + 1,), **i32)
        self.sorted_ids = torch.empty((R,), **i32)
        self.inv_pos = torch.empty((R,), **i32)
        self.xq = torch.empty((R, H), dtype=torch.int8, device=dev)
        self.xs = torch.empty((R,), dtype=torch.float32, device=dev)
        n13 = 2 * I if self.ffn else I
        self.h = torch.empty((R, n13), dtype=torch.bfloat16, device=dev)
        if self.ffn:
            self.aq = torch.empty((R, I), dtype=torch.int8, device=dev)
            self.as_ = torch.empty((R,), dtype=torch.float32, device=dev)
            if not self.fused_combine:
                self.y = torch.empty((R, H), dtype=torch.bfloat16, device=dev)
        width = H if self.ffn else I
        self.out = torch.empty((max_tokens, width), dtype=torch.bfloat16, device=dev)
        # fused combine: fp32 token accumulator, zero between batches (the
        # finishing kernel clears the rows it converts)
        self.acc = torch.zeros((max_tokens, width), dtype=torch.float32, device=dev) if self.fused_combine else None

    # number of library kernel launches per forward (for launch accounting)
    def launches_per_forward(self, tokens: int | None = None) -> int:
        # align: 3, quant_scatter: 1, each grouped GEMM: 1 or 2 (AUTO dispatch),
        # silu: (1), combine: 1
        R = (tokens if tokens is not None else self.max_tokens) * self.topk
        g = len(ops.gemm_auto_kernels(R, self.E))
        return 3 + 1 + g + ((1 + g) if self.ffn else 0) + 1

    def forward(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                out: torch.Tensor | None = None, events: list | None = None) -> torch.Tensor:
        """Routed forward.  ``events``: optional list; when given, (name, start,
        end) CUDA-event pairs recorded on the current stream around each stage
        (align, quant_scatter, gemm_gate_up, silu_mul_requant, gemm_down,
        combine) are appended to it (used for per-stage timing)."""
        T, H = x.shape
        if T > self.max_tokens:
            self._alloc(T)
        k = self.topk
        if H != self.H or tuple(topk_ids.shape) != (T, k):
            raise ValueError("x must be [T, H] and topk_ids [T, topk]")
        R = T * k
        dev = x.device
        lib = _lib.load()
        stream = torch.cuda.current_stream(dev).cuda_stream
        ev = _Ev(events)
        ev.start("align")
        ids = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
        ids = ids.contiguous()
        rc = lib.w4a8_moe_align(ids.data_ptr(), T, k, self.E, self.align_block, self.offsets.data_ptr(),
                                self.sorted_ids.data_ptr(), self.inv_pos.data_ptr(), None, None, None,
                                self.ws.data_ptr(),
                                self.ws.numel(), stream)
        _lib.check(rc, "moe_align")
        ev.stop()
        xq, xs = self.xq[:R], self.xs[:R]
        ev.start("quant_scatter")
        ops.quant_scatter(x, self.inv_pos[:R], k, xq, xs)
        ev.stop()
        if out is None:
            out = self.out[:T]
        fuse = self.fused_combine
        tw = topk_weights if topk_weights.dtype == torch.float32 else topk_weights.float()
        tw = tw.contiguous()
        h = self.h[:R]
        ev.start("gemm_gate_up")
        if fuse and not self.ffn:
            ops.w4a8_group_gemm_moe_combine(xq, xs, self.w13.packed, self.w13.scale, self.w13.zero, self.offsets,
                                            self.sorted_ids, tw, self.acc, self.gs)
        else:
            ops.w4a8_group_gemm_moe_ex(xq, xs, self.w13.packed, self.w13.scale, self.w13.zero, self.offsets, h,
                                       self.gs, prepacked=self.prepacked)
        ev.stop()
        y = h
        if self.ffn:
            aq, as_ = self.aq[:R], self.as_[:R]
            ev.start("silu_mul_requant")
            ops.silu_mul_requant(h, aq, as_)
            ev.stop()
            ev.start("gemm_down")
            if fuse:
                ops.w4a8_group_gemm_moe_combine(aq, as_, self.w2.packed, self.w2.scale, self.w2.zero, self.offsets,
                                                self.sorted_ids, tw, self.acc, self.gs)
            else:
                y = self.y[:R]
                ops.w4a8_group_gemm_moe_ex(aq, as_, self.w2.packed, self.w2.scale, self.w2.zero, self.offsets, y,
                                           self.gs, prepacked=self.prepacked)
            ev.stop()
        ev.start("combine")
        if fuse:
            out = ops.combine_finish(self.acc, out)
        else:
            out = ops.moe_combine(y, self.inv_pos[:R], tw, out)
        ev.stop()
        return out

    __call__ = forward


class HostPipeline:
    """Serves batches that live in (pinned) host memory through a layer with
    the host<->device copies overlapped with compute.

    ``submit(x, topk_ids, topk_weights, out)`` queues one batch: its inputs
    are copied to the device on one side stream, the layer runs on the
    caller's current stream, and its output is copied back into ``out`` on a
    second side stream, so batch i+1's inputs and batch i-1's output move
    while batch i computes.  Every batch's copies still happen in full; only
    their placement in time changes.  ``depth`` device slots are recycled
    (a slot is refilled only after its previous batch has consumed its inputs
    and sent its output).  ``flush()`` makes the current stream wait until
    every submitted output has reached host memory.  Works with any layer
    whose forward is ``layer(x, topk_ids, topk_weights, out=...)``."""

    def __init__(self, layer, device=None, depth: int = 2):
        self.layer = layer
        self.depth = depth
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.copy_in = torch.cuda.Stream(self.dev)
        self.copy_out = torch.cuda.Stream(self.dev)
        self.slots = None
        self.n = 0

    def _alloc(self, x, ids, w, out):
        def dev_like(t):
            return torch.empty(t.shape, dtype=t.dtype, device=self.dev)
        self.slots = [dict(x=dev_like(x), ids=dev_like(ids), w=dev_like(w), out=dev_like(out),
                           loaded=torch.cuda.Event(), computed=torch.cuda.Event(), sent=torch.cuda.Event())
                      for _ in range(self.depth)]

    def submit(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
               out: torch.Tensor) -> None:
        if self.slots is None or x.shape[0] > self.slots[0]["x"].shape[0]:
            if self.slots is not None:
                self.flush()
            self._alloc(x, topk_ids, topk_weights, out)
            self.n = 0
        T = x.shape[0]
        s = self.slots[self.n % self.depth]
        compute = torch.cuda.current_stream(self.dev)
        if self.n < self.depth:
            self.copy_in.wait_stream(compute)        # nothing earlier used this slot
        else:
            self.copy_in.wait_event(s["computed"])   # the slot's previous batch consumed its inputs
        with torch.cuda.stream(self.copy_in):
            s["x"][:T].copy_(x, non_blocking=True)
            s["ids"][:T].copy_(topk_ids, non_blocking=True)
            s["w"][:T].copy_(topk_weights, non_blocking=True)
            s["loaded"].record(self.copy_in)
        compute.wait_event(s["loaded"])
        if self.n >= self.depth:
            compute.wait_event(s["sent"])            # the slot's previous output left the device
        o = self.layer(s["x"][:T], s["ids"][:T], s["w"][:T], out=s["out"][:T])
        s["computed"].record(compute)
        self.copy_out.wait_event(s["computed"])
        with torch.cuda.stream(self.copy_out):
            out.copy_(o, non_blocking=True)
            s["sent"].record(self.copy_out)
        if o.data_ptr() != s["out"].data_ptr():      # a layer that returns its own buffer
            o.record_stream(self.copy_out)
        self.n += 1

    def flush(self) -> None:
        torch.cuda.current_stream(self.dev).wait_stream(self.copy_out)


def w4a8_moe(x, topk_ids, topk_weights, w13: W4A8Weights, w2: W4A8Weights | None, group_size: int):
    """One-shot routed MoE forward (allocates its buffers; use MoELayer in a loop)."""
    layer = MoELayer(w13, w2, group_size, topk_ids.shape[1], x.shape[0])
    return layer(x, topk_ids, topk_weights).clone()
