"""Expert-parallel (EP) W4A8 MoE over one process per GPU.

Experts are sharded evenly: rank r owns experts [r*E/P, (r+1)*E/P).  One
forward does, per rank (P = world size, R = T*k routed slots):

  1. dest = topk_ids // (E/P); align the R slots by destination rank
     (the same counting-sort kernel as the expert align, with P "experts")
  2. quantise each token once and write it to its slots in destination order
  3. counts all-to-all (P ints), then NCCL all-to-all of the int8 rows, their
     fp32 scales and their local expert ids
  4. align the received rows by local expert, permute them into expert order
  5. local grouped GEMMs (gate/up -> SiLU-mul requant -> down)
  6. permute the outputs back to arrival order, NCCL all-to-all them home
  7. weighted top-k combine in token order

The split sizes of the all-to-all are read on the host (one small
device-to-host copy per forward), as NCCL's all_to_all_single needs them.
The fabric is NVSwitch, so the exchange is one flat all-to-all.  No TMA
multicast is used anywhere on this path.

The device work goes through an ``ops`` backend (the CUDA library by
default); a CPU backend built from the oracle lets the same host logic run on
gloo ranks in tests.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops as cuda_ops
from .moe import W4A8Weights


class CudaEPOps:
    """Device stages of the EP forward, all in this package's CUDA library."""

    def align(self, ids: torch.Tensor, n: int):
        al = cuda_ops.moe_align(ids, n)
        return al.expert_offsets, al.sorted_ids, al.inv_pos

    def quant_scatter(self, x, inv_pos, k):
        return cuda_ops.quant_scatter(x, inv_pos, k)

    def gather_rows(self, src, index):
        return cuda_ops.gather_rows(src, index)

    def grouped_gemm(self, xq, xs, w: W4A8Weights, offsets, out, gs):
        self.gemm_launches += len(cuda_ops.gemm_auto_kernels(xq.shape[0], w.packed.shape[0]))
        return cuda_ops.w4a8_group_gemm_moe(xq, xs, w.packed, w.scale, w.zero, offsets, out, gs)

    def silu_mul_requant(self, h):
        return cuda_ops.silu_mul_requant(h)

    def combine(self, y, inv_pos, topk_w):
        return cuda_ops.moe_combine(y, inv_pos, topk_w)

    # launches of this package's kernels per forward besides the grouped GEMMs:
    # align x2 (3 each), quant_scatter, 3 row gathers (rows, scales, outputs),
    # SiLU-mul requant, combine; the GEMMs (1 or 2 launches each, AUTO dispatch)
    # are counted as they are issued
    fixed_launches_per_forward = 6 + 1 + 3 + 1 + 1
    gemm_launches = 0


class ExpertParallelMoE:
    """Routed W4A8 MoE with experts sharded over the ranks of ``group``."""

    def __init__(self, w13_local: W4A8Weights, w2_local: W4A8Weights | None, num_experts: int, group_size: int,
                 topk: int, group=None, ops=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not shard evenly over {self.world} ranks")
        self.E = num_experts
        self.epr = num_experts // self.world
        if w13_local.packed.shape[0] != self.epr:
            raise ValueError("w13_local must hold this rank's E/P experts")
        self.w13, self.w2 = w13_local, w2_local
        self.gs, self.topk = group_size, topk
        self._last_gemm_launches = 0
        self.ops = ops if ops is not None else CudaEPOps()
        self.offsets = None          # last local expert offsets (for reporting)
        self.out = w13_local.packed.new_empty((0,))

    # -- helpers ---------------------------------------------------------------
    def launches_per_forward(self) -> int:
        """Library launches of the last forward (0 for a backend that is not the CUDA library)."""
        return getattr(self.ops, "fixed_launches_per_forward", 0) + self._last_gemm_launches

    @property
    def local(self):
        return self

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        return out

    # -- forward ---------------------------------------------------------------
    def forward(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, out=None,
                events: list | None = None) -> torch.Tensor:
        T, H = x.shape
        k = self.topk
        dev = x.device
        ops = self.ops
        g0 = getattr(ops, "gemm_launches", 0)
        ev = _events(events)
        ev.start("dispatch_prep")
        ids = topk_ids.to(torch.int32)
        # 1. destination rank of every slot; ids outside [0, E) are dropped (-1)
        dest = torch.where((ids >= 0) & (ids < self.E), ids // self.epr, torch.full_like(ids, -1))
        send_off, send_sorted, send_inv = ops.align(dest, self.world)
        # 2. quantise once, rows in destination order
        xq_send, xs_send = ops.quant_scatter(x, send_inv, k)
        lid_send = (ids.reshape(-1)[send_sorted.long()] % self.epr).to(torch.int32)
        ev.stop()
        # 3. exchange counts, then rows / scales / local expert ids
        ev.start("a2a_counts")
        send_counts = (send_off[1:] - send_off[:-1]).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        counts = torch.stack([send_counts, recv_counts]).cpu()
        in_splits = counts[0].tolist()
        out_splits = counts[1].tolist()
        n_send = sum(in_splits)
        n_recv = sum(out_splits)
        xq_recv = torch.empty((n_recv, H), dtype=torch.int8, device=dev)
        xs_recv = torch.empty((n_recv,), dtype=torch.float32, device=dev)
        lid_recv = torch.empty((n_recv,), dtype=torch.int32, device=dev)
        ev.stop()
        ev.start("a2a_dispatch")
        self._a2a(xq_recv, xq_send[:n_send], out_splits, in_splits)
        self._a2a(xs_recv, xs_send[:n_send], out_splits, in_splits)
        self._a2a(lid_recv, lid_send[:n_send], out_splits, in_splits)
        ev.stop()
        # 4. local expert order
        ev.start("local_align_gather")
        loc_off, loc_sorted, loc_inv = ops.align(lid_recv.view(-1, 1), self.epr)
        self.offsets = loc_off
        xq_loc = ops.gather_rows(xq_recv, loc_sorted)
        xs_loc = ops.gather_rows(xs_recv, loc_sorted)
        # 5. local grouped GEMMs
        n13 = self.w13.packed.shape[1]
        h = torch.empty((n_recv, n13), dtype=torch.bfloat16, device=dev)
        ev.stop()
        ev.start("gemm_gate_up")
        ops.grouped_gemm(xq_loc, xs_loc, self.w13, loc_off, h, self.gs)
        ev.stop()
        if self.w2 is not None:
            ev.start("silu_mul_requant")
            aq, as_ = ops.silu_mul_requant(h)
            ev.stop()
            y_loc = torch.empty((n_recv, H), dtype=torch.bfloat16, device=dev)
            ev.start("gemm_down")
            ops.grouped_gemm(aq, as_, self.w2, loc_off, y_loc, self.gs)
            ev.stop()
        else:
            y_loc = h
        # 6. back to arrival order, then home
        ev.start("gather_back")
        y_recv = ops.gather_rows(y_loc, loc_inv)
        y_home = torch.empty((n_send, y_loc.shape[1]), dtype=torch.bfloat16, device=dev)
        ev.stop()
        ev.start("a2a_combine")
        self._a2a(y_home, y_recv, in_splits, out_splits)
        ev.stop()
        # 7. combine in token order
        ev.start("combine")
        y_full = y_home
        if n_send < T * k:   # dropped slots have inv = -1 and are never read
            y_full = torch.empty((T * k, y_home.shape[1]), dtype=torch.bfloat16, device=dev)
            y_full[:n_send] = y_home
        self.out = ops.combine(y_full, send_inv, topk_weights)
        ev.stop()
        self.n_recv = n_recv
        self._last_gemm_launches = getattr(ops, "gemm_launches", 0) - g0
        return self.out

    __call__ = forward

    # -- construction for benchmarks --------------------------------------------
    @classmethod
    def with_synthetic_weights(cls, cfg, T, rank, world, dev, gen):
        from . import workloads as W
        epr = cfg.experts // world
        n13 = 2 * cfg.inter if cfg.ffn else cfg.inter
        w13 = W4A8Weights(*W.make_int4_weights(epr, n13, cfg.hidden, cfg.group_size, gen, dev))
        w2 = W4A8Weights(*W.make_int4_weights(epr, cfg.hidden, cfg.inter, cfg.group_size, gen, dev)) \
            if cfg.ffn else None
        return cls(w13, w2, cfg.experts, cfg.group_size, cfg.topk)


class _events:
    def __init__(self, events):
        self.events = events

    def start(self, name):
        if self.events is not None:
            self.s = torch.cuda.Event(enable_timing=True)
            self.s.record()
            self.name = name

    def stop(self):
        if self.events is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.events.append((self.name, self.s, e))
