"""Expert-parallel (EP) W4A8 MoE over one process per GPU.

Two transports with the same results (bit for bit):

* ``P2PExpertParallelMoE`` (the product on B200): the token rows travel over
  NVLink peer memory, written by this package's own kernels -- a counts
  exchange, a fused quantise + dispatch that stores each token's int8 rows
  straight into the owning rank's expert-sorted receive buffer, the local
  grouped GEMMs on that buffer, a return of the result rows into the home
  rank's slot buffer, and a local combine.  Waits on peers are bounded
  device-side barriers; there is no host synchronisation and no NCCL call on
  the data path, so a forward can be queued behind the previous one.
* ``ExpertParallelMoE`` (NCCL all-to-all, described below): the baseline
  transport, and the one whose host logic the gloo tests run on CPU with the
  oracle as its device backend.

Experts are sharded evenly: rank r owns experts [r*E/P, (r+1)*E/P).  The NCCL
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


class P2PExpertParallelMoE:
    """Routed W4A8 MoE with experts sharded over the ranks of ``group``, the
    token rows moved over NVLink peer memory by this package's kernels.

    One receive buffer per rank of one layout (torch symmetric memory, so
    every rank can store into every other's): flags, counts matrix, int8
    rows / scales / return addresses of the tokens it serves, and the bf16
    results of its own slots.  Its row capacity is world x max_tokens x topk
    (a rank may serve every slot of every rank), so no routing can overflow
    it.  Per forward, on every rank: align by global expert, exchange the
    per-expert row counts, dispatch, barrier, gate/up GEMM -> SiLU-mul
    requant -> down GEMM on the receive buffer, return, barrier, combine.
    With ``fused_return`` (default) the last GEMM returns every result row
    to its sender's slot buffer over NVLink itself (a row-address table
    built on the device after the dispatch; the GEMM's transform warpgroup
    copies each finished tile's rows while later tiles run) instead of a
    separate return pass: 14.56 against 14.72 ms per step at 2 GPUs, 14.25
    against 15.55 at 8.  With ``dedup_dispatch`` (default) a token's int8 row
    crosses to each remote rank once, however many of its experts that rank
    owns; the owner copies it into the other slots' rows after the barrier.
    """

    def __init__(self, w13_local: W4A8Weights, w2_local: W4A8Weights | None, num_experts: int, group_size: int,
                 topk: int, max_tokens: int, group=None, fused_return: bool = True, dedup_dispatch: bool = True):
        import torch.distributed._symmetric_memory as symm_mem
        from . import _lib
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not shard evenly over {self.world} ranks")
        self.E = num_experts
        self.epr = num_experts // self.world
        if w13_local.packed.shape[0] != self.epr:
            raise ValueError("w13_local must hold this rank's E/P experts")
        self.w13, self.w2 = w13_local, w2_local
        self.gs, self.topk = group_size, topk
        self.ffn = w2_local is not None
        _, n13, H = w13_local.shape
        self.H, self.n13 = H, n13
        self.I = n13 // 2 if self.ffn else n13
        self.width = H if self.ffn else n13     # columns of a result row
        dev = w13_local.packed.device
        self.device = dev
        self.max_tokens = max_tokens
        self.fused_return = fused_return
        self.dedup = dedup_dispatch
        self.tk_max = max_tokens * topk
        self.cap = self.world * self.tk_max
        lib = _lib.load()
        self._lib = lib

        def rup(n):
            return (n + 255) // 256 * 256
        off = 0
        self.flags_off = off
        off += rup(4 * self.world)
        self.counts_off = off
        off += rup(4 * self.world * self.E)
        self.xq_off = off
        off += rup(self.cap * H)
        self.xs_off = off
        off += rup(4 * self.cap)
        self.src_off = off
        off += rup(4 * self.cap)
        self.yhome_off = off
        off += rup(2 * self.tk_max * self.width)
        self.dup_off = off
        off += rup(4 * self.cap)
        self.buf_bytes = off
        if hasattr(symm_mem, "enable_symm_mem_for_group"):
            try:
                symm_mem.enable_symm_mem_for_group(self.group.group_name)
            except Exception:  # noqa: BLE001  (already enabled, or not needed by this torch)
                pass
        self.buf = symm_mem.empty(self.buf_bytes, dtype=torch.uint8, device=dev)
        self.hdl = symm_mem.rendezvous(self.buf, self.group)
        self.peers = torch.tensor([int(p) for p in self.hdl.buffer_ptrs], dtype=torch.int64, device=dev)
        self.buf[: self.counts_off].zero_()              # flags start at epoch 0
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)
        self.epoch = 0
        b = self.buf
        self.xq = b[self.xq_off:self.xq_off + self.cap * H].view(self.cap, H).view(torch.int8)
        self.xs = b[self.xs_off:self.xs_off + 4 * self.cap].view(torch.float32)
        self.src = b[self.src_off:self.src_off + 4 * self.cap].view(torch.int32)
        self.yhome = b[self.yhome_off:self.yhome_off + 2 * self.tk_max * self.width].view(torch.bfloat16).view(
            self.tk_max, self.width)
        i32 = dict(dtype=torch.int32, device=dev)
        ws_bytes = max(int(lib.w4a8_moe_align_workspace_size(max_tokens, topk, self.E)), 4)
        self.ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
        self.off_g = torch.empty((self.E + 1,), **i32)
        self.sorted = torch.empty((self.tk_max,), **i32)
        self.inv = torch.empty((self.tk_max,), **i32)
        self.dest_base = torch.empty((self.E,), **i32)
        self.local_off = torch.empty((self.epr + 1,), **i32)
        self.home_pos = torch.empty((self.tk_max,), **i32)
        self.h = torch.empty((self.cap, n13), dtype=torch.bfloat16, device=dev)
        if self.ffn:
            self.aq = torch.empty((self.cap, self.I), dtype=torch.int8, device=dev)
            self.as_ = torch.empty((self.cap,), dtype=torch.float32, device=dev)
            self.y = torch.empty((self.cap, H), dtype=torch.bfloat16, device=dev)
        if fused_return:
            self.row_addr = torch.empty((self.cap,), dtype=torch.int64, device=dev)   # uint64 addresses
        self.out = torch.empty((max_tokens, self.width), dtype=torch.bfloat16, device=dev)
        self._last_gemm_launches = 0

    @property
    def local(self):
        return self

    @property
    def offsets(self):
        """Segments of this rank's experts in its receive buffer (last forward)."""
        return self.local_off

    @property
    def n_recv(self) -> int:
        """Rows this rank served in the last forward (reads the device)."""
        return int(self.local_off[self.epr].item())

    def launches_per_forward(self, tokens: int | None = None) -> int:
        R = (tokens if tokens is not None else self.max_tokens) * self.topk
        g = len(cuda_ops.gemm_auto_kernels(R, self.epr))
        # align 3, exchange, dispatch, barrier, (replicate), GEMMs, (SiLU, GEMMs), return, barrier, combine
        return 3 + 3 + int(self.dedup) + g + ((1 + g) if self.ffn else 0) + 3

    def _next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def forward(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, out=None,
                events: list | None = None) -> torch.Tensor:
        from . import _lib
        lib = self._lib
        T, H = x.shape
        k = self.topk
        if T > self.max_tokens or H != self.H or tuple(topk_ids.shape) != (T, k):
            raise ValueError(f"x must be [T <= {self.max_tokens}, {self.H}] and topk_ids [T, {k}]")
        if x.dtype != torch.bfloat16 or x.stride(1) != 1:
            x = x.to(torch.bfloat16).contiguous()
        st = torch.cuda.current_stream(x.device).cuda_stream
        ids = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
        ids = ids.contiguous()
        tw = topk_weights if topk_weights.dtype == torch.float32 else topk_weights.float()
        tw = tw.contiguous()
        R = T * k
        peers = self.peers.data_ptr()
        ev = _events(events)
        ev.start("dispatch_prep")
        _lib.check(lib.w4a8_moe_align(ids.data_ptr(), T, k, self.E, 128, self.off_g.data_ptr(), self.sorted.data_ptr(),
                                      self.inv.data_ptr(), None, None, None, self.ws.data_ptr(), self.ws.numel(), st),
                   "moe_align")
        ev.stop()
        ev.start("a2a_counts")
        _lib.check(lib.w4a8_ep_exchange(self.off_g.data_ptr(), self.E, self.world, self.rank, peers, self.counts_off,
                                        self.flags_off, self._next_epoch(), self.cap, self.dest_base.data_ptr(),
                                        self.local_off.data_ptr(), st), "ep_exchange")
        ev.stop()
        ev.start("a2a_dispatch")
        if self.dedup:
            _lib.check(lib.w4a8_ep_dispatch_dedup(x.data_ptr(), x.stride(0), T, H, ids.data_ptr(), k, self.E,
                                                  self.world, self.rank, self.tk_max, self.off_g.data_ptr(),
                                                  self.inv.data_ptr(), self.dest_base.data_ptr(), peers, self.xq_off,
                                                  self.xs_off, self.src_off, self.dup_off, self.home_pos.data_ptr(),
                                                  st), "ep_dispatch_dedup")
        else:
            _lib.check(lib.w4a8_ep_dispatch(x.data_ptr(), x.stride(0), T, H, ids.data_ptr(), k, self.E, self.world,
                                            self.rank, self.tk_max, self.off_g.data_ptr(), self.inv.data_ptr(),
                                            self.dest_base.data_ptr(), peers, self.xq_off, self.xs_off, self.src_off,
                                            self.home_pos.data_ptr(), st), "ep_dispatch")
        _lib.check(lib.w4a8_ep_barrier(peers, self.flags_off, self.world, self.rank, self._next_epoch(), st),
                   "ep_barrier")
        # rows this rank serves are counted on the device; the kernels' choice
        # assumes the average, R (every rank routes R slots)
        rows_hint = min(R, self.cap)
        total = self.local_off.data_ptr() + 4 * self.epr
        if self.dedup:
            _lib.check(lib.w4a8_ep_replicate(self.buf.data_ptr(), self.xq_off, self.dup_off, H, total, rows_hint, st),
                       "ep_replicate")
        if self.fused_return:
            _lib.check(lib.w4a8_ep_row_addresses(self.src.data_ptr(), total, self.cap, self.width, self.tk_max, peers,
                                                 self.yhome_off, self.row_addr.data_ptr(), st), "ep_row_addresses")
        ev.stop()
        w = self.w13
        ev.start("gemm_gate_up")
        if self.fused_return and not self.ffn:
            _lib.check(lib.w4a8_group_gemm_moe_rows(self.xq.data_ptr(), H, self.xs.data_ptr(), w.packed.data_ptr(),
                                                    w.scale.data_ptr(), w.zero.data_ptr(), self.local_off.data_ptr(),
                                                    self.h.data_ptr(), self.row_addr.data_ptr(), self.cap, self.epr,
                                                    self.n13, H, self.gs, rows_hint, st), "w4a8_group_gemm_moe_rows")
        else:
            _lib.check(lib.w4a8_group_gemm_moe_hint(self.xq.data_ptr(), H, self.xs.data_ptr(), w.packed.data_ptr(),
                                                    w.scale.data_ptr(), w.zero.data_ptr(), self.local_off.data_ptr(),
                                                    self.h.data_ptr(), self.n13, 1, self.cap, self.epr, self.n13, H,
                                                    self.gs, rows_hint, st), "w4a8_group_gemm_moe")
        ev.stop()
        res = self.h
        if self.ffn:
            ev.start("silu_mul_requant")
            _lib.check(lib.w4a8_silu_mul_requant_rows(self.h.data_ptr(), self.n13, self.cap, self.I,
                                                      self.aq.data_ptr(), self.as_.data_ptr(), total, st),
                       "silu_mul_requant")
            ev.stop()
            w = self.w2
            ev.start("gemm_down")
            if self.fused_return:
                _lib.check(lib.w4a8_group_gemm_moe_rows(self.aq.data_ptr(), self.I, self.as_.data_ptr(),
                                                        w.packed.data_ptr(), w.scale.data_ptr(), w.zero.data_ptr(),
                                                        self.local_off.data_ptr(), self.y.data_ptr(),
                                                        self.row_addr.data_ptr(), self.cap, self.epr, H, self.I,
                                                        self.gs, rows_hint, st),
                           "w4a8_group_gemm_moe_rows")
            else:
                _lib.check(lib.w4a8_group_gemm_moe_hint(self.aq.data_ptr(), self.I, self.as_.data_ptr(),
                                                        w.packed.data_ptr(), w.scale.data_ptr(), w.zero.data_ptr(),
                                                        self.local_off.data_ptr(), self.y.data_ptr(), H, 1, self.cap,
                                                        self.epr, H, self.I, self.gs, rows_hint, st),
                           "w4a8_group_gemm_moe")
                res = self.y
            ev.stop()
        ev.start("a2a_combine")
        if not self.fused_return:
            _lib.check(lib.w4a8_ep_return(res.data_ptr(), res.stride(0), self.width, self.src.data_ptr(), total,
                                          rows_hint, self.tk_max, peers, self.yhome_off, st), "ep_return")
        _lib.check(lib.w4a8_ep_barrier(peers, self.flags_off, self.world, self.rank, self._next_epoch(), st),
                   "ep_barrier")
        ev.stop()
        if out is None:
            out = self.out[:T]
        ev.start("combine")
        out = cuda_ops.moe_combine(self.yhome, self.home_pos[:R], tw, out)
        ev.stop()
        self._last_gemm_launches = len(cuda_ops.gemm_auto_kernels(rows_hint, self.epr)) * (2 if self.ffn else 1)
        return out

    __call__ = forward

    @classmethod
    def with_synthetic_weights(cls, cfg, T, rank, world, dev, gen, fused_return: bool = True,
                               dedup_dispatch: bool = True):
        from . import workloads as W
        epr = cfg.experts // world
        n13 = 2 * cfg.inter if cfg.ffn else cfg.inter
        w13 = W4A8Weights(*W.make_int4_weights(epr, n13, cfg.hidden, cfg.group_size, gen, dev))
        w2 = W4A8Weights(*W.make_int4_weights(epr, cfg.hidden, cfg.inter, cfg.group_size, gen, dev)) \
            if cfg.ffn else None
        return cls(w13, w2, cfg.experts, cfg.group_size, cfg.topk, T, fused_return=fused_return,
                   dedup_dispatch=dedup_dispatch)
