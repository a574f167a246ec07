#!/usr/bin/env python
"""Benchmark of the W4A8 MoE layer (grouped GEMM hot path) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload deepseek_ep] [--tokens T]

One "step" is one routed MoE layer forward over one batch of synthetic tokens:
align -> quantise+dispatch -> gate/up grouped GEMM -> SiLU-mul requant ->
down grouped GEMM -> combine (and, for N > 1, the expert-parallel NCCL
all-to-all dispatch and combine).  Default workload: the DeepSeek-V3-shaped
layer (hidden 7168, moe intermediate 2048, 256 experts, top-8, group 128) at
16384 tokens per GPU, i.e. the per-GPU shape of the expert-parallel
configuration; at N = 1 all 256 experts are local.

Prints ONE JSON line on rank 0.  `value` is whole-job tokens/s (device time,
max over ranks), `e2e` the same through host buffers (pinned H2D of every
step's tokens and routing, D2H of its output, through the package's
HostPipeline, which overlaps each step's copies with its neighbours'
compute), `roofline` describes the
dominant kernel (the gate/up grouped GEMM), `cpu_baseline` the reference
algorithm restated on the CPU (oracle/, torch CPU, all host threads) timed on
a bounded sample of the same workload.

--impl reference times that CPU restatement alone (rank 0; other ranks exit 0).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import re
import statistics
import subprocess
import sys
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
PKG_NAME = "flagos-kernel-gen_b200"
METRIC = "MoE layer tokens/s"


def load_peaks() -> dict:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return dict(hbm_gbs=float(d["hbm_gbs"]), bf16_tflops=float(d["bf16_tflops"]),
                    bf16_tflops_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), src="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, src="fallback")


def parse_workload(name: str, tokens: int | None):
    W = importlib.import_module(PKG_NAME).workloads
    m = re.fullmatch(r"([a-z0-9_]+?)(?:_T(\d+))?", name)
    base, t = m.group(1), m.group(2)
    ep = False
    if base.endswith("_ep"):
        base, ep = base[:-3], True
    cfg = W.CONFIGS[base]
    T = tokens or (int(t) if t else (16384 if ep else 8192))
    return cfg, T


def traffic_from_profiles(workload: str, kernel: str):
    """Per-launch DRAM bytes of `kernel` on `workload` from the committed ncu
    summaries (line format: `traffic_per_launch <workload> <kernel> <bytes>`)."""
    d = os.path.join(REPO, "profiles")
    if not os.path.isdir(d):
        return None
    for f in sorted(os.listdir(d)):
        if not f.endswith((".md", ".txt")):
            continue
        for line in open(os.path.join(d, f), encoding="utf-8"):
            parts = line.strip().strip("`").split()
            if len(parts) == 4 and parts[0] == "traffic_per_launch" and parts[1] == workload and parts[2] == kernel:
                return float(parts[3])
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ["clocks.sm", "clocks.max.sm", "clocks_event_reasons.hw_slowdown",
              "clocks_event_reasons.hw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown",
              "clocks_event_reasons.sw_power_cap"]

    def __init__(self, device_index: int):
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={','.join(self.FIELDS)}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", ident], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            p = [x.strip() for x in line.split(",")]
            if len(p) != 6:
                continue
            try:
                sm.append(float(p[0]))
                smax = max(smax, float(p[1]))
            except ValueError:
                continue
            for n, v in zip(names, p[2:]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU legs (oracle)
def cpu_sample_step(O, cfg, inp, off, experts, T):
    """One CPU pass of the reference algorithm over the routed rows of `experts`
    (full per-expert work: unpack, per-group fp32 einsum, scales, SiLU-mul
    requant, down projection).  Returns (seconds, rows)."""
    rows = 0
    t0 = time.perf_counter()
    for e in experts:
        m0, m1 = int(off[e]), int(off[e + 1])
        if m1 <= m0:
            continue
        rows += m1 - m0
        xq, xs = inp["xq"][m0:m1], inp["xs"][m0:m1]
        sub = torch.tensor([0, m1 - m0], dtype=torch.int32)
        w13 = [t[e:e + 1] for t in inp["w13"]]
        h = O.group_gemm(xq, xs, *w13, sub, torch.empty((m1 - m0, w13[0].shape[1]), dtype=torch.bfloat16),
                         cfg.group_size)
        if inp["w2"] is not None:
            aq, as_ = O.silu_mul_requant(h)
            w2 = [t[e:e + 1] for t in inp["w2"]]
            O.group_gemm(torch.from_numpy(aq), torch.from_numpy(as_), *w2, sub,
                         torch.empty((m1 - m0, w2[0].shape[1]), dtype=torch.bfloat16), cfg.group_size)
    return time.perf_counter() - t0, rows


def cpu_inputs(cfg, T, seed=0):
    """CPU copies of the workload for the oracle legs: routing and quantised,
    expert-sorted rows come from the CPU restatements; weights only for the
    experts a sample touches are materialised (generated per expert)."""
    from oracle import w4a8_oracle as O
    W = importlib.import_module(PKG_NAME).workloads
    inp = W.make_moe_inputs(cfg, T, seed=seed, weights=False)
    al = O.moe_align(inp.topk_ids, cfg.experts, 128)
    xq_tok, xs_tok = O.act_quant(inp.x)
    src = al["sorted_ids"] // cfg.topk
    return O, dict(xq=torch.from_numpy(xq_tok[src]), xs=torch.from_numpy(xs_tok[src])), al["expert_offsets"]


def cpu_weights_for(cfg, experts, seed=1):
    W = importlib.import_module(PKG_NAME).workloads
    g = W.make_generator(seed)
    n13 = 2 * cfg.inter if cfg.ffn else cfg.inter
    w13 = [[], [], []]
    w2 = [[], [], []]
    for _ in experts:
        for i, t in enumerate(W.make_int4_weights(1, n13, cfg.hidden, cfg.group_size, g)):
            w13[i].append(t)
        if cfg.ffn:
            for i, t in enumerate(W.make_int4_weights(1, cfg.hidden, cfg.inter, cfg.group_size, g)):
                w2[i].append(t)
    cat = lambda L: [torch.cat(x, 0) for x in L]  # noqa: E731
    return cat(w13), (cat(w2) if cfg.ffn else None)


def run_cpu_leg(cfg, T, steps, warmup, budget_s):
    """Times the CPU restatement: each step processes whole experts (the
    busiest first) within a per-step time budget, the same sample every step.
    Returns the measured step time, the sampled rows and the tokens/s the
    sample stands for (tokens x sampled rows / routed rows, per second)."""
    torch.set_num_threads(os.cpu_count() or 1)
    O, inp, off = cpu_inputs(cfg, T)
    counts = off[1:] - off[:-1]
    order = [int(e) for e in sorted(range(cfg.experts), key=lambda e: -int(counts[e])) if counts[e] > 0]
    R = int(off[-1])
    # calibrate with one expert
    w13, w2 = cpu_weights_for(cfg, order[:1])
    inp1 = dict(inp, w13=w13, w2=w2)
    off1 = torch.tensor([0, int(counts[order[0]])], dtype=torch.int64)
    inp1["xq"] = inp["xq"][int(off[order[0]]):int(off[order[0] + 1])]
    inp1["xs"] = inp["xs"][int(off[order[0]]):int(off[order[0] + 1])]
    t1 = min(cpu_sample_step(O, cfg, inp1, off1, [0], T)[0] for _ in range(2))   # the first call is cold
    n_exp = max(1, min(len(order), int(budget_s / max(t1, 1e-3))))
    sample = order[:n_exp]
    w13, w2 = cpu_weights_for(cfg, sample)
    # re-index the sample's rows contiguously
    xq = torch.cat([inp["xq"][int(off[e]):int(off[e + 1])] for e in sample])
    xs = torch.cat([inp["xs"][int(off[e]):int(off[e + 1])] for e in sample])
    c = torch.tensor([int(counts[e]) for e in sample])
    soff = torch.cat([torch.zeros(1, dtype=torch.int64), torch.cumsum(c, 0)])
    sinp = dict(xq=xq, xs=xs, w13=w13, w2=w2)
    times, rows = [], 0
    for i in range(warmup + steps):
        dt, rows = cpu_sample_step(O, cfg, sinp, soff, list(range(len(sample))), T)
        if i >= warmup:
            times.append(dt)
    t = statistics.median(times)
    tok_s = T * (rows / R) / t
    return {"value": tok_s, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(sample)} of {int((counts > 0).sum())} active experts ({rows} of {R} routed rows, "
                      f"busiest first), full gate/up + SiLU-mul requant + down per expert, median of {steps} "
                      f"step(s); tokens/s = tokens x sampled rows / routed rows per second",
            "seconds_per_step": t, "seconds_timed": sum(times), "sample_rows": rows, "routed_rows": R,
            "scale_factor": R / rows, "steps_timed": len(times)}


def cpu_full_step(cfg, T, seed=0):
    """One whole layer step of the CPU restatement (every routed row of every
    active expert), for workloads small enough to run in full: (seconds,
    tokens/s).  Weights are generated for the active experts only (the
    restatement never reads the others; the reference unpacks all E experts'
    weights every call, docs/Task1.md:78-85, so its own step costs more)."""
    torch.set_num_threads(os.cpu_count() or 1)
    from oracle import w4a8_oracle as O
    W = importlib.import_module(PKG_NAME).workloads
    inp = W.make_moe_inputs(cfg, T, seed=seed, weights=False)
    ids = inp.topk_ids.to(torch.int64)
    used = torch.unique(ids)
    remap = torch.full((cfg.experts,), -1, dtype=torch.int64)
    remap[used] = torch.arange(used.numel())
    ids_c = remap[ids].to(torch.int32)
    w13, w2 = cpu_weights_for(cfg, used.tolist())
    t0 = time.perf_counter()
    O.moe_layer(inp.x, ids_c, inp.topk_weights, w13, w2, cfg.group_size)
    dt = time.perf_counter() - t0
    return dt, T / dt


# ----------------------------------------------------------------------------- GPU leg
def build_layer(pkg, cfg, T, rank, world, dev, transport="p2p", fused_combine=False, prepack=False):
    W = pkg.workloads
    gen = W.make_generator(1000 + rank, dev)
    if world == 1:
        n13 = 2 * cfg.inter if cfg.ffn else cfg.inter
        w13 = pkg.W4A8Weights(*W.make_int4_weights(cfg.experts, n13, cfg.hidden, cfg.group_size, gen, dev))
        w2 = pkg.W4A8Weights(*W.make_int4_weights(cfg.experts, cfg.hidden, cfg.inter, cfg.group_size, gen, dev)) \
            if cfg.ffn else None
        return pkg.MoELayer(w13, w2, cfg.group_size, cfg.topk, T, fused_combine=fused_combine, prepack=prepack)
    ep = importlib.import_module(PKG_NAME + ".ep")
    if transport == "nccl":
        return ep.ExpertParallelMoE.with_synthetic_weights(cfg, T, rank, world, dev, gen)
    return ep.P2PExpertParallelMoE.with_synthetic_weights(cfg, T, rank, world, dev, gen,
                                                           fused_return=(transport != "p2p_return_pass"),
                                                           dedup_dispatch=(transport != "p2p_plain_dispatch"))


def kernel_bench(pkg, spec: str, steps: int, warmup: int, kernel: int):
    """Kernel-only mode: one grouped GEMM launch per step on the 8-argument
    operator (E experts x M rows each, N x K weights, group 128), e.g.
    ``--workload gemm_E32_M256_N4096_K7168``.  Used for ncu captures."""
    m = re.fullmatch(r"gemm_E(\d+)_M(\d+)_N(\d+)_K(\d+)(?:_G(\d+))?", spec)
    E, M, N, K = (int(m.group(i)) for i in range(1, 5))
    gs = int(m.group(5) or 128)
    W = pkg.workloads
    dev = torch.device("cuda", 0)
    gen = W.make_generator(0, dev)
    w, ws, wz = W.make_int4_weights(E, N, K, gs, gen, dev)
    R = E * M
    x_q = torch.randint(-127, 128, (R, K), generator=gen, device=dev, dtype=torch.int8)
    xs = torch.empty((R,), device=dev).uniform_(0.001, 0.05, generator=gen)
    off = torch.arange(0, R + 1, M, device=dev, dtype=torch.int32)
    out = torch.empty((R, N), dtype=torch.bfloat16, device=dev)
    for _ in range(warmup):
        pkg.w4a8_group_gemm_moe_ex(x_q, xs, w, ws, wz, off, out, gs, kernel=kernel)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        pkg.w4a8_group_gemm_moe_ex(x_q, xs, w, ws, wz, off, out, gs, kernel=kernel)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    peaks = load_peaks()
    byts = W.gemm_roofline_bytes(E, R, N, K, gs)
    ops_ = W.gemm_ops(R, N, K)
    print(json.dumps({"metric": "grouped GEMM rows/s", "value": R / (ms * 1e-3), "unit": "rows/s",
                      "ms_per_launch": ms, "workload": spec, "kernel": kernel, "steps": steps,
                      "hbm_frac": byts / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                      "int8_frac": ops_ / (ms * 1e-3) / 1e12 / (2 * peaks["bf16_tflops"]),
                      "GBps": byts / (ms * 1e-3) / 1e9, "TOPS": ops_ / (ms * 1e-3) / 1e12,
                      "device_status": pkg.device_status()}), flush=True)


# ----------------------------------------------------------------------------- parity checks
def parity_single(pkg, layer, cfg, x, ids, tw, dev):
    """Checks the benchmark's own layer on its own inputs before timing (the
    oracle only as the checker): sampled tokens of the whole layer against the
    oracle layer, and the int32 partials of the busiest expert's gate/up and
    down rows bit for bit (the tensor-core kernel in the configuration the
    layer's launch uses, whose bf16 rows must equal the layer's own)."""
    from oracle import w4a8_oracle as O
    t0 = time.perf_counter()
    out = layer(x, ids, tw).clone()
    torch.cuda.synchronize()
    T = x.shape[0]
    tokens = sorted({0, T // 2, T - 1})
    ref = O.moe_layer_tokens(x, ids, tw, (layer.w13.packed, layer.w13.scale, layer.w13.zero),
                             (layer.w2.packed, layer.w2.scale, layer.w2.zero) if layer.w2 is not None else None,
                             cfg.group_size, tokens)
    o = out[torch.tensor(tokens, device=dev)].cpu().float()
    r = ref.float()
    width = o.shape[1]
    elem_ok = bool(((o - r).abs() <= 0.016 * r.abs() + 1e-4 * width).all())
    mean_norm = float((o - r).abs().mean() / r.abs().mean().clamp_min(1e-30))
    checks = {"layer_tokens": {"tokens": tokens, "elementwise_ok": elem_ok, "mean_err_norm": mean_norm,
                               "ok": elem_ok and mean_norm <= 1e-3}}
    off = layer.offsets.cpu()
    counts = off[1:] - off[:-1]
    e = int(torch.argmax(counts))
    m0, m1 = int(off[e]), int(off[e + 1])
    idx = torch.tensor([e], device=dev)
    sub_off = torch.tensor([0, m1 - m0], dtype=torch.int32, device=dev)
    stages = [("gate_up", layer.xq, layer.xs, layer.w13, layer.h)]
    if layer.w2 is not None:
        stages.append(("down", layer.aq, layer.as_, layer.w2, layer.y))
    for name, xq, xs, w, layer_out in stages:
        wp, ws, wz = (t.index_select(0, idx).contiguous() for t in (w.packed, w.scale, w.zero))
        N, K = wp.shape[1], 2 * wp.shape[2]
        G = K // cfg.group_size
        sub_out = torch.empty((m1 - m0, N), dtype=torch.bfloat16, device=dev)
        parts = torch.empty((m1 - m0, N, G), dtype=torch.int32, device=dev)
        pkg.w4a8_group_gemm_moe_ex(xq[m0:m1], xs[m0:m1], wp, ws, wz, sub_off, sub_out, cfg.group_size,
                                   kernel=pkg.KERNEL_TC, partials=parts)
        torch.cuda.synchronize()
        same_as_layer = bool(torch.equal(sub_out.view(torch.int16), layer_out[m0:m1].view(torch.int16)))
        ref_p = O.group_partials(xq[m0:m1].cpu().numpy(), O.signed_weights(wp[0].cpu(), wz[0].cpu(),
                                                                           cfg.group_size), cfg.group_size)
        exact = bool((parts.cpu().numpy() == ref_p).all())
        checks[f"{name}_partials"] = {"expert": e, "rows": m1 - m0, "bit_exact": exact,
                                      "bf16_rows_equal_layer_launch": same_as_layer, "ok": exact and same_as_layer}
        del parts, ref_p
    torch.cuda.empty_cache()
    ok = all(c["ok"] for c in checks.values()) and pkg.device_status() == 0
    return {"ok": ok, "kind": "oracle (sampled tokens + one expert's exact partials)", "checks": checks,
            "seconds": time.perf_counter() - t0}


def parity_ep(pkg, layer, cfg, rank, world, dev, tokens_per_rank=64):
    """Expert parallelism: every rank's EP output on a small batch equals, bit
    for bit, a single-GPU layer over all ranks' tokens with the union of the
    ranks' expert shards (regenerated from the ranks' weight seeds)."""
    W = pkg.workloads
    t0 = time.perf_counter()
    toks = [W.make_moe_inputs(cfg, tokens_per_rank, seed=900 + r, device=dev, weights=False) for r in range(world)]
    mine = toks[rank]
    out = layer(mine.x, mine.topk_ids, mine.topk_weights).clone()
    torch.cuda.synchronize()
    parts13, parts2 = [], []
    for r in range(world):
        gen = W.make_generator(1000 + r, dev)
        epr = cfg.experts // world
        n13 = 2 * cfg.inter if cfg.ffn else cfg.inter
        parts13.append(W.make_int4_weights(epr, n13, cfg.hidden, cfg.group_size, gen, dev))
        if cfg.ffn:
            parts2.append(W.make_int4_weights(epr, cfg.hidden, cfg.inter, cfg.group_size, gen, dev))
    w13 = pkg.W4A8Weights(*[torch.cat([p[i] for p in parts13]) for i in range(3)])
    w2 = pkg.W4A8Weights(*[torch.cat([p[i] for p in parts2]) for i in range(3)]) if cfg.ffn else None
    del parts13, parts2
    single = pkg.MoELayer(w13, w2, cfg.group_size, cfg.topk, tokens_per_rank * world)
    ref = single(torch.cat([t.x for t in toks]), torch.cat([t.topk_ids for t in toks]),
                 torch.cat([t.topk_weights for t in toks]))
    ref = ref[rank * tokens_per_rank:(rank + 1) * tokens_per_rank]
    same = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
    del single, w13, w2, ref
    torch.cuda.empty_cache()
    flag = torch.tensor([1 if same else 0], device=dev)
    torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
    ok = bool(flag.item()) and pkg.device_status() == 0
    return {"ok": ok, "kind": f"EP output bit-exact against a single-GPU layer ({tokens_per_rank} tokens per "
                              f"rank, every rank checked)", "seconds": time.perf_counter() - t0}


# ----------------------------------------------------------------------------- timing helpers
def timed_steps(layer, x, ids, tw, steps, world):
    """Device time of `steps` forwards (max over ranks) and the mean per-stage
    times of rank-local CUDA events."""
    events = []
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        layer(x, ids, tw, events=events)
    t1.record()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    stages = {}
    for name, s, e in events:
        stages.setdefault(name, []).append(s.elapsed_time(e))
    stages = {k: statistics.mean(v) for k, v in stages.items()}
    if world > 1:
        tt = torch.tensor([ms], device=x.device)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        ms = float(tt.item())
    return ms, stages


def gemm_fracs(W, peaks, counts, cfg, gu_ms, dn_ms):
    """Roofline fractions of the gate/up and down GEMMs of one layer step."""
    active = int((counts > 0).sum())
    R = int(counts.sum())
    n13 = 2 * cfg.inter if cfg.ffn else cfg.inter
    int8_peak = 2.0 * peaks["bf16_tflops"]
    gu_b = W.gemm_roofline_bytes(active, R, n13, cfg.hidden, cfg.group_size)
    gu_o = W.gemm_ops(R, n13, cfg.hidden)
    d = {"active_experts": active, "routed_rows": R, "gate_up_ms": gu_ms,
         "gate_up_hbm_frac": gu_b / (gu_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
         "gate_up_int8_frac": gu_o / (gu_ms * 1e-3) / 1e12 / int8_peak}
    if dn_ms is not None:
        dn_b = W.gemm_roofline_bytes(active, R, cfg.hidden, cfg.inter, cfg.group_size)
        dn_o = W.gemm_ops(R, cfg.hidden, cfg.inter)
        d.update({"down_ms": dn_ms, "down_hbm_frac": dn_b / (dn_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                  "down_int8_frac": dn_o / (dn_ms * 1e-3) / 1e12 / int8_peak,
                  "both_hbm_frac": (gu_b + dn_b) / ((gu_ms + dn_ms) * 1e-3) / 1e9 / peaks["hbm_gbs"],
                  "both_int8_frac": (gu_o + dn_o) / ((gu_ms + dn_ms) * 1e-3) / 1e12 / int8_peak})
    return d


def north_star_targets(pkg, layer, cfg, dev, steps, peaks):
    """The two target points of the DeepSeek-V3 config, timed on the benchmark
    layer's own weights: T = 16 (weight-streaming bound; target >= 0.70 of
    HBM) and T = 8192 (tensor bound; target >= 0.60 of dense int8)."""
    W = pkg.workloads
    out = {}
    for T in (16, 8192):
        inp = W.make_moe_inputs(cfg, T, seed=11, device=dev, weights=False)
        for _ in range(3):
            layer(inp.x, inp.topk_ids, inp.topk_weights)
        ms, st = timed_steps(layer, inp.x, inp.topk_ids, inp.topk_weights, steps, 1)
        off = layer.offsets.cpu()
        d = gemm_fracs(W, peaks, (off[1:] - off[:-1]), cfg, st["gemm_gate_up"], st.get("gemm_down"))
        d.update({"tokens": T, "layer_ms": ms, "layer_tokens_per_s": T / (ms * 1e-3),
                  "kernels": list(pkg.ops.gemm_auto_kernels(T * cfg.topk, cfg.experts))})
        out[f"T{T}"] = d
    out["T16_hbm_frac"] = out["T16"]["both_hbm_frac"]
    out["T8192_int8_frac"] = out["T8192"]["both_int8_frac"]
    out["note"] = ("GEMM time over both projections (gate/up + down), CUDA events per launch inside timed layer "
                   "steps; HBM peak = hbm_gbs, int8 peak = 2 x bf16_tflops (burst) of MEASURED_PEAKS.json")
    return out


def router_stage(pkg, cfg, T, dev, steps, peaks):
    """The router + top-k kernel fused with the token quantisation, at the
    layer's token count: CUDA-event time per launch, HBM fraction of its
    algorithmic bytes (logits and bf16 rows in; int8 rows, scales, ids and
    weights out), and its expert ids against the oracle on sampled tokens."""
    from oracle import w4a8_oracle as O
    W = pkg.workloads
    g = W.make_generator(5, dev)
    logits = torch.randn((T, cfg.experts), generator=g, device=dev, dtype=torch.float32)
    x = torch.randn((T, cfg.hidden), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    for _ in range(3):
        pkg.router_topk(logits, cfg.topk, cfg.scoring, x=x)
    evs = []
    for _ in range(max(steps, 5)):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        res = pkg.router_topk(logits, cfg.topk, cfg.scoring, x=x)
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)
    byts = T * cfg.experts * 4 + T * cfg.hidden * 2 + T * cfg.hidden + T * 4 + T * cfg.topk * 8
    rows = torch.linspace(0, T - 1, steps=min(T, 64)).long()
    ids_o, _ = O.route_topk(logits[rows].cpu(), cfg.topk, cfg.scoring)
    return {"kernel": "router_quant_kernel", "tokens": T, "ms_per_launch": ms,
            "hbm_frac": byts / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "algorithmic_bytes": byts,
            "ids_match_oracle": bool((res[0][rows].cpu().numpy() == ids_o).all())}


def routing_variant(pkg, layer, cfg, T, rank, world, dev, steps):
    """The other routing of the same layer (Zipf(1.2) popularity for a uniform
    workload, uniform for a Zipf one): tokens/s (max over ranks) and the load
    skew it causes (rows per rank under EP, rows per expert on one GPU)."""
    import dataclasses
    W = pkg.workloads
    zipf = 0.0 if cfg.zipf else 1.2
    vcfg = dataclasses.replace(cfg, zipf=zipf, name=cfg.name + ("_uniform" if cfg.zipf else "_zipf"))
    inp = W.make_moe_inputs(vcfg, T, seed=7 + rank, device=dev, weights=False)
    for _ in range(3):
        layer(inp.x, inp.topk_ids, inp.topk_weights)
    ms, _ = timed_steps(layer, inp.x, inp.topk_ids, inp.topk_weights, steps, world)
    d = {"routing": f"{cfg.scoring}" + (f"+zipf{zipf}" if zipf else " uniform"), "value": world * T / (ms * 1e-3),
         "unit": "tokens/s", "ms_per_step": ms}
    if world > 1:
        rows = torch.tensor([float(layer.n_recv)], device=dev)
        allr = [torch.zeros_like(rows) for _ in range(world)]
        torch.distributed.all_gather(allr, rows)
        per_rank = [int(t.item()) for t in allr]
        d.update({"rows_per_rank": per_rank, "load_skew": max(per_rank) / (sum(per_rank) / world)})
    else:
        off = layer.offsets.cpu()
        c = (off[1:] - off[:-1]).float()
        d.update({"max_rows_per_expert": int(c.max()), "load_skew": float(c.max() / c[c > 0].mean())})
    return d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="deepseek_ep")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the parity check, the target points and the routing variant")
    ap.add_argument("--cpu-budget", type=float, default=6.0, help="seconds of CPU work per baseline step")
    ap.add_argument("--kernel", type=int, default=0, help="kernel-only mode: 0 auto, 1 tensor core, 2 CUDA core")
    ap.add_argument("--prepack", action="store_true",
                    help="single GPU: the layer's weights in the prepacked nibble layout (w4a8_prepack_weights)")
    ap.add_argument("--fused-combine", action="store_true",
                    help="single GPU: top-k combine fused into the down GEMM's epilogue (fp32 atomics)")
    ap.add_argument("--ep-transport", default="p2p", choices=["p2p", "p2p_return_pass", "p2p_plain_dispatch", "nccl"],
                    help="expert-parallel transport for N > 1: peer-memory kernels (default) or NCCL all-to-all")
    args = ap.parse_args()
    if args.workload.startswith("gemm_"):
        kernel_bench(importlib.import_module(PKG_NAME), args.workload, args.steps, args.warmup, args.kernel)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    cfg, T = parse_workload(args.workload, args.tokens)
    config = {"workload": args.workload, "tokens_per_gpu": T, "hidden": cfg.hidden, "moe_inter": cfg.inter,
              "experts": cfg.experts, "topk": cfg.topk, "group_size": cfg.group_size,
              "routing": f"{cfg.scoring}" + (f"+zipf{cfg.zipf}" if cfg.zipf else " uniform"),
              "parallelism": f"ep{world} ({args.ep_transport})" if world > 1 else "single", "l2": "inputs larger than L2 "
              "(expert weights are GBs; no flush needed)"}
    if args.prepack and world == 1:
        config["weights"] = "prepacked nibble layout"
    if args.fused_combine and world == 1:
        config["combine"] = "fused into the down GEMM epilogue (fp32 atomics)"

    if args.impl == "reference":
        if rank != 0:
            return
        # every requested step is run and timed; each is the same bounded
        # sample of the workload, sized so the whole run stays within minutes
        budget = min(args.cpu_budget, 150.0 / max(1, args.steps + args.warmup))
        cb = run_cpu_leg(cfg, T, args.steps, args.warmup, budget_s=budget)
        full = {}
        if cfg.name.startswith("deepseek"):
            dt, tps = cpu_full_step(importlib.import_module(PKG_NAME).workloads.CONFIGS["deepseek"], 16)
            full["deepseek_T16"] = {"seconds": dt, "tokens_per_s": tps}
        dt, tps = cpu_full_step(importlib.import_module(PKG_NAME).workloads.CONFIGS["small"], 64)
        full["small_T64"] = {"seconds": dt, "tokens_per_s": tps}
        line = {"metric": METRIC, "value": cb["value"], "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * cb["seconds_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8 x int4 -> int32/fp32 -> bf16",
                "data": "synthetic (seeded; BASELINE.json distributions)", "config": config, "impl": "reference",
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "sample": {k: cb[k] for k in ("seconds_timed", "steps_timed", "sample_rows", "routed_rows",
                                              "scale_factor", "seconds_per_step")},
                "full_steps": full,
                "note": "each step is the same sample of the workload (whole experts, busiest first); ms_per_step "
                        "is the measured time of that sample and value = tokens x sampled rows / routed rows per "
                        "second.  Reference algorithm (docs/Task1.md:53-114 + FFN glue) restated in oracle/, torch "
                        "CPU; the reference tree itself is Python and is not present on the GPU box"}
        print(json.dumps(line), flush=True)
        return

    pkg = importlib.import_module(PKG_NAME)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    W = pkg.workloads
    layer = build_layer(pkg, cfg, T, rank, world, dev, args.ep_transport, args.fused_combine, args.prepack)
    inp = W.make_moe_inputs(cfg, T, seed=7 + rank, device=dev, weights=False)
    x, ids, tw = inp.x, inp.topk_ids, inp.topk_weights

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    parity = None
    if not args.no_extras:
        parity = parity_single(pkg, layer, cfg, x, ids, tw, dev) if world == 1 else \
            parity_ep(pkg, layer, cfg, rank, world, dev)

    for _ in range(args.warmup):
        layer(x, ids, tw)
    barrier()
    if pkg.device_status() != 0:
        raise RuntimeError("device status error after warm-up")

    # ---- device-timed steps (inputs resident in HBM)
    sampler = ClockSampler(local_rank)
    time.sleep(0.2)
    ms, stages = timed_steps(layer, x, ids, tw, args.steps, world)
    clocks = sampler.stop()

    # ---- end to end through the public API with host buffers
    x_h = x.cpu().pin_memory()
    ids_h = ids.cpu().pin_memory()
    tw_h = tw.cpu().pin_memory()
    out_h = torch.empty((T, cfg.hidden if cfg.ffn else cfg.inter), dtype=torch.bfloat16).pin_memory()
    # the package's host pipeline: each step's H2D and D2H run on side streams,
    # overlapped with the neighbouring steps' compute
    pipe = pkg.HostPipeline(layer, dev)

    def e2e_step():
        pipe.submit(x_h, ids_h, tw_h, out_h)

    for _ in range(2):
        e2e_step()
    pipe.flush()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    pipe.flush()
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    h2d = x.numel() * 2 + ids.numel() * 4 + tw.numel() * 4
    d2h = out_h.numel() * 2
    status = pkg.device_status()

    # ---- roofline of the dominant kernel (gate/up grouped GEMM), from the
    # first timed region (the e2e steps ran the same routing)
    peaks = load_peaks()
    off = layer.offsets.cpu() if world == 1 else layer.local.offsets.cpu()
    counts = (off[1:] - off[:-1])
    active = int((counts > 0).sum())
    R = int(off[-1])
    n13 = 2 * cfg.inter if cfg.ffn else cfg.inter
    gu_bytes = W.gemm_roofline_bytes(active, R, n13, cfg.hidden, cfg.group_size)
    gu_ops = W.gemm_ops(R, n13, cfg.hidden)
    gu_ms = stages["gemm_gate_up"]
    # kernels of the gate/up launch under the AUTO dispatch; with both, the
    # streaming kernel takes the experts with <= 4 rows and the tensor-core
    # kernel the rest, and the one holding most of the rows dominates
    kernels = pkg.ops.gemm_auto_kernels(R, int(counts.numel()))
    if len(kernels) == 2:
        small_rows = int(counts[counts <= pkg.ops.GEMV_AUTO_ROWS].sum())
        kernels = kernels if small_rows * 2 >= R else kernels[::-1]
    dominant = kernels[0]
    int8_peak = 2.0 * peaks["bf16_tflops"]
    t_hbm = gu_bytes / (peaks["hbm_gbs"] * 1e9)
    t_tc = gu_ops / (int8_peak * 1e12)
    if t_tc >= t_hbm:
        achieved = gu_ops / (gu_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOPS",
                "frac": achieved / int8_peak}
    else:
        achieved = gu_bytes / (gu_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"]}
    # per-launch DRAM traffic from the committed ncu summaries: recorded for
    # the single-GPU workload only (under EP the rank's routed rows, hence its
    # traffic, differ with N)
    traffic = traffic_from_profiles(args.workload, dominant) if world == 1 else None
    roof.update({"kernel": "w4a8 grouped GEMM (gate/up), " + " + ".join(kernels), "ms_per_launch": gu_ms,
                 "algorithmic_bytes": gu_bytes, "algorithmic_ops": gu_ops,
                 "hbm_frac": gu_bytes / (gu_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                 "int8_frac": gu_ops / (gu_ms * 1e-3) / 1e12 / int8_peak,
                 "int8_frac_of_sustained": gu_ops / (gu_ms * 1e-3) / 1e12 / (2.0 * peaks["bf16_tflops_sustained"]),
                 "traffic": traffic,
                 "peak_source": f"{peaks['src']}: HBM = hbm_gbs; int8 = 2 x bf16_tflops (dense int8 rate is "
                                f"twice bf16 on sm_100)"})
    if world > 1:
        roof["traffic_note"] = "per-launch DRAM bytes are profiled for the single-GPU workload only"
    if "gemm_down" in stages:
        dn_ms = stages["gemm_down"]
        roof["down_ms_per_launch"] = dn_ms
        roof["down_int8_frac"] = W.gemm_ops(R, cfg.hidden, cfg.inter) / (dn_ms * 1e-3) / 1e12 / int8_peak

    targets = variant = router = None
    if not args.no_extras:
        if world == 1 and cfg.name.startswith("deepseek") and cfg.ffn:
            targets = north_star_targets(pkg, layer, W.CONFIGS["deepseek"], dev, max(5, args.steps), peaks)
        if world == 1:
            router = router_stage(pkg, cfg, T, dev, args.steps, peaks)
        variant = routing_variant(pkg, layer, cfg, T, rank, world, dev, args.steps)

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cb = run_cpu_leg(cfg, T, steps=1, warmup=0, budget_s=args.cpu_budget)
        cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}

    if rank == 0:
        line = {"metric": METRIC, "value": world * T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int4 -> int32/fp32 -> bf16",
                "data": "synthetic (seeded; BASELINE.json distributions; random-init weights)",
                "config": config,
                "e2e": {"value": world * T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
                "gpu_launches": args.steps * layer.launches_per_forward(),
                "roofline": roof, "cpu_baseline": cpu, "clocks": clocks, "device_status": status,
                "parity": parity, "stages_ms": stages, "targets": targets, "routing_variant": variant,
                "router": router,
                "active_experts": active, "routed_rows": R}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
