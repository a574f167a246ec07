"""Seeded synthetic workloads with the shapes and value distributions of the
benchmark configurations (there is no network, so no checkpoints or datasets):

* weights: int4 uniform in [-8, 7] stored as nibble = q + 8 (so ``w_zero`` is 8
  everywhere), packed two per byte along K with the low nibble holding the
  even k (docs/Task1.md:78-81); fp32 per-(expert, channel, K-group) scales
  uniform in [0.005, 0.02];
* activations: bf16 N(0, 1);
* router: logits N(0, 1) (plus a per-expert bias -s*ln(rank) for Zipf(s)
  popularity), softmax or sigmoid scores, top-k, weights renormalised to sum 1.

Also the ten operator shapes of docs/Task1.md:30-41 for the 8-argument entry
point, with uniformly random expert splits.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class MoEConfig:
    name: str
    hidden: int          # H (K of the gate/up GEMM, N of the down GEMM)
    inter: int           # I (expert intermediate size); gate/up produces 2I columns
    experts: int         # E
    topk: int
    group_size: int = 128
    scoring: str = "softmax"   # "softmax" | "sigmoid"
    zipf: float = 0.0          # 0 = uniform routing, else Zipf exponent of expert popularity
    ffn: bool = True           # False: single up-projection GEMM (config 0)


CONFIGS = {
    # config 0: single up-projection GEMM, CPU-runnable
    "small": MoEConfig("small", hidden=1024, inter=512, experts=8, topk=2, ffn=False),
    "mixtral": MoEConfig("mixtral", hidden=4096, inter=14336, experts=8, topk=2),
    "deepseek": MoEConfig("deepseek", hidden=7168, inter=2048, experts=256, topk=8, scoring="sigmoid"),
    "qwen3_zipf": MoEConfig("qwen3_zipf", hidden=2048, inter=768, experts=128, topk=8, zipf=1.2),
    "deepseek_zipf": MoEConfig("deepseek_zipf", hidden=7168, inter=2048, experts=256, topk=8,
                               scoring="sigmoid", zipf=1.2),
}

# docs/Task1.md:30-41: (E, M_total, N, K, group_size)
TASK1_SHAPES = [
    (4, 32, 512, 512, 128),
    (8, 64, 1024, 1024, 128),
    (8, 128, 1408, 2048, 128),
    (8, 256, 2048, 2048, 128),
    (16, 128, 1024, 1536, 64),
    (16, 256, 1536, 2048, 128),
    (32, 256, 1408, 2048, 128),
    (32, 512, 2048, 4096, 128),
    (64, 512, 1024, 2048, 128),
    (64, 1024, 2048, 4096, 128),
]


def make_generator(seed: int, device: str | torch.device = "cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def pack_nibbles(nib: torch.Tensor) -> torch.Tensor:
    """uint8 nibbles [..., K] (0..15) -> packed uint8 [..., K/2], low nibble = even k."""
    lo = nib[..., 0::2].to(torch.uint8)
    hi = nib[..., 1::2].to(torch.uint8)
    return lo | (hi << 4)


def make_int4_weights(E: int, N: int, K: int, group_size: int, gen: torch.Generator,
                      device: str | torch.device = "cpu", zero_mode: str = "symmetric"):
    """Packed int4 expert weights [E, N, K/2] with scales and zero points [E, N, K/gs].

    zero_mode: "symmetric" (w_zero = 8, i.e. int4 in [-8, 7]), "random" (w_zero
    uniform in [0, 15]) or "wrap" (w_zero over the whole int8 range, which
    exercises the int8 wrap of the zero fold).
    """
    G = K // group_size
    # two nibbles per byte drawn as one uniform byte: identical distribution to two uniform nibbles
    packed = torch.randint(0, 256, (E, N, K // 2), generator=gen, device=device, dtype=torch.uint8)
    scale = torch.empty((E, N, G), device=device, dtype=torch.float32).uniform_(0.005, 0.02, generator=gen)
    if zero_mode == "symmetric":
        zero = torch.full((E, N, G), 8, device=device, dtype=torch.int8)
    elif zero_mode == "random":
        zero = torch.randint(0, 16, (E, N, G), generator=gen, device=device, dtype=torch.int32).to(torch.int8)
    elif zero_mode == "wrap":
        zero = torch.randint(-128, 128, (E, N, G), generator=gen, device=device, dtype=torch.int32).to(torch.int8)
    else:
        raise ValueError(zero_mode)
    return packed, scale, zero


def zipf_bias(E: int, s: float, gen: torch.Generator, device="cpu") -> torch.Tensor:
    rank = torch.randperm(E, generator=gen, device=device).to(torch.float32) + 1.0
    return -s * torch.log(rank)


def route(logits: torch.Tensor, topk: int, scoring: str):
    """Router used to make test inputs (not part of the kernel path): scores,
    top-k, weights renormalised to sum to 1.  Returns (ids int32, weights fp32)."""
    scores = torch.softmax(logits, dim=-1) if scoring == "softmax" else torch.sigmoid(logits)
    w, ids = torch.topk(scores, topk, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    return ids.to(torch.int32), w.to(torch.float32)


@dataclass
class MoEInputs:
    x: torch.Tensor            # bf16 [T, H]
    topk_ids: torch.Tensor     # int32 [T, k]
    topk_weights: torch.Tensor  # fp32 [T, k]
    w13: tuple                 # (packed [E, 2I or I, H/2], scale, zero)
    w2: tuple | None           # (packed [E, H, I/2], scale, zero) or None for single-GEMM configs


def make_moe_inputs(cfg: MoEConfig, T: int, seed: int = 0, device: str | torch.device = "cpu",
                    zero_mode: str = "symmetric", weights: bool = True) -> MoEInputs:
    gen = make_generator(seed, device)
    E, H, I = cfg.experts, cfg.hidden, cfg.inter
    w13 = w2 = None
    if weights:
        n13 = 2 * I if cfg.ffn else I
        w13 = make_int4_weights(E, n13, H, cfg.group_size, gen, device, zero_mode)
        if cfg.ffn:
            w2 = make_int4_weights(E, H, I, cfg.group_size, gen, device, zero_mode)
    x = torch.randn((T, H), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=gen, device=device, dtype=torch.float32)
    if cfg.zipf > 0:
        logits = logits + zipf_bias(E, cfg.zipf, gen, device)[None, :]
    ids, w = route(logits, cfg.topk, cfg.scoring)
    return MoEInputs(x, ids, w, w13, w2)


def random_splits(E: int, M_total: int, gen: torch.Generator, device="cpu") -> torch.Tensor:
    """Monotone expert_offsets [E+1] from E-1 uniform cut points in [0, M_total]."""
    cuts = torch.randint(0, M_total + 1, (E - 1,), generator=gen, device=device, dtype=torch.int64)
    cuts, _ = torch.sort(cuts)
    off = torch.cat([torch.zeros(1, dtype=torch.int64, device=device), cuts,
                     torch.full((1,), M_total, dtype=torch.int64, device=device)])
    return off.to(torch.int32)


def make_gemm_inputs(E: int, M_total: int, N: int, K: int, group_size: int, seed: int = 0,
                     device="cpu", zero_mode: str = "random", offsets: torch.Tensor | None = None):
    """Inputs of the 8-argument entry point: x_q uniform over the whole int8
    range, x_scale uniform in [0.001, 0.05], random expert splits."""
    gen = make_generator(seed, device)
    packed, scale, zero = make_int4_weights(E, N, K, group_size, gen, device, zero_mode)
    x_q = torch.randint(-128, 128, (M_total, K), generator=gen, device=device, dtype=torch.int32).to(torch.int8)
    x_scale = torch.empty((M_total,), device=device, dtype=torch.float32).uniform_(0.001, 0.05, generator=gen)
    if offsets is None:
        offsets = random_splits(E, M_total, gen, device)
    return x_q, x_scale, packed, scale, zero, offsets


def gemm_roofline_bytes(active_experts: int, R: int, N: int, K: int, group_size: int) -> int:
    """Algorithmic HBM bytes of one grouped GEMM: every active expert's packed
    weights, scales and zero points once, plus activations, token scales and
    bf16 output once."""
    G = K // group_size
    return active_experts * (N * K // 2 + N * G * 4 + N * G) + R * K + R * 4 + R * N * 2


def gemm_ops(R: int, N: int, K: int) -> int:
    return 2 * R * N * K


def cdiv(a: int, b: int) -> int:
    return -(-a // b)


def log2i(x: int) -> int:
    return int(math.log2(x))
