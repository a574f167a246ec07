"""Generates the golden fixtures of this directory by running the REFERENCE's
own PyTorch implementations (read from the reference checkout, executed here
on the CPU).  It needs the reference tree, so it runs only where that tree is
mounted; the fixtures it writes are committed and travel instead.

    python tests/golden/make_golden.py /path/to/reference-checkout
    (or set W4A8_REFERENCE_ROOT and omit the argument)

Sources executed:
  * docs/Task1.md:49-115  -- ``w4a8_group_gemm_moe`` (the operator contract).
    Its internal per-group partial sums (the einsum of :104) are captured by
    giving the executed code a ``torch`` whose ``einsum`` records its result.
  * docs/Task3.md:53-80   -- ``_quantize_rows`` (the repository's int8
    quantiser; with a 128-wide row the group is the whole row, i.e. exactly
    the per-token convention of the activation quantiser).

Each fixture stores the inputs, the reference outputs (bf16 as uint16 bits),
and the captured int32 partials.
"""
from __future__ import annotations

import hashlib
import os
import re
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import importlib  # noqa: E402

pkg = importlib.import_module("flagos-kernel-gen_b200")
W = pkg.workloads


def _python_block(md_path: str) -> str:
    text = open(md_path, encoding="utf-8").read()
    blocks = re.findall(r"```python\n(.*?)```", text, flags=re.S)
    # the implementation block is the one that defines functions
    return [b for b in blocks if "def " in b and "import torch" in b][0]


class _RecordingTorch:
    """Forwards to torch; records every einsum result."""

    def __init__(self):
        self.einsums = []

    def __getattr__(self, name):
        return getattr(torch, name)

    def einsum(self, *args, **kw):
        r = torch.einsum(*args, **kw)
        self.einsums.append(r.clone())
        return r


def load_reference(ref_root: str):
    ns1: dict = {}
    exec(compile(_python_block(os.path.join(ref_root, "docs", "Task1.md")), "docs/Task1.md", "exec"), ns1)
    ns3: dict = {}
    exec(compile(_python_block(os.path.join(ref_root, "docs", "Task3.md")), "docs/Task3.md", "exec"), ns3)
    return ns1, ns3


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def run_gemm_case(ns1, name, x_q, x_scale, packed, scale, zero, offsets, gs, out_init=None):
    rec = _RecordingTorch()
    ns1["torch"] = rec
    fn = ns1["w4a8_group_gemm_moe"]
    M, K = x_q.shape
    E, N, _ = packed.shape
    out = out_init.clone() if out_init is not None else torch.zeros((M, N), dtype=torch.bfloat16)
    fn(x_q, x_scale, packed, scale, zero, offsets, out, gs)
    ns1["torch"] = torch
    G = K // gs
    partials = np.zeros((M, N, G), dtype=np.int32)
    off = offsets.numpy()
    it = iter(rec.einsums)
    for e in range(E):
        m0, m1 = int(off[e]), int(off[e + 1])
        if m1 <= m0:
            continue
        p = next(it)
        pi = p.to(torch.int64)
        assert torch.equal(pi.to(torch.float32), p), "einsum partial is not an exact integer"
        partials[m0:m1] = pi.to(torch.int32).numpy()
    return out, partials


def main(ref_root: str):
    ns1, ns3 = load_reference(ref_root)
    fixtures = {}

    def gemm_fixture(name, E, M, N, K, gs, zero_mode, offsets=None, seed=0, untouched_fill=False, store_inputs=True):
        x_q, x_scale, packed, scale, zero, off = W.make_gemm_inputs(E, M, N, K, gs, seed=seed, zero_mode=zero_mode,
                                                                    offsets=offsets)
        out_init = None
        if untouched_fill:
            out_init = torch.full((M, N), -3.0, dtype=torch.bfloat16)
        out, partials = run_gemm_case(ns1, name, x_q, x_scale, packed, scale, zero, off, gs, out_init)
        d = dict(gs=np.int32(gs), out_bits=bf16_bits(out), partials=partials)
        if store_inputs:
            d.update(x_q=x_q.numpy(), x_scale=x_scale.numpy(), packed=packed.numpy(), scale=scale.numpy(),
                     zero=zero.numpy(), offsets=off.numpy())
        if out_init is not None:
            d["out_init_bits"] = bf16_bits(out_init)
        fixtures[name] = d

    gemm_fixture("gemm_empty_expert", 4, 32, 256, 512, 128, "random",
                 offsets=torch.tensor([0, 10, 10, 25, 32], dtype=torch.int32), seed=1)
    gemm_fixture("gemm_gs64", 3, 24, 128, 384, 64, "random", seed=2)
    gemm_fixture("gemm_zero_wrap", 2, 16, 128, 256, 128, "wrap",
                 offsets=torch.tensor([0, 7, 16], dtype=torch.int32), seed=3)
    gemm_fixture("gemm_untouched_rows", 2, 20, 128, 256, 128, "symmetric",
                 offsets=torch.tensor([2, 9, 15], dtype=torch.int32), seed=4, untouched_fill=True)

    # config 0 (routed single up-projection GEMM, seed 0): inputs are regenerated
    # by the package's seeded generator; the fixture pins their hash and the
    # reference output on the expert-sorted rows.
    cfg = W.CONFIGS["small"]
    inp = W.make_moe_inputs(cfg, 64, seed=0)
    sys.path.insert(0, REPO)
    from oracle import w4a8_oracle as O  # the quantiser/align restatements (pinned separately)
    al = O.moe_align(inp.topk_ids, cfg.experts, 128)
    xq_tok, xs_tok = O.act_quant(inp.x)
    src = al["sorted_ids"] // cfg.topk
    xq = torch.from_numpy(xq_tok[src])
    xs = torch.from_numpy(xs_tok[src])
    off = torch.from_numpy(al["expert_offsets"])
    packed, scale, zero = inp.w13
    out, partials = run_gemm_case(ns1, "cfg0", xq, xs, packed, scale, zero, off, cfg.group_size)
    h = hashlib.sha256()
    for t in (inp.x.view(torch.int16), inp.topk_ids, inp.topk_weights, packed, scale, zero):
        h.update(t.contiguous().numpy().tobytes())
    fixtures["cfg0_gemm"] = dict(gs=np.int32(cfg.group_size), out_bits=bf16_bits(out),
                                 partials_sha256=np.frombuffer(hashlib.sha256(partials.tobytes()).digest(), np.uint8),
                                 inputs_sha256=np.frombuffer(h.digest(), np.uint8))

    # quantiser of docs/Task3.md:58-67 on 128-wide rows (one group per row)
    g = W.make_generator(5)
    xq_in = torch.randn((48, 128), generator=g).to(torch.bfloat16)
    xq_in[3] = 0.0                        # all-zero row: scale clamps to 1e-10
    xq_in[7] *= 1e-6                      # tiny row
    xq_in[11] *= 300.0                    # large row
    xq_in[13, 5] = 127.0                  # exact multiple
    q, s = ns3["_quantize_rows"](xq_in.to(torch.float32))
    fixtures["quant_rows"] = dict(x_bits=bf16_bits(xq_in), q=q.numpy(), s=s.numpy().reshape(-1))

    for name, d in fixtures.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
        print("wrote", name, {k: v.shape for k, v in d.items()})


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("W4A8_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <reference checkout> (or set W4A8_REFERENCE_ROOT)")
    main(root)
