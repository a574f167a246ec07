"""Expert-parallel host logic on CPU ranks (torch.distributed gloo, world 2 and
4): the dispatch / combine bookkeeping of ep.ExpertParallelMoE, run with the
oracle as the device backend, must reproduce the single-process oracle layer
exactly on every rank.  Also: a rank that dies before the exchange makes the
survivors fail with an error within the process-group timeout (no hang)."""
import datetime
import importlib
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class OracleEPOps:
    """CPU stand-in for the CUDA stages, built from the oracle restatements."""

    def __init__(self, O):
        self.O = O

    def align(self, ids, n):
        a = self.O.moe_align(ids.numpy(), n, 1)
        return (torch.from_numpy(a["expert_offsets"]), torch.from_numpy(a["sorted_ids"]),
                torch.from_numpy(a["inv_pos"]))

    def quant_scatter(self, x, inv_pos, k):
        q, s = self.O.act_quant(x)
        R = inv_pos.numel()
        xq = torch.zeros((R, x.shape[1]), dtype=torch.int8)
        xs = torch.zeros((R,), dtype=torch.float32)
        inv = inv_pos.numpy()
        ok = inv >= 0
        f = np.nonzero(ok)[0]
        xq[torch.from_numpy(inv[ok]).long()] = torch.from_numpy(q[f // k])
        xs[torch.from_numpy(inv[ok]).long()] = torch.from_numpy(s[f // k])
        return xq, xs

    def gather_rows(self, src, index):
        out = torch.zeros((index.numel(),) + tuple(src.shape[1:]), dtype=src.dtype)
        ok = index >= 0
        out[ok] = src[index[ok].long()]
        return out

    def grouped_gemm(self, xq, xs, w, off, out, gs):
        return self.O.group_gemm(xq, xs, w.packed, w.scale, w.zero, off, out, gs)

    def silu_mul_requant(self, h):
        q, s = self.O.silu_mul_requant(h)
        return torch.from_numpy(q), torch.from_numpy(s)

    def combine(self, y, inv, w):
        return self.O.combine(y, inv.numpy(), w)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, case, q):
    try:
        sys.path.insert(0, REPO)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        pkg = importlib.import_module("flagos-kernel-gen_b200")
        ep = importlib.import_module("flagos-kernel-gen_b200.ep")
        from oracle import w4a8_oracle as O
        W = pkg.workloads
        cfg = W.MoEConfig("t", hidden=256, inter=128, experts=8, topk=3, zipf=case.get("zipf", 0.0),
                          ffn=case.get("ffn", True))
        # same global weights on every rank; each keeps its shard
        full = W.make_moe_inputs(cfg, 1, seed=123, zero_mode="random")
        epr = cfg.experts // world
        sl = slice(rank * epr, (rank + 1) * epr)
        w13 = pkg.W4A8Weights(*[t[sl].contiguous() for t in full.w13])
        w2 = pkg.W4A8Weights(*[t[sl].contiguous() for t in full.w2]) if cfg.ffn else None
        T = case["tokens"][rank]
        inp = W.make_moe_inputs(cfg, max(T, 1), seed=500 + rank, weights=False)
        x, ids, tw = inp.x[:T], inp.topk_ids[:T].clone(), inp.topk_weights[:T]
        if case.get("drop") and T > 2:
            ids[1, 0] = -1
            ids[2, 1] = cfg.experts   # out of range: dropped as well
        layer = ep.ExpertParallelMoE(w13, w2, cfg.experts, cfg.group_size, cfg.topk, ops=OracleEPOps(O))
        if case.get("die") == rank:
            os._exit(3)   # a rank that vanishes before the exchange
        out = layer(x, ids, tw)
        ref = O.moe_layer(x, ids, tw, full.w13, full.w2, cfg.group_size)
        same = torch.equal(out.view(torch.int16), ref.view(torch.int16))
        q.put((rank, "ok", bool(same), float((out.float() - ref.float()).abs().max()) if T else 0.0))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", type(e).__name__, traceback.format_exc()[-400:]))


def _run(world, case, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    res = []
    while not q.empty():
        res.append(q.get())
    return sorted(res), [p.exitcode for p in procs], alive


@pytest.mark.parametrize("world,case", [
    (2, dict(tokens=[40, 24])),
    (4, dict(tokens=[16, 0, 33, 5], zipf=1.2, drop=True)),
    (2, dict(tokens=[12, 30], ffn=False)),
])
def test_ep_matches_single_process_oracle(world, case):
    res, codes, alive = _run(world, case)
    assert not alive, "EP ranks hung"
    assert len(res) == world, (res, codes)
    for rank, status, *rest in res:
        assert status == "ok", rest
        same, maxdiff = rest
        assert same, f"rank {rank}: EP output differs from the oracle (max diff {maxdiff})"


def test_ep_rank_failure_is_detected():
    """Rank 1 exits before the exchange; rank 0's collective must fail (error
    raised before the process-group timeout expires the test), not hang."""
    res, codes, alive = _run(2, dict(tokens=[8, 8], die=1), timeout=90)
    assert not alive, "surviving rank hung"
    assert codes[1] == 3
    r0 = [r for r in res if r[0] == 0]
    assert r0 and r0[0][1] == "error", res
