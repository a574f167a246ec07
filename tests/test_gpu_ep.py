"""Expert parallelism on 2 GPUs (skipped with fewer), both transports (the
peer-memory kernels -- with the return streamed by the down GEMM or as its own
pass, with the deduplicated or the per-slot dispatch -- and NCCL
all-to-all): every rank's output equals, bit for
bit, a single-GPU MoELayer run over the tokens of all ranks (same weights),
and a second forward through the same buffers gives the same bits.  Rows reach an expert in a
different order under EP, but each row's result does not depend on the other
rows of its segment, and the combine sums in the same slot order."""
import datetime
import importlib
import os
import socket
import sys
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, zipf, transport):
    try:
        sys.path.insert(0, REPO)
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        pkg = importlib.import_module("flagos-kernel-gen_b200")
        ep = importlib.import_module("flagos-kernel-gen_b200.ep")
        W = pkg.workloads
        cfg = W.MoEConfig("t", hidden=1024, inter=512, experts=16, topk=4, zipf=zipf)
        full = W.make_moe_inputs(cfg, 1, seed=77, zero_mode="random")      # same weights everywhere (CPU seed)
        epr = cfg.experts // world
        sl = slice(rank * epr, (rank + 1) * epr)
        w13 = pkg.W4A8Weights(*[t[sl].contiguous().to(dev) for t in full.w13])
        w2 = pkg.W4A8Weights(*[t[sl].contiguous().to(dev) for t in full.w2])
        T = 96 + 32 * rank
        toks = [W.make_moe_inputs(cfg, 96 + 32 * r, seed=300 + r, weights=False) for r in range(world)]
        mine = toks[rank]
        if transport.startswith("p2p"):
            layer = ep.P2PExpertParallelMoE(w13, w2, cfg.experts, cfg.group_size, cfg.topk, max_tokens=256,
                                            fused_return=(transport != "p2p_return_pass"),
                                            dedup_dispatch=(transport != "p2p_plain_dispatch"))
        else:
            layer = ep.ExpertParallelMoE(w13, w2, cfg.experts, cfg.group_size, cfg.topk)
        out = layer(mine.x.to(dev), mine.topk_ids.to(dev), mine.topk_weights.to(dev)).clone()
        out2 = layer(mine.x.to(dev), mine.topk_ids.to(dev), mine.topk_weights.to(dev)).clone()   # buffers reused
        torch.cuda.synchronize()
        repeat_same = torch.equal(out.view(torch.int16), out2.view(torch.int16))
        torch.cuda.synchronize()
        # single-GPU reference over all ranks' tokens
        ref_layer = pkg.MoELayer(pkg.W4A8Weights(*[t.to(dev) for t in full.w13]),
                                 pkg.W4A8Weights(*[t.to(dev) for t in full.w2]), cfg.group_size, cfg.topk,
                                 sum(t.x.shape[0] for t in toks))
        ref = ref_layer(torch.cat([t.x for t in toks]).to(dev), torch.cat([t.topk_ids for t in toks]).to(dev),
                        torch.cat([t.topk_weights for t in toks]).to(dev))
        start = sum(t.x.shape[0] for t in toks[:rank])
        ref = ref[start:start + T]
        torch.cuda.synchronize()
        same = torch.equal(out.view(torch.int16), ref.view(torch.int16)) and repeat_same
        q.put((rank, "ok", bool(same), float((out.float() - ref.float()).abs().max()), pkg.device_status()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc()[-600:]))


@pytest.mark.parametrize("transport", ["p2p", "p2p_return_pass", "p2p_plain_dispatch", "nccl"])
@pytest.mark.parametrize("zipf", [0.0, 1.2])
def test_ep_two_gpus_matches_single_gpu(zipf, transport):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, zipf, transport)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "EP ranks did not finish"
    res = sorted(q.get() for _ in range(q.qsize()))
    assert len(res) == 2, res
    for r in res:
        assert r[1] == "ok", r
        assert r[2], f"rank {r[0]}: EP differs from single GPU (max diff {r[3]})"
        assert r[4] == 0
