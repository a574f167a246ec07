"""GPU parity of the routed W4A8 layer at the benchmark configurations, on the
weights and inputs the benchmark itself uses (weights drawn on the device
from generator seed 1000, tokens from seed 7, as ``bench.py`` does on rank 0):

* DeepSeek-V3 shape (H 7168, I 2048, 256 experts, top-8 sigmoid): the whole
  layer at T = 16 (every active expert), sampled tokens at T = 256, 8192 and
  16384 (the default benchmark workload), uniform and Zipf routing;
* full-size slices at T = 16384: three experts' gate/up (K 7168) and down
  (K 2048, N 7168) rows through the tensor-core kernel in its widest tile
  configuration, int32 partials bit-exact against the oracle, bf16 outputs
  identical to the layer's own launch and within the GEMM rule;
* Mixtral-8x7B shape (H 4096, I 14336, 8 experts, top-2): the whole layer at
  T = 1, 16 and 128;
* Qwen3-30B-A3B shape with Zipf(1.2) routing at T = 4096: tokens of the
  hottest and of the coldest expert.

Layer outputs use the tolerance stated in ``gpu_util`` (the reference's bf16
rule elementwise, and mean|out - ref| <= 1e-3 mean|ref|).  Checking sampled
tokens is exact in scope: a token's output depends only on its own
activations, its experts and their weights (``oracle.moe_layer_tokens``)."""
import numpy as np
import pytest
import torch

from gpu_util import O, assert_gemm_close, assert_layer_close

pytestmark = pytest.mark.gpu

WEIGHT_SEED = 1000   # bench.py build_layer: make_generator(1000 + rank)
INPUT_SEED = 7       # bench.py: make_moe_inputs(..., seed=7 + rank)
MID_TILE_AVG_ROWS = 160   # gemm_tc.cu: above this many rows per expert the 256-token tiles run


def _weights(pkg, cfg, dev):
    W = pkg.workloads
    gen = W.make_generator(WEIGHT_SEED, dev)
    n13 = 2 * cfg.inter if cfg.ffn else cfg.inter
    w13 = pkg.W4A8Weights(*W.make_int4_weights(cfg.experts, n13, cfg.hidden, cfg.group_size, gen, dev))
    w2 = pkg.W4A8Weights(*W.make_int4_weights(cfg.experts, cfg.hidden, cfg.inter, cfg.group_size, gen, dev))
    return w13, w2


def _as_tuple(w):
    return (w.packed, w.scale, w.zero)


def _forward(pkg, layer, cfg, T, dev, seed=INPUT_SEED):
    inp = pkg.workloads.make_moe_inputs(cfg, T, seed=seed, device=dev, weights=False)
    out = layer(inp.x, inp.topk_ids, inp.topk_weights).clone()
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    return inp, out


def _check_tokens(layer, cfg, inp, out, tokens, what):
    ref = O.moe_layer_tokens(inp.x, inp.topk_ids, inp.topk_weights, _as_tuple(layer.w13), _as_tuple(layer.w2),
                             cfg.group_size, tokens)
    return assert_layer_close(out[torch.as_tensor(tokens, device=out.device)], ref, cfg.hidden, what)


@pytest.fixture(scope="module")
def deepseek(pkg, cuda):
    cfg = pkg.workloads.CONFIGS["deepseek"]
    w13, w2 = _weights(pkg, cfg, cuda)
    layer = pkg.MoELayer(w13, w2, cfg.group_size, cfg.topk, 16384)
    yield cfg, layer
    del layer, w13, w2
    torch.cuda.empty_cache()


def test_deepseek_T16_whole_layer(pkg, cuda, deepseek):
    """Config 2 at T = 16 (decode: the streaming kernel, ~100 active experts
    of 1-4 rows), every token against the oracle layer."""
    cfg, layer = deepseek
    inp, out = _forward(pkg, layer, cfg, 16, cuda)
    active = int(((layer.offsets[1:] - layer.offsets[:-1]) > 0).sum())
    assert active > 90
    _check_tokens(layer, cfg, inp, out, list(range(16)), "deepseek T=16")


@pytest.mark.parametrize("T,tokens", [(256, [0, 31, 100, 200, 255]), (8192, [0, 4095, 8191])])
def test_deepseek_sampled_tokens(pkg, cuda, deepseek, T, tokens):
    """Config 2 at T = 256 (streaming + 64-token tensor-core tiles) and
    T = 8192 (256-token tiles)."""
    cfg, layer = deepseek
    inp, out = _forward(pkg, layer, cfg, T, cuda)
    _check_tokens(layer, cfg, inp, out, tokens, f"deepseek T={T}")


def _slice_check(pkg, cuda, x_sorted, s_sorted, offsets, w, experts, layer_out, gs):
    """Runs the tensor-core kernel on the rows of `experts` alone and checks
    partials (bit-exact vs the oracle), the bf16 output (identical to the
    layer's launch over all experts, within the GEMM rule vs the oracle)."""
    off = offsets.cpu().numpy()
    segs = [(int(off[e]), int(off[e + 1])) for e in experts]
    xq = torch.cat([x_sorted[a:b] for a, b in segs])
    xs = torch.cat([s_sorted[a:b] for a, b in segs])
    counts = [b - a for a, b in segs]
    M = sum(counts)
    assert M > MID_TILE_AVG_ROWS * len(experts), "slice must run the 256-token tile configuration"
    sub_off = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int32, device=cuda)
    idx = torch.tensor(experts, device=cuda)
    wp, ws, wz = (t.index_select(0, idx).contiguous() for t in (w.packed, w.scale, w.zero))
    E, N, K = len(experts), wp.shape[1], 2 * wp.shape[2]
    G = K // gs
    out = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    parts = torch.empty((M, N, G), dtype=torch.int32, device=cuda)
    pkg.w4a8_group_gemm_moe_ex(xq, xs, wp, ws, wz, sub_off, out, gs, kernel=pkg.KERNEL_TC, partials=parts)
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    # the slice's rows equal the layer's own launch over all experts bit for bit
    ref_rows = torch.cat([layer_out[a:b] for a, b in segs])
    assert torch.equal(out.view(torch.int16), ref_rows.view(torch.int16))
    out_c, parts_c, xq_c, xs_c = out.cpu(), parts.cpu().numpy(), xq.cpu(), xs.cpu()
    wp_c, ws_c, wz_c = wp.cpu(), ws.cpu(), wz.cpu()
    ref64 = np.empty((M, N), dtype=np.float64)
    for i, e in enumerate(experts):
        m0 = int(sum(counts[:i]))
        m1 = m0 + counts[i]
        p = O.group_partials(xq_c[m0:m1].numpy(), O.signed_weights(wp_c[i], wz_c[i], gs), gs)
        np.testing.assert_array_equal(parts_c[m0:m1], p, err_msg=f"expert {e}: int32 partials differ")
        ref64[m0:m1] = (p.astype(np.float64) * ws_c[i].numpy().astype(np.float64)[None]).sum(-1) \
            * xs_c[m0:m1].numpy().astype(np.float64)[:, None]
        del p
    oracle_out = torch.zeros((M, N), dtype=torch.bfloat16)
    O.group_gemm(xq_c, xs_c, wp_c, ws_c, wz_c, sub_off.cpu(), oracle_out, gs)
    assert_gemm_close(out_c, oracle_out, ref64, N)


@pytest.mark.parametrize("routing", ["deepseek", "deepseek_zipf"])
def test_deepseek_T16384_headline(pkg, cuda, deepseek, routing):
    """The default benchmark workload (config 4's per-GPU shape, 131072
    routed rows, 256-token tiles): sampled tokens of the whole layer, then
    full-size slices of the hottest, a median and the coldest expert through
    gate/up (K 7168) and down (K 2048, N 7168)."""
    _, layer = deepseek
    cfg = pkg.workloads.CONFIGS[routing]
    inp, out = _forward(pkg, layer, cfg, 16384, cuda)
    _check_tokens(layer, cfg, inp, out, [0, 5000, 16383], f"{routing} T=16384")
    off = layer.offsets.cpu()
    counts = (off[1:] - off[:-1]).numpy()
    order = [int(e) for e in np.argsort(-counts, kind="stable") if counts[e] > 0]
    if routing == "deepseek":
        experts = [order[0], order[len(order) // 2], order[-1]]
    else:
        # Zipf: the hottest experts hold 5k-16k rows each (their int32 partials
        # would take GBs); take the three largest below 1000 rows, still in the
        # 256-token tile configuration
        experts = [e for e in order if counts[e] <= 1000][:3]
    R = int(off[-1])
    _slice_check(pkg, cuda, layer.xq[:R], layer.xs[:R], layer.offsets, layer.w13, experts, layer.h[:R],
                 cfg.group_size)
    _slice_check(pkg, cuda, layer.aq[:R], layer.as_[:R], layer.offsets, layer.w2, experts, layer.y[:R],
                 cfg.group_size)


@pytest.fixture(scope="module")
def mixtral(pkg, cuda):
    cfg = pkg.workloads.CONFIGS["mixtral"]
    w13, w2 = _weights(pkg, cfg, cuda)
    layer = pkg.MoELayer(w13, w2, cfg.group_size, cfg.topk, 128)
    yield cfg, layer
    del layer, w13, w2
    torch.cuda.empty_cache()


def test_mixtral_whole_layers(pkg, cuda, mixtral):
    """Config 1 (gate/up N 28672, down K 14336) at T = 1 (streaming only),
    16 (streaming + tensor core) and 128 (tensor core): every token of each
    batch against one oracle run over the three batches' tokens."""
    cfg, layer = mixtral
    outs, inps = [], []
    for T in (1, 16, 128):
        inp, out = _forward(pkg, layer, cfg, T, cuda, seed=INPUT_SEED + T)
        inps.append(inp)
        outs.append(out)
    x = torch.cat([i.x.cpu() for i in inps])
    ids = torch.cat([i.topk_ids.cpu() for i in inps])
    tw = torch.cat([i.topk_weights.cpu() for i in inps])
    ref = O.moe_layer_tokens(x, ids, tw, _as_tuple(layer.w13), _as_tuple(layer.w2), cfg.group_size,
                             list(range(x.shape[0])))
    start = 0
    for out in outs:
        T = out.shape[0]
        assert_layer_close(out, ref[start:start + T], cfg.hidden, f"mixtral T={T}")
        start += T


def test_qwen3_zipf_hottest_and_coldest_experts(pkg, cuda):
    """Config 3 (Zipf(1.2) routing: one expert takes almost every token,
    others a handful): tokens of the hottest and of the coldest active expert."""
    cfg = pkg.workloads.CONFIGS["qwen3_zipf"]
    w13, w2 = _weights(pkg, cfg, cuda)
    layer = pkg.MoELayer(w13, w2, cfg.group_size, cfg.topk, 4096)
    inp, out = _forward(pkg, layer, cfg, 4096, cuda)
    off = layer.offsets.cpu()
    counts = (off[1:] - off[:-1]).numpy()
    assert counts.max() > 2000 and counts[counts > 0].min() < 100, "routing must be skewed"
    hot = int(np.argmax(counts))
    cold = int(np.argmin(np.where(counts > 0, counts, 1 << 30)))
    ids = inp.topk_ids.cpu()
    hot_toks = torch.nonzero((ids == hot).any(1)).flatten()[:12].tolist()
    cold_toks = torch.nonzero((ids == cold).any(1)).flatten()[:12].tolist()
    _check_tokens(layer, cfg, inp, out, sorted(set(hot_toks + cold_toks)), "qwen3 zipf T=4096")
