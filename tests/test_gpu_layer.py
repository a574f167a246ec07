"""GPU parity of the routed-MoE stages and of the whole layer.

Bit-exact against the oracle: activation quantisation (also against the
reference's own quantiser fixture), align (all outputs), fused quantise +
dispatch, combine.  Within tolerance: SiLU-mul requant (expf differs from the
CPU's by ulps, which can move an int8 by one step) and the full layer."""
import numpy as np
import pytest
import torch

from gpu_util import O, assert_layer_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,H", [(1, 7168), (37, 4096), (64, 2048), (5, 1000), (3, 16392), (0, 128)])
def test_act_quant_bit_exact(pkg, cuda, T, H):
    g = pkg.workloads.make_generator(T * 7 + H)
    x = (torch.randn((T, H), generator=g) * 3).to(torch.bfloat16)
    if T > 2:
        x[1] = 0
        x[2] *= 1e-30
    q, s = pkg.act_quant(x.to(cuda))
    torch.cuda.synchronize()
    rq, rs = O.act_quant(x)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_act_quant_matches_reference_quantiser(pkg, cuda, golden):
    g = golden("quant_rows")
    x = O.bits_to_bf16(g["x_bits"]).to(cuda)
    q, s = pkg.act_quant(x)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q.cpu().numpy(), g["q"])
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), g["s"].astype(np.float32).view(np.uint32))


def _check_align(pkg, cuda, ids, E, bs):
    al = pkg.moe_align(ids.to(cuda), E, bs)
    torch.cuda.synchronize()
    ref = O.moe_align(ids, E, bs)
    np.testing.assert_array_equal(al.expert_offsets.cpu().numpy(), ref["expert_offsets"])
    n = int(ref["expert_offsets"][-1])
    np.testing.assert_array_equal(al.sorted_ids.cpu().numpy()[:n], ref["sorted_ids"])
    np.testing.assert_array_equal(al.inv_pos.cpu().numpy(), ref["inv_pos"])
    np.testing.assert_array_equal(al.padded_ids.cpu().numpy(), ref["padded_ids"])
    np.testing.assert_array_equal(al.block_expert.cpu().numpy(), ref["block_expert"])
    assert int(al.num_post_pad.item()) == ref["num_post_pad"]


@pytest.mark.parametrize("cfg,T", [("small", 64), ("deepseek", 16), ("deepseek", 16384), ("qwen3_zipf", 4096),
                                   ("mixtral", 1), ("deepseek_zipf", 3000)])
def test_align_bit_exact(pkg, cuda, cfg, T):
    c = pkg.workloads.CONFIGS[cfg]
    inp = pkg.workloads.make_moe_inputs(c, T, seed=0, weights=False)
    _check_align(pkg, cuda, inp.topk_ids, c.experts, 128)


@pytest.mark.parametrize("bs", [1, 16, 64])
def test_align_dropped_ids_and_block_sizes(pkg, cuda, bs):
    rng = np.random.default_rng(bs)
    ids = torch.from_numpy(rng.integers(-1, 33, size=(777, 6)).astype(np.int32))   # -1 and 32 are dropped
    _check_align(pkg, cuda, ids, 32, bs)
    _check_align(pkg, cuda, torch.zeros((0, 4), dtype=torch.int32), 8, bs)


def test_align_many_experts(pkg, cuda):
    """More experts than the scan's 1024 threads (its serial offset path),
    a skewed split and dropped ids."""
    rng = np.random.default_rng(5)
    E = 3000
    ids = rng.zipf(1.3, size=(4000, 8)) % (E + 7) - 3   # values in [-3, E+3]: some dropped
    _check_align(pkg, cuda, torch.from_numpy(ids.astype(np.int32)), E, 64)


def test_align_without_padded_outputs(pkg, cuda):
    """The routed layer asks for no padded block map (NULL padded_ids,
    block_expert, num_post_pad): offsets, sorted ids and inverse positions
    must equal those of the full call."""
    c = pkg.workloads.CONFIGS["deepseek"]
    inp = pkg.workloads.make_moe_inputs(c, 777, seed=4, weights=False)
    ids = inp.topk_ids.to(torch.int32).contiguous().to(cuda)
    T, k = ids.shape
    E, R = c.experts, T * k
    full = pkg.moe_align(ids, E, 128)
    lib = pkg._lib.load()
    need = lib.w4a8_moe_align_workspace_size(T, k, E)
    ws = torch.empty((need,), dtype=torch.uint8, device=cuda)
    off = torch.full((E + 1,), -7, dtype=torch.int32, device=cuda)
    srt = torch.full((R,), -7, dtype=torch.int32, device=cuda)
    inv = torch.full((R,), -7, dtype=torch.int32, device=cuda)
    rc = lib.w4a8_moe_align(ids.data_ptr(), T, k, E, 128, off.data_ptr(), srt.data_ptr(), inv.data_ptr(),
                            None, None, None, ws.data_ptr(), need, torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(off, full.expert_offsets)
    assert torch.equal(srt, full.sorted_ids)
    assert torch.equal(inv, full.inv_pos)


def test_quant_scatter_and_combine(pkg, cuda):
    c = pkg.workloads.CONFIGS["deepseek"]
    T = 200
    inp = pkg.workloads.make_moe_inputs(c, T, seed=2, weights=False)
    al = pkg.moe_align(inp.topk_ids.to(cuda), c.experts)
    xq, xs = pkg.quant_scatter(inp.x.to(cuda), al.inv_pos, c.topk)
    torch.cuda.synchronize()
    rq, rs = O.act_quant(inp.x)
    src = al.sorted_ids.cpu().numpy() // c.topk
    np.testing.assert_array_equal(xq.cpu().numpy(), rq[src])
    np.testing.assert_array_equal(xs.cpu().numpy(), rs[src])
    y = torch.randn((T * c.topk, c.hidden), generator=pkg.workloads.make_generator(9)).to(torch.bfloat16)
    out = pkg.moe_combine(y.to(cuda), al.inv_pos, inp.topk_weights.to(cuda))
    torch.cuda.synchronize()
    ref = O.combine(y, al.inv_pos.cpu().numpy(), inp.topk_weights)
    np.testing.assert_array_equal(O.bf16_bits(out.cpu()), O.bf16_bits(ref))


@pytest.mark.parametrize("R,I", [(64, 2048), (17, 768), (3, 14336), (5, 999)])
def test_silu_mul_requant(pkg, cuda, R, I):
    h = (torch.randn((R, 2 * I), generator=pkg.workloads.make_generator(R + I)) * 4).to(torch.bfloat16)
    q, s = pkg.silu_mul_requant(h.to(cuda))
    torch.cuda.synchronize()
    rq, rs = O.silu_mul_requant(h)
    np.testing.assert_allclose(s.cpu().numpy(), rs, rtol=1e-6, atol=0)
    d = np.abs(q.cpu().numpy().astype(np.int32) - rq.astype(np.int32))
    assert d.max() <= 1
    assert (d > 0).mean() <= 1e-3


def _layer_case(pkg, cuda, cfg_name, T, seed):
    W = pkg.workloads
    c = W.CONFIGS[cfg_name]
    inp = W.make_moe_inputs(c, T, seed=seed, zero_mode="random")
    w13 = pkg.W4A8Weights(*[t.to(cuda) for t in inp.w13])
    w2 = pkg.W4A8Weights(*[t.to(cuda) for t in inp.w2]) if inp.w2 is not None else None
    layer = pkg.MoELayer(w13, w2, c.group_size, c.topk, T)
    out = layer(inp.x.to(cuda), inp.topk_ids.to(cuda), inp.topk_weights.to(cuda))
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    ref, inter = O.moe_layer(inp.x, inp.topk_ids, inp.topk_weights, inp.w13, inp.w2, c.group_size,
                             return_intermediates=True)
    return out.cpu(), ref, layer, inter


def test_layer_single_gemm_config0(pkg, cuda):
    """Config 0: routed up-projection [64 x 1024] x [8, 512, 1024], top-2, combined."""
    out, ref, layer, inter = _layer_case(pkg, cuda, "small", 64, 0)
    # the gate/up GEMM output on sorted rows equals the oracle's within the GEMM tolerance
    np.testing.assert_array_equal(layer.xq[:128].cpu().numpy(), inter["xq"].numpy())
    torch.testing.assert_close(out.float(), ref.float(), rtol=0.016, atol=1e-4 * 512)
    o, r = out.float(), ref.float()
    assert (o - r).abs().mean() <= 1e-3 * r.abs().mean()


def test_layer_ffn_small(pkg, cuda):
    """A small gate/up -> SiLU-mul requant -> down FFN with every stage on the GPU."""
    W = pkg.workloads
    W.CONFIGS["_test_ffn"] = W.MoEConfig("_test_ffn", hidden=512, inter=256, experts=16, topk=4, zipf=1.2)
    try:
        out, ref, layer, inter = _layer_case(pkg, cuda, "_test_ffn", 96, 3)
    finally:
        del W.CONFIGS["_test_ffn"]
    assert_layer_close(out, ref, 512, "small FFN")


def test_host_pipeline_matches_direct_forward(pkg, cuda):
    """HostPipeline (copies on side streams, overlapped with compute) returns,
    for every batch, exactly what a direct forward on device tensors returns."""
    W = pkg.workloads
    gen = W.make_generator(5, cuda)
    E, H, I, gs, k = 16, 1024, 256, 128, 4
    w13 = pkg.W4A8Weights(*W.make_int4_weights(E, 2 * I, H, gs, gen, cuda))
    w2 = pkg.W4A8Weights(*W.make_int4_weights(E, H, I, gs, gen, cuda))
    layer = pkg.MoELayer(w13, w2, gs, k, 64)
    batches = []
    for b in range(5):
        T = 48 + 4 * b
        x = torch.randn((T, H), generator=gen, device=cuda).to(torch.bfloat16)
        probs = torch.softmax(torch.randn((T, E), generator=gen, device=cuda), -1)
        tw, ids = torch.topk(probs, k, dim=-1)
        batches.append((x, ids.to(torch.int32), (tw / tw.sum(-1, keepdim=True)).float()))
    direct = [layer(x, ids, tw).clone() for x, ids, tw in batches]
    pipe = pkg.HostPipeline(layer, cuda)
    outs = []
    for x, ids, tw in batches:
        o = torch.empty((x.shape[0], H), dtype=torch.bfloat16).pin_memory()
        pipe.submit(x.cpu().pin_memory(), ids.cpu().pin_memory(), tw.cpu().pin_memory(), o)
        outs.append(o)
    pipe.flush()
    torch.cuda.synchronize()
    for d, o in zip(direct, outs):
        assert torch.equal(d.cpu(), o)


@pytest.mark.parametrize("kernel", ["AUTO", "TC", "GEMV", "SIMT"])
def test_fused_combine_gemm_each_kernel(pkg, cuda, kernel):
    """w4a8_group_gemm_moe_combine: each kernel's epilogue adds topk_w * bf16(y)
    into the token rows.  Against the unfused GEMM followed by the j-ascending
    combine it may differ only by the order of the fp32 additions: every
    element within the layer rule, and nearly all bit-identical."""
    W = pkg.workloads
    c = W.MoEConfig("t", hidden=1024, inter=768, experts=16, topk=4, zipf=1.2)
    T = 200
    inp = W.make_moe_inputs(c, T, seed=12, zero_mode="random")
    al = pkg.moe_align(inp.topk_ids.to(cuda), c.experts)
    xq, xs = pkg.quant_scatter(inp.x.to(cuda), al.inv_pos, c.topk)
    w = [t.to(cuda) for t in inp.w2]             # down projection: [E, 1024, 768]
    aq = xq[:, :768].contiguous()
    sel = getattr(pkg, f"KERNEL_{kernel}")
    R = T * c.topk
    y = torch.empty((R, c.hidden), dtype=torch.bfloat16, device=cuda)
    pkg.w4a8_group_gemm_moe_ex(aq, xs, *w, al.expert_offsets, y, c.group_size, kernel=sel)
    tw = inp.topk_weights.to(cuda)
    ref = pkg.moe_combine(y, al.inv_pos, tw)
    acc = torch.zeros((T, c.hidden), dtype=torch.float32, device=cuda)
    pkg.w4a8_group_gemm_moe_combine(aq, xs, *w, al.expert_offsets, al.sorted_ids, tw, acc, c.group_size,
                                    kernel=sel)
    out = torch.empty((T, c.hidden), dtype=torch.bfloat16, device=cuda)
    pkg.combine_finish(acc, out)
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    assert int(torch.count_nonzero(acc)) == 0, "combine_finish must clear the accumulator"
    assert_layer_close(out, ref, c.hidden, f"fused combine ({kernel})")
    same = (out.view(torch.int16) == ref.view(torch.int16)).float().mean().item()
    assert same >= 0.99, same


@pytest.mark.parametrize("cfg_name,T", [("_ffn", 96), ("small", 64)])
def test_layer_fused_combine_against_oracle(pkg, cuda, cfg_name, T):
    """MoELayer(fused_combine=True) against the oracle layer, twice in a row
    (the accumulator must come back cleared), FFN and single-GEMM forms."""
    W = pkg.workloads
    c = W.MoEConfig("_ffn", hidden=512, inter=256, experts=16, topk=4, zipf=1.2) if cfg_name == "_ffn" \
        else W.CONFIGS[cfg_name]
    inp = W.make_moe_inputs(c, T, seed=3, zero_mode="random")
    w13 = pkg.W4A8Weights(*[t.to(cuda) for t in inp.w13])
    w2 = pkg.W4A8Weights(*[t.to(cuda) for t in inp.w2]) if inp.w2 is not None else None
    layer = pkg.MoELayer(w13, w2, c.group_size, c.topk, T, fused_combine=True)
    outs = [layer(inp.x.to(cuda), inp.topk_ids.to(cuda), inp.topk_weights.to(cuda)).clone() for _ in range(2)]
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    ref = O.moe_layer(inp.x, inp.topk_ids, inp.topk_weights, inp.w13, inp.w2, c.group_size)
    width = c.hidden if inp.w2 is not None else c.inter
    for o in outs:
        assert_layer_close(o, ref, width, "fused layer")


@pytest.mark.parametrize("I", [512, 768, 2048, 14336])   # one warp per row (<= 1024) and one CTA per row
def test_silu_requant_rows_counted_on_device(pkg, cuda, I):
    """w4a8_silu_mul_requant_rows (the expert-parallel receive buffer's form:
    the row count read on the device) writes exactly the bits of
    w4a8_silu_mul_requant on its first rows and leaves the rows past the count
    untouched."""
    R, valid = 700, 523
    g = pkg.workloads.make_generator(I)
    h = (torch.randn((R, 2 * I), generator=g) * 2).to(torch.bfloat16).to(cuda)
    q_ref = torch.zeros((R, I), dtype=torch.int8, device=cuda)
    s_ref = torch.zeros((R,), dtype=torch.float32, device=cuda)
    pkg.silu_mul_requant(h, q_ref, s_ref)
    q = torch.full((R, I), 77, dtype=torch.int8, device=cuda)
    s = torch.full((R,), -1.0, dtype=torch.float32, device=cuda)
    cnt = torch.tensor([valid], dtype=torch.int32, device=cuda)
    lib = pkg._lib.load()
    rc = lib.w4a8_silu_mul_requant_rows(h.data_ptr(), 2 * I, R, I, q.data_ptr(), s.data_ptr(), cnt.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    pkg._lib.check(rc, "w4a8_silu_mul_requant_rows")
    torch.cuda.synchronize()
    assert torch.equal(q[:valid], q_ref[:valid])
    assert torch.equal(s[:valid].view(torch.int32), s_ref[:valid].view(torch.int32))
    assert bool((q[valid:] == 77).all()) and bool((s[valid:] == -1.0).all())
