"""GPU parity of the grouped W4A8 GEMM (both kernels, called through the C ABI)
against the CPU oracle, which is itself pinned to the reference's outputs.

Bit-exact: the int32 per-group partial sums.  Within tolerance (gpu_util):
the bf16 outputs.  Edge cases: empty experts, rows outside every segment,
int8 wrap of the zero fold, group size 64, N = 1408, M not a multiple of the
tile, strided / transposed outputs, strided activations, M_total = 0."""
import numpy as np
import pytest
import torch

from gpu_util import O, assert_gemm_close, segment_rows, to_dev

pytestmark = pytest.mark.gpu

KERNELS = {"auto": 0, "tc": 1, "simt": 2, "gemv": 3}
GOLDEN = ["gemm_empty_expert", "gemm_gs64", "gemm_zero_wrap", "gemm_untouched_rows"]


def run(pkg, dev, x_q, xs, w, ws, wz, off, gs, kernel, out=None, partials=True):
    x_q, xs, w, ws, wz, off = to_dev(dev, x_q, xs, w, ws, wz, off)
    M, K = x_q.shape
    E, N, _ = w.shape
    if out is None:
        out = torch.zeros((M, N), dtype=torch.bfloat16, device=dev)
    parts = torch.zeros((M, N, K // gs), dtype=torch.int32, device=dev) if partials else None
    pkg.w4a8_group_gemm_moe_ex(x_q, xs, w, ws, wz, off, out, gs, kernel=kernel, partials=parts)
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    return out, parts


@pytest.mark.parametrize("kernel", list(KERNELS))
@pytest.mark.parametrize("name", GOLDEN)
def test_gemm_reference_golden(pkg, cuda, golden, name, kernel):
    g = golden(name)
    gs = int(g["gs"])
    M, N = g["out_bits"].shape
    t = {k: torch.from_numpy(g[k]) for k in ("x_q", "x_scale", "packed", "scale", "zero", "offsets")}
    init = O.bits_to_bf16(g["out_init_bits"]) if "out_init_bits" in g else torch.zeros((M, N), dtype=torch.bfloat16)
    out, parts = run(pkg, cuda, t["x_q"], t["x_scale"], t["packed"], t["scale"], t["zero"], t["offsets"], gs,
                     KERNELS[kernel], out=init.clone().to(cuda))
    rows = segment_rows(g["offsets"], M)
    np.testing.assert_array_equal(parts.cpu().numpy()[rows], g["partials"][rows])
    ref = O.bits_to_bf16(g["out_bits"])
    # rows outside every segment keep the caller's values, bit for bit
    np.testing.assert_array_equal(O.bf16_bits(out.cpu())[~rows], g["out_bits"][~rows])
    ref64 = O.group_gemm_f64(g["x_q"], g["x_scale"], g["packed"], g["scale"], g["zero"], g["offsets"], gs)
    assert_gemm_close(out, ref, ref64, N, rows)


@pytest.mark.parametrize("kernel", list(KERNELS))
@pytest.mark.parametrize("shape", [(4, 32, 512, 512, 128), (8, 64, 1024, 1024, 128), (8, 128, 1408, 2048, 128),
                                   (8, 256, 2048, 2048, 128), (16, 128, 1024, 1536, 64), (16, 256, 1536, 2048, 128),
                                   (32, 256, 1408, 2048, 128), (32, 512, 2048, 4096, 128),
                                   (64, 512, 1024, 2048, 128), (64, 1024, 2048, 4096, 128)])
def test_gemm_task1_shapes(pkg, cuda, shape, kernel):
    """The ten operator shapes of docs/Task1.md:30-41, random zero points and splits."""
    E, M, N, K, gs = shape
    x_q, xs, w, ws, wz, off = pkg.workloads.make_gemm_inputs(E, M, N, K, gs, seed=11, zero_mode="random")
    out, parts = run(pkg, cuda, x_q, xs, w, ws, wz, off, gs, KERNELS[kernel])
    ref = torch.zeros((M, N), dtype=torch.bfloat16)
    ref, ref_parts = O.group_gemm(x_q, xs, w, ws, wz, off, ref, gs, with_partials=True)
    rows = segment_rows(off, M)
    np.testing.assert_array_equal(parts.cpu().numpy()[rows], ref_parts[rows])
    ref64 = O.group_gemm_f64(x_q, xs, w, ws, wz, off, gs)
    assert_gemm_close(out, ref, ref64, N, rows)


@pytest.mark.parametrize("kernel", list(KERNELS))
def test_gemm_ragged_tiles_and_skew(pkg, cuda, kernel):
    """Segments of 1, 15, 16, 17, 127, 128, 129, 300 rows, an empty expert in
    the middle and at the end, K = 64 * odd (a half-filled last K block)."""
    counts = [1, 15, 0, 16, 17, 127, 128, 129, 300, 0]
    E = len(counts)
    off = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int32)
    M, N, K, gs = int(off[-1]), 256, 576, 64
    x_q, xs, w, ws, wz, _ = pkg.workloads.make_gemm_inputs(E, M, N, K, gs, seed=3, zero_mode="wrap", offsets=off)
    out, parts = run(pkg, cuda, x_q, xs, w, ws, wz, off, gs, KERNELS[kernel])
    ref, ref_parts = O.group_gemm(x_q, xs, w, ws, wz, off, torch.zeros((M, N), dtype=torch.bfloat16), gs,
                                  with_partials=True)
    np.testing.assert_array_equal(parts.cpu().numpy(), ref_parts)
    assert_gemm_close(out, ref, O.group_gemm_f64(x_q, xs, w, ws, wz, off, gs), N)


@pytest.mark.parametrize("kernel", list(KERNELS))
def test_gemm_strided_operands(pkg, cuda, kernel):
    E, M, N, K, gs = 4, 96, 384, 512, 128
    x_q, xs, w, ws, wz, off = pkg.workloads.make_gemm_inputs(E, M, N, K, gs, seed=5)
    ref = O.group_gemm(x_q, xs, w, ws, wz, off, torch.zeros((M, N), dtype=torch.bfloat16), gs)
    ref_bits = O.bf16_bits(ref)
    # x_q as a column slice of a wider buffer (row stride 2K), out as a slice with row stride 3N
    xbig = torch.zeros((M, 2 * K), dtype=torch.int8)
    xbig[:, K:] = x_q
    big = torch.full((M, 3 * N), 7.0, dtype=torch.bfloat16, device=cuda)
    out_view = big[:, N:2 * N]
    run(pkg, cuda, xbig[:, K:].to(cuda), xs, w, ws, wz, off, gs, KERNELS[kernel], out=out_view, partials=False)
    simt, _ = run(pkg, cuda, x_q, xs, w, ws, wz, off, gs, KERNELS["simt"], partials=False)
    if kernel in ("tc", "simt"):   # same fp32 recurrence -> identical bits
        np.testing.assert_array_equal(O.bf16_bits(out_view.cpu()), O.bf16_bits(simt.cpu()))
    else:
        assert_gemm_close(out_view, ref, O.group_gemm_f64(x_q, xs, w, ws, wz, off, gs), N)
    assert (big[:, :N] == 7.0).all() and (big[:, 2 * N:] == 7.0).all()
    # transposed output (column stride M)
    outT = torch.zeros((N, M), dtype=torch.bfloat16, device=cuda).t()
    run(pkg, cuda, x_q, xs, w, ws, wz, off, gs, KERNELS[kernel], out=outT, partials=False)
    if kernel in ("tc", "simt"):
        np.testing.assert_array_equal(O.bf16_bits(outT.cpu()), O.bf16_bits(simt.cpu()))
    else:
        assert_gemm_close(outT, ref, O.group_gemm_f64(x_q, xs, w, ws, wz, off, gs), N)
    assert_gemm_close(simt, ref, O.group_gemm_f64(x_q, xs, w, ws, wz, off, gs), N)
    del ref_bits


@pytest.mark.parametrize("shape,counts", [
    ((256, 512, 128), [16, 3, 40, 5]),          # <= 48 rows per expert: 64-token tiles
    ((256, 512, 128), [100, 129, 64, 111]),     # <= 160: 128-token tiles, a 1-row tail tile
    ((256, 512, 128), [300, 257, 0, 511]),      # > 160: 256-token tiles, tails of 44, 1 and 255 rows
    ((384, 1024, 64), [260, 0, 433]),           # > 160 with group size 64
])
def test_tc_tile_configurations(pkg, cuda, shape, counts):
    """The tensor-core kernel's three tile widths (chosen by the average rows
    per expert): exact int32 partials against the oracle, bf16 outputs
    identical to the CUDA-core kernel's (same fp32 group-scale recurrence)."""
    N, K, gs = shape
    E = len(counts)
    off = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int32)
    M = int(off[-1])
    x_q, xs, w, ws, wz, _ = pkg.workloads.make_gemm_inputs(E, M, N, K, gs, seed=M, zero_mode="wrap", offsets=off)
    out, parts = run(pkg, cuda, x_q, xs, w, ws, wz, off, gs, KERNELS["tc"])
    simt, _ = run(pkg, cuda, x_q, xs, w, ws, wz, off, gs, KERNELS["simt"], partials=False)
    ref, ref_parts = O.group_gemm(x_q, xs, w, ws, wz, off, torch.zeros((M, N), dtype=torch.bfloat16), gs,
                                  with_partials=True)
    np.testing.assert_array_equal(parts.cpu().numpy(), ref_parts)
    np.testing.assert_array_equal(O.bf16_bits(out.cpu()), O.bf16_bits(simt.cpu()))
    assert_gemm_close(out, ref, O.group_gemm_f64(x_q, xs, w, ws, wz, off, gs), N)


def test_gemm_empty_inputs(pkg, cuda):
    E, N, K, gs = 4, 256, 512, 128
    _, _, w, ws, wz, _ = pkg.workloads.make_gemm_inputs(E, 8, N, K, gs, seed=0)
    # M_total = 0
    x0 = torch.zeros((0, K), dtype=torch.int8, device=cuda)
    out0 = torch.zeros((0, N), dtype=torch.bfloat16, device=cuda)
    pkg.w4a8_group_gemm_moe(x0, torch.zeros(0, device=cuda), w.to(cuda), ws.to(cuda), wz.to(cuda),
                            torch.zeros(E + 1, dtype=torch.int32, device=cuda), out0, gs)
    # all experts empty: nothing written
    x = torch.ones((8, K), dtype=torch.int8, device=cuda)
    out = torch.full((8, N), 5.0, dtype=torch.bfloat16, device=cuda)
    pkg.w4a8_group_gemm_moe(x, torch.ones(8, device=cuda), w.to(cuda), ws.to(cuda), wz.to(cuda),
                            torch.zeros(E + 1, dtype=torch.int32, device=cuda), out, gs)
    torch.cuda.synchronize()
    assert (out == 5.0).all()
    assert pkg.device_status() == 0


def test_tc_and_simt_agree_at_full_size(pkg, cuda):
    """DeepSeek-V3 gate/up shape (E=256, N=4096, K=7168) at T=256 tokens x top-8:
    both kernels apply the same fp32 group-scale recurrence to exact int32
    partials, so their bf16 outputs agree bit for bit (size-independent check)."""
    W = pkg.workloads
    cfg = W.CONFIGS["deepseek"]
    gen = W.make_generator(0, cuda)
    E, N, K, gs = cfg.experts, 2 * cfg.inter, cfg.hidden, cfg.group_size
    w, ws, wz = W.make_int4_weights(E, N, K, gs, gen, cuda)
    inp = W.make_moe_inputs(cfg, 256, seed=1, device=cuda, weights=False)
    al = pkg.moe_align(inp.topk_ids, E)
    xq, xs = pkg.quant_scatter(inp.x, al.inv_pos, cfg.topk)
    R = xq.shape[0]
    a = torch.empty((R, N), dtype=torch.bfloat16, device=cuda)
    b = torch.empty((R, N), dtype=torch.bfloat16, device=cuda)
    pkg.w4a8_group_gemm_moe_ex(xq, xs, w, ws, wz, al.expert_offsets, a, gs, kernel=1)
    pkg.w4a8_group_gemm_moe_ex(xq, xs, w, ws, wz, al.expert_offsets, b, gs, kernel=2)
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    # spot-check a few rows against the CPU oracle
    off = al.expert_offsets.cpu()
    e = int(torch.argmax(off[1:] - off[:-1]))
    m0, m1 = int(off[e]), int(off[e + 1])
    sub_off = torch.tensor([0, m1 - m0], dtype=torch.int32)
    ref = O.group_gemm(xq[m0:m1].cpu(), xs[m0:m1].cpu(), w[e:e + 1].cpu(), ws[e:e + 1].cpu(), wz[e:e + 1].cpu(),
                       sub_off, torch.zeros((m1 - m0, N), dtype=torch.bfloat16), gs)
    ref64 = O.group_gemm_f64(xq[m0:m1].cpu(), xs[m0:m1].cpu(), w[e:e + 1].cpu(), ws[e:e + 1].cpu(),
                             wz[e:e + 1].cpu(), sub_off, gs)
    assert_gemm_close(a[m0:m1], ref, ref64, N)


@pytest.mark.parametrize("T", [16, 3])
def test_streaming_and_tc_partials_agree_at_decode_size(pkg, cuda, T):
    """DeepSeek-V3 gate/up (E=256, N=4096, K=7168) at decode token counts: the
    streaming kernel, the tensor-core kernel and the AUTO dispatch (which splits
    experts between them on the device) produce identical int32 partials; bf16
    outputs agree within the GEMM tolerance (different fp32 summation order)."""
    W = pkg.workloads
    cfg = W.CONFIGS["deepseek"]
    gen = W.make_generator(0, cuda)
    E, N, K, gs = cfg.experts, 2 * cfg.inter, cfg.hidden, cfg.group_size
    w, ws, wz = W.make_int4_weights(E, N, K, gs, gen, cuda, zero_mode="random")
    inp = W.make_moe_inputs(cfg, T, seed=4, device=cuda, weights=False)
    al = pkg.moe_align(inp.topk_ids, E)
    xq, xs = pkg.quant_scatter(inp.x, al.inv_pos, cfg.topk)
    R = xq.shape[0]
    G = K // gs
    res = {}
    for name, kern in (("gemv", 3), ("tc", 1), ("auto", 0)):
        out = torch.empty((R, N), dtype=torch.bfloat16, device=cuda)
        parts = torch.empty((R, N, G), dtype=torch.int32, device=cuda)
        pkg.w4a8_group_gemm_moe_ex(xq, xs, w, ws, wz, al.expert_offsets, out, gs, kernel=kern, partials=parts)
        torch.cuda.synchronize()
        res[name] = (out, parts)
    assert pkg.device_status() == 0
    assert torch.equal(res["gemv"][1], res["tc"][1])
    assert torch.equal(res["auto"][1], res["tc"][1])
    off = al.expert_offsets.cpu()
    e = int(torch.argmax(off[1:] - off[:-1]))
    m0, m1 = int(off[e]), int(off[e + 1])
    sub = torch.tensor([0, m1 - m0], dtype=torch.int32)
    args = (xq[m0:m1].cpu(), xs[m0:m1].cpu(), w[e:e + 1].cpu(), ws[e:e + 1].cpu(), wz[e:e + 1].cpu(), sub)
    ref = O.group_gemm(*args, torch.zeros((m1 - m0, N), dtype=torch.bfloat16), gs)
    ref64 = O.group_gemm_f64(*args, gs)
    for name in res:
        assert_gemm_close(res[name][0][m0:m1], ref, ref64, N)


@pytest.mark.parametrize("rows_per_expert", [1, 3, 40, 300])   # streaming, mixed, 64- and 256-token tiles
def test_gemm_row_address_store(pkg, cuda, rows_per_expert):
    """w4a8_group_gemm_moe_rows stores each row through a table of addresses
    (the tensor-core kernel via its staging output and 16-byte copies): rows
    sent to a permutation of another buffer's rows (0 = not stored) hold
    exactly the bits the strided store writes."""
    E, N, K = 8, 512, 1024
    M = E * rows_per_expert
    g = pkg.workloads.make_generator(M)
    x, xs, w, ws, wz, off = pkg.workloads.make_gemm_inputs(E, M, N, K, 128, seed=M)
    x, xs, w, ws, wz, off = (t.to(cuda) for t in (x, xs, w, ws, wz, off))
    ref = torch.zeros((M, N), dtype=torch.bfloat16, device=cuda)
    pkg.w4a8_group_gemm_moe(x, xs, w, ws, wz, off, ref, 128)
    perm = torch.randperm(M, generator=g).to(cuda)
    dst = torch.full((M, N), -1.0, dtype=torch.bfloat16, device=cuda)
    addr = dst.data_ptr() + perm.to(torch.int64) * (N * 2)
    skip = torch.arange(M, device=cuda) % 7 == 3
    addr[skip] = 0
    stage = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    lib = pkg._lib.load()
    rc = lib.w4a8_group_gemm_moe_rows(x.data_ptr(), K, xs.data_ptr(), w.data_ptr(), ws.data_ptr(), wz.data_ptr(),
                                      off.data_ptr(), stage.data_ptr(), addr.data_ptr(), M, E, N, K, 128, 0,
                                      torch.cuda.current_stream().cuda_stream)
    pkg._lib.check(rc, "w4a8_group_gemm_moe_rows")
    torch.cuda.synchronize()
    got = dst[perm]
    keep = ~skip & (torch.arange(M, device=cuda) < int(off[-1]))
    assert torch.equal(got[keep].view(torch.int16), ref[keep].view(torch.int16))
    assert bool((got[skip].float() == -1.0).all())
    assert pkg.device_status() == 0
