"""GPU parity of the offline weight prepack (w4a8_prepack_weights) and of the
grouped GEMMs on prepacked weights (w4a8_group_gemm_moe_prepacked): the
prepack kernel's bytes equal the oracle's restatement of the layout, and
every kernel gives the same int32 partials and bf16 bits on prepacked
weights as on the reference layout (the layout changes no arithmetic)."""
import numpy as np
import pytest
import torch

from gpu_util import O

pytestmark = pytest.mark.gpu

KERNELS = {"auto": 0, "tc": 1, "simt": 2, "gemv": 3}


def test_prepack_kernel_matches_oracle(pkg, cuda):
    g = pkg.workloads.make_generator(11)
    w, _, _ = pkg.workloads.make_int4_weights(4, 96, 1024, 128, g)
    got = pkg.prepack_weights(w.to(cuda))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), O.prepack(w))
    inplace = w.to(cuda)
    pkg.prepack_weights(inplace, out=inplace)
    torch.cuda.synchronize()
    assert torch.equal(inplace.cpu(), got.cpu())


@pytest.mark.parametrize("kernel", list(KERNELS))
@pytest.mark.parametrize("E,M,N,K,gs,zero_mode", [
    (8, 256, 512, 1024, 128, "random"),   # tensor-core tiles
    (16, 20, 384, 2048, 64, "wrap"),       # gs 64, zero points that wrap int8
    (32, 2, 1024, 4096, 128, "random"),    # decode: streaming kernel
])
def test_prepacked_gemm_matches_reference_layout(pkg, cuda, kernel, E, M, N, K, gs, zero_mode):
    x, xs, w, ws, wz, off = pkg.workloads.make_gemm_inputs(E, E * M, N, K, gs, seed=E + K, zero_mode=zero_mode)
    x, xs, w, ws, wz, off = (t.to(cuda) for t in (x, xs, w, ws, wz, off))
    R, G = E * M, K // gs
    ref = torch.zeros((R, N), dtype=torch.bfloat16, device=cuda)
    ref_p = torch.zeros((R, N, G), dtype=torch.int32, device=cuda)
    pkg.w4a8_group_gemm_moe_ex(x, xs, w, ws, wz, off, ref, gs, kernel=KERNELS[kernel], partials=ref_p)
    wp = pkg.prepack_weights(w)
    got = torch.zeros_like(ref)
    got_p = torch.zeros_like(ref_p)
    pkg.w4a8_group_gemm_moe_ex(x, xs, wp, ws, wz, off, got, gs, kernel=KERNELS[kernel], partials=got_p,
                               prepacked=True)
    torch.cuda.synchronize()
    assert torch.equal(got_p, ref_p)
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    assert pkg.device_status() == 0


def test_prepacked_layer_matches(pkg, cuda):
    cfg = pkg.workloads.MoEConfig("t", hidden=1024, inter=512, experts=16, topk=4)
    inp = pkg.workloads.make_moe_inputs(cfg, 200, seed=9)
    w13 = pkg.W4A8Weights(*[t.to(cuda) for t in inp.w13])
    w2 = pkg.W4A8Weights(*[t.to(cuda) for t in inp.w2])
    args = (inp.x.to(cuda), inp.topk_ids.to(cuda), inp.topk_weights.to(cuda))
    ref = pkg.MoELayer(w13, w2, cfg.group_size, cfg.topk, 200)(*args).clone()
    got = pkg.MoELayer(w13, w2, cfg.group_size, cfg.topk, 200, prepack=True)(*args)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
