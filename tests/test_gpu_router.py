"""GPU parity of the router + top-k kernel (w4a8_router_topk) against the
oracle's restatement and the torch router that makes the benchmark inputs:
expert ids exact (order included), renormalised weights within a few ulps
(the GPU's expf and its summation order differ from the CPU's by ulps), and
the fused quantisation bit-exact against the act-quant oracle."""
import numpy as np
import pytest
import torch

from gpu_util import O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("scoring,E,k,T", [
    ("sigmoid", 256, 8, 16384),   # DeepSeek-V3 routing at the benchmark's token count
    ("softmax", 8, 2, 64),        # configs 0 / 1
    ("softmax", 128, 8, 4096),    # Qwen3 shape
    ("sigmoid", 3, 3, 7),         # topk == E
    ("softmax", 1024, 32, 33),    # largest E and topk
    ("sigmoid", 300, 5, 0),       # empty batch
])
def test_router_matches_oracle_and_torch(pkg, cuda, scoring, E, k, T):
    g = pkg.workloads.make_generator(E * 31 + k)
    logits = torch.randn((T, E), generator=g, dtype=torch.float32)
    ids, w = pkg.router_topk(logits.to(cuda), k, scoring)
    torch.cuda.synchronize()
    ids_o, w_o = O.route_topk(logits, k, scoring)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    np.testing.assert_allclose(w.cpu().numpy(), w_o, rtol=4e-6, atol=0)
    if T:
        ids_t, w_t = pkg.workloads.route(logits, k, scoring)
        np.testing.assert_array_equal(ids.cpu().numpy(), ids_t.numpy())
        np.testing.assert_allclose(w.cpu().numpy(), w_t.numpy(), rtol=4e-6, atol=0)


def test_router_ties_masked_experts_and_no_renormalisation(pkg, cuda):
    logits = torch.tensor([[1.0, 3.0, 3.0, float("-inf"), 2.0, 3.0],
                           [float("-inf")] * 5 + [0.5],
                           [0.0] * 6], dtype=torch.float32)
    ids, w = pkg.router_topk(logits.to(cuda), 4, "sigmoid", renormalize=False)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), [[1, 2, 5, 4], [5, 0, 1, 2], [0, 1, 2, 3]])
    ids_o, w_o = O.route_topk(logits, 4, "sigmoid", renormalize=False)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    np.testing.assert_allclose(w.cpu().numpy(), w_o, rtol=4e-6, atol=0)


@pytest.mark.parametrize("T,H", [(16, 7168), (257, 4096), (5, 1000)])
def test_router_fused_quantisation_is_bit_exact(pkg, cuda, T, H):
    g = pkg.workloads.make_generator(T + H)
    logits = torch.randn((T, 256), generator=g, dtype=torch.float32)
    x = (torch.randn((T, H), generator=g) * 2).to(torch.bfloat16)
    ids, w, xq, xs = pkg.router_topk(logits.to(cuda), 8, "sigmoid", x=x.to(cuda))
    torch.cuda.synchronize()
    rq, rs = O.act_quant(x)
    np.testing.assert_array_equal(xq.cpu().numpy(), rq)
    np.testing.assert_array_equal(xs.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    np.testing.assert_array_equal(ids.cpu().numpy(), O.route_topk(logits, 8, "sigmoid")[0])


def test_router_rejects_bad_arguments(pkg, cuda):
    logits = torch.zeros((4, 16), dtype=torch.float32, device=cuda)
    for k in (0, 17, 33):
        with pytest.raises(RuntimeError):
            pkg.router_topk(logits, k, "softmax")
    with pytest.raises(RuntimeError):
        pkg.router_topk(torch.zeros((4, 1025), dtype=torch.float32, device=cuda), 8, "softmax")
