"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch

from oracle import w4a8_oracle as O

# Tolerances for bf16 outputs of the grouped GEMM (written here, used by every test):
#  * the reference's own rule: gems_assert_close rtol=0.016, atol=1e-4*N (docs/Task1.md:45)
#  * max relative error <= 1e-2 against the float64 dequant reference, with the
#    relative error defined as |out - ref| / (|ref| + 1e-2 * max|ref|)
#  * mean |out - oracle| <= 1e-3 * mean|oracle| against the reference-identical
#    bf16 oracle (an absolute 1e-3 is below the bf16 rounding floor at these
#    magnitudes, so the bound is normalised by the output scale)
#  * mean abs error against float64 no worse than 1.25x that of bf16 rounding itself
MAX_REL = 1e-2
MEAN_ABS_NORM = 1e-3
FLOOR_FACTOR = 1.25


def to_dev(dev, *ts):
    return [t.to(dev) if isinstance(t, torch.Tensor) else t for t in ts]


def assert_gemm_close(out_gpu: torch.Tensor, out_oracle: torch.Tensor, ref64: np.ndarray, N: int,
                      rows: np.ndarray | None = None):
    g = out_gpu.cpu()
    o = out_oracle.cpu()
    if rows is not None:
        g, o, ref64 = g[rows], o[rows], ref64[rows]
    if g.numel() == 0:
        return
    O.gems_assert_close(g, o, N)
    st = O.error_stats(g, ref64)
    assert st["max_rel"] <= MAX_REL, st
    assert st["mean_abs"] <= FLOOR_FACTOR * st["bf16_floor_mean_abs"] + 1e-12, st
    gf, of = g.float(), o.float()
    assert (gf - of).abs().mean().item() <= MEAN_ABS_NORM * of.abs().mean().item() + 1e-12


def segment_rows(offsets, M):
    rows = np.zeros(M, dtype=bool)
    for _, m0, m1 in O.segments(offsets, M):
        rows[m0:m1] = True
    return rows


# Tolerance of a routed layer's bf16 output against the oracle layer (used by
# every layer test):
#  * elementwise the reference's bf16 rule, rtol 0.016 and atol 1e-4 * N with
#    N the output width (docs/Task1.md:45);
#  * on average mean|out - ref| <= 1e-3 * mean|ref| (a quarter of one bf16
#    rounding step).
# Why a correct implementation meets it: the GPU layer and the oracle compute
# the same exact integer partials and the same quantisers; they differ only in
# fp32 summation order and in expf against the CPU's sigmoid.  Such a
# difference can move one bf16 rounding of h or y, or one int8 truncation of
# the requant, by a single step, and one step of one of the I inputs of a
# down-GEMM row changes that row by a fraction of a percent of one term.  A CPU
# emulation of exactly these differences (float64 group-scale sums and
# sigmoid in the oracle) moved layer outputs by 2.5e-5 to 6e-5 of mean|ref| on
# average, within the elementwise rule everywhere.
LAYER_MEAN_NORM = 1e-3


def assert_layer_close(out: torch.Tensor, ref: torch.Tensor, N: int, what: str = "layer"):
    o = out.cpu().float()
    r = ref.cpu().float()
    assert o.shape == r.shape, (o.shape, r.shape)
    O.gems_assert_close(o, r, N)
    mean_err = (o - r).abs().mean().item()
    mean_ref = r.abs().mean().item()
    assert mean_err <= LAYER_MEAN_NORM * mean_ref + 1e-12, f"{what}: mean|out-ref| {mean_err:.4g} vs mean|ref| {mean_ref:.4g}"
    return mean_err / max(mean_ref, 1e-30)
