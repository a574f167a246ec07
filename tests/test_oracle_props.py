"""Properties of the oracle's restatements that have no reference code (align,
combine, quantiser edge cases), and of the seeded workloads."""
import numpy as np
import pytest
import torch
from hypothesis import given, settings, strategies as st


@settings(max_examples=40, deadline=None)
@given(T=st.integers(0, 40), k=st.integers(1, 8), E=st.integers(1, 20), bs=st.sampled_from([1, 16, 64, 128]),
       seed=st.integers(0, 1000), drop=st.booleans())
def test_align_is_a_stable_counting_sort(O, T, k, E, bs, seed, drop):
    rng = np.random.default_rng(seed)
    lo = -1 if drop else 0
    ids = rng.integers(lo, E + (1 if drop else 0), size=(T, k)).astype(np.int32)
    a = O.moe_align(ids, E, bs)
    flat = ids.reshape(-1)
    valid = (flat >= 0) & (flat < E)
    off = a["expert_offsets"]
    assert off[0] == 0 and off[-1] == valid.sum()
    for e in range(E):
        seg = a["sorted_ids"][off[e]:off[e + 1]]
        assert (flat[seg] == e).all()
        assert (np.diff(seg) > 0).all()          # stable: ascending flat index
    inv = a["inv_pos"]
    assert (inv[~valid] == -1).all()
    np.testing.assert_array_equal(a["sorted_ids"][inv[valid]], np.nonzero(valid)[0])
    # padded form
    R = T * k
    cap = R + E * (bs - 1)
    assert a["padded_ids"].shape[0] == cap
    assert a["num_post_pad"] % bs == 0
    real = a["padded_ids"][a["padded_ids"] != R]
    np.testing.assert_array_equal(np.sort(real), np.sort(a["sorted_ids"]))
    for b, e in enumerate(a["block_expert"]):
        rows = a["padded_ids"][b * bs:(b + 1) * bs]
        rows = rows[rows != R]
        if e < 0:
            assert b * bs >= a["num_post_pad"] and rows.size == 0
        else:
            assert (flat[rows] == e).all()


def test_combine_is_the_weighted_sum(O):
    rng = np.random.default_rng(0)
    T, k, H = 5, 3, 16
    y = torch.from_numpy(rng.standard_normal((T * k, H)).astype(np.float32)).to(torch.bfloat16)
    w = rng.random((T, k)).astype(np.float32)
    inv = rng.permutation(T * k).astype(np.int32)
    out = O.combine(y, inv, w)
    yf = y.to(torch.float32).numpy()
    ref = np.zeros((T, H), np.float32)
    for t in range(T):
        for j in range(k):
            ref[t] = ref[t] + np.float32(w[t, j]) * yf[inv[t * k + j]]
    np.testing.assert_array_equal(out.to(torch.float32).numpy(), torch.from_numpy(ref).to(torch.bfloat16).float().numpy())


def test_quantiser_edge_cases(O):
    x = torch.zeros((3, 256), dtype=torch.bfloat16)
    x[1, 0] = -5.0
    x[2] = torch.linspace(-1, 1, 256).to(torch.bfloat16)
    q, s = O.act_quant(x)
    assert s[0] == np.float32(1e-10) and (q[0] == 0).all()
    assert q[1, 0] == -127 and (q[1, 1:] == 0).all()
    assert q.min() >= -127 and q.max() <= 127
    # truncation toward zero, not rounding
    y = np.array([[127.0, 0.99, -0.99, 1.5, -1.5]], np.float32)
    qq, ss = O.quant_rows(y)
    assert ss[0] == 1.0 and list(qq[0]) == [127, 0, 0, 1, -1]


def test_workload_generators(pkg):
    W = pkg.workloads
    for name, cfg in W.CONFIGS.items():
        if cfg.experts * cfg.hidden * cfg.inter > 2 ** 28:
            continue
        inp = W.make_moe_inputs(cfg, 32, seed=0)
        assert inp.topk_ids.shape == (32, cfg.topk) and inp.topk_ids.dtype == torch.int32
        torch.testing.assert_close(inp.topk_weights.sum(-1), torch.ones(32))
        packed, scale, zero = inp.w13
        assert packed.dtype == torch.uint8 and (zero == 8).all()
        assert float(scale.min()) >= 0.005 and float(scale.max()) <= 0.02
    off = W.random_splits(16, 100, W.make_generator(0))
    assert off[0] == 0 and off[-1] == 100 and (off[1:] >= off[:-1]).all()


def test_zipf_routing_is_skewed(pkg):
    W = pkg.workloads
    cfg = W.CONFIGS["qwen3_zipf"]
    inp = W.make_moe_inputs(cfg, 1024, seed=0, weights=False)
    counts = np.bincount(inp.topk_ids.numpy().reshape(-1), minlength=cfg.experts)
    assert counts.max() > 10 * np.median(counts)


@pytest.mark.parametrize("seed,zipf", [(3, 1.2), (4, 0.0)])
def test_layer_on_a_token_subset_equals_the_full_layer(pkg, O, seed, zipf):
    """``moe_layer_tokens`` (used to check full-size layers on sampled
    tokens) gives exactly the full layer's rows for those tokens, with dropped
    slots and experts the subset does not use."""
    W = pkg.workloads
    cfg = W.MoEConfig("t", hidden=512, inter=256, experts=16, topk=4, zipf=zipf)
    inp = W.make_moe_inputs(cfg, 64, seed=seed, zero_mode="random")
    ids = inp.topk_ids.clone()
    ids[7, 1] = -1                     # a dropped slot
    full = O.moe_layer(inp.x, ids, inp.topk_weights, inp.w13, inp.w2, 128)
    toks = [5, 0, 63, 7, 17]
    sub = O.moe_layer_tokens(inp.x, ids, inp.topk_weights, inp.w13, inp.w2, 128, toks)
    np.testing.assert_array_equal(O.bf16_bits(full[toks]), O.bf16_bits(sub))


@pytest.mark.parametrize("scoring,E,k,T", [("softmax", 8, 2, 64), ("sigmoid", 256, 8, 300), ("softmax", 128, 8, 97),
                                           ("sigmoid", 3, 3, 5)])
def test_router_restatement_matches_the_benchmark_router(pkg, O, scoring, E, k, T):
    """The oracle's router (ranking by logit, ties to the lower index) picks the
    same experts in the same order as the torch router that makes the benchmark
    inputs (scores -> torch.topk -> renormalise), with weights within a few ulps."""
    g = pkg.workloads.make_generator(T + E)
    logits = torch.randn((T, E), generator=g, dtype=torch.float32)
    ids_t, w_t = pkg.workloads.route(logits, k, scoring)
    ids_o, w_o = O.route_topk(logits, k, scoring)
    np.testing.assert_array_equal(ids_o, ids_t.numpy())
    np.testing.assert_allclose(w_o, w_t.numpy(), rtol=2e-6, atol=0)


def test_router_ties_go_to_the_lower_index(O):
    logits = np.array([[1.0, 3.0, 3.0, -np.inf, 2.0, 3.0]], dtype=np.float32)
    ids, w = O.route_topk(logits, 4, "sigmoid")
    np.testing.assert_array_equal(ids, [[1, 2, 5, 4]])
    assert abs(float(w.sum()) - 1.0) < 1e-6


@pytest.mark.parametrize("fault", ["dropped_group", "scale_1pct", "swapped_rows"])
def test_layer_tolerance_rejects_planted_errors(pkg, O, fault):
    """The layer tolerance of the GPU tests (mean|out - ref| <= 1e-3 mean|ref|)
    rejects the errors it is meant to catch: a layer computed by the oracle
    with one K-group missing, every weight scale 1 % off, or two tokens'
    results swapped differs from the true layer by well over the bound."""
    cfg = pkg.workloads.CONFIGS["small"]
    inp = pkg.workloads.make_moe_inputs(cfg, 64, seed=3)
    ref = O.moe_layer(inp.x, inp.topk_ids, inp.topk_weights, inp.w13, None, cfg.group_size).float()
    packed, scale, zero = inp.w13
    if fault == "dropped_group":
        scale = scale.clone()
        scale[:, :, 3] = 0
    elif fault == "scale_1pct":
        scale = scale * 1.01
    bad = O.moe_layer(inp.x, inp.topk_ids, inp.topk_weights, (packed, scale, zero), None, cfg.group_size).float()
    if fault == "swapped_rows":
        bad = bad.clone()
        bad[[5, 9]] = bad[[9, 5]]
    rel = (bad - ref).abs().mean().item() / ref.abs().mean().item()
    assert rel > 5e-3, f"{fault}: relative mean error {rel:.3g} would pass a 1e-3 bound"


def test_prepack_layout_round_trip(O):
    """The prepack layout holds the same nibbles: unpacking it gives the
    reference layout's nibbles in k order, and it differs from the input
    (so a kernel reading it with the wrong layout would be caught)."""
    rng = np.random.default_rng(5)
    packed = rng.integers(0, 256, size=(3, 7, 64), dtype=np.uint8)
    pp = O.prepack(packed)
    assert pp.shape == packed.shape and pp.dtype == np.uint8
    np.testing.assert_array_equal(O.unpack_prepacked(pp), O.unpack_int4(packed))
    assert not np.array_equal(pp, packed)
