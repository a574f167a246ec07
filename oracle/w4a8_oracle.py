"""CPU restatement of the W4A8 MoE path -- TEST INFRASTRUCTURE ONLY (see
``oracle/__init__.py``: imported only by tests, smoke() and bench.py's CPU
legs, never by the product path).

Integer work (nibble unpack, zero fold, exact per-group partial sums, counting
sort) is numpy; the floating-point epilogue of the grouped GEMM uses the same
torch CPU operations, in the same order and on the same per-expert shapes, as
the reference implementation, so its bf16 output is identical to the
reference's on the same machine.
"""
from __future__ import annotations

import numpy as np
import torch


# ----------------------------------------------------------------------------- helpers
def _np(t):
    if isinstance(t, torch.Tensor):
        return t.detach().cpu().numpy()
    return np.asarray(t)


def _t(a):
    return a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit pattern (numpy has no bfloat16)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def bits_to_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


# ----------------------------------------------------------------------------- weights
def unpack_int4(packed) -> np.ndarray:
    """uint8 [..., K/2] -> int16 [..., K]; low nibble = even k, high nibble = odd k
    (docs/Task1.md:78-81)."""
    p = _np(packed).astype(np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.int16)
    out[..., 0::2] = p & 0x0F
    out[..., 1::2] = (p >> 4) & 0x0F
    return out


def prepack(packed) -> np.ndarray:
    """The word-interleaved prepack layout of ``w4a8_prepack_weights``: in
    each 32-bit word q of a row (k = 8q .. 8q + 7), byte b holds k = 8q + b
    in its low nibble and k = 8q + 4 + b in its high nibble."""
    nib = unpack_int4(packed).astype(np.uint8)                  # [..., K]
    w = nib.reshape(nib.shape[:-1] + (-1, 2, 4))                # [..., K/8, half, b]
    return (w[..., 0, :] | (w[..., 1, :] << 4)).reshape(nib.shape[:-1] + (-1,)).astype(np.uint8)


def unpack_prepacked(packed) -> np.ndarray:
    """uint8 [..., K/2] in the prepack layout -> nibbles int16 [..., K] in k order."""
    p = _np(packed).astype(np.uint8).reshape(_np(packed).shape[:-1] + (-1, 4))
    lo, hi = p & 0x0F, (p >> 4) & 0x0F
    return np.concatenate([lo, hi], axis=-1).reshape(p.shape[:-2] + (-1,)).astype(np.int16)


def fold_zero(w_int4: np.ndarray, w_zero, group_size: int) -> np.ndarray:
    """int8(nibble - zero) with the per-group zero broadcast over K; the int16
    difference wraps on the cast exactly like ``.to(torch.int8)``
    (docs/Task1.md:84-85)."""
    z = _np(w_zero).astype(np.int16)
    zz = np.repeat(z, group_size, axis=-1)
    return (w_int4.astype(np.int16) - zz).astype(np.int8)


def signed_weights(w_q4_packed, w_zero, group_size: int) -> np.ndarray:
    """int8(nibble - zero) [..., K]: ``unpack_int4`` then ``fold_zero``, written
    with the reference's own torch operations (nibbles widened to int16, the
    per-group zero subtracted, ``.to(torch.int8)`` wrapping;
    docs/Task1.md:78-85) because they run multi-threaded: ten times faster
    than the numpy pair on the multi-GB expert tensors of the large configs.
    The golden tests check both forms against the reference bit for bit."""
    p = _t(w_q4_packed).to(torch.uint8)
    nib = torch.stack([p & 0x0F, p >> 4], dim=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)
    z = _t(w_zero).to(torch.int16).repeat_interleave(group_size, dim=-1)
    return (nib.to(torch.int16) - z).to(torch.int8).numpy()


# ----------------------------------------------------------------------------- grouped GEMM
def group_partials(x_q, w_signed: np.ndarray, group_size: int) -> np.ndarray:
    """Exact int32 partial sums P[m, n, g] = sum_{k in g} x[m,k] * w[n,k]
    (the einsum of docs/Task1.md:100-104).  float64 BLAS products are exact
    here: |terms| <= 2^14 and |sums| <= 2^21 < 2^53."""
    x = _np(x_q).astype(np.float64)
    w = w_signed.astype(np.float64)
    m, K = x.shape
    N = w.shape[0]
    G = K // group_size
    xg = x.reshape(m, G, group_size).transpose(1, 0, 2)      # [G, m, gs]
    wg = w.reshape(N, G, group_size).transpose(1, 2, 0)      # [G, gs, N]
    p = np.matmul(xg, wg)                                    # [G, m, N]
    return np.ascontiguousarray(p.transpose(1, 2, 0)).astype(np.int32)


def segments(expert_offsets, M_total: int):
    """(e, m0, m1) for non-empty segments, following the reference loop
    (docs/Task1.md:88-92) with Python-slice clamping to [0, M_total]."""
    off = _np(expert_offsets).astype(np.int64)
    E = off.shape[0] - 1
    for e in range(E):
        m0 = int(min(max(off[e], 0), M_total))
        m1 = int(min(max(off[e + 1], 0), M_total))
        if m1 <= m0:
            continue
        yield e, m0, m1


def group_gemm(x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, out: torch.Tensor,
               group_size: int, with_partials: bool = False):
    """Restatement of the reference W4A8 grouped GEMM (docs/Task1.md:53-114).

    Per expert (the reference loops experts independently, so unpacking one
    expert's slice at a time is the same computation without the E*N*K
    temporaries): unpack + zero fold (:78-85), per-group partials as an fp32
    einsum (:100-104), fp32 group-scale reduction (:107), token scale (:110),
    bf16 store into ``out`` (:112).  Rows outside every segment are untouched.
    Returns ``out`` (and the int32 partials [M_total, N, G] when asked; rows
    outside segments are zero there).
    """
    x_q = _t(x_q)
    x_scale = _t(x_scale).to(torch.float32)
    packed = _t(w_q4_packed)
    ws = _t(w_scale).to(torch.float32)
    wz = _t(w_zero)
    M_total, K = x_q.shape
    E, N, K_half = packed.shape
    assert K_half * 2 == K
    assert K % group_size == 0
    G = K // group_size
    parts = np.zeros((M_total, N, G), dtype=np.int32) if with_partials else None
    for e, m0, m1 in segments(expert_offsets, M_total):
        w_signed = torch.from_numpy(signed_weights(packed[e], wz[e], group_size))
        xg = x_q[m0:m1].reshape(-1, G, group_size).to(torch.float32)
        wg = w_signed.reshape(N, G, group_size).to(torch.float32)
        partial = torch.einsum("mgk,ngk->mng", xg, wg)
        acc = (partial * ws[e].unsqueeze(0)).sum(dim=-1)
        acc = acc * x_scale[m0:m1].unsqueeze(-1)
        out[m0:m1].copy_(acc.to(out.dtype))
        if parts is not None:
            parts[m0:m1] = partial.to(torch.int32).numpy()
    if with_partials:
        return out, parts
    return out


def group_gemm_f64(x_q, x_scale, w_q4_packed, w_scale, w_zero, expert_offsets, group_size: int) -> np.ndarray:
    """High-precision dequant reference: out[m, n] = xs[m] * sum_g ws[e,n,g] * P[m,n,g]
    evaluated in float64 from the exact integer partials (rows outside every
    segment are NaN).  Used to measure the error of bf16 outputs."""
    x_q = _np(x_q)
    xs = _np(x_scale).astype(np.float64)
    ws = _np(w_scale).astype(np.float64)
    M_total, K = x_q.shape
    E, N, _ = _np(w_q4_packed).shape
    out = np.full((M_total, N), np.nan, dtype=np.float64)
    for e, m0, m1 in segments(expert_offsets, M_total):
        p = group_partials(x_q[m0:m1], signed_weights(_np(w_q4_packed)[e], _np(w_zero)[e], group_size), group_size)
        out[m0:m1] = (p.astype(np.float64) * ws[e][None]).sum(-1) * xs[m0:m1, None]
    return out


# ----------------------------------------------------------------------------- quantisers
def quant_rows(y32: np.ndarray):
    """Per-row symmetric int8 (docs/Task3.md:58-67 with the group = the whole
    row): scale = max(amax / 127, 1e-10) in fp32, q = trunc(clamp(y/scale, -127, 127))."""
    y = y32.astype(np.float32)
    amax = np.abs(y).max(axis=-1) if y.shape[-1] else np.zeros(y.shape[:-1], np.float32)
    s = np.maximum(amax / np.float32(127.0), np.float32(1e-10)).astype(np.float32)
    q = np.clip(y / s[..., None], np.float32(-127.0), np.float32(127.0))
    return np.trunc(q).astype(np.int8), s


def act_quant(x_bf16: torch.Tensor):
    """bf16 [T, H] -> (int8 [T, H], fp32 [T]) with the per-token quantiser."""
    return quant_rows(x_bf16.to(torch.float32).numpy())


def silu_mul_requant(h_bf16: torch.Tensor):
    """gate = h[:, :I], up = h[:, I:]; y = (gate * sigmoid(gate)) * up in fp32
    (docs/Task3.md:99-110), then the per-row quantiser."""
    I = h_bf16.shape[1] // 2
    gate = h_bf16[:, :I].to(torch.float32)
    up = h_bf16[:, I:].to(torch.float32)
    y = (gate * torch.sigmoid(gate)) * up
    return quant_rows(y.numpy())


# ----------------------------------------------------------------------------- router
def route_topk(logits, topk: int, scoring: str, renormalize: bool = True):
    """Routing of the benchmark inputs (softmax or sigmoid of fp32 logits [T, E]
    -> top-k -> weights / their sum; the reference takes routing as given,
    docs/Task1.md:13).  Ranking: descending logit, ties to the lower expert
    index (the scores are increasing functions of the logits, so this is their
    top-k order).  Scores are fp32; returns (ids int32 [T, k], weights fp32 [T, k])."""
    lg = np.asarray(_np(logits), dtype=np.float32)
    T, E = lg.shape
    order = np.lexsort((np.broadcast_to(np.arange(E), (T, E)), -lg), axis=-1)[:, :topk]
    top = np.take_along_axis(lg, order, axis=-1)
    if scoring == "softmax":
        mx = lg.max(axis=-1, keepdims=True)
        den = np.exp(lg - mx, dtype=np.float32).sum(axis=-1, keepdims=True, dtype=np.float32)
        sc = (np.exp(top - mx, dtype=np.float32) / den).astype(np.float32)
    else:
        sc = (np.float32(1.0) / (np.float32(1.0) + np.exp(-top, dtype=np.float32))).astype(np.float32)
    if renormalize:
        sc = (sc / sc.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return order.astype(np.int32), sc


# ----------------------------------------------------------------------------- align / combine
def moe_align(topk_ids, E: int, block_size: int):
    """Stable counting sort of flat (token, slot) indices by expert.

    Returns dict with expert_offsets [E+1], sorted_ids [R], inv_pos [R] (-1 for
    ids outside [0, E)), padded_ids [R + E*(bs-1)] (sentinel R), block_expert
    [ceil(cap/bs)] (-1 past the end), num_post_pad."""
    ids = _np(topk_ids).astype(np.int64).reshape(-1)
    R = ids.shape[0]
    valid = (ids >= 0) & (ids < E)
    counts = np.bincount(ids[valid], minlength=E).astype(np.int64)
    off = np.zeros(E + 1, dtype=np.int64)
    off[1:] = np.cumsum(counts)
    order = np.argsort(np.where(valid, ids, E), kind="stable")[: int(valid.sum())]
    sorted_ids = order.astype(np.int32)
    inv = np.full(R, -1, dtype=np.int32)
    inv[order] = np.arange(order.shape[0], dtype=np.int32)
    padded_counts = (counts + block_size - 1) // block_size * block_size
    poff = np.zeros(E + 1, dtype=np.int64)
    poff[1:] = np.cumsum(padded_counts)
    cap = R + E * (block_size - 1)
    padded = np.full(cap, R, dtype=np.int32)
    for e in range(E):
        padded[poff[e]: poff[e] + counts[e]] = sorted_ids[off[e]: off[e + 1]]
    nblk = (cap + block_size - 1) // block_size
    block_expert = np.full(nblk, -1, dtype=np.int32)
    for e in range(E):
        block_expert[poff[e] // block_size: poff[e + 1] // block_size] = e
    return dict(expert_offsets=off.astype(np.int32), sorted_ids=sorted_ids, inv_pos=inv,
                padded_ids=padded, block_expert=block_expert, num_post_pad=int(poff[E]))


def combine(y_bf16: torch.Tensor, inv_pos, topk_w) -> torch.Tensor:
    """out[t] = bf16(sum_{j ascending} w[t, j] * y[inv_pos[t*k + j]]); each
    product and sum rounded to fp32."""
    w = _np(topk_w).astype(np.float32)
    T, k = w.shape
    pos = _np(inv_pos).reshape(T, k)
    y = y_bf16.to(torch.float32).numpy()
    acc = np.zeros((T, y.shape[1]), dtype=np.float32)
    for j in range(k):
        p = pos[:, j]
        ok = p >= 0
        term = np.zeros_like(acc)
        term[ok] = (w[ok, j][:, None] * y[p[ok]]).astype(np.float32)
        acc = (acc + term).astype(np.float32)
    return torch.from_numpy(acc).to(torch.bfloat16)


# ----------------------------------------------------------------------------- routed layer
def moe_layer(x_bf16: torch.Tensor, topk_ids, topk_w, w13, w2, group_size: int, block_size: int = 128,
              return_intermediates: bool = False):
    """Routed W4A8 MoE on the CPU, composed from the restatements above and the
    reference GEMM (gate/up -> SiLU-mul requant -> down -> combine; or a single
    up GEMM when ``w2`` is None)."""
    T, H = x_bf16.shape
    k = topk_ids.shape[1]
    E = w13[0].shape[0]
    al = moe_align(topk_ids, E, block_size)
    R = int(al["expert_offsets"][-1])
    xq_tok, xs_tok = act_quant(x_bf16)
    src_tok = al["sorted_ids"] // k
    xq = torch.from_numpy(xq_tok[src_tok])
    xs = torch.from_numpy(xs_tok[src_tok])
    off = torch.from_numpy(al["expert_offsets"])
    n13 = w13[0].shape[1]
    h = torch.zeros((R, n13), dtype=torch.bfloat16)
    group_gemm(xq, xs, w13[0], w13[1], w13[2], off, h, group_size)
    inter = dict(align=al, xq=xq, xs=xs, h=h)
    if w2 is not None:
        aq, as_ = silu_mul_requant(h)
        y = torch.zeros((R, w2[0].shape[1]), dtype=torch.bfloat16)
        group_gemm(torch.from_numpy(aq), torch.from_numpy(as_), w2[0], w2[1], w2[2], off, y, group_size)
        inter.update(aq=aq, as_=as_, y=y)
    else:
        y = h
    out = combine(y, al["inv_pos"], topk_w)
    return (out, inter) if return_intermediates else out


# ----------------------------------------------------------------------------- tolerance
def gems_assert_close(actual: torch.Tensor, expected: torch.Tensor, N: int) -> None:
    """The reference's correctness rule for bf16 outputs: rtol = 0.016,
    atol = 1e-4 * N (docs/Task1.md:45; flag_gems itself is not installed, so
    the check is restated with torch.testing.assert_close)."""
    torch.testing.assert_close(actual.to(torch.float32), expected.to(torch.float32), rtol=0.016,
                               atol=1e-4 * N)


def error_stats(out_bf16: torch.Tensor, ref64: np.ndarray) -> dict:
    """max rel err with floor 1e-2 * max|ref|, mean abs err (vs the float64 reference),
    and the same for the bf16 rounding of the reference itself (the floor any
    bf16 output has)."""
    o = out_bf16.to(torch.float32).numpy().astype(np.float64)
    mask = ~np.isnan(ref64)
    r = ref64[mask]
    o = o[mask]
    floor = 1e-2 * np.abs(r).max() if r.size else 1.0
    rel = np.abs(o - r) / (np.abs(r) + floor)
    r_bf = torch.from_numpy(r.astype(np.float32)).to(torch.bfloat16).to(torch.float64).numpy()
    return dict(max_rel=float(rel.max()) if r.size else 0.0,
                mean_abs=float(np.abs(o - r).mean()) if r.size else 0.0,
                bf16_floor_mean_abs=float(np.abs(r_bf - r).mean()) if r.size else 0.0,
                mean_abs_ref=float(np.abs(r).mean()) if r.size else 0.0)


def moe_layer_tokens(x_bf16: torch.Tensor, topk_ids, topk_w, w13, w2, group_size: int, tokens,
                     block_size: int = 128) -> torch.Tensor:
    """``moe_layer`` for the tokens listed in ``tokens`` only (rows in that order).

    A token's output depends only on its own activations, its k (expert,
    weight) pairs and those experts' weights: the other tokens change only the
    order of rows inside an expert segment, and every row of the reference
    GEMM is computed on its own.  So the layer restricted to a token subset,
    with the experts that subset uses renumbered densely, gives the same
    output rows.  ``w13`` / ``w2`` may live on any device; only the used
    experts' slices are copied to the CPU, which keeps full-size checks of the
    large configurations (GBs of expert weights) cheap."""
    sel = torch.as_tensor(tokens, dtype=torch.long)
    ids = _t(topk_ids).cpu().to(torch.int64)[sel]
    E = w13[0].shape[0]
    ok = (ids >= 0) & (ids < E)
    used = torch.unique(ids[ok])
    remap = torch.full((E,), -1, dtype=torch.int64)
    remap[used] = torch.arange(used.numel())
    ids_c = torch.where(ok, remap[ids.clamp(0, E - 1)], torch.full_like(ids, -1)).to(torch.int32)

    def take(w):
        if w is None:
            return None
        idx = used.to(w[0].device)
        return tuple(t.index_select(0, idx).cpu() for t in w)

    return moe_layer(x_bf16.cpu()[sel], ids_c, _t(topk_w).cpu()[sel], take(w13), take(w2), group_size, block_size)
