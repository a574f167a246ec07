"""w4a8_moe_align_noalloc: the align entry point for callers that cannot
allocate device memory (for example a server whose memory pool already owns
all free device memory, or a plain C caller without an allocator).  It keeps
its scratch in a fixed array inside the library instead of a caller
workspace.

Called through the C ABI, it must give the same outputs as w4a8_moe_align
(integer outputs: bit for bit) on two calls in a row, since every call reuses
the same scratch array.  This file is named so that pytest collects it last.
"""
import ctypes
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


def _outputs(R, E, bs, dev):
    cap = R + E * (bs - 1)
    nblk = (cap + bs - 1) // bs
    i32 = dict(dtype=torch.int32, device=dev)
    return dict(off=torch.full((E + 1,), -7, **i32), sorted=torch.full((R,), -7, **i32),
                inv=torch.full((R,), -7, **i32), padded=torch.full((cap,), -7, **i32),
                blk=torch.full((nblk,), -7, **i32), npp=torch.full((1,), -7, **i32))


def _call(lib, ids, E, bs, o, stream, workspace=None):
    T, k = ids.shape
    args = [ids.data_ptr(), T, k, E, bs, o["off"].data_ptr(), o["sorted"].data_ptr(), o["inv"].data_ptr(),
            o["padded"].data_ptr(), o["blk"].data_ptr(), o["npp"].data_ptr()]
    if workspace is None:
        return lib.w4a8_moe_align_noalloc(*args, stream)
    return lib.w4a8_moe_align(*args, workspace.data_ptr(), workspace.numel(), stream)


def test_noalloc_align_matches_workspace_align_twice(cuda):
    L = importlib.import_module("flagos-kernel-gen_b200._lib")
    W = importlib.import_module("flagos-kernel-gen_b200.workloads")
    lib = L.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    cases = [("deepseek", 4096, 128), ("qwen3_zipf", 3000, 64)]   # second call reuses the scratch
    for name, T, bs in cases:
        cfg = W.CONFIGS[name]
        ids = W.make_moe_inputs(cfg, T, seed=21, weights=False).topk_ids.to(cuda).contiguous()
        E, R = cfg.experts, ids.numel()
        ws = torch.empty((lib.w4a8_moe_align_workspace_size(T, cfg.topk, E),), dtype=torch.uint8, device=cuda)
        ref = _outputs(R, E, bs, cuda)
        got = _outputs(R, E, bs, cuda)
        assert _call(lib, ids, E, bs, ref, stream, workspace=ws) == L.W4A8_OK, lib.w4a8_last_error()
        rc = _call(lib, ids, E, bs, got, stream)
        assert rc == L.W4A8_OK, lib.w4a8_last_error()
        torch.cuda.synchronize()
        for key in ref:
            assert torch.equal(got[key], ref[key]), f"{name}: {key} differs"
    # the documented maximum (T*topk = 131072 slots over E = 512 experts, which
    # fills almost all of the fixed scratch), then a call that asks for no
    # padded outputs (padded_ids, block_expert, num_post_pad = NULL)
    T, k, E, bs = 16384, 8, 512, 128
    gen = torch.Generator(device=cuda)
    gen.manual_seed(3)
    ids = torch.randint(0, E, (T, k), generator=gen, device=cuda, dtype=torch.int32)
    ws = torch.empty((lib.w4a8_moe_align_workspace_size(T, k, E),), dtype=torch.uint8, device=cuda)
    ref = _outputs(T * k, E, bs, cuda)
    got = _outputs(T * k, E, bs, cuda)
    assert _call(lib, ids, E, bs, ref, stream, workspace=ws) == L.W4A8_OK, lib.w4a8_last_error()
    assert _call(lib, ids, E, bs, got, stream) == L.W4A8_OK, lib.w4a8_last_error()
    torch.cuda.synchronize()
    for key in ref:
        assert torch.equal(got[key], ref[key]), f"maximum size: {key} differs"
    part = _outputs(T * k, E, bs, cuda)
    rc = lib.w4a8_moe_align_noalloc(ids.data_ptr(), T, k, E, bs, part["off"].data_ptr(), part["sorted"].data_ptr(),
                                    part["inv"].data_ptr(), None, None, None, stream)
    assert rc == L.W4A8_OK, lib.w4a8_last_error()
    torch.cuda.synchronize()
    for key in ("off", "sorted", "inv"):
        assert torch.equal(part[key], ref[key]), f"without padded outputs: {key} differs"
    # beyond the fixed scratch size: a clear error, and nothing launched
    big = torch.zeros((16385, 8), dtype=torch.int32, device=cuda)
    o = _outputs(8, 8, 1, cuda)
    rc = lib.w4a8_moe_align_noalloc(big.data_ptr(), 16385, 8, 256, 128, o["off"].data_ptr(), o["sorted"].data_ptr(),
                                    o["inv"].data_ptr(), None, None, None, stream)
    assert rc == L.W4A8_ERR_INVALID
    assert b"131072" in lib.w4a8_last_error()
