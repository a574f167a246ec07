"""CPU-only checks of the drop-in boundary: the C-ABI library loads, exports
every entry point declared in include/w4a8moe.h, validates arguments without
touching a GPU, and the Python mirror keeps the reference's signature and
error behaviour (docs/Task1.md:8-17, :74-75).  No compute call is made."""
import ctypes
import inspect
import os
import re
import subprocess

import pytest
import torch

from conftest import REPO

HEADER = os.path.join(REPO, "include", "w4a8moe.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(w4a8_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for required in ("w4a8_group_gemm_moe", "w4a8_group_gemm_moe_ex", "w4a8_act_quant", "w4a8_quant_scatter",
                     "w4a8_moe_align", "w4a8_moe_align_workspace_size", "w4a8_silu_mul_requant",
                     "w4a8_moe_combine", "w4a8_device_status", "w4a8_last_error", "w4a8_abi_version"):
        assert required in names


def test_library_exports_every_declared_symbol(pkg):
    from importlib import import_module
    lib_mod = import_module("flagos-kernel-gen_b200._lib")
    lib = lib_mod.load()
    out = subprocess.run(["nm", "-D", "--defined-only", lib_mod.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT\s+(w4a8_\w+)", out))
    for name in declared_functions():
        assert name in exported, f"{name} declared in the header but not exported"
        assert hasattr(lib, name)
        assert name in lib_mod.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.w4a8_abi_version() == 1


def _call_gemm(lib, **over):
    args = dict(x_q=1 << 20, x_stride0=512, x_scale=1 << 20, w=1 << 20, ws=1 << 20, wz=1 << 20, off=1 << 20,
                out=1 << 20, os0=512, os1=1, M=32, E=4, N=512, K=512, gs=128, kernel=0, partials=None, stream=None)
    args.update(over)
    return lib.w4a8_group_gemm_moe_ex(*args.values())


def test_capi_rejects_bad_arguments_without_a_gpu(pkg):
    from importlib import import_module
    L = import_module("flagos-kernel-gen_b200._lib")
    lib = L.load()
    assert _call_gemm(lib, gs=96) == L.W4A8_ERR_INVALID
    assert b"group_size" in lib.w4a8_last_error()
    assert _call_gemm(lib, K=448) == L.W4A8_ERR_INVALID           # 448 % 128 != 0
    assert b"group_size" in lib.w4a8_last_error()
    assert _call_gemm(lib, x_stride0=100) == L.W4A8_ERR_INVALID   # stride < K
    assert _call_gemm(lib, kernel=7) == L.W4A8_ERR_INVALID
    assert _call_gemm(lib, w=None) == L.W4A8_ERR_INVALID
    # nothing to do is not an error
    assert _call_gemm(lib, M=0) == L.W4A8_OK
    ws = ctypes.c_size_t(lib.w4a8_moe_align_workspace_size(16, 8, 256)).value
    assert ws >= 4 * (256 + 128)
    assert lib.w4a8_moe_align(None, 16, 8, 256, 128, 1 << 20, 1 << 20, 1 << 20, None, None, None, 1 << 20, 4,
                              None) == L.W4A8_ERR_INVALID
    assert b"workspace" in lib.w4a8_last_error() or b"null" in lib.w4a8_last_error()


@pytest.mark.parametrize("bs", [0, -3, 4097, 1 << 31, (1 << 32) + 128])
def test_align_rejects_block_sizes_outside_the_index_range(pkg, bs):
    """block_size is bounded in both align entry points: a value that would
    truncate in a 32-bit cast, or make the padded index range overflow, is an
    argument error and no kernel is launched (no GPU is touched here)."""
    from importlib import import_module
    L = import_module("flagos-kernel-gen_b200._lib")
    lib = L.load()
    p = 1 << 20
    assert lib.w4a8_moe_align(p, 16, 8, 256, bs, p, p, p, None, None, None, p, 1 << 30, None) == L.W4A8_ERR_INVALID
    assert b"block_size" in lib.w4a8_last_error()
    assert lib.w4a8_moe_align_noalloc(p, 16, 8, 256, bs, p, p, p, None, None, None, None) == L.W4A8_ERR_INVALID
    assert b"block_size" in lib.w4a8_last_error()


def test_align_rejects_padded_range_overflow(pkg):
    """T*topk + E*(block_size-1) beyond the 32-bit padded index range."""
    from importlib import import_module
    L = import_module("flagos-kernel-gen_b200._lib")
    lib = L.load()
    p = 1 << 20
    # T*topk = 2^30 - 2^20 slots is accepted on its own, but 8192 experts x 4095
    # padding entries (33.5 M) push the padded range past 2^30
    T = (1 << 24) - (1 << 14)
    assert lib.w4a8_moe_align(p, T, 64, 8192, 4096, p, p, p, None, None, None, p, 1 << 40, None) \
        == L.W4A8_ERR_INVALID
    assert b"block_size" in lib.w4a8_last_error()


def test_python_signature_matches_reference(pkg):
    sig = inspect.signature(pkg.w4a8_group_gemm_moe)
    assert list(sig.parameters) == ["x_q", "x_scale", "w_q4_packed", "w_scale", "w_zero", "expert_offsets", "out",
                                    "group_size"]


def test_reference_asserts_are_kept(pkg):
    E, N, K, M, gs = 2, 128, 256, 8, 128
    x_q = torch.zeros((M, K), dtype=torch.int8)
    xs = torch.ones(M)
    w_bad = torch.zeros((E, N, K // 2 + 1), dtype=torch.uint8)
    wsc = torch.ones((E, N, K // gs))
    wz = torch.zeros((E, N, K // gs), dtype=torch.int8)
    off = torch.tensor([0, 4, 8], dtype=torch.int32)
    out = torch.zeros((M, N), dtype=torch.bfloat16)
    with pytest.raises(AssertionError):                 # K_half * 2 == K  (docs/Task1.md:74)
        pkg.w4a8_group_gemm_moe(x_q, xs, w_bad, wsc, wz, off, out, gs)
    w = torch.zeros((E, N, K // 2), dtype=torch.uint8)
    with pytest.raises(AssertionError):                 # K % group_size == 0  (docs/Task1.md:75)
        pkg.w4a8_group_gemm_moe(x_q, xs, w, wsc, wz, off, out, 96)


def test_no_cpu_fallback(pkg):
    E, N, K, M, gs = 2, 128, 256, 8, 128
    args = (torch.zeros((M, K), dtype=torch.int8), torch.ones(M), torch.zeros((E, N, K // 2), dtype=torch.uint8),
            torch.ones((E, N, K // gs)), torch.zeros((E, N, K // gs), dtype=torch.int8),
            torch.tensor([0, 4, 8], dtype=torch.int32), torch.zeros((M, N), dtype=torch.bfloat16), gs)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.w4a8_group_gemm_moe(*args)


def test_product_path_never_imports_the_oracle():
    pkg_dir = os.path.join(REPO, "flagos-kernel-gen_b200")
    for root, _, files in os.walk(pkg_dir):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                text = open(os.path.join(root, f), encoding="utf-8").read()
                assert "import oracle" not in text and "from oracle" not in text, f


def test_newer_entry_points_reject_bad_arguments_without_a_gpu(pkg):
    """Router, prepack, row-address GEMM and return-address entry points check
    their arguments on the host before any launch."""
    from importlib import import_module
    L = import_module("flagos-kernel-gen_b200._lib")
    lib = L.load()
    P = 1 << 20   # a stand-in pointer value: every call below fails validation before using it

    def router(**over):
        a = dict(logits=P, ls0=256, T=16, E=256, topk=8, scoring=1, renorm=1, ids=P, w=P, x=None, xs0=0, H=0,
                 xq=None, qs0=0, xscale=None, stream=None)
        a.update(over)
        return lib.w4a8_router_topk(*a.values())
    for bad in (dict(topk=0), dict(topk=257, E=256), dict(topk=33, E=64), dict(E=1025, ls0=1025), dict(scoring=2),
                dict(ls0=100), dict(x=P, H=0), dict(x=P, H=7168, xs0=7168, qs0=7168, xq=None, xscale=P)):
        assert router(**bad) == L.W4A8_ERR_INVALID, bad
    assert router(T=0) == L.W4A8_OK

    assert lib.w4a8_prepack_weights(P, P, 4, 100, None) == L.W4A8_ERR_INVALID      # K not a multiple of 64
    assert lib.w4a8_prepack_weights(P + 8, P, 4, 128, None) == L.W4A8_ERR_INVALID  # unaligned input
    assert lib.w4a8_prepack_weights(P, P, 0, 128, None) == L.W4A8_OK

    def rows(**over):
        a = dict(x_q=P, xs0=512, x_scale=P, w=P, ws=P, wz=P, off=P, stage=P, addr=P, M=32, E=4, N=512, K=512,
                 gs=128, hint=0, stream=None)
        a.update(over)
        return lib.w4a8_group_gemm_moe_rows(*a.values())
    for bad in (dict(addr=None), dict(stage=None), dict(N=500), dict(stage=P + 8), dict(hint=33), dict(gs=96)):
        assert rows(**bad) == L.W4A8_ERR_INVALID, bad
    assert rows(M=0) == L.W4A8_OK

    assert lib.w4a8_ep_row_addresses(P, P, 16, 7168, 0, P, 0, P, None) == L.W4A8_ERR_INVALID   # tk_max 0
    assert lib.w4a8_ep_row_addresses(None, P, 16, 7168, 8, P, 0, P, None) == L.W4A8_ERR_INVALID
    assert lib.w4a8_ep_row_addresses(P, P, 0, 7168, 8, P, 0, P, None) == L.W4A8_OK

    def dedup(**over):
        a = dict(x=P, xs0=7168, T=16, H=7168, ids=P, topk=8, E=256, world=2, rank=0, tk_max=128, off=P, inv=P,
                 base=P, peers=P, xq_off=0, xs_off=0, src_off=0, dup_off=256, home=P, stream=None)
        a.update(over)
        return lib.w4a8_ep_dispatch_dedup(*a.values())
    for bad in (dict(dup_off=-1), dict(tk_max=127), dict(rank=2), dict(E=255), dict(H=0), dict(ids=None)):
        assert dedup(**bad) == L.W4A8_ERR_INVALID, bad
    assert dedup(T=0) == L.W4A8_OK
    assert lib.w4a8_ep_replicate(P, 0, -1, 7168, P, 16, None) == L.W4A8_ERR_INVALID
    assert lib.w4a8_ep_replicate(P, 0, 256, 7168, None, 16, None) == L.W4A8_ERR_INVALID


def _header_declarations():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = {}
    for name, params in re.findall(r"\b(w4a8_\w+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        ps = [p.strip() for p in params.split(",") if p.strip()]
        out[name] = [] if ps == ["void"] else ps
    return out


def test_ctypes_signatures_match_the_header(pkg):
    """Every entry point's ctypes argument list has the header's arity and,
    parameter by parameter, the same kind: pointer, 64-bit integer, 32-bit
    integer, size_t.  A shifted or missing argument would otherwise reach the
    library as a wrong pointer or stream without any error on the host."""
    from importlib import import_module
    L = import_module("flagos-kernel-gen_b200._lib")
    decls = _header_declarations()
    assert set(decls) == set(declared_functions())
    scalar = {"int64_t": ctypes.c_int64, "int32_t": ctypes.c_int32, "int": ctypes.c_int, "size_t": ctypes.c_size_t}
    for name, params in decls.items():
        _, argtypes = L.SIGNATURES[name]
        assert len(argtypes) == len(params), f"{name}: header has {len(params)} parameters, ctypes {len(argtypes)}"
        for i, (p, t) in enumerate(zip(params, argtypes)):
            if "*" in p:
                assert t is ctypes.c_void_p or issubclass(t, ctypes._Pointer), f"{name} arg {i} ({p}) is {t}"
            else:
                ctype = re.sub(r"^const\s+", "", p).rsplit(None, 1)[0]
                assert ctypes.sizeof(t) == ctypes.sizeof(scalar[ctype]), f"{name} arg {i} ({p}) is {t}"
