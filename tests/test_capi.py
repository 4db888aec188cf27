"""The C ABI library loads, exports every declared symbol, and validates on
the host (these calls return before touching a GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from sglang_restomod_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "b200moe.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|int64_t|const char\*)\s+(b200_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), f"{name} declared in b200moe.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)
    assert lib.b200_abi_version() == 1


def test_ctypes_signatures_match_the_header_arity():
    """Every declaration's parameter count equals its ctypes signature's, so a
    binding cannot silently shift arguments."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    decls = re.findall(r"^(?:int|int64_t|const char\*)\s+(b200_\w+)\(([^;]*?)\);", text,
                       re.M | re.S)
    assert {name for name, _ in decls} == set(declared_functions())
    for name, params in decls:
        p = params.strip()
        count = 0 if p in ("", "void") else len(p.split(","))
        assert count == len(_lib.SIGNATURES[name][1]), name


def test_library_has_no_torch_dependency():
    """The C ABI .so stands alone: no libtorch / libc10 in its dependencies."""
    import subprocess

    out = subprocess.run(["ldd", str(_lib.library_path())], capture_output=True, text=True).stdout
    deps = [line.split()[0] for line in out.splitlines() if line.strip()]
    assert not [d for d in deps if "torch" in d or "c10" in d], out


def _err(status):
    assert status != 0
    return _lib.load().b200_last_error().decode()


def test_shape_guards_match_the_reference_messages():
    lib = _lib.load()
    # K must cover whole 128-wide quantization groups (sm70_fp8_moe/__init__.py:48-73).
    st = lib.b200_fp8_prepack(ctypes.c_void_p(16), 1, 256, 100, 0, ctypes.c_void_p(16), None)
    assert st == _lib.ERR_INVALID
    assert "needs K a multiple of the 128-wide quantization group" in _err(st)
    st = lib.b200_fp8_prepack(ctypes.c_void_p(16), 1, 96, 128, 0, ctypes.c_void_p(16), None)
    assert "needs N a multiple of 128" in _err(st)
    st = lib.b200_fp8_prepack(ctypes.c_void_p(16), 1, 128, 128, 1, ctypes.c_void_p(16), None)
    assert "gate/up bank needs N a multiple of 256" in _err(st)
    st = lib.b200_nvfp4_prepack(None, None, 1, 128, 128, 0, None, None)
    assert st == _lib.ERR_INVALID and "null pointer" in _err(st)


def test_align_validation():
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    assert lib.b200_moe_align_block_size(p, 10, 0, 8, p, 100, p, 100, p, None) == _lib.ERR_UNSUPPORTED
    assert lib.b200_moe_align_block_size(p, 10, 2000, 8, p, 100, p, 100, p, None) == _lib.ERR_UNSUPPORTED
    st = lib.b200_moe_align_block_size(p, 40, 16, 8, p, 50, p, 100, p, None)
    # 40 routes over 16 experts: at most 40 + 16 * 7 = 152 padded slots
    assert st == _lib.ERR_INVALID and "sorted_token_ids holds 50 slots, needs 152" in _err(st)
    st = lib.b200_moe_align_block_size(p, 40, 16, 8, p, 152, p, 18, p, None)
    assert st == _lib.ERR_INVALID and "expert_ids holds 18 blocks, needs 19" in _err(st)


def test_gemm_validation():
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    # unsupported block size
    st = lib.b200_moe_gemm(0, p, 0, 8, 128, p, p, None, 4, 256, 0, p, p, 4, p, 12, 1, 8, None, 0,
                           p, 0, 256, p, 1 << 30, None)
    assert st == _lib.ERR_UNSUPPORTED and "block_size" in _err(st)
    # fp32 activations are not an input this library takes
    st = lib.b200_linear(0, p, 2, 1, 128, p, p, None, 128, 0, p, 0, p, 1 << 30, None)
    assert st == _lib.ERR_UNSUPPORTED
    # FP8 needs scales, NVFP4 needs its global scale
    st = lib.b200_linear(0, p, 0, 1, 128, p, None, None, 128, 0, p, 0, p, 1 << 30, None)
    assert "block scales" in _err(st)
    st = lib.b200_linear(1, p, 0, 1, 128, p, None, None, 128, 0, p, 0, p, 1 << 30, None)
    assert "global scale" in _err(st)
    # a workspace below the fixed size is refused
    st = lib.b200_linear(0, p, 0, 1, 128, p, p, None, 128, 0, p, 0, p, 16, None)
    assert st == _lib.ERR_INVALID and "workspace" in _err(st)


def test_fused_shared_validation():
    lib = _lib.load()
    p, q, r = ctypes.c_void_p(256), ctypes.c_void_p(512), ctypes.c_void_p(1024)

    def call(ids_out, w_out):
        return lib.b200_moe_layer_forward_fused_shared(
            0, p, 0, 4, 256, 128, p, q, 4, 16, 1.0, ids_out, w_out, p, p, None, p, p, None, 16,
            1.0, p, 0, p, 1 << 30, None)

    st = call(None, r)
    assert st == _lib.ERR_INVALID and "null pointer" in _err(st)
    st = call(p, r)  # extended ids would overwrite the input ids
    assert st == _lib.ERR_INVALID and "overwrite" in _err(st)
    st = call(r, q)  # extended weights would overwrite the input weights
    assert st == _lib.ERR_INVALID and "overwrite" in _err(st)


def test_sizes():
    lib = _lib.load()
    assert lib.b200_fp8_packed_bytes(3, 256, 512) == 3 * 256 * 512
    assert lib.b200_nvfp4_packed_bytes(2, 256, 512) == 2 * 2 * 4 * 9216
    assert lib.b200_nvfp4_packed_bytes(1, 100, 128) == -1
    fixed = lib.b200_gemm_workspace_bytes(0)
    assert fixed > 0 and lib.b200_gemm_workspace_bytes(1000) == fixed + 2048


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setenv(_lib.ENV_LIB, str(tmp_path / "nope.so"))
    monkeypatch.setattr(_lib, "_LIB", None)
    with pytest.raises(FileNotFoundError):
        _lib.load()


def test_ep_validation_without_a_gpu():
    """The expert-parallel entry points refuse bad arguments on the host,
    before any device call (so this runs without a GPU)."""
    import ctypes

    from sglang_restomod_b200 import _lib

    lib = _lib.load()
    region = ctypes.create_string_buffer(4096 + 256)
    base = ctypes.addressof(region)
    aligned = ctypes.c_void_p((base + 255) // 256 * 256)
    misaligned = ctypes.c_void_p((base + 255) // 256 * 256 + 8)
    peers = (ctypes.c_uint64 * 8)()
    x = (ctypes.c_uint16 * 1024)()
    ids = (ctypes.c_int32 * 64)()
    w = (ctypes.c_float * 64)()
    # world too large, rank outside world, hidden not a multiple of 128
    assert lib.b200_ep_dispatch(x, 0, 4, 256, ids, w, 4, 16, 0, 0, 65, peers, aligned, 8, None) == _lib.ERR_INVALID
    assert lib.b200_ep_dispatch(x, 0, 4, 256, ids, w, 4, 16, 0, 2, 2, peers, aligned, 8, None) == _lib.ERR_INVALID
    assert lib.b200_ep_dispatch(x, 0, 4, 100, ids, w, 4, 16, 0, 0, 2, peers, aligned, 8, None) == _lib.ERR_INVALID
    # more tokens than the region was sized for, experts not divisible by world
    assert lib.b200_ep_dispatch(x, 0, 9, 256, ids, w, 4, 16, 0, 0, 2, peers, aligned, 8, None) == _lib.ERR_INVALID
    assert lib.b200_ep_dispatch(x, 0, 4, 256, ids, w, 4, 15, 0, 0, 2, peers, aligned, 8, None) == _lib.ERR_INVALID
    # region not 256-byte aligned, peer table missing
    assert lib.b200_ep_dispatch(x, 0, 4, 256, ids, w, 4, 16, 0, 0, 2, peers, misaligned, 8, None) == _lib.ERR_INVALID
    assert lib.b200_ep_dispatch(x, 0, 4, 256, ids, w, 4, 16, 0, 0, 2, None, aligned, 8, None) == _lib.ERR_INVALID
    # unsupported activation dtype
    assert lib.b200_ep_dispatch(x, 2, 4, 256, ids, w, 4, 16, 0, 0, 2, peers, aligned, 8, None) == _lib.ERR_UNSUPPORTED
    # combine: tokens beyond max_tokens; expert forward: workspace too small
    out = (ctypes.c_uint16 * 1024)()
    assert lib.b200_ep_combine(9, 256, ids, 4, 16, 1.0, None, 0, out, 0, 2, aligned, 8, None) == _lib.ERR_INVALID
    wq = (ctypes.c_uint8 * 16)()
    assert lib.b200_ep_expert_forward(0, 256, 128, 8, wq, None, None, wq, None, None, 16, 0, 2,
                                      peers, aligned, 8, 4, aligned, 16, None) == _lib.ERR_INVALID
    assert "workspace" in lib.b200_last_error().decode()


def test_ep_region_layout_sizes():
    from sglang_restomod_b200 import ops

    for world, tokens, k, h in [(1, 1, 1, 128), (2, 24, 4, 256), (8, 128, 9, 7168), (8, 4096, 8, 7168)]:
        lay = ops.ep_region_layout(world, tokens, k, h)
        assert lay["total"] == ops.ep_region_bytes(world, tokens, k, h)
        rows = world * tokens  # one row per (source token, owner), top_k slots each
        offs = [lay[n] for n in ("ids", "weights", "orig", "rows", "recv", "comb")]
        assert all(o % 256 == 0 for o in offs) and offs == sorted(offs)
        assert lay["weights"] - lay["ids"] >= 4 * rows * k
        assert lay["orig"] - lay["weights"] >= 4 * rows * k
        assert lay["recv"] - lay["rows"] >= 8 * rows
        assert lay["comb"] - lay["recv"] >= 2 * rows * h
        assert lay["total"] - lay["comb"] >= 2 * rows * h + 8 * tokens


def test_w8a8_validation():
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    assert lib.b200_w8a8_workspace_bytes(10, 100) == -1
    assert lib.b200_w8a8_workspace_bytes(10, 256) > lib.b200_gemm_workspace_bytes(0)
    st = lib.b200_w8a8_linear(p, _lib.DTYPE_BF16, 4, 200, p, p, 256, 0, p, _lib.DTYPE_BF16, p,
                              1 << 30, None)
    assert st == _lib.ERR_INVALID and "128-wide quantization group" in _err(st)
    # workspace smaller than the quantized activations need
    need = lib.b200_w8a8_workspace_bytes(64, 512)
    st = lib.b200_w8a8_linear(p, _lib.DTYPE_BF16, 64, 512, p, p, 256, 0, p, _lib.DTYPE_BF16, p,
                              need - 4096, None)
    assert st == _lib.ERR_INVALID and "b200_w8a8_workspace_bytes" in _err(st)
    st = lib.b200_w8a8_moe_gemm(p, _lib.DTYPE_BF16, 4, 256, p, p, 4, 256, 0, p, p, 1, p, 12, 1, 4,
                                None, 0, p, _lib.DTYPE_BF16, 256, p, 1 << 30, None)
    assert st == _lib.ERR_UNSUPPORTED and "block_size" in _err(st)
    st = lib.b200_fp8_act_quant(p, _lib.DTYPE_BF16, 4, 256, p, p, 2, None)
    assert st == _lib.ERR_INVALID and "scales_ld" in _err(st)


def test_grouped_router_validation():
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    st = lib.b200_topk_route_grouped(p, _lib.DTYPE_F32, 4, 100, 8, 0, 1, None, 8, 2, p, p, None)
    assert st == _lib.ERR_INVALID and "divide" in _err(st)
    st = lib.b200_topk_route_grouped(p, _lib.DTYPE_F32, 4, 64, 8, 0, 1, None, 8, 9, p, p, None)
    assert st == _lib.ERR_INVALID and "topk_group" in _err(st)
    st = lib.b200_topk_route_grouped(p, _lib.DTYPE_F32, 4, 64, 20, 0, 1, None, 8, 2, p, p, None)
    assert st == _lib.ERR_INVALID and "kept groups" in _err(st)
