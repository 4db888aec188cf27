"""ctypes binding of libb200moe.so (the C ABI declared in include/b200moe.h).

The library is the only compute path: if it is missing or fails to load,
every op raises. There is no CPU or PyTorch fallback.

Search order for the library: ``$B200_MOE_LIB`` (an explicit path), then the
in-tree build next to this file.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

ENV_LIB = "B200_MOE_LIB"
LIB_NAME = "libb200moe.so"

OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3

DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_F32 = 2

QUANT_FP8_BLOCK = 0
QUANT_NVFP4 = 1

SCORING_SOFTMAX = 0
SCORING_SIGMOID = 1

GATED_NONE = 0
GATED_FUSED = 1
GATED_SPLIT = 2

PATH_STREAM = 16
PATH_TCGEN05 = 17

_LOCK = threading.Lock()
_LIB = None

c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_float = ctypes.c_float
c_void_p = ctypes.c_void_p

# name -> (restype, argtypes); kept in the order of include/b200moe.h
SIGNATURES = {
    "b200_abi_version": (c_int32, []),
    "b200_last_error": (ctypes.c_char_p, []),
    "b200_num_sms": (c_int32, []),
    "b200_workspace_status": (c_int32, [c_void_p, ctypes.POINTER(c_int32), c_int32, c_void_p]),
    "b200_moe_align_block_size": (
        c_int32,
        [c_void_p, c_int64, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p],
    ),
    "b200_topk_route": (
        c_int32,
        [c_void_p, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
         c_void_p, c_void_p],
    ),
    "b200_topk_route_grouped": (
        c_int32,
        [c_void_p, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int32,
         c_int32, c_void_p, c_void_p, c_void_p],
    ),
    "b200_append_shared_route": (
        c_int32, [c_void_p, c_void_p, c_int64, c_int32, c_int32, c_float, c_void_p, c_void_p, c_void_p]
    ),
    "b200_moe_sum_reduce": (
        c_int32,
        [c_void_p, c_void_p, c_int64, c_int32, c_int64, c_int32, c_float, c_void_p],
    ),
    "b200_moe_combine": (
        c_int32,
        [c_void_p, c_int32, c_void_p, c_int32, c_int64, c_int32, c_int64, c_float, c_void_p,
         c_int32, c_void_p, c_int32, c_void_p],
    ),
    "b200_fp8_packed_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "b200_fp8_prepack": (c_int32, [c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p, c_void_p]),
    "b200_nvfp4_packed_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "b200_nvfp4_prepack": (
        c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p, c_void_p]
    ),
    "b200_gemm_workspace_bytes": (c_int64, [c_int64]),
    "b200_linear": (
        c_int32,
        [c_int32, c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64,
         c_int32, c_void_p, c_int32, c_void_p, c_int64, c_void_p],
    ),
    "b200_linear_noalloc_scratch_bytes": (c_int64, []),
    "b200_linear_noalloc": (
        c_int32,
        [c_int32, c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64,
         c_int32, c_void_p, c_int32, c_void_p],
    ),
    "b200_linear_noalloc_status": (c_int32, [ctypes.POINTER(c_int32), c_int32, c_void_p]),
    "b200_linear_loads_only": (
        c_int32,
        [c_int32, c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64,
         c_int32, c_void_p, c_int32, c_void_p, c_int64, c_void_p],
    ),
    "b200_moe_gemm_loads_only": (
        c_int32,
        [c_int32, c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int32,
         c_int64, c_int32, c_void_p, c_void_p, c_int64, c_void_p, c_int32, c_int32, c_int64,
         c_void_p, c_int32, c_void_p, c_int32, c_int64, c_void_p, c_int64, c_void_p],
    ),
    "b200_linear_path": (
        c_int32, [c_int64, c_int64, c_int64, ctypes.POINTER(c_int32), ctypes.POINTER(c_int32)]
    ),
    "b200_moe_path": (c_int32, [c_int32, c_int32, c_int64, ctypes.POINTER(c_int32)]),
    "b200_moe_gemm": (
        c_int32,
        [c_int32, c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int32,
         c_int64, c_int32, c_void_p, c_void_p, c_int64, c_void_p, c_int32, c_int32, c_int64,
         c_void_p, c_int32, c_void_p, c_int32, c_int64, c_void_p, c_int64, c_void_p],
    ),
    "b200_moe_layer_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64, c_int32, c_int32, c_int32]),
    "b200_moe_layer_forward": (
        c_int32,
        [c_int32, c_void_p, c_int32, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int32,
         c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_float,
         c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_int64, c_void_p],
    ),
    "b200_moe_layer_forward_fused_shared": (
        c_int32,
        [c_int32, c_void_p, c_int32, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int32,
         c_int32, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_int32, c_float, c_void_p, c_int32, c_void_p, c_int64, c_void_p],
    ),
    "b200_moe_layer_forward_logits": (
        c_int32,
        [c_int32, c_void_p, c_int32, c_int64, c_int64, c_int64, c_void_p, c_int32, c_int32,
         c_int32, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_int32, c_float, c_void_p, c_int32, c_void_p, c_int32,
         c_void_p, c_int64, c_void_p],
    ),
    "b200_w8a8_workspace_bytes": (c_int64, [c_int64, c_int64]),
    "b200_fp8_act_quant": (
        c_int32, [c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p]
    ),
    "b200_w8a8_linear": (
        c_int32,
        [c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int32, c_void_p,
         c_int32, c_void_p, c_int64, c_void_p],
    ),
    "b200_w8a8_moe_gemm": (
        c_int32,
        [c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p, c_int32, c_int64, c_int32,
         c_void_p, c_void_p, c_int64, c_void_p, c_int32, c_int32, c_int64, c_void_p, c_int32,
         c_void_p, c_int32, c_int64, c_void_p, c_int64, c_void_p],
    ),
    "b200_ep_region_bytes": (c_int64, [c_int32, c_int64, c_int32, c_int64]),
    "b200_ep_region_layout": (c_int32, [c_int32, c_int64, c_int32, c_int64, ctypes.POINTER(c_int64)]),
    "b200_ipc_get_handle": (c_int32, [c_void_p, c_void_p, ctypes.POINTER(c_int64)]),
    "b200_ipc_open_handle": (c_int32, [c_void_p, c_int64, ctypes.POINTER(c_void_p)]),
    "b200_ipc_close_handle": (c_int32, [c_void_p, c_int64]),
    "b200_ep_dispatch": (
        c_int32,
        [c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p, c_int32, c_int32, c_int32,
         c_int32, c_int32, c_void_p, c_void_p, c_int64, c_void_p],
    ),
    "b200_ep_expert_workspace_bytes": (
        c_int64, [c_int32, c_int64, c_int32, c_int64, c_int64, c_int32, c_int32]
    ),
    "b200_ep_expert_forward": (
        c_int32,
        [c_int32, c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_int64, c_int32, c_void_p,
         c_int64, c_void_p],
    ),
    "b200_ep_combine": (
        c_int32,
        [c_int64, c_int64, c_void_p, c_int32, c_int32, c_float, c_void_p, c_int32, c_void_p,
         c_int32, c_int32, c_void_p, c_int64, c_void_p],
    ),
}


class B200Error(RuntimeError):
    """A non-zero status from libb200moe."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class Unsupported(B200Error):
    """The library declined a valid call (shape or dtype it does not cover)."""


def library_path() -> Path:
    explicit = os.environ.get(ENV_LIB)
    if explicit:
        return Path(explicit)
    return Path(__file__).resolve().with_name(LIB_NAME)


def load():
    """Load (once) and return the ctypes handle; raises if it cannot."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if not path.is_file():
            raise FileNotFoundError(
                f"{LIB_NAME} not found at {path}; build it with "
                "`python sglang-restomod_b200/build.py` (or set B200_MOE_LIB)"
            )
        lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.b200_abi_version() != 1:
            raise RuntimeError(f"{path} has ABI {lib.b200_abi_version()}, expected 1")
        _LIB = lib
        return lib


def check(status: int) -> None:
    """Raise for a non-zero status, carrying the library's message."""
    if status == OK:
        return
    msg = load().b200_last_error().decode(errors="replace")
    if status == ERR_UNSUPPORTED:
        raise Unsupported(status, msg)
    raise B200Error(status, msg)
