"""b200_linear_noalloc checked against b200_linear through the C ABI.

Some callers of this library cannot allocate device memory themselves: an
engine that reserved all of it for its own pool before loading plugins, or a
binding with no access to the device allocator. b200_linear_noalloc serves
them from a fixed array compiled into the library instead of a caller-owned
workspace. This test calls it twice in a row (the second call reuses the
array the first one left behind) and checks both results against the
ordinary entry point's, within the tolerance the other GEMM tests use.

It lives in its own file, collected last, so that a run stopping at the
first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from sglang_restomod_b200 import _lib, ops, synth
from tests.conftest import ATOL, RTOL, assert_close

pytestmark = pytest.mark.gpu

_CODE = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def _noalloc(x, packed, scales, n, y, gated_mode=_lib.GATED_NONE):
    lib = _lib.load()
    m, k = x.shape
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.b200_linear_noalloc(
        _lib.QUANT_FP8_BLOCK, ctypes.c_void_p(x.data_ptr()), _CODE[x.dtype], m, k,
        ctypes.c_void_p(packed.data_ptr()), ctypes.c_void_p(scales.data_ptr()), None, n,
        gated_mode, ctypes.c_void_p(y.data_ptr()), _CODE[y.dtype], stream,
    )


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k,n,gated", [(4, 1024, 768, False), (24, 512, 1024, True)])
def test_noalloc_matches_linear_twice(cuda_device, x_dtype, m, k, n, gated):
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=31)
    packed = ops.fp8_prepack(q[0], gated=gated)
    x = synth.activations(m, k, cuda_device, seed=32, dtype=x_dtype)
    mode = _lib.GATED_FUSED if gated else _lib.GATED_NONE
    cols = n // 2 if gated else n
    want = ops.linear(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, scales=s[0], gated_mode=mode,
                      out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    for call in range(2):
        y = torch.full((m, cols), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        rc = _noalloc(x, packed, s[0], n, y, mode)
        assert rc == _lib.OK, _lib.load().b200_last_error().decode()
        torch.cuda.synchronize()
        assert_close(y, want, rtol=RTOL, atol=ATOL, what=f"no-alloc call {call + 1}")


def test_noalloc_refuses_calls_beyond_its_array(cuda_device):
    lib = _lib.load()
    cap = lib.b200_linear_noalloc_scratch_bytes()
    assert cap == 16 << 20
    # bf16 activations are converted inside the array; 64 x 131072 do not fit.
    p = ctypes.c_void_p(256)
    rc = lib.b200_linear_noalloc(_lib.QUANT_FP8_BLOCK, p, _lib.DTYPE_BF16, 64, 131072, p, p, None,
                                 128, 0, p, _lib.DTYPE_BF16, None)
    assert rc == _lib.ERR_INVALID
    assert "static array" in lib.b200_last_error().decode()
