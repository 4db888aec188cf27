"""b200_linear_noalloc checked against b200_linear and the CPU oracle.

Some callers of this library cannot allocate device memory themselves: an
engine that reserved all of it for its own pool before loading plugins, or a
binding with no access to the device allocator. b200_linear_noalloc serves
them from a fixed array compiled into the library instead of a caller-owned
workspace. These tests call it twice in a row (the second call reuses the
array the first one left behind) and check both results against the
ordinary entry point's and against the oracle, within the tolerance the
other GEMM tests use. The cases cover the weight-streaming GEMM (M <= 32)
and the tensor-core GEMM (M >= 33), including shapes whose K is split into
parts that sum their fp32 partials inside the array.

The file is collected last, so that a run stopping at the first failure has
already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import oracle
from sglang_restomod_b200 import _lib, ops, synth
from sglang_restomod_b200.layer import dense_k_parts
from tests.conftest import ATOL, RTOL, assert_close

pytestmark = pytest.mark.gpu

_CODE = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _noalloc(x, packed, scales, n, y, gated_mode=_lib.GATED_NONE):
    lib = _lib.load()
    m, k = x.shape
    return lib.b200_linear_noalloc(
        _lib.QUANT_FP8_BLOCK, ctypes.c_void_p(x.data_ptr()), _CODE[x.dtype], m, k,
        ctypes.c_void_p(packed.data_ptr()), ctypes.c_void_p(scales.data_ptr()), None, n,
        gated_mode, ctypes.c_void_p(y.data_ptr()), _CODE[y.dtype], _stream(),
    )


def _status(reset=1):
    bits = ctypes.c_int32(-1)
    rc = _lib.load().b200_linear_noalloc_status(ctypes.byref(bits), reset, _stream())
    assert rc == _lib.OK, _lib.load().b200_last_error().decode()
    return int(bits.value)


CASES = [
    (4, 1024, 768, False),    # weight-streaming GEMM
    (24, 512, 1024, True),    # weight-streaming GEMM, fused gate/up
    (64, 5120, 1024, False),  # tcgen05 GEMM, K split into parts (fp32 partials in the array)
    (130, 5120, 1024, True),  # tcgen05 GEMM, two row chunks, split K, fused gate/up
    (33, 768, 1024, False),   # tcgen05 GEMM, first row count past the decode range
]


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k,n,gated", CASES)
def test_noalloc_matches_linear_twice(cuda_device, x_dtype, m, k, n, gated):
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=31)
    packed = ops.fp8_prepack(q[0], gated=gated)
    x = synth.activations(m, k, cuda_device, seed=32, dtype=x_dtype)
    mode = _lib.GATED_FUSED if gated else _lib.GATED_NONE
    cols = n // 2 if gated else n
    if m >= 64:
        assert dense_k_parts(m, n, k, ops.num_sms()) > 1  # the split-K partials are exercised
    want = ops.linear(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, scales=s[0], gated_mode=mode,
                      out_dtype=torch.bfloat16)
    ref = oracle.fp8_linear_ref(x.cpu(), q[0].cpu(), s[0].cpu(), gated=gated)
    torch.cuda.synchronize()
    for call in range(2):
        y = torch.full((m, cols), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        rc = _noalloc(x, packed, s[0], n, y, mode)
        assert rc == _lib.OK, _lib.load().b200_last_error().decode()
        torch.cuda.synchronize()
        assert_close(y, want, rtol=RTOL, atol=ATOL, what=f"no-alloc call {call + 1} vs b200_linear")
        assert_close(y, ref, rtol=RTOL, atol=ATOL, what=f"no-alloc call {call + 1} vs oracle")
    assert _status() == 0


def test_noalloc_status_reads_and_resets(cuda_device):
    """The status accessor reads the array's error word: zero after clean
    calls, still zero after a reset."""
    m, k, n = 4, 512, 256
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=33)
    packed = ops.fp8_prepack(q[0], gated=False)
    x = synth.activations(m, k, cuda_device, seed=34)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_device)
    assert _noalloc(x, packed, s[0], n, y) == _lib.OK
    assert _status(reset=0) == 0
    assert _status(reset=1) == 0
    assert _lib.load().b200_linear_noalloc_status(None, 0, _stream()) == _lib.ERR_INVALID


def test_noalloc_refuses_calls_beyond_its_array(cuda_device):
    lib = _lib.load()
    cap = lib.b200_linear_noalloc_scratch_bytes()
    assert cap == 16 << 20
    # The documented limit: (array - fixed workspace) / 2 bf16 elements.
    room = (cap - lib.b200_gemm_workspace_bytes(0)) // 2
    if ops.num_sms() == 148:
        assert room == 3405568
    p = ctypes.c_void_p(256)
    # bf16 activations are converted inside the array; 64 x 131072 do not fit.
    rc = lib.b200_linear_noalloc(_lib.QUANT_FP8_BLOCK, p, _lib.DTYPE_BF16, 64, 131072, p, p, None,
                                 128, 0, p, _lib.DTYPE_BF16, None)
    assert rc == _lib.ERR_INVALID
    assert "static array" in lib.b200_last_error().decode()
