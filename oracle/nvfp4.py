"""NVFP4 (E2M1 codes, E4M3 scale per 16 K, fp32 global) references.

Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import torch

# E2M1 magnitudes (``quant/sm70_fp4_moe/check.py:31-32``).
E2M1_GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def quantize_nvfp4(w: torch.Tensor, global_scale: float = 1.0):
    """[N, K] -> (packed uint8 [N, K/2], e4m3 scales [N, K/16]).

    Restates ``quant/sm70_fp4_moe/check.py:35-51`` step for step (the amax
    and the division by 6 run in the weight's dtype, fp16 in the reference;
    nearest grid value; low nibble = even K; bit 3 = sign). A global scale
    other than 1 divides the group scale before its E4M3 rounding.
    """
    n, k = w.shape
    groups = w.reshape(n, k // 16, 16)
    amax = groups.abs().amax(dim=-1).clamp_min(1e-8) / 6.0
    if global_scale != 1.0:
        amax = amax.float() / global_scale
    scales = amax.to(torch.float8_e4m3fn)
    q = groups.float() / (scales.to(torch.float32) * global_scale)[..., None]
    idx = (q.abs()[..., None] - E2M1_GRID.to(q.device)).abs().argmin(dim=-1)
    code = torch.where(q < 0, -idx, idx)
    nibble = code.abs().to(torch.uint8) | ((code < 0).to(torch.uint8) << 3)
    nibble = nibble.reshape(n, k // 2, 2)
    packed = (nibble[..., 0] | (nibble[..., 1] << 4)).contiguous()
    return packed, scales.contiguous()


def dequant_nvfp4(packed: torch.Tensor, scales: torch.Tensor, global_scale: float = 1.0):
    """Dense fp32 [N, K] with the reference's rounding points.

    ``docs/qpn2-layout.md`` section 3 (applied by
    ``csrc/decode_gemv_qpn2.cu:40-61``): the group scale is
    ``fp16_rne(float(e4m3) * global)``, the code value is exact, and the
    weight is their product rounded to fp16. With ``global_scale == 1`` this
    is ``quant/sm70_fp4_moe/check.py:54-64``.
    """
    n, k = packed.shape[0], packed.shape[1] * 2
    nib = packed.to(torch.int32)
    codes = torch.stack([nib & 0xF, nib >> 4], dim=-1).reshape(n, k)
    mag = E2M1_GRID[codes & 7]
    values = torch.where((codes & 8) != 0, -mag, mag).to(torch.float16)
    scale16 = (scales.to(torch.float32) * float(global_scale)).to(torch.float16)
    scale16 = scale16.repeat_interleave(16, dim=1)
    return (values * scale16).to(torch.float32)


def nvfp4_linear_ref(x, packed, scales, global_scale: float = 1.0, gated: bool = False):
    y = x.float() @ dequant_nvfp4(packed, scales, global_scale).T
    if gated:
        half = y.shape[1] // 2
        y = torch.nn.functional.silu(y[:, :half]) * y[:, half:]
    return y


def encode_scales(scales: torch.Tensor) -> torch.Tensor:
    """Q0.7 scale bytes of the SM70 Marlin iterator (``scales.py:20-56``).

    Each byte is the high byte of ``fp16(scale * 2**7)`` with the low pad bit
    dropped, and every group of four along N is stored in the order 0, 2, 1, 3.
    Input ``[E, K/16, N]`` e4m3; output the same shape as uint8.
    """
    logical = scales.to(torch.float16)
    e, g, n = logical.shape
    flat = logical.reshape(-1, n).view(-1, 4)[:, [0, 2, 1, 3]].reshape(-1, n)
    bits = (flat.float() * 128.0).to(torch.float16).view(torch.int16).to(torch.int32) & 0xFFFF
    return ((bits >> 7) & 0xFF).to(torch.uint8).reshape(e, g, n)


def encode_global_scale(global_scale: torch.Tensor) -> torch.Tensor:
    """Global scale compensation of ``scales.py:59-73``: x * 2**(14 - 7)."""
    return global_scale.to(torch.float32) * (2.0 ** (2**4 - 2**1 - 7))
