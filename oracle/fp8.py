"""Block-FP8 (E4M3, 128x128 fp32 scales) quantization and dense references.

Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import torch

BLOCK = 128
E4M3_MAX = 448.0


def quant_block_fp8(w: torch.Tensor, clamp_min: float = 1e-6):
    """[N, K] -> (e4m3 [N, K], fp32 scales [N/128, K/128]).

    Restates ``quant/sm70_fp8_moe/check.py:18-24``: fp32 math, the block amax
    clamped to ``clamp_min`` *before* the division by 448, q = e4m3(w / s).
    """
    n, k = w.shape
    blocks = w.float().reshape(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    scale = blocks.abs().amax(dim=(1, 3)).clamp_min(clamp_min) / E4M3_MAX
    q = (blocks / scale[:, None, :, None]).to(torch.float8_e4m3fn)
    return q.reshape(n, k), scale


def quant_block_fp8_lm_head(weight: torch.Tensor):
    """LM-head rule of ``quant/sm70_fp8_lm_head/__init__.py:33-41``.

    The arithmetic runs in the weight's own dtype (fp16 in the reference);
    the scale is ``amax / 448`` clamped to 1e-8 *after* the division.
    """
    n, k = weight.shape
    if n % BLOCK or k % BLOCK:
        raise ValueError(f"shape {tuple(weight.shape)} is not a multiple of {BLOCK}")
    wb = weight.view(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    scale = (wb.abs().amax(dim=(1, 3)) / E4M3_MAX).clamp(min=1e-8)
    q = (wb / scale[:, None, :, None]).to(torch.float8_e4m3fn).view(n, k)
    return q.contiguous(), scale.to(torch.float32).contiguous()


def dequant_block_fp8(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp32 W[n, k] = e4m3[n, k] * s[n/128, k/128] (``check.py:27-31``)."""
    n, k = q.shape
    return (
        q.float().reshape(n // BLOCK, BLOCK, k // BLOCK, BLOCK) * s.float()[:, None, :, None]
    ).reshape(n, k)


def fp8_linear_ref(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor, gated: bool = False):
    """y = x . dequant(W)^T in fp32 (the dense reference of
    ``tests/test_sm70_fp8_dense_gpu.py:22-34``, there in fp64).

    ``gated``: W is a [2I, K] gate/up bank and the result is
    ``silu(y[:, :I]) * y[:, I:]`` (``quant/sm70_fp8_moe/README.md:53-56``).
    """
    y = x.float() @ dequant_block_fp8(q, s).T
    if gated:
        half = y.shape[1] // 2
        y = torch.nn.functional.silu(y[:, :half]) * y[:, half:]
    return y
