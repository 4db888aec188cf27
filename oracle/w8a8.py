"""W8A8 block-FP8 references (test infrastructure only).

The reference's FP8 paths are W8A16; the W8A8 entry points of the library
follow upstream SGLang's block-FP8 W8A8 arithmetic instead (activations
quantized per token and 128-wide K group, weights per 128x128 block). The
activation scale uses the block rule the reference applies to its LM head
(``quant/sm70_fp8_lm_head/__init__.py:33-41``: ``scale = clamp(amax / 448,
1e-8)``, ``q = (w / scale).to(e4m3)``), here on 1x128 groups.
"""

from __future__ import annotations

import torch

from .fp8 import dequant_block_fp8

GROUP = 128


def act_quant_fp8(x: torch.Tensor):
    """(e4m3 [rows, K], fp32 scales [rows, K/128]) of ``x`` per 1x128 group."""
    rows, k = x.shape
    xf = x.float().reshape(rows, k // GROUP, GROUP)
    scale = (xf.abs().amax(dim=-1) / 448.0).clamp(min=1e-8)
    q = (xf / scale[..., None]).to(torch.float8_e4m3fn).reshape(rows, k)
    return q, scale


def act_dequant_fp8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    rows, k = q.shape
    return (q.float().reshape(rows, k // GROUP, GROUP) * scale[..., None]).reshape(rows, k)


def w8a8_linear_ref(x: torch.Tensor, w_q: torch.Tensor, w_s: torch.Tensor,
                    gated: bool = False) -> torch.Tensor:
    """fp32 ``y = dequant(quant(x)) . dequant(W)^T``; ``gated``: the bank is
    ``[gate | up]`` and the result ``silu(gate) * up``."""
    xq = act_dequant_fp8(*act_quant_fp8(x))
    y = xq @ dequant_block_fp8(w_q, w_s).T
    if gated:
        half = y.shape[-1] // 2
        y = torch.nn.functional.silu(y[..., :half]) * y[..., half:]
    return y


def quantized_activations(x: torch.Tensor) -> torch.Tensor:
    """``x`` as the W8A8 GEMMs see it (quantized and dequantized, fp32)."""
    return act_dequant_fp8(*act_quant_fp8(x))
