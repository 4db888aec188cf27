"""Load-time weight quantizers (run on the weights' device with torch ops).

These produce checkpoint-format tensors - the same formats a block-FP8 or
ModelOpt NVFP4 checkpoint carries - which the prepack kernels then re-lay.
They are load-time tools (LM-head / dense post-load quantization and the
synthetic benchmark weights), not part of the per-token path.
"""

from __future__ import annotations

import torch

BLOCK = 128
E4M3_MAX = 448.0
E2M1_MAX = 6.0


def quantize_block_fp8(weight: torch.Tensor, clamp_min: float = 1e-8):
    """[N, K] -> (e4m3 [N, K], fp32 scale [N/128, K/128]).

    scale = max(block amax / 448, clamp_min), q = e4m3(w / scale), in fp32:
    the rule of ``quant/sm70_fp8_lm_head/__init__.py:33-41`` (clamp after the
    division), computed in fp32 rather than the weight's own dtype.
    """
    n, k = weight.shape
    if n % BLOCK or k % BLOCK:
        raise ValueError(f"shape {tuple(weight.shape)} is not a multiple of {BLOCK}")
    wb = weight.float().view(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    scale = (wb.abs().amax(dim=(1, 3)) / E4M3_MAX).clamp(min=clamp_min)
    q = (wb / scale[:, None, :, None]).to(torch.float8_e4m3fn).view(n, k)
    return q.contiguous(), scale.contiguous()


def quantize_nvfp4(weight: torch.Tensor, global_scale: torch.Tensor | float | None = None):
    """[N, K] -> (packed uint8 [N, K/2], e4m3 [N, K/16], fp32 global scale).

    ModelOpt convention: global = amax(W) / (448 * 6) unless given; group
    scale = e4m3(group amax / 6 / global); codes are the nearest E2M1 value
    of w / (scale * global); byte j holds K 2j (low nibble) and 2j+1 (high),
    bit 3 of a nibble is the sign (``quant/sm70_fp4_moe/check.py:35-51``).
    """
    n, k = weight.shape
    if k % 16:
        raise ValueError(f"K must be a multiple of 16, got {k}")
    w = weight.float()
    if global_scale is None:
        gs = (w.abs().amax() / (E4M3_MAX * E2M1_MAX)).clamp(min=1e-12)
    else:
        gs = torch.as_tensor(global_scale, dtype=torch.float32, device=w.device)
    groups = w.view(n, k // 16, 16)
    amax = groups.abs().amax(dim=-1).clamp(min=1e-12)
    scales = (amax / E2M1_MAX / gs).to(torch.float8_e4m3fn)
    eff = scales.float() * gs
    q = groups / torch.where(eff > 0, eff, torch.ones_like(eff))[..., None]
    mag = q.abs()
    # Nearest of {0, .5, 1, 1.5, 2, 3, 4, 6}: midpoints, ties toward the lower code.
    bounds = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=w.device)
    idx = torch.bucketize(mag, bounds, right=False).to(torch.uint8)
    nib = idx | ((q < 0) & (idx > 0)).to(torch.uint8) << 3
    nib = nib.view(n, k // 2, 2)
    packed = (nib[..., 0] | (nib[..., 1] << 4)).contiguous()
    return packed, scales.contiguous(), gs.reshape(()).float()
