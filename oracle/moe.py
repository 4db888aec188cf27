"""Fused-MoE references (test infrastructure only).

Weights are passed already dequantized to fp32 (``dequant_block_fp8`` /
``dequant_nvfp4``), ``[E, N, K]`` with the logical row order (a gate/up bank
is ``[gate rows | up rows]``).
"""

from __future__ import annotations

import numpy as np
import torch


def _silu_mul(y: torch.Tensor) -> torch.Tensor:
    half = y.shape[-1] // 2
    return torch.nn.functional.silu(y[..., :half]) * y[..., half:]


def moe_layer_ref(
    x: torch.Tensor,
    topk_ids: torch.Tensor,
    topk_weights: torch.Tensor,
    w13: torch.Tensor,
    w2: torch.Tensor,
    routed_scaling_factor: float = 1.0,
    shared_out: torch.Tensor | None = None,
    inter_dtype: torch.dtype | None = torch.bfloat16,
) -> torch.Tensor:
    """fp32 result of one fused-MoE layer.

    Per token and slot, an id outside ``[0, E)`` is skipped (the -1 of
    expert parallelism, ``quant/sm70_fp8_moe/check.py:34-48`` and
    ``method.py:269-283``); otherwise ``silu(x W13g^T) * (x W13u^T)`` (rounded
    to ``inter_dtype``, the activation dtype the intermediate is stored in),
    times ``W2^T``, times the router weight, summed over slots; then the
    routed scaling factor (``method.py:307-308``) and the shared expert.
    Vectorised per expert so it doubles as the CPU baseline. ``w13`` may be
    a callable ``e -> (w13_e, w2_e)`` with ``w2`` then the expert count.
    """
    tokens, top_k = topk_ids.shape
    # w13 / w2 are stacked banks, or w13 is a callable e -> (w13[e], w2[e])
    # that dequantizes one expert on demand (bounded memory for big banks).
    fetch = w13 if callable(w13) else (lambda e: (w13[e], w2[e]))
    num_experts = int(w2) if callable(w13) else w13.shape[0]
    hidden_out = None if callable(w13) else w2.shape[1]
    ids = topk_ids.reshape(-1).long()
    wts = topk_weights.reshape(-1).float()
    tok = torch.arange(tokens).repeat_interleave(top_k)
    valid = (ids >= 0) & (ids < num_experts)
    out = None if hidden_out is None else torch.zeros(tokens, hidden_out, dtype=torch.float32)
    xf = x.float()
    for e in torch.unique(ids[valid]).tolist():
        sel = torch.nonzero(valid & (ids == e)).flatten()
        we13, we2 = fetch(e)
        h = _silu_mul(xf[tok[sel]] @ we13.T)
        if inter_dtype is not None:
            h = h.to(inter_dtype).float()
        y = (h @ we2.T) * wts[sel, None]
        if out is None:
            out = torch.zeros(tokens, y.shape[1], dtype=torch.float32)
        out.index_add_(0, tok[sel], y)
    if out is None:
        out = torch.zeros(tokens, x.shape[1], dtype=torch.float32)
    out = out * routed_scaling_factor
    if shared_out is not None:
        out = out + shared_out.float()
    return out


def fp8_moe_method_ref(x, topk_ids, topk_weights, w13, w2, output_scale=None):
    """Semantics of ``SM70Fp8MoEMethod.apply`` (``quant/sm70_fp8_moe/method.py:239-309``).

    Both of its expert-parallel branches - compaction of valid routes
    (``:269-276``) and the clamp onto expert 0 with a zero weight
    (``:277-283``) - drop every route whose local id is -1; the result is the
    weighted sum over the remaining slots, times ``output_scale`` when set.
    """
    out = moe_layer_ref(x, topk_ids, topk_weights, w13, w2, inter_dtype=None)
    if output_scale is not None:
        out = out * output_scale
    return out


def moe_gemm_ref(
    a: torch.Tensor,
    w: torch.Tensor,
    sorted_token_ids,
    expert_ids,
    num_tokens_post_pad: int,
    block_size: int,
    top_k: int,
    num_routes: int,
    topk_weights: torch.Tensor | None = None,
    mul_topk_weights: bool = False,
    gated_mode: int = 0,
):
    """``moe_wna16_marlin_gemm`` semantics (``quant/sm70_fp4_moe/method.py:385-564``).

    Slot ``p`` of block ``b`` (``p < num_tokens_post_pad``) holding route
    ``r < num_routes`` computes ``a[r // top_k] . w[expert_ids[b]]^T`` into
    output row ``r`` (times ``topk_weights[r]`` when ``mul_topk_weights``).
    ``gated_mode`` 1 applies ``silu(gate) * up``. Returns (fp32 rows
    [num_routes, cols], bool mask of the rows written).
    """
    sorted_token_ids = np.asarray(sorted_token_ids)
    expert_ids = np.asarray(expert_ids)
    n = w.shape[1]
    cols = n // 2 if gated_mode == 1 else n
    out = torch.zeros(num_routes, cols, dtype=torch.float32)
    written = torch.zeros(num_routes, dtype=torch.bool)
    flat_w = None if topk_weights is None else topk_weights.reshape(-1).float()
    af = a.float()
    for b in range(num_tokens_post_pad // block_size):
        e = int(expert_ids[b])
        slots = sorted_token_ids[b * block_size : (b + 1) * block_size]
        routes = [int(r) for r in slots if 0 <= int(r) < num_routes]
        if not routes:
            continue
        r_t = torch.tensor(routes)
        y = af[r_t // top_k] @ w[e].T
        if gated_mode == 1:
            y = _silu_mul(y)
        if mul_topk_weights:
            y = y * flat_w[r_t, None]
        out[r_t] = y
        written[r_t] = True
    return out, written


def moe_sum_reduce_ref(inp: torch.Tensor, routed_scaling_factor: float = 1.0) -> torch.Tensor:
    """``quant/sm70_fp4_moe/sum_reduce.py:84-123``: fp32 sum over top-k,
    times the scaling factor, stored in the input dtype."""
    return (inp.float().sum(dim=1) * routed_scaling_factor).to(inp.dtype)
