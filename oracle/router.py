"""Softmax -> top-k -> renormalise router (test infrastructure only).

The router is upstream SGLang (``StandardTopKOutput`` as built in
``quant/sm70_fp8_moe/check.py:106-114``); the benchmark configurations define
it as fp32 softmax over the logits, top-k, weights renormalised to sum 1.
"""

from __future__ import annotations

import torch


def route_topk(logits: torch.Tensor, top_k: int):
    """(topk_ids int32 [T, k], topk_weights fp32 [T, k])."""
    probs = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(probs, top_k, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    return ids.to(torch.int32), w.to(torch.float32)


def route_topk_general(logits: torch.Tensor, top_k: int, scoring: str = "softmax",
                       renormalize: bool = True, bias: torch.Tensor | None = None):
    """Top-k routing with a deterministic tie order (lower expert id first).

    ``scoring`` "softmax": weights are softmax probabilities, chosen by
    probability; "sigmoid": weights are sigmoid(logit), chosen by
    sigmoid(logit) + ``bias`` (upstream SGLang's biased top-k selection, where
    the correction bias steers the choice but not the weights). Selection is a
    stable descending sort of the key, so equal keys keep expert order.
    """
    x = logits.float()
    if scoring == "softmax":
        scores = torch.softmax(x, dim=-1)
        key = x  # same order as the probabilities
    else:
        scores = torch.sigmoid(x)
        key = scores + (bias.float() if bias is not None else 0.0)
    order = torch.sort(-key, dim=-1, stable=True).indices[:, :top_k]
    w = scores.gather(1, order)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    return order.to(torch.int32), w.to(torch.float32)


def route_topk_grouped(logits: torch.Tensor, top_k: int, num_expert_group: int, topk_group: int,
                       scoring: str = "softmax", renormalize: bool = True,
                       bias: torch.Tensor | None = None):
    """Grouped top-k of upstream SGLang (``grouped_topk`` / ``biased_grouped_topk``,
    the routing ``select_experts`` feeds into ``StandardTopKOutput``,
    ``quant/sm70_fp8_moe/check.py:106-114``): the experts form
    ``num_expert_group`` contiguous groups; a group scores its largest
    selection key, or with ``bias`` the sum of its two largest biased keys;
    the ``topk_group`` best groups stay selectable and the top-k is taken among
    their experts. Stable orders (lower group / expert first) on ties."""
    x = logits.float()
    tokens, experts = x.shape
    if scoring == "softmax":
        scores = torch.softmax(x, dim=-1)
        key = x
    else:
        scores = torch.sigmoid(x)
        key = scores + (bias.float() if bias is not None else 0.0)
    g = key.view(tokens, num_expert_group, experts // num_expert_group)
    if bias is not None:
        srt = torch.sort(-g, dim=-1, stable=True).values  # ascending of -key
        group_score = -(srt[..., 0] + srt[..., 1])         # largest + second largest
    else:
        group_score = g.max(dim=-1).values
    keep = torch.sort(-group_score, dim=-1, stable=True).indices[:, :topk_group]
    mask = torch.zeros(tokens, num_expert_group, dtype=torch.bool)
    mask.scatter_(1, keep, True)
    mask = mask.repeat_interleave(experts // num_expert_group, dim=1)
    masked = torch.where(mask, key, torch.full_like(key, float("-inf")))
    order = torch.sort(-masked, dim=-1, stable=True).indices[:, :top_k]
    w = scores.gather(1, order)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    return order.to(torch.int32), w.to(torch.float32)
