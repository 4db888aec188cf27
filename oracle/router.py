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
