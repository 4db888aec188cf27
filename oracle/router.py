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
