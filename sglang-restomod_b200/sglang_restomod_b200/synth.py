"""Seeded synthetic inputs for the benchmark configurations.

No dataset or checkpoint is involved: the configurations are defined by
their shapes and value distributions - activations bf16 ~ N(0, 1), router
logits fp32 ~ N(0, 1) -> softmax -> top-k -> renormalised, weights
~ N(0, 0.02) quantized to block FP8 (128x128 fp32 scales, amax / 448) or
NVFP4 (E2M1, E4M3 per 16 K, fp32 global per expert-matrix).

Generation runs on the target device with a seeded generator, one expert at
a time, so even the 11 GB expert-parallel bank is built in seconds.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .quant.quantize import quantize_block_fp8, quantize_nvfp4

WEIGHT_STD = 0.02


@dataclass(frozen=True)
class MoEShape:
    hidden: int
    inter: int
    experts: int
    top_k: int
    shared_inter: int = 0


# The configurations named by the benchmark definition.
CONFIG0 = MoEShape(hidden=1024, inter=512, experts=16, top_k=4)
CONFIG2 = MoEShape(hidden=2048, inter=512, experts=512, top_k=10, shared_inter=512)
CONFIG4 = MoEShape(hidden=7168, inter=2048, experts=256, top_k=8, shared_inter=2048)
DENSE_SHAPES = ((5120, 25600), (25600, 5120), (5120, 152064))  # (K, N)


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def activations(tokens: int, hidden: int, device, seed: int = 0, dtype=torch.bfloat16):
    g = _gen(device, seed)
    return torch.randn(tokens, hidden, generator=g, device=device).to(dtype)


def route(tokens: int, experts: int, top_k: int, device, seed: int = 1):
    """(topk_ids int32 [T, k], topk_weights fp32 [T, k])."""
    g = _gen(device, seed)
    logits = torch.randn(tokens, experts, generator=g, device=device)
    probs = torch.softmax(logits, dim=-1)
    w, ids = torch.topk(probs, top_k, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    return ids.to(torch.int32).contiguous(), w.float().contiguous()


def _expert_gen(device, seed: int, expert: int) -> torch.Generator:
    # One generator per global expert: a rank holding experts [a, b) builds
    # exactly the experts a single GPU would, whatever the world size.
    return _gen(device, seed * 1_000_003 + expert)


def fp8_bank(experts: int, n: int, k: int, device, seed: int, first_expert: int = 0):
    """(e4m3 [E, N, K], fp32 scales [E, N/128, K/128]) for global experts
    [first_expert, first_expert + experts)."""
    q = torch.empty(experts, n, k, dtype=torch.float8_e4m3fn, device=device)
    s = torch.empty(experts, n // 128, k // 128, dtype=torch.float32, device=device)
    for e in range(experts):
        g = _expert_gen(device, seed, first_expert + e)
        w = torch.randn(n, k, generator=g, device=device) * WEIGHT_STD
        q[e], s[e] = quantize_block_fp8(w)
    return q, s


def nvfp4_bank(experts: int, n: int, k: int, device, seed: int, first_expert: int = 0):
    """(packed uint8 [E, N, K/2], e4m3 [E, N, K/16], fp32 global [E])."""
    p = torch.empty(experts, n, k // 2, dtype=torch.uint8, device=device)
    s = torch.empty(experts, n, k // 16, dtype=torch.float8_e4m3fn, device=device)
    gs = torch.empty(experts, dtype=torch.float32, device=device)
    for e in range(experts):
        g = _expert_gen(device, seed, first_expert + e)
        w = torch.randn(n, k, generator=g, device=device) * WEIGHT_STD
        p[e], s[e], gs[e] = quantize_nvfp4(w)
    return p, s, gs
