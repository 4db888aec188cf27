"""A quantized fused-MoE layer (routed experts + optional shared expert).

This is the object the method classes and the benchmark drive: it holds the
prepacked banks and runs one forward through the torch custom ops
``torch.ops.b200_moe.*`` (:mod:`.torch_ops`), whose CUDA implementations call
the C ABI (``b200_moe_layer_forward`` plus the shared expert's two dense
calls).
Semantics follow ``SM70Fp8MoEMethod.apply``
(``sglang_restomod/quant/sm70_fp8_moe/method.py:239-309``): stable
expert-major routing, gated SiLU*up, router-weighted down projection,
top-k sum, ``routed_scaling_factor``; routes whose local id is -1 (expert
parallelism) contribute nothing.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib, ops, synth, torch_ops  # noqa: F401 - torch_ops registers torch.ops.b200_moe

B = torch.ops.b200_moe


def block_size_for(routes: int, experts: int) -> int:
    """Route slots per expert group for the streaming kernel.

    A group re-reads its expert's weights, so the block should hold the
    usual per-expert route count; larger blocks waste tensor-core rows,
    which the decode regime can afford (it is HBM-bound).

    Measured on B200 (block FP8, H=7168, I=2048, 1024 routes spread evenly
    over 256 / 128 / 64 / 32 experts, graph replay, ms per layer; blocks of 64
    run on the tensor-core GEMM, re-measured after its single-thread MMA loop):

    ============  =====  =====  =====  =====
    routes/expert   4      8     16     32
    blocks of 8   1.765  1.305  1.095  0.876
    blocks of 16  1.843  1.067  0.770  0.717
    blocks of 32  2.929  1.807  1.088  0.957
    blocks of 64  2.941  1.338  0.714  0.409
    ============  =====  =====  =====  =====

    and on the E=512 bank (H=2048, I=512, top-10; FP8 / NVFP4): 8 slots
    0.300 / 0.262 against 16 slots 0.309 / 0.302 ms at 5 routes per expert,
    0.377 / 0.328 against 0.331 / 0.329 ms at 7.5, so 8-slot groups up to 6
    routes per expert on average, 16-slot groups below 12, and from 12 on
    blocks of 64 on the tensor-core GEMM.
    """
    avg = routes / max(experts, 1)
    if avg <= 6:
        return 8
    if avg < 12:
        return 16
    return 64


@dataclass
class SharedExpert:
    """Always-on expert (weight 1): gate/up bank [2I, H] + down [H, I]."""

    quant: int
    inter: int
    w13: torch.Tensor
    w2: torch.Tensor
    w13_scales: torch.Tensor | None = None
    w2_scales: torch.Tensor | None = None
    w13_global: torch.Tensor | None = None
    w2_global: torch.Tensor | None = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = B.linear(x, self.w13, 2 * self.inter, self.quant, self.w13_scales, self.w13_global,
                     _lib.GATED_FUSED, torch.float16)
        return B.linear(h, self.w2, x.shape[-1], self.quant, self.w2_scales, self.w2_global,
                        _lib.GATED_NONE, x.dtype)

    launches_per_forward = 3  # bf16->f16 conversion, gate/up(+SiLU), down (decode rows)

    def launches(self, m: int, hidden: int, x_dtype=torch.bfloat16) -> int:
        """Kernels of one forward on m rows: the library's dense linear runs
        m > 32 on the tcgen05 GEMM and, when splitting K pays, adds a
        finishing kernel (the rule of b200_linear, `dense_k_parts`)."""
        n = 1 if x_dtype == torch.bfloat16 else 0
        sms = ops.num_sms()
        for rows_n, k in ((2 * self.inter, hidden), (hidden, self.inter)):
            n += 1
            if m >= 33:
                n += 1 if dense_k_parts(m, rows_n, k, sms) > 1 else 0
        return n


def dense_k_parts(m: int, n: int, k: int, sms: int) -> int:
    """K parts b200_linear's tcgen05 path uses for [m, k] x [n, k]^T (the
    library's rule, restated for launch accounting): items of 192 rows x 128
    weight rows go round-robin over the SMs; K is split when that cuts the
    busiest SM's 128-K units by a quarter or more, each part charged 3x the
    streaming time of its m*n fp32 partial sums, and only while the partials
    fit the workspace (2 CTAs per SM x 128 x 64 floats)."""
    if m * n > 2 * sms * 128 * 64:
        return 1
    kch = k // 128
    items = (m + 191) // 192 * (n // 128)
    part_cost = 3.0 * m * n * 4.0 / 16384.0 / sms
    whole = float((items + sms - 1) // sms * kch)
    best, best_parts = whole, 1
    for ks in range(2, min(16, kch) + 1):
        kpart = -(-kch // ks)
        parts = -(-kch // kpart)
        cost = (items * parts + sms - 1) // sms * kpart + part_cost * parts
        if cost < best:
            best, best_parts = cost, parts
    return best_parts if best < 0.75 * whole else 1


@dataclass
class QuantMoELayer:
    quant: int
    hidden: int
    inter: int
    num_experts: int  # experts held by this layer (local experts under EP)
    top_k: int
    w13: torch.Tensor
    w2: torch.Tensor
    w13_scales: torch.Tensor | None = None
    w2_scales: torch.Tensor | None = None
    w13_global: torch.Tensor | None = None
    w2_global: torch.Tensor | None = None
    shared: SharedExpert | None = None
    routed_scaling_factor: float = 1.0
    block_size: int | None = None
    # The banks hold the shared expert as one more expert (index num_experts)
    # after fuse_shared(): one routed launch computes it with the rest.
    shared_fused: bool = False
    # Grouped routing for forward_logits (upstream's num_expert_group /
    # topk_group): only the topk_group best expert groups are selectable.
    num_expert_group: int | None = None
    topk_group: int | None = None

    def can_fuse_shared(self) -> bool:
        s = self.shared
        return s is not None and s.quant == self.quant and s.inter == self.inter and \
            self.quant == _lib.QUANT_FP8_BLOCK

    def fuse_shared(self) -> "QuantMoELayer":
        """Append the shared expert to the routed banks (same shapes and block
        FP8). The separate SharedExpert stays for callers that run the routed
        experts alone (the NCCL expert-parallel transport)."""
        if self.shared_fused or not self.can_fuse_shared():
            return self
        s = self.shared
        self.w13 = torch.cat([self.w13, s.w13.reshape(1, -1)])
        self.w2 = torch.cat([self.w2, s.w2.reshape(1, -1)])
        self.w13_scales = torch.cat([self.w13_scales, s.w13_scales.unsqueeze(0)])
        self.w2_scales = torch.cat([self.w2_scales, s.w2_scales.unsqueeze(0)])
        self.shared_fused = True
        return self

    def fused_routes(self, topk_ids, topk_weights, shared_id=None):
        """Routes plus one shared route per token (weight 1 / rsf: the combine
        scales every route by rsf, the shared expert's output is unscaled)."""
        sid = self.num_experts if shared_id is None else shared_id
        return B.append_shared_route(topk_ids, topk_weights, sid, 1.0 / self.routed_scaling_factor)

    def fused_block_size(self, tokens: int, block_size=None) -> int | None:
        """Block size of the fused forward, or None when it should not be used.
        The shared expert's weights are streamed once per group of its tokens:
        fused when all tokens fit one group (small decode batches, saving the
        dense MLP's launches) or on the tensor-core GEMM (blocks of 64+, one
        item per weight block); with several 8-16-slot groups its weights
        would be streamed several times (measured 3 % slower at 128 tokens)."""
        if not self.shared_fused:
            return None
        bs = block_size or self.block_size or block_size_for(tokens * (self.top_k + 1),
                                                             self.num_experts + 1)
        return bs if bs >= 64 or tokens <= bs else None

    def forward(self, x, topk_ids, topk_weights, out=None, shared_out=None, block_size=None,
                use_shared=True):
        tokens, top_k = topk_ids.shape
        bs = self.fused_block_size(tokens, block_size) if use_shared and shared_out is None else None
        if bs is not None:
            # the shared route is appended inside the library call
            if out is None:
                out = torch.empty_like(x)
            B.moe_layer_forward_fused_shared(
                x, topk_ids, topk_weights, self.quant, self.num_experts, self.inter, self.w13,
                self.w2, self.w13_scales, self.w2_scales, bs, self.routed_scaling_factor,
                1.0 / self.routed_scaling_factor, out)
            return out
        if use_shared and shared_out is None and self.shared is not None:
            shared_out = self.shared.forward(x)
        bs = block_size or self.block_size or block_size_for(tokens * top_k, self.num_experts)
        args = (x, topk_ids, topk_weights, self.quant, self.num_experts, self.inter, self.w13,
                self.w2, self.w13_scales, self.w2_scales, self.w13_global, self.w2_global, bs,
                self.routed_scaling_factor, shared_out)
        if out is None:
            return B.moe_layer_forward(*args)
        B.moe_layer_forward_out(*args, out)
        return out

    def forward_logits(self, x, router_logits, out=None, scoring: int = _lib.SCORING_SOFTMAX,
                       renormalize: bool = True, correction_bias=None):
        """Route with the library's top-k kernel, then forward (the routing of
        the benchmark: softmax -> top-k -> renormalise). Without a fused
        shared expert this is one library call, whose router and moe_align
        share a launch for decode batches."""
        tokens = x.shape[0]
        if self.num_expert_group:
            ids, w = B.topk_route_grouped(router_logits, self.top_k, self.num_expert_group,
                                          self.topk_group or self.num_expert_group, scoring,
                                          renormalize, correction_bias)
            return self.forward(x, ids, w, out=out)
        if self.fused_block_size(tokens) is None:
            shared_out = self.shared.forward(x) if self.shared is not None else None
            bs = self.block_size or block_size_for(tokens * self.top_k, self.num_experts)
            if out is None:
                out = torch.empty_like(x)
            B.moe_layer_forward_logits(
                x, router_logits, self.top_k, self.quant, self.num_experts, self.inter, self.w13,
                self.w2, self.w13_scales, self.w2_scales, self.w13_global, self.w2_global, bs,
                self.routed_scaling_factor, shared_out, scoring, renormalize, correction_bias,
                out)
            return out
        ids, w = B.topk_route(router_logits, self.top_k, scoring, renormalize, correction_bias)
        return self.forward(x, ids, w, out=out)

    def launches_per_forward(self, x_dtype=torch.bfloat16, tokens: int | None = None) -> int:
        """Kernels of one forward on ``tokens`` rows, following the library's
        rules: up to 4095 routes one preparation kernel ([shared-route
        append +] align [+ bf16 conversion]), from 4096 on the three-kernel
        align with the append and the conversion as their own launches;
        blocks of 64+ run the tcgen05 GEMMs, which add their plan and the
        slot-order copy of the activations (instead of the conversion); then
        gate/up, down and the combine, plus the separate shared MLP when the
        shared expert is not fused into this forward."""
        bf16 = x_dtype == torch.bfloat16
        fused = tokens is not None and self.fused_block_size(tokens) is not None
        if fused:
            routes = tokens * (self.top_k + 1)
            bs = self.fused_block_size(tokens)
        elif tokens is not None:
            routes = tokens * self.top_k
            bs = self.block_size or block_size_for(routes, self.num_experts)
        else:
            routes, bs = 0, self.block_size or 16
        tc = bs >= 64
        n = 3  # gate/up, down, combine
        if routes >= 4096:
            n += 3 + (1 if fused else 0) + (1 if bf16 and not tc else 0)
        else:
            n += 1
        if tc:
            n += 2
        if not fused and self.shared is not None:
            n += (self.shared.launches(tokens, self.hidden, x_dtype) if tokens is not None
                  else SharedExpert.launches_per_forward)
        return n

    def weight_bytes_per_expert(self) -> int:
        if self.quant == _lib.QUANT_FP8_BLOCK:
            return 3 * self.hidden * self.inter + 3 * (self.hidden // 128) * (self.inter // 128) * 4
        return 3 * self.hidden * self.inter // 2 + 3 * self.hidden * self.inter // 16

    @classmethod
    def synthetic(cls, shape: synth.MoEShape, quant: int, device, first_expert: int = 0,
                  num_experts: int | None = None, seed: int = 10,
                  fuse_shared: bool = False) -> "QuantMoELayer":
        """Random-init layer of ``shape`` holding experts [first, first + num)
        (the shared expert appended to the banks when ``fuse_shared`` and the
        shapes allow)."""
        e = shape.experts if num_experts is None else num_experts
        h, i = shape.hidden, shape.inter
        if quant == _lib.QUANT_FP8_BLOCK:
            q13, s13 = synth.fp8_bank(e, 2 * i, h, device, seed, first_expert)
            w13 = B.fp8_prepack(q13, True)
            del q13
            q2, s2 = synth.fp8_bank(e, h, i, device, seed + 1, first_expert)
            w2 = B.fp8_prepack(q2, False)
            del q2
            kw = dict(w13_scales=s13, w2_scales=s2)
        else:
            p13, s13, g13 = synth.nvfp4_bank(e, 2 * i, h, device, seed, first_expert)
            w13 = B.nvfp4_prepack(p13, s13, True)
            del p13, s13
            p2, s2, g2 = synth.nvfp4_bank(e, h, i, device, seed + 1, first_expert)
            w2 = B.nvfp4_prepack(p2, s2, False)
            del p2, s2
            kw = dict(w13_global=g13, w2_global=g2)
        shared = None
        if shape.shared_inter:
            si = shape.shared_inter
            # The shared expert stays block-FP8 in both checkpoints
            # (its dense path is the FP8 linear).
            q13, s13 = synth.fp8_bank(1, 2 * si, h, device, seed + 2, 0)
            q2, s2 = synth.fp8_bank(1, h, si, device, seed + 3, 0)
            shared = SharedExpert(
                quant=_lib.QUANT_FP8_BLOCK, inter=si, w13=B.fp8_prepack(q13[0], True),
                w2=B.fp8_prepack(q2[0], False), w13_scales=s13[0], w2_scales=s2[0],
            )
        layer = cls(quant=quant, hidden=h, inter=i, num_experts=e, top_k=shape.top_k, w13=w13,
                    w2=w2, shared=shared, **kw)
        return layer.fuse_shared() if fuse_shared else layer
