"""The library's operations as torch custom ops: ``torch.ops.b200_moe.*``.

The reference exposes its kernels to SGLang through the torch dispatcher
(``TORCH_LIBRARY(sglang_sm70_fp8_moe, ...)`` with ``ops.impl(..., kCUDA, ...)``
in ``quant/sm70_fp8_moe/shim.cpp:50-56``; ``torch.ops.sglang_sm70_turbomind.*``
in ``quant/sm70_fp8_dense/_method.py:750-772``). This module does the same
for libb200moe: every op has a schema, a CUDA implementation that calls the
C ABI through :mod:`ops` on the current stream, and a fake (meta)
implementation, so the dispatcher, fake-tensor propagation and
``torch.compile`` tracing see the ops' shapes, dtypes and the buffers they
write. The C ABI library itself has no torch dependency; the registration
lives here, on the torch side of the boundary.

Two kinds of ops:

* functional ones return new tensors (``linear``, ``moe_layer_forward``,
  ``moe_align_block_size``, ``topk_route``, the prepacks, ...);
* out-variants write caller-owned buffers and return nothing, marked
  ``Tensor(a!)`` in their schema as the reference marks ``out``
  (``moe_gemm``, ``moe_sum_reduce``, ``linear_out``,
  ``moe_layer_forward_out``, the expert-parallel exchange).

Importing the package registers the namespace once.
"""

from __future__ import annotations

import torch

from . import _lib, census, ops

NAMESPACE = "b200_moe"

_DEF = torch.library.Library(NAMESPACE, "DEF")

_SCHEMAS = {
    # routing
    "moe_align_block_size":
        "moe_align_block_size(Tensor topk_ids, int block_size, int num_experts)"
        " -> (Tensor, Tensor, Tensor)",
    "topk_route":
        "topk_route(Tensor router_logits, int top_k, int scoring=0, bool renormalize=True,"
        " Tensor? correction_bias=None) -> (Tensor, Tensor)",
    "topk_route_grouped":
        "topk_route_grouped(Tensor router_logits, int top_k, int num_expert_group, int topk_group,"
        " int scoring=0, bool renormalize=True, Tensor? correction_bias=None) -> (Tensor, Tensor)",
    "append_shared_route":
        "append_shared_route(Tensor topk_ids, Tensor topk_weights, int shared_id,"
        " float shared_weight) -> (Tensor, Tensor)",
    # combine
    "moe_sum_reduce":
        "moe_sum_reduce(Tensor input, Tensor(a!) output, float routed_scaling_factor) -> ()",
    "moe_combine":
        "moe_combine(Tensor routed, Tensor topk_ids, int num_experts, float routed_scaling_factor,"
        " Tensor? shared_out, ScalarType out_dtype) -> Tensor",
    # load-time prepacks
    "fp8_prepack": "fp8_prepack(Tensor w, bool gated) -> Tensor",
    "nvfp4_prepack": "nvfp4_prepack(Tensor w, Tensor scales, bool gated) -> Tensor",
    # GEMMs
    "linear":
        "linear(Tensor x, Tensor packed, int n, int quant, Tensor? scales=None,"
        " Tensor? global_scale=None, int gated_mode=0, ScalarType? out_dtype=None) -> Tensor",
    "linear_out":
        "linear_out(Tensor x, Tensor packed, int n, int quant, Tensor? scales,"
        " Tensor? global_scale, int gated_mode, Tensor(a!) out) -> ()",
    "moe_gemm":
        "moe_gemm(Tensor a, Tensor packed, int n, int quant, int num_experts,"
        " Tensor sorted_token_ids, Tensor expert_ids, Tensor num_tokens_post_pad, int block_size,"
        " int top_k, int num_routes, Tensor(a!) c, Tensor? scales=None,"
        " Tensor? global_scale=None, Tensor? topk_weights=None, bool mul_topk_weights=False,"
        " int gated_mode=0) -> ()",
    # the fused layer
    "moe_layer_forward":
        "moe_layer_forward(Tensor x, Tensor topk_ids, Tensor topk_weights, int quant,"
        " int num_experts, int inter, Tensor w13, Tensor w2, Tensor? w13_scales=None,"
        " Tensor? w2_scales=None, Tensor? w13_global=None, Tensor? w2_global=None,"
        " int block_size=16, float routed_scaling_factor=1.0, Tensor? shared_out=None) -> Tensor",
    "moe_layer_forward_out":
        "moe_layer_forward_out(Tensor x, Tensor topk_ids, Tensor topk_weights, int quant,"
        " int num_experts, int inter, Tensor w13, Tensor w2, Tensor? w13_scales,"
        " Tensor? w2_scales, Tensor? w13_global, Tensor? w2_global, int block_size,"
        " float routed_scaling_factor, Tensor? shared_out, Tensor(a!) out) -> ()",
    "moe_layer_forward_fused_shared":
        "moe_layer_forward_fused_shared(Tensor x, Tensor topk_ids, Tensor topk_weights, int quant,"
        " int num_experts, int inter, Tensor w13, Tensor w2, Tensor? w13_scales,"
        " Tensor? w2_scales, int block_size, float routed_scaling_factor,"
        " float shared_route_weight, Tensor(a!) out) -> (Tensor, Tensor)",
    "moe_layer_forward_logits":
        "moe_layer_forward_logits(Tensor x, Tensor router_logits, int top_k, int quant,"
        " int num_experts, int inter, Tensor w13, Tensor w2, Tensor? w13_scales,"
        " Tensor? w2_scales, Tensor? w13_global, Tensor? w2_global, int block_size,"
        " float routed_scaling_factor, Tensor? shared_out, int scoring, bool renormalize,"
        " Tensor? correction_bias, Tensor(a!) out) -> (Tensor, Tensor)",
    # W8A8 block FP8 (opt-in: quantizes the activations)
    "fp8_act_quant": "fp8_act_quant(Tensor x, int? scales_ld=None) -> (Tensor, Tensor)",
    "w8a8_linear":
        "w8a8_linear(Tensor x, Tensor w, Tensor w_scales, int gated_mode=0,"
        " ScalarType? out_dtype=None) -> Tensor",
    "w8a8_moe_gemm":
        "w8a8_moe_gemm(Tensor a, Tensor w, Tensor w_scales, int num_experts,"
        " Tensor sorted_token_ids, Tensor expert_ids, Tensor num_tokens_post_pad, int block_size,"
        " int top_k, int num_routes, Tensor(a!) c, Tensor? topk_weights=None,"
        " bool mul_topk_weights=False, int gated_mode=0) -> ()",
    # expert parallelism over peer memory
    "ep_dispatch":
        "ep_dispatch(Tensor x, Tensor topk_ids, Tensor topk_weights, int num_experts, int rank,"
        " int world, Tensor peers, Tensor(a!) region, int max_tokens, bool shared_expert) -> ()",
    "ep_expert_forward":
        "ep_expert_forward(int quant, int hidden, int inter, int local_experts, Tensor w13,"
        " Tensor w2, Tensor? w13_scales, Tensor? w2_scales, Tensor? w13_global,"
        " Tensor? w2_global, int block_size, int rank, int world, Tensor peers,"
        " Tensor(a!) region, int max_tokens, int top_k) -> ()",
    "ep_combine":
        "ep_combine(Tensor topk_ids, int hidden, int num_experts, int world, Tensor(a!) region,"
        " int max_tokens, float routed_scaling_factor, Tensor? shared_out,"
        " Tensor(b!) out) -> ()",
}

for _schema in _SCHEMAS.values():
    _DEF.define(_schema)


def _impl(name):
    def deco(fn):
        _DEF.impl(name, fn, "CUDA")
        return fn

    return deco


def _fake(name):
    return torch.library.register_fake(f"{NAMESPACE}::{name}")


# ------------------------------------------------------------------ routing
@_impl("moe_align_block_size")
def _align_cuda(topk_ids, block_size, num_experts):
    return ops.moe_align_block_size(topk_ids, block_size, num_experts)


@_fake("moe_align_block_size")
def _align_fake(topk_ids, block_size, num_experts):
    cap, blocks = ops.align_capacity(topk_ids.numel(), num_experts, block_size)
    i32 = dict(dtype=torch.int32, device=topk_ids.device)
    return topk_ids.new_empty(cap, **i32), topk_ids.new_empty(blocks, **i32), \
        topk_ids.new_empty(1, **i32)


@_impl("topk_route")
def _topk_cuda(router_logits, top_k, scoring=0, renormalize=True, correction_bias=None):
    return ops.topk_route(router_logits, top_k, scoring=scoring, renormalize=renormalize,
                          correction_bias=correction_bias)


@_fake("topk_route")
def _topk_fake(router_logits, top_k, scoring=0, renormalize=True, correction_bias=None):
    t = router_logits.shape[0]
    return (router_logits.new_empty(t, top_k, dtype=torch.int32),
            router_logits.new_empty(t, top_k, dtype=torch.float32))


@_impl("topk_route_grouped")
def _topk_grouped_cuda(router_logits, top_k, num_expert_group, topk_group, scoring=0,
                       renormalize=True, correction_bias=None):
    return ops.topk_route_grouped(router_logits, top_k, num_expert_group, topk_group,
                                  scoring=scoring, renormalize=renormalize,
                                  correction_bias=correction_bias)


@_fake("topk_route_grouped")
def _topk_grouped_fake(router_logits, top_k, num_expert_group, topk_group, scoring=0,
                       renormalize=True, correction_bias=None):
    t = router_logits.shape[0]
    return (router_logits.new_empty(t, top_k, dtype=torch.int32),
            router_logits.new_empty(t, top_k, dtype=torch.float32))


@_impl("append_shared_route")
def _append_cuda(topk_ids, topk_weights, shared_id, shared_weight):
    return ops.append_shared_route(topk_ids, topk_weights, shared_id, shared_weight)


@_fake("append_shared_route")
def _append_fake(topk_ids, topk_weights, shared_id, shared_weight):
    t, k = topk_ids.shape
    return topk_ids.new_empty(t, k + 1), topk_weights.new_empty(t, k + 1)


# ------------------------------------------------------------------ combine
@_impl("moe_sum_reduce")
def _sum_reduce_cuda(input, output, routed_scaling_factor):  # noqa: A002 - upstream's name
    ops.moe_sum_reduce(input, output, routed_scaling_factor)


@_fake("moe_sum_reduce")
def _sum_reduce_fake(input, output, routed_scaling_factor):  # noqa: A002
    return None


@_impl("moe_combine")
def _combine_cuda(routed, topk_ids, num_experts, routed_scaling_factor, shared_out, out_dtype):
    return ops.moe_combine(routed, topk_ids, num_experts, routed_scaling_factor,
                           shared_out=shared_out, out_dtype=out_dtype)


@_fake("moe_combine")
def _combine_fake(routed, topk_ids, num_experts, routed_scaling_factor, shared_out, out_dtype):
    return routed.new_empty(topk_ids.shape[0], routed.shape[-1], dtype=out_dtype)


# ------------------------------------------------------------------ prepack
@_impl("fp8_prepack")
def _fp8_prepack_cuda(w, gated):
    return ops.fp8_prepack(w, gated)


@_fake("fp8_prepack")
def _fp8_prepack_fake(w, gated):
    w3 = w.unsqueeze(0) if w.dim() == 2 else w
    e, n, k = w3.shape
    return w.new_empty(e, n * k, dtype=torch.uint8)


@_impl("nvfp4_prepack")
def _nvfp4_prepack_cuda(w, scales, gated):
    return ops.nvfp4_prepack(w, scales, gated)


@_fake("nvfp4_prepack")
def _nvfp4_prepack_fake(w, scales, gated):
    w3 = w.unsqueeze(0) if w.dim() == 2 else w
    e, n, half_k = w3.shape
    per_expert = (n // 128) * (2 * half_k // 128) * 9216
    return w.new_empty(e, per_expert, dtype=torch.uint8)


# -------------------------------------------------------------------- GEMMs
def _linear_cols(n, gated_mode):
    return n // 2 if gated_mode == _lib.GATED_FUSED else n


@_impl("linear")
def _linear_cuda(x, packed, n, quant, scales=None, global_scale=None, gated_mode=0,
                 out_dtype=None):
    census.note_linear("linear", x.numel() // max(x.shape[-1], 1), n, x.shape[-1])
    return ops.linear(x, packed, n, quant=quant, scales=scales, global_scale=global_scale,
                      gated_mode=gated_mode, out_dtype=out_dtype)


@_fake("linear")
def _linear_fake(x, packed, n, quant, scales=None, global_scale=None, gated_mode=0,
                 out_dtype=None):
    return x.new_empty(*x.shape[:-1], _linear_cols(n, gated_mode), dtype=out_dtype or x.dtype)


@_impl("linear_out")
def _linear_out_cuda(x, packed, n, quant, scales, global_scale, gated_mode, out):
    census.note_linear("linear", x.numel() // max(x.shape[-1], 1), n, x.shape[-1])
    ops.linear(x, packed, n, quant=quant, scales=scales, global_scale=global_scale,
               gated_mode=gated_mode, out=out)


@_fake("linear_out")
def _linear_out_fake(x, packed, n, quant, scales, global_scale, gated_mode, out):
    return None


@_impl("moe_gemm")
def _moe_gemm_cuda(a, packed, n, quant, num_experts, sorted_token_ids, expert_ids,
                   num_tokens_post_pad, block_size, top_k, num_routes, c, scales=None,
                   global_scale=None, topk_weights=None, mul_topk_weights=False, gated_mode=0):
    census.note_moe("moe_gemm", quant, a.shape[0], num_routes, num_experts, block_size,
                    min(expert_ids.numel(), sorted_token_ids.numel() // block_size), n,
                    a.shape[-1])
    ops.moe_gemm(a, packed, n, quant=quant, num_experts=num_experts,
                 sorted_token_ids=sorted_token_ids, expert_ids=expert_ids,
                 num_tokens_post_pad=num_tokens_post_pad, block_size=block_size, top_k=top_k,
                 num_routes=num_routes, c=c, scales=scales, global_scale=global_scale,
                 topk_weights=topk_weights, mul_topk_weights=mul_topk_weights,
                 gated_mode=gated_mode)


@_fake("moe_gemm")
def _moe_gemm_fake(a, packed, n, quant, num_experts, sorted_token_ids, expert_ids,
                   num_tokens_post_pad, block_size, top_k, num_routes, c, scales=None,
                   global_scale=None, topk_weights=None, mul_topk_weights=False, gated_mode=0):
    return None


# ---------------------------------------------------------------- the layer
def _note_layer(op, quant, topk_ids, num_experts, block_size, inter, hidden):
    t, k = topk_ids.shape
    census.note_moe(op, quant, t, t * k, num_experts, block_size,
                    ops.align_capacity(t * k, num_experts, block_size)[1], 2 * inter, hidden)


def _layer_kw(quant, num_experts, inter, w13, w2, w13_scales, w2_scales, w13_global, w2_global,
              block_size, routed_scaling_factor, shared_out):
    return dict(quant=quant, num_experts=num_experts, inter=inter, w13=w13, w2=w2,
                w13_scales=w13_scales, w2_scales=w2_scales, w13_global=w13_global,
                w2_global=w2_global, block_size=block_size,
                routed_scaling_factor=routed_scaling_factor, shared_out=shared_out)


@_impl("moe_layer_forward")
def _layer_cuda(x, topk_ids, topk_weights, quant, num_experts, inter, w13, w2, w13_scales=None,
                w2_scales=None, w13_global=None, w2_global=None, block_size=16,
                routed_scaling_factor=1.0, shared_out=None):
    _note_layer("moe_layer", quant, topk_ids, num_experts, block_size, inter, x.shape[-1])
    return ops.moe_layer_forward(x, topk_ids, topk_weights, **_layer_kw(
        quant, num_experts, inter, w13, w2, w13_scales, w2_scales, w13_global, w2_global,
        block_size, routed_scaling_factor, shared_out))


@_fake("moe_layer_forward")
def _layer_fake(x, topk_ids, topk_weights, quant, num_experts, inter, w13, w2, w13_scales=None,
                w2_scales=None, w13_global=None, w2_global=None, block_size=16,
                routed_scaling_factor=1.0, shared_out=None):
    return torch.empty_like(x)


@_impl("moe_layer_forward_out")
def _layer_out_cuda(x, topk_ids, topk_weights, quant, num_experts, inter, w13, w2, w13_scales,
                    w2_scales, w13_global, w2_global, block_size, routed_scaling_factor,
                    shared_out, out):
    _note_layer("moe_layer", quant, topk_ids, num_experts, block_size, inter, x.shape[-1])
    ops.moe_layer_forward(x, topk_ids, topk_weights, out=out, **_layer_kw(
        quant, num_experts, inter, w13, w2, w13_scales, w2_scales, w13_global, w2_global,
        block_size, routed_scaling_factor, shared_out))


@_fake("moe_layer_forward_out")
def _layer_out_fake(x, topk_ids, topk_weights, quant, num_experts, inter, w13, w2, w13_scales,
                    w2_scales, w13_global, w2_global, block_size, routed_scaling_factor,
                    shared_out, out):
    return None


@_impl("moe_layer_forward_fused_shared")
def _layer_fused_cuda(x, topk_ids, topk_weights, quant, num_experts, inter, w13, w2, w13_scales,
                      w2_scales, block_size, routed_scaling_factor, shared_route_weight, out):
    t, k = topk_ids.shape
    census.note_moe("moe_layer+shared", quant, t, t * (k + 1), num_experts + 1, block_size,
                    ops.align_capacity(t * (k + 1), num_experts + 1, block_size)[1], 2 * inter,
                    x.shape[-1])
    _, ids, w = ops.moe_layer_forward_fused_shared(
        x, topk_ids, topk_weights, quant=quant, num_experts=num_experts, inter=inter, w13=w13,
        w2=w2, w13_scales=w13_scales, w2_scales=w2_scales, block_size=block_size,
        routed_scaling_factor=routed_scaling_factor, shared_route_weight=shared_route_weight,
        out=out)
    return ids, w


@_fake("moe_layer_forward_fused_shared")
def _layer_fused_fake(x, topk_ids, topk_weights, quant, num_experts, inter, w13, w2, w13_scales,
                      w2_scales, block_size, routed_scaling_factor, shared_route_weight, out):
    t, k = topk_ids.shape
    return topk_ids.new_empty(t, k + 1), topk_weights.new_empty(t, k + 1)


@_impl("moe_layer_forward_logits")
def _layer_logits_cuda(x, router_logits, top_k, quant, num_experts, inter, w13, w2, w13_scales,
                       w2_scales, w13_global, w2_global, block_size, routed_scaling_factor,
                       shared_out, scoring, renormalize, correction_bias, out):
    _, ids, w = ops.moe_layer_forward_logits(
        x, router_logits, top_k, out=out, scoring=scoring, renormalize=renormalize,
        correction_bias=correction_bias, **_layer_kw(
            quant, num_experts, inter, w13, w2, w13_scales, w2_scales, w13_global, w2_global,
            block_size, routed_scaling_factor, shared_out))
    return ids, w


@_fake("moe_layer_forward_logits")
def _layer_logits_fake(x, router_logits, top_k, quant, num_experts, inter, w13, w2, w13_scales,
                       w2_scales, w13_global, w2_global, block_size, routed_scaling_factor,
                       shared_out, scoring, renormalize, correction_bias, out):
    t = x.shape[0]
    return (x.new_empty(t, top_k, dtype=torch.int32), x.new_empty(t, top_k, dtype=torch.float32))


# ------------------------------------------------------------------- W8A8
@_impl("fp8_act_quant")
def _act_quant_cuda(x, scales_ld=None):
    return ops.fp8_act_quant(x, scales_ld)


@_fake("fp8_act_quant")
def _act_quant_fake(x, scales_ld=None):
    rows, k = x.shape
    ld = rows if scales_ld is None else scales_ld
    return (x.new_empty(rows, k, dtype=torch.float8_e4m3fn),
            x.new_empty(k // 128, ld, dtype=torch.float32))


@_impl("w8a8_linear")
def _w8a8_linear_cuda(x, w, w_scales, gated_mode=0, out_dtype=None):
    census.note("w8a8_linear", f"m={x.numel() // max(x.shape[-1], 1)}", f"n={w.shape[-2]}",
                f"k={x.shape[-1]}")
    return ops.w8a8_linear(x, w, w_scales, gated_mode=gated_mode, out_dtype=out_dtype)


@_fake("w8a8_linear")
def _w8a8_linear_fake(x, w, w_scales, gated_mode=0, out_dtype=None):
    return x.new_empty(*x.shape[:-1], _linear_cols(w.shape[-2], gated_mode),
                       dtype=out_dtype or x.dtype)


@_impl("w8a8_moe_gemm")
def _w8a8_moe_cuda(a, w, w_scales, num_experts, sorted_token_ids, expert_ids,
                   num_tokens_post_pad, block_size, top_k, num_routes, c, topk_weights=None,
                   mul_topk_weights=False, gated_mode=0):
    census.note("w8a8_moe_gemm", f"routes={num_routes}", f"experts={num_experts}",
                f"block={block_size}", f"n={w.shape[-2]}", f"k={a.shape[-1]}")
    ops.w8a8_moe_gemm(a, w, w_scales, num_experts=num_experts, sorted_token_ids=sorted_token_ids,
                      expert_ids=expert_ids, num_tokens_post_pad=num_tokens_post_pad,
                      block_size=block_size, top_k=top_k, num_routes=num_routes, c=c,
                      topk_weights=topk_weights, mul_topk_weights=mul_topk_weights,
                      gated_mode=gated_mode)


@_fake("w8a8_moe_gemm")
def _w8a8_moe_fake(a, w, w_scales, num_experts, sorted_token_ids, expert_ids,
                   num_tokens_post_pad, block_size, top_k, num_routes, c, topk_weights=None,
                   mul_topk_weights=False, gated_mode=0):
    return None


# ------------------------------------------------------ expert parallelism
@_impl("ep_dispatch")
def _ep_dispatch_cuda(x, topk_ids, topk_weights, num_experts, rank, world, peers, region,
                      max_tokens, shared_expert):
    ops.ep_dispatch(x, topk_ids, topk_weights, num_experts=num_experts, rank=rank, world=world,
                    peers=peers, region=region, max_tokens=max_tokens,
                    shared_expert=shared_expert)


@_fake("ep_dispatch")
def _ep_dispatch_fake(x, topk_ids, topk_weights, num_experts, rank, world, peers, region,
                      max_tokens, shared_expert):
    return None


@_impl("ep_expert_forward")
def _ep_experts_cuda(quant, hidden, inter, local_experts, w13, w2, w13_scales, w2_scales,
                     w13_global, w2_global, block_size, rank, world, peers, region, max_tokens,
                     top_k):
    ops.ep_expert_forward(quant=quant, hidden=hidden, inter=inter, local_experts=local_experts,
                          w13=w13, w2=w2, w13_scales=w13_scales, w2_scales=w2_scales,
                          w13_global=w13_global, w2_global=w2_global, block_size=block_size,
                          rank=rank, world=world, peers=peers, region=region,
                          max_tokens=max_tokens, top_k=top_k)


@_fake("ep_expert_forward")
def _ep_experts_fake(quant, hidden, inter, local_experts, w13, w2, w13_scales, w2_scales,
                     w13_global, w2_global, block_size, rank, world, peers, region, max_tokens,
                     top_k):
    return None


@_impl("ep_combine")
def _ep_combine_cuda(topk_ids, hidden, num_experts, world, region, max_tokens,
                     routed_scaling_factor, shared_out, out):
    ops.ep_combine(topk_ids, hidden=hidden, num_experts=num_experts, world=world, region=region,
                   max_tokens=max_tokens, routed_scaling_factor=routed_scaling_factor,
                   shared_out=shared_out, out=out)


@_fake("ep_combine")
def _ep_combine_fake(topk_ids, hidden, num_experts, world, region, max_tokens,
                     routed_scaling_factor, shared_out, out):
    return None


def op(name: str):
    """``torch.ops.b200_moe.<name>`` (the default overload)."""
    return getattr(getattr(torch.ops, NAMESPACE), name).default


def names() -> list[str]:
    return list(_SCHEMAS)
