"""The library's ops as torch custom ops (``torch.ops.b200_moe.*``).

CPU: every op is registered with its schema, out-arguments are marked as
written (``Tensor(a!)``, as the reference marks ``out`` in
``quant/sm70_fp8_moe/shim.cpp:50-56``), and the fake implementations give
the right shapes and dtypes on meta tensors (what fake-tensor propagation and
``torch.compile`` tracing see).

GPU: ``torch.library.opcheck`` on small cases (schema, fake tensors, AOT
dispatch), and one layer forward through ``torch.ops`` captured in a CUDA
graph and replayed.
"""

from __future__ import annotations

import pytest
import torch

from sglang_restomod_b200 import _lib, ops, synth, torch_ops
from tests.conftest import assert_close

B = torch.ops.b200_moe
META = torch.device("meta")


def test_every_op_is_registered_with_its_schema():
    names = torch_ops.names()
    assert {"moe_align_block_size", "moe_gemm", "moe_layer_forward", "linear", "moe_sum_reduce",
            "topk_route", "ep_dispatch", "ep_expert_forward", "ep_combine"} <= set(names)
    for name in names:
        schema = torch_ops.op(name)._schema
        assert schema.name == f"b200_moe::{name}"
    mutated = {
        "moe_sum_reduce": {"output"}, "moe_gemm": {"c"}, "linear_out": {"out"},
        "moe_layer_forward_out": {"out"}, "moe_layer_forward_fused_shared": {"out"},
        "moe_layer_forward_logits": {"out"}, "ep_dispatch": {"region"},
        "ep_expert_forward": {"region"}, "ep_combine": {"region", "out"},
        "w8a8_moe_gemm": {"c"},
    }
    for name in names:
        schema = torch_ops.op(name)._schema
        written = {a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write}
        assert written == mutated.get(name, set()), name


def test_fake_implementations_propagate_shapes():
    x = torch.empty(5, 256, dtype=torch.bfloat16, device=META)
    packed = torch.empty(1, 384 * 256, dtype=torch.uint8, device=META)
    assert B.linear(x, packed, 384, 0).shape == (5, 384)
    y = B.linear(x, packed, 384, 0, None, None, _lib.GATED_FUSED, torch.float16)
    assert y.shape == (5, 192) and y.dtype == torch.float16
    ids = torch.empty(5, 4, dtype=torch.int32, device=META)
    w = torch.empty(5, 4, dtype=torch.float32, device=META)
    sorted_ids, expert_ids, ntpp = B.moe_align_block_size(ids, 16, 8)
    cap, blocks = ops.align_capacity(20, 8, 16)
    assert sorted_ids.shape == (cap,) and expert_ids.shape == (blocks,) and ntpp.shape == (1,)
    assert sorted_ids.dtype == torch.int32
    out = B.moe_layer_forward(x, ids, w, 0, 8, 128, packed, packed)
    assert out.shape == x.shape and out.dtype == x.dtype
    ids2, w2 = B.moe_layer_forward_fused_shared(x, ids, w, 0, 8, 128, packed, packed, None, None,
                                                64, 1.0, 1.0, torch.empty_like(x))
    assert ids2.shape == (5, 5) and ids2.dtype == torch.int32 and w2.dtype == torch.float32
    r_ids, r_w = B.topk_route(torch.empty(5, 8, device=META), 2)
    assert r_ids.shape == (5, 2) and r_w.dtype == torch.float32
    q = torch.empty(3, 256, 384, dtype=torch.float8_e4m3fn, device=META)
    assert B.fp8_prepack(q, False).shape == (3, 256 * 384)
    wq = torch.empty(512, 256, dtype=torch.float8_e4m3fn, device=META)
    ws = torch.empty(4, 2, dtype=torch.float32, device=META)
    assert B.w8a8_linear(x, wq, ws, _lib.GATED_FUSED).shape == (5, 256)
    q8, s8 = B.fp8_act_quant(x, 8)
    assert q8.dtype == torch.float8_e4m3fn and q8.shape == (5, 256) and s8.shape == (2, 8)
    p4 = torch.empty(2, 256, 192, dtype=torch.uint8, device=META)
    s4 = torch.empty(2, 256, 24, dtype=torch.float8_e4m3fn, device=META)
    assert B.nvfp4_prepack(p4, s4, False).shape == (2, 2 * 3 * 9216)


# ---------------------------------------------------------------- on a B200
@pytest.mark.gpu
def test_opcheck_small_cases(cuda_device):
    dev = cuda_device
    k, n, m = 256, 384, 5
    q, s = synth.fp8_bank(1, n, k, dev, seed=1)
    packed = B.fp8_prepack(q[0], False)
    x = synth.activations(m, k, dev, seed=2)
    # (fp8_prepack is left out: opcheck's schema test multiplies the inputs,
    # which torch does not implement for float8 tensors)
    torch.library.opcheck(B.linear.default, (x, packed, n, _lib.QUANT_FP8_BLOCK, s[0]))
    torch.library.opcheck(B.linear_out.default,
                          (x, packed, n, _lib.QUANT_FP8_BLOCK, s[0], None, _lib.GATED_NONE,
                           torch.empty(m, n, dtype=torch.bfloat16, device=dev)))
    ids, w = synth.route(7, 8, 2, dev, seed=3)
    torch.library.opcheck(B.moe_align_block_size.default, (ids, 16, 8))
    logits = torch.randn(7, 8, device=dev)
    torch.library.opcheck(B.topk_route.default, (logits, 2))
    inp = torch.randn(7, 2, 256, device=dev, dtype=torch.bfloat16)
    torch.library.opcheck(B.moe_sum_reduce.default,
                          (inp, torch.empty(7, 256, device=dev, dtype=torch.bfloat16), 1.5))

    from sglang_restomod_b200.layer import QuantMoELayer

    shape = synth.MoEShape(hidden=256, inter=128, experts=8, top_k=2)
    layer = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, dev)
    xl = synth.activations(7, shape.hidden, dev, seed=4)
    args = (xl, ids, w, layer.quant, layer.num_experts, layer.inter, layer.w13, layer.w2,
            layer.w13_scales, layer.w2_scales, None, None, 16, 1.0, None)
    torch.library.opcheck(B.moe_layer_forward.default, args)
    torch.library.opcheck(B.moe_layer_forward_out.default, args + (torch.empty_like(xl),))
    sorted_ids, expert_ids, ntpp = B.moe_align_block_size(ids, 16, 8)
    c = torch.zeros(14, 2 * shape.inter, dtype=torch.bfloat16, device=dev)
    torch.library.opcheck(
        B.moe_gemm.default,
        (xl, layer.w13, 2 * shape.inter, layer.quant, 8, sorted_ids, expert_ids, ntpp, 16, 2, 14,
         c, layer.w13_scales))


@pytest.mark.gpu
def test_layer_forward_through_torch_ops_in_cuda_graph(cuda_device):
    """A layer forward (routed + shared expert, all through torch.ops.b200_moe)
    captured in a CUDA graph, replayed on new inputs, equals eager."""
    from sglang_restomod_b200.layer import QuantMoELayer

    dev = cuda_device
    shape = synth.MoEShape(hidden=512, inter=256, experts=16, top_k=4, shared_inter=256)
    layer = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, dev)
    tokens = 12
    x = synth.activations(tokens, shape.hidden, dev, seed=5)
    ids, w = synth.route(tokens, shape.experts, shape.top_k, dev, seed=6)
    out = torch.empty_like(x)
    layer.forward(x, ids, w, out=out)  # sizes the workspace before capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer.forward(x, ids, w, out=out)
    for seed in (7, 8):
        x.copy_(synth.activations(tokens, shape.hidden, dev, seed=seed))
        i2, w2 = synth.route(tokens, shape.experts, shape.top_k, dev, seed=seed + 10)
        ids.copy_(i2)
        w.copy_(w2)
        graph.replay()
        want = layer.forward(x, ids, w)
        torch.cuda.synchronize()
        assert_close(out, want, what=f"graph replay {seed}")
    assert ops.workspace_status() == 0
