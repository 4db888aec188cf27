"""GPU: the plugin-surface components, driven the way SGLang drives the
reference's, against the CPU oracle (rtol / atol 2e-2)."""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

import oracle
from sglang_restomod_b200 import ops, synth
from sglang_restomod_b200.quant import fp8_moe
from sglang_restomod_b200.quant.fp8_moe.method import B200Fp8MoEMethod
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu


def _runner_cfg(top_k, experts, local, rsf=1.0):
    return SimpleNamespace(activation="silu", is_gated=True, top_k=top_k, num_experts=experts,
                           num_local_experts=local, routed_scaling_factor=rsf,
                           swiglu_limit=None, gemm1_clamp_limit=None, gemm1_alpha=None,
                           gemm1_beta=None, apply_router_weight_on_input=False, no_combine=False)


def _fp8_layer(experts, hidden, inter, dev):
    q13, s13 = synth.fp8_bank(experts, 2 * inter, hidden, dev, seed=40)
    q2, s2 = synth.fp8_bank(experts, hidden, inter, dev, seed=41)
    P = torch.nn.Parameter
    layer = torch.nn.Module()
    layer.w13_weight = P(q13.clone(), requires_grad=False)
    layer.w2_weight = P(q2.clone(), requires_grad=False)
    layer.w13_weight_scale_inv = P(s13.clone(), requires_grad=False)
    layer.w2_weight_scale_inv = P(s2.clone(), requires_grad=False)
    layer.should_fuse_routed_scaling_factor_in_topk = False
    d13 = torch.stack([oracle.dequant_block_fp8(q13[e].cpu(), s13[e].cpu()) for e in range(experts)])
    d2 = torch.stack([oracle.dequant_block_fp8(q2[e].cpu(), s2[e].cpu()) for e in range(experts)])
    return layer, d13, d2


@pytest.mark.parametrize("case", ["dense", "ep", "scaled", "empty_routes", "prefill"])
def test_fp8_moe_method_apply(cuda_device, case):
    """B200Fp8MoEMethod.process_weights_after_loading + apply, as SGLang calls them
    (the reference's method check: dense, EP with -1 ids, routed scaling, all dropped)."""
    local, hidden, inter, top_k = 8, 256, 256, 3
    experts = 2 * local if case == "ep" else local
    tokens = 100 if case == "prefill" else 9
    rsf = 2.5 if case == "scaled" else 1.0
    layer, d13, d2 = _fp8_layer(local, hidden, inter, cuda_device)
    method = B200Fp8MoEMethod(SimpleNamespace(weight_block_size=[128, 128]))
    method.moe_runner_config = _runner_cfg(top_k, experts, local, rsf)
    method.process_weights_after_loading(layer)
    assert layer.w13_weight is None  # checkpoint layout released
    g = torch.Generator(device=cuda_device).manual_seed(7)
    x = (torch.randn(tokens, hidden, generator=g, device=cuda_device) * 0.5).bfloat16()
    ids = torch.stack([torch.randperm(local, generator=g, device=cuda_device)[:top_k]
                       for _ in range(tokens)]).int()
    if case == "ep":
        ids[0, 0] = -1
        ids[1, -1] = -1
        ids[5, :] = -1
    if case == "empty_routes":
        ids[:] = -1
    w = torch.rand(tokens, top_k, generator=g, device=cuda_device)
    out = method.apply(layer, SimpleNamespace(hidden_states=x,
                                              topk_output=SimpleNamespace(topk_ids=ids, topk_weights=w)))
    out = out.hidden_states
    want = oracle.fp8_moe_method_ref(x.cpu(), ids.cpu(), w.cpu(), d13, d2, output_scale=rsf)
    assert_close(out, want, what=f"method {case}")
    if case == "empty_routes":
        assert int(torch.count_nonzero(out)) == 0


def test_fp8_moe_offsets_api(cuda_device):
    """prepare_experts + apply over expert-sorted rows and offsets[E+1]
    (the reference's selftest pattern, quant/sm70_fp8_moe/selftest.py:19-45)."""
    experts, n, k, per = 4, 256, 128, 3
    q, s = synth.fp8_bank(experts, n, k, cuda_device, seed=50)
    prepared = fp8_moe.prepare_experts(q, s)
    counts = [per, per + 2, 0, per]
    x = synth.activations(sum(counts), k, cuda_device, seed=51, dtype=torch.float16)
    offsets = torch.tensor([0, *torch.tensor(counts).cumsum(0).tolist()], dtype=torch.int32,
                           device=cuda_device)
    out = torch.empty(x.shape[0], n // 2, dtype=torch.float16, device=cuda_device)
    fp8_moe.apply(out, x, offsets, prepared)
    want = torch.empty(x.shape[0], n // 2)
    for e in range(experts):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            want[lo:hi] = oracle.fp8_linear_ref(x[lo:hi].cpu(), q[e].cpu(), s[e].cpu(), gated=True)
    assert_close(out, want, what="offsets api")


def _nvfp4_layer(experts, hidden, inter, dev):
    p13, s13, g13 = synth.nvfp4_bank(experts, 2 * inter, hidden, dev, seed=60)
    p2, s2, g2 = synth.nvfp4_bank(experts, hidden, inter, dev, seed=61)
    P = torch.nn.Parameter
    layer = SimpleNamespace(
        params_dtype=torch.bfloat16, moe_runner_config=SimpleNamespace(is_gated=True),
        quant_config=SimpleNamespace(group_size=16), w13_bias=None, w2_bias=None,
        w13_weight=P(p13.clone(), requires_grad=False), w13_weight_scale=P(s13.clone(), requires_grad=False),
        w13_weight_scale_2=P(torch.stack([g13, g13], 1), requires_grad=False),
        w2_weight=P(p2.clone(), requires_grad=False), w2_weight_scale=P(s2.clone(), requires_grad=False),
        w2_weight_scale_2=P(g2.clone(), requires_grad=False),
    )
    d13 = torch.stack([oracle.dequant_nvfp4(p13[e].cpu(), s13[e].cpu(), float(g13[e])) for e in range(experts)])
    d2 = torch.stack([oracle.dequant_nvfp4(p2[e].cpu(), s2[e].cpu(), float(g2[e])) for e in range(experts)])
    return layer, d13, d2


@pytest.mark.parametrize("block", [8, 16, 48])
def test_nvfp4_marlin_hook_chain(cuda_device, block):
    """prepare_moe_nvfp4, then upstream fused_marlin_moe's call sequence:
    align -> moe_wna16_marlin_gemm (gate/up) -> SiLU*up -> moe_wna16_marlin_gemm
    (down, mul_topk_weights, size_m = M*top_k, top_k = 1) -> moe_sum_reduce."""
    from sglang_restomod_b200.moe.align import moe_align_block_size
    from sglang_restomod_b200.moe.sum_reduce import moe_sum_reduce
    from sglang_restomod_b200.quant.fp4_moe.method import moe_wna16_marlin_gemm, prepare_moe_nvfp4

    experts, hidden, inter, top_k, tokens = 6, 256, 128, 3, 11
    layer, d13, d2 = _nvfp4_layer(experts, hidden, inter, cuda_device)
    prepare_moe_nvfp4(layer)
    x = synth.activations(tokens, hidden, cuda_device, seed=62)
    ids, w = synth.route(tokens, experts, top_k, cuda_device, seed=63)
    sorted_ids, expert_ids, ntpp = moe_align_block_size(ids, block, experts)
    common = dict(b_bias_or_none=None, b_scales=layer.w13_weight_scale, b_zeros_or_none=None,
                  g_idx_or_none=None, perm_or_none=None, workspace=None,
                  sorted_token_ids=sorted_ids, expert_ids=expert_ids,
                  num_tokens_post_padded=ntpp, topk_weights=w, moe_block_size=block,
                  is_ep=False, b_q_type=None)
    c1 = torch.empty(tokens * top_k, 2 * inter, dtype=x.dtype, device=cuda_device)
    moe_wna16_marlin_gemm(x, c1, layer.w13_weight, global_scale_or_none=layer.w13_weight_scale_2,
                          top_k=top_k, mul_topk_weights=False, size_m=tokens, size_n=2 * inter,
                          size_k=hidden, **common)
    h = (torch.nn.functional.silu(c1[:, :inter].float()) * c1[:, inter:].float()).to(x.dtype)
    c2 = torch.empty(tokens * top_k, hidden, dtype=x.dtype, device=cuda_device)
    moe_wna16_marlin_gemm(h, c2, layer.w2_weight, global_scale_or_none=layer.w2_weight_scale_2,
                          top_k=1, mul_topk_weights=True, size_m=tokens * top_k, size_n=hidden,
                          size_k=inter, **common)
    out = torch.empty(tokens, hidden, dtype=x.dtype, device=cuda_device)
    moe_sum_reduce(c2.view(tokens, top_k, hidden), out, 1.0)
    want = oracle.moe_layer_ref(x.cpu(), ids.cpu(), w.cpu(), d13, d2)
    assert_close(out, want, what=f"nvfp4 hook chain block={block}")


def test_fp8_dense_apply_and_fused(cuda_device):
    from sglang_restomod_b200.quant.fp8_dense import (
        apply_b200_fp8_fused_silu_and_mul, apply_b200_fp8_linear, prepare_b200_fp8_linear)

    n, k = 512, 768
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=70)
    plain = SimpleNamespace(weight=q[0], weight_scale_inv=s[0])
    prepare_b200_fp8_linear(plain)
    gated = SimpleNamespace(weight=q[0], weight_scale_inv=s[0])
    prepare_b200_fp8_linear(gated, gated_silu=True)
    x = synth.activations(6, k, cuda_device, seed=71).view(2, 3, k)
    bias = torch.randn(n, device=cuda_device).bfloat16()
    want = oracle.fp8_linear_ref(x.reshape(-1, k).cpu(), q[0].cpu(), s[0].cpu())
    assert_close(apply_b200_fp8_linear(plain, x).reshape(-1, n), want, what="dense")
    assert_close(apply_b200_fp8_linear(plain, x, bias).reshape(-1, n),
                 want + bias.float().cpu(), what="dense+bias")
    assert_close(apply_b200_fp8_linear(gated, x).reshape(-1, n), want, what="gated bank, plain contract")
    fused = apply_b200_fp8_fused_silu_and_mul(gated, x).reshape(-1, n // 2)
    assert_close(fused, oracle.fp8_linear_ref(x.reshape(-1, k).cpu(), q[0].cpu(), s[0].cpu(), gated=True),
                 what="fused silu")
    assert apply_b200_fp8_fused_silu_and_mul(plain, x) is None


def test_lm_head_quantize_and_serve(cuda_device):
    from sglang_restomod_b200.quant.fp8_dense import apply_b200_fp8_linear
    from sglang_restomod_b200.quant.fp8_lm_head import _quantize, quantize_lm_head

    vocab, hidden = 4096, 1024
    g = torch.Generator(device=cuda_device).manual_seed(80)
    head_w = (torch.randn(vocab, hidden, generator=g, device=cuda_device) * 0.05).half()
    model = SimpleNamespace(lm_head=torch.nn.Linear(hidden, vocab, bias=False, device=cuda_device,
                                                     dtype=torch.float16))
    model.lm_head.weight.data.copy_(head_w)
    assert quantize_lm_head(model)
    q, s = _quantize(head_w)
    x = synth.activations(4, hidden, cuda_device, seed=81, dtype=torch.float16)
    y = apply_b200_fp8_linear(model.lm_head, x)
    assert_close(y, oracle.fp8_linear_ref(x.cpu(), q.cpu(), s.cpu()), what="lm_head")


def test_nvfp4_dense(cuda_device):
    from sglang_restomod_b200.quant.fp4_dense import apply_b200_nvfp4_linear, prepare_b200_nvfp4_linear

    n, k = 384, 512
    p, s, gs = synth.nvfp4_bank(1, n, k, cuda_device, seed=90)
    layer = SimpleNamespace(weight=p[0], weight_scale=s[0], weight_scale_2=gs[:1])
    prepare_b200_nvfp4_linear(layer)
    x = synth.activations(5, k, cuda_device, seed=91)
    want = oracle.nvfp4_linear_ref(x.cpu(), p[0].cpu(), s[0].cpu(), float(gs[0]))
    assert_close(apply_b200_nvfp4_linear(layer, x), want, what="nvfp4 dense")
    assert ops.workspace_status() == 0


def test_dense_quant_converts_admitted_linears(cuda_device):
    """fp8_dense_quant after load: admitted bf16 linears are quantized with the
    LM-head rule and served by the B200 GEMV; refused ones keep their path."""
    from sglang_restomod_b200.quant.fp8_dense_quant import quantize_dense_linears
    from sglang_restomod_b200.quant.fp8_lm_head import _quantize

    torch.manual_seed(0)
    model = torch.nn.Module()
    model.up = torch.nn.Linear(512, 768, bias=True)
    model.odd = torch.nn.Linear(200, 256, bias=False)
    model.lm_head = torch.nn.Linear(512, 384, bias=False)
    for p in model.parameters():
        p.data.normal_(0, 0.02)
    model = model.to(cuda_device, torch.bfloat16)
    w_up = model.up.weight.detach().clone()
    outcome = quantize_dense_linears(model)
    assert outcome["converted"] == 1 and outcome["lm_head"] == 1 and outcome["shape:256x200"] == 1
    assert model.up.weight.numel() == 0 and model.lm_head.weight.numel() > 0
    x = synth.activations(3, 512, cuda_device, seed=9)
    y = model.up(x)
    q, s = _quantize(w_up.to(torch.float16))
    want = oracle.fp8_linear_ref(x.cpu(), q.cpu(), s.cpu()) + model.up.bias.float().cpu()
    assert_close(y, want, what="converted linear")
