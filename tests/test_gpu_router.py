"""Router top-k kernel (b200_topk_route) against the CPU oracle.

Ids must match exactly (distinct keys, or ties resolved to the lower expert
id as the oracle's stable sort does); weights within 1e-5 relative (the
kernel and torch sum the softmax denominator in different orders).
"""

from __future__ import annotations

import pytest
import torch

import oracle
from sglang_restomod_b200 import _lib, ops

pytestmark = pytest.mark.gpu

W_RTOL, W_ATOL = 1e-5, 1e-6


def _check(got, want, what):
    ids, w = got
    wids, ww = want
    assert torch.equal(ids.cpu(), wids), f"{what}: ids differ"
    torch.testing.assert_close(w.cpu(), ww, rtol=W_RTOL, atol=W_ATOL, msg=what)


@pytest.mark.parametrize("experts,top_k", [(16, 4), (256, 8), (512, 10), (1000, 8), (33, 1), (64, 32)])
@pytest.mark.parametrize("tokens", [1, 37, 1024])
def test_softmax_renormalised_matches_oracle(cuda_device, experts, top_k, tokens):
    g = torch.Generator().manual_seed(experts * 7 + tokens)
    logits = torch.randn(tokens, experts, generator=g)
    got = ops.topk_route(logits.to(cuda_device), top_k)
    _check(got, oracle.route_topk_general(logits, top_k), f"E={experts} k={top_k} T={tokens}")
    # the benchmark's own router (torch.topk) agrees on distinct keys
    ids, w = oracle.route_topk(logits, top_k)
    assert torch.equal(got[0].cpu(), ids)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_precision_logits(cuda_device, dtype):
    g = torch.Generator().manual_seed(3)
    logits = (torch.randn(300, 256, generator=g) * 3).to(dtype)
    got = ops.topk_route(logits.to(cuda_device), 8)
    _check(got, oracle.route_topk_general(logits, 8), str(dtype))


def test_softmax_without_renormalisation(cuda_device):
    g = torch.Generator().manual_seed(4)
    logits = torch.randn(64, 512, generator=g)
    got = ops.topk_route(logits.to(cuda_device), 10, renormalize=False)
    _check(got, oracle.route_topk_general(logits, 10, renormalize=False), "no renorm")


@pytest.mark.parametrize("with_bias", [False, True])
def test_sigmoid_with_correction_bias(cuda_device, with_bias):
    g = torch.Generator().manual_seed(5)
    logits = torch.randn(200, 256, generator=g)
    bias = torch.randn(256, generator=g) * 0.1 if with_bias else None
    got = ops.topk_route(logits.to(cuda_device), 8, scoring=_lib.SCORING_SIGMOID,
                         correction_bias=bias.to(cuda_device) if with_bias else None)
    _check(got, oracle.route_topk_general(logits, 8, scoring="sigmoid", bias=bias), "sigmoid")


def test_ties_go_to_the_lower_expert(cuda_device):
    logits = torch.zeros(5, 64)
    logits[:, 10] = 2.0
    logits[:, 3] = 1.0
    logits[:, 40] = 1.0  # ties with expert 3
    got = ops.topk_route(logits.to(cuda_device), 4)
    _check(got, oracle.route_topk_general(logits, 4), "ties")
    assert got[0][0].tolist() == [10, 3, 40, 0]


def test_routed_layer_from_logits(cuda_device):
    """Router + layer forward equal the layer fed by the oracle's routing."""
    from sglang_restomod_b200 import synth
    from sglang_restomod_b200.layer import QuantMoELayer
    from tests.conftest import assert_close

    shape = synth.MoEShape(hidden=256, inter=128, experts=16, top_k=4)
    layer = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, cuda_device)
    x = synth.activations(40, shape.hidden, cuda_device, seed=9)
    g = torch.Generator().manual_seed(9)
    logits = torch.randn(40, shape.experts, generator=g)
    out = layer.forward_logits(x, logits.to(cuda_device))
    ids, w = oracle.route_topk(logits, shape.top_k)
    want = layer.forward(x, ids.to(cuda_device), w.to(cuda_device))
    assert_close(out, want, what="router + layer")


def test_empty_batch(cuda_device):
    ids, w = ops.topk_route(torch.empty(0, 16, device=cuda_device), 4)
    assert ids.shape == (0, 4) and w.shape == (0, 4)


@pytest.mark.parametrize("tokens,experts,top_k,block", [(1, 16, 4, 8), (32, 512, 10, 16), (37, 64, 6, 16),
                                                         (128, 256, 8, 16), (300, 512, 10, 64),
                                                         (1000, 64, 8, 64)])
def test_layer_forward_from_logits(cuda_device, tokens, experts, top_k, block):
    """b200_moe_layer_forward_logits (router + align in one kernel up to 32
    tokens, separate kernels above) gives the routes of b200_topk_route and
    the output of the layer fed those routes."""
    from sglang_restomod_b200 import synth
    from tests.conftest import assert_close

    shape = synth.MoEShape(hidden=256, inter=128, experts=experts, top_k=top_k)
    q13, s13 = synth.fp8_bank(experts, 256, 256, cuda_device, 40)
    q2, s2 = synth.fp8_bank(experts, 256, 128, cuda_device, 41)
    bank = dict(w13=ops.fp8_prepack(q13, True), w2=ops.fp8_prepack(q2, False), w13_scales=s13,
                w2_scales=s2)
    x = synth.activations(tokens, 256, cuda_device, seed=tokens)
    g = torch.Generator().manual_seed(tokens + experts)
    logits = torch.randn(tokens, experts, generator=g).to(cuda_device)
    out, ids, w = ops.moe_layer_forward_logits(x, logits, top_k, quant=0, num_experts=experts,
                                               inter=128, block_size=block, **bank)
    ref_ids, ref_w = ops.topk_route(logits, top_k)
    torch.cuda.synchronize()
    assert torch.equal(ids, ref_ids) and torch.equal(w, ref_w)
    want = ops.moe_layer_forward(x, ref_ids, ref_w, quant=0, num_experts=experts, inter=128,
                                 block_size=block, **bank)
    assert_close(out, want, rtol=1e-3, atol=1e-3, what=f"from logits T={tokens}")
    assert ops.workspace_status() == 0


# --------------------------------------------- grouped (expert-group) top-k
@pytest.mark.parametrize("experts,groups,topk_group,top_k,scoring,with_bias",
                         [(256, 8, 4, 8, "sigmoid", True),    # DeepSeek-V3's routing
                          (256, 8, 4, 8, "sigmoid", False),
                          (64, 8, 3, 6, "softmax", False),
                          (160, 32, 6, 12, "softmax", False),
                          (96, 4, 1, 4, "sigmoid", True)])
def test_grouped_topk_matches_oracle(cuda_device, experts, groups, topk_group, top_k, scoring,
                                     with_bias):
    g = torch.Generator().manual_seed(experts + groups + top_k)
    logits = torch.randn(77, experts, generator=g)
    bias = torch.randn(experts, generator=g) * 0.5 if with_bias else None
    code = _lib.SCORING_SIGMOID if scoring == "sigmoid" else _lib.SCORING_SOFTMAX
    got = ops.topk_route_grouped(logits.to(cuda_device), top_k, groups, topk_group, scoring=code,
                                 correction_bias=None if bias is None else bias.to(cuda_device))
    want = oracle.route_topk_grouped(logits, top_k, groups, topk_group, scoring=scoring,
                                     bias=bias)
    _check(got, want, f"grouped {experts}/{groups}/{topk_group}/{top_k} {scoring}")
    # every chosen expert lies in one of the topk_group kept groups
    per = experts // groups
    chosen_groups = got[0].cpu().long() // per
    assert int(max(len(set(r.tolist())) for r in chosen_groups)) <= topk_group


def test_grouped_topk_groups_matter(cuda_device):
    """One group holds the single best expert but weak others; with a top-2
    group score it loses to groups whose two best are strong."""
    experts, groups = 16, 4
    logits = torch.full((1, experts), -4.0)
    logits[0, 0] = 4.0          # group 0: one strong expert
    logits[0, 4:6] = 3.0        # group 1: two good experts
    logits[0, 8:10] = 2.9       # group 2
    bias = torch.zeros(experts)
    ids, _ = ops.topk_route_grouped(logits.to(cuda_device), 2, groups, 1,
                                    scoring=_lib.SCORING_SIGMOID,
                                    correction_bias=bias.to(cuda_device))
    assert sorted(ids[0].tolist()) == [4, 5]
    ids_max, _ = ops.topk_route_grouped(logits.to(cuda_device), 2, groups, 1,
                                        scoring=_lib.SCORING_SIGMOID)
    assert ids_max[0].tolist()[0] == 0  # by group maximum, group 0 wins
