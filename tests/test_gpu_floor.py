"""The loads-only twins of b200_linear / b200_moe_gemm (the data-movement
floor used for measurement): they run on both kernels (weight-streaming and
tcgen05), report no device error, and leave the outputs untouched."""

from __future__ import annotations

import pytest
import torch

from sglang_restomod_b200 import _lib, ops, synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("quant", [_lib.QUANT_FP8_BLOCK, _lib.QUANT_NVFP4])
@pytest.mark.parametrize("m", [1, 16, 64, 200])
def test_linear_loads_only_leaves_output(cuda_device, quant, m):
    k, n = 512, 768
    if quant == _lib.QUANT_FP8_BLOCK:
        q, s = synth.fp8_bank(1, n, k, cuda_device, seed=1)
        packed, kw = ops.fp8_prepack(q[0], False), dict(scales=s[0])
    else:
        p4, s8, gs = synth.nvfp4_bank(1, n, k, cuda_device, seed=1)
        packed, kw = ops.nvfp4_prepack(p4[0], s8[0], False), dict(global_scale=gs[:1])
    x = synth.activations(m, k, cuda_device, seed=2)
    y = torch.full((m, n), 7.0, dtype=torch.bfloat16, device=cuda_device)
    ops.linear(x, packed, n, quant=quant, out=y, loads_only=True, **kw)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0
    assert bool((y == 7.0).all())
    ops.linear(x, packed, n, quant=quant, out=y, **kw)  # the real call still works after it
    torch.cuda.synchronize()
    assert not bool((y == 7.0).all())


@pytest.mark.parametrize("block", [8, 16, 64, 256])
def test_moe_gemm_loads_only_leaves_output(cuda_device, block):
    experts, tokens, top_k, k, n = 6, 150, 3, 384, 512
    ids, w = synth.route(tokens, experts, top_k, cuda_device, seed=3)
    x = synth.activations(tokens, k, cuda_device, seed=4)
    q, s = synth.fp8_bank(experts, n, k, cuda_device, seed=5)
    packed = ops.fp8_prepack(q, True)
    sid, eid, ntpp = ops.moe_align_block_size(ids, block, experts)
    c = torch.full((tokens * top_k, n // 2), 3.0, dtype=torch.bfloat16, device=cuda_device)
    ops.moe_gemm(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, num_experts=experts,
                 sorted_token_ids=sid, expert_ids=eid, num_tokens_post_pad=ntpp,
                 block_size=block, top_k=top_k, num_routes=tokens * top_k, c=c, scales=s,
                 gated_mode=_lib.GATED_FUSED, loads_only=True)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0
    assert bool((c == 3.0).all())
