"""GPU parity of the opt-in W8A8 block-FP8 path against the CPU oracle.

The activation quantization is compared bit-exactly (e4m3 bytes and fp32
scales); the GEMMs within rtol / atol 2e-2 against the oracle's
dequantize(quantize(x)) . dequantize(W)^T, i.e. the same activation
quantization, fp32 arithmetic.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from sglang_restomod_b200 import _lib, ops, synth
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,k", [(1, 128), (7, 384), (300, 1024), (64, 7168)])
def test_fp8_act_quant_bit_exact(cuda_device, x_dtype, rows, k):
    x = synth.activations(rows, k, cuda_device, seed=rows + k, dtype=x_dtype)
    x[0, :128] = 0  # an all-zero group takes the 1e-8 floor
    if rows > 2:
        x[2, 128:256] *= 1e4  # a large group
    q, s = ops.fp8_act_quant(x, scales_ld=rows + 5)
    want_q, want_s = oracle.act_quant_fp8(x.cpu())
    torch.cuda.synchronize()
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), want_q.view(torch.uint8).numpy())
    assert np.array_equal(s[:, :rows].cpu().numpy(), want_s.T.contiguous().numpy())


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k,n,gated", [(1, 256, 384, False), (33, 512, 256, True),
                                         (128, 384, 640, False), (200, 1024, 512, True),
                                         (300, 768, 1024, False), (5, 7168, 256, True)])
def test_w8a8_linear(cuda_device, x_dtype, m, k, n, gated):
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=m + n)
    x = synth.activations(m, k, cuda_device, seed=3, dtype=x_dtype)
    mode = _lib.GATED_FUSED if gated else _lib.GATED_NONE
    y = ops.w8a8_linear(x, q[0], s[0], gated_mode=mode, out_dtype=torch.bfloat16)
    want = oracle.w8a8_linear_ref(x.cpu(), q[0].cpu(), s[0].cpu(), gated=gated)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0
    assert_close(y, want, what=f"w8a8 linear m={m} k={k} n={n} gated={gated}")


@pytest.mark.parametrize("block", [8, 16, 64, 128, 256])
@pytest.mark.parametrize("gated_mode", [_lib.GATED_NONE, _lib.GATED_FUSED])
def test_w8a8_moe_gemm(cuda_device, block, gated_mode):
    experts, tokens, top_k, k, n = 6, 150, 3, 384, 512
    ids, weights = synth.route(tokens, experts, top_k, cuda_device, seed=block + gated_mode)
    ids[3, 1] = -1  # an expert-parallel drop
    x = synth.activations(tokens, k, cuda_device, seed=11)
    q, s = synth.fp8_bank(experts, n, k, cuda_device, seed=4)
    sorted_ids, expert_ids, ntpp = ops.moe_align_block_size(ids, block, experts)
    routes = tokens * top_k
    cols = n // 2 if gated_mode == _lib.GATED_FUSED else n
    c = torch.zeros(routes, cols, dtype=torch.bfloat16, device=cuda_device)
    mul = gated_mode == _lib.GATED_NONE
    ops.w8a8_moe_gemm(x, q, s, num_experts=experts, sorted_token_ids=sorted_ids,
                      expert_ids=expert_ids, num_tokens_post_pad=ntpp, block_size=block,
                      top_k=top_k, num_routes=routes, c=c, topk_weights=weights,
                      mul_topk_weights=mul, gated_mode=gated_mode)
    dense = torch.stack([oracle.dequant_block_fp8(q[e].cpu(), s[e].cpu()) for e in range(experts)])
    want, written = oracle.moe_gemm_ref(
        oracle.quantized_activations(x.cpu()), dense, sorted_ids.cpu().numpy(),
        expert_ids.cpu().numpy(), int(ntpp.item()), block, top_k, routes, weights.cpu(), mul,
        1 if gated_mode == _lib.GATED_FUSED else 0)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0
    assert not bool(written[3 * top_k + 1])
    assert_close(c.cpu()[written], want[written], what=f"w8a8 moe bs={block} g={gated_mode}")
    # dropped routes are never written
    assert int(torch.count_nonzero(c[3 * top_k + 1])) == 0


def test_w8a8_moe_gemm_prefill_shape(cuda_device):
    """Config-2 shapes (H=2048, gate/up N=1024, 512 experts) at 2048 tokens,
    blocks of 64; 256 routes' rows checked."""
    shape = synth.CONFIG2
    tokens = 2048
    ids, weights = synth.route(tokens, shape.experts, shape.top_k, cuda_device, seed=5)
    x = synth.activations(tokens, shape.hidden, cuda_device, seed=6)
    q, s = synth.fp8_bank(shape.experts, 2 * shape.inter, shape.hidden, cuda_device, seed=7)
    sorted_ids, expert_ids, ntpp = ops.moe_align_block_size(ids, 64, shape.experts)
    routes = tokens * shape.top_k
    c = torch.zeros(routes, shape.inter, dtype=torch.bfloat16, device=cuda_device)
    ops.w8a8_moe_gemm(x, q, s, num_experts=shape.experts, sorted_token_ids=sorted_ids,
                      expert_ids=expert_ids, num_tokens_post_pad=ntpp, block_size=64,
                      top_k=shape.top_k, num_routes=routes, c=c, gated_mode=_lib.GATED_FUSED)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0
    pick = torch.randperm(routes, generator=torch.Generator().manual_seed(0))[:256]
    xq = oracle.quantized_activations(x.cpu())
    ids_c = ids.cpu().reshape(-1)
    for r in pick.tolist():
        e = int(ids_c[r])
        w = oracle.dequant_block_fp8(q[e].cpu(), s[e].cpu())
        y = xq[r // shape.top_k] @ w.T
        want = torch.nn.functional.silu(y[: shape.inter]) * y[shape.inter:]
        assert_close(c[r].cpu(), want, what=f"route {r}")
