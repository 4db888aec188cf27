"""GPU parity: every kernel through the C ABI against the CPU oracle.

moe_align is compared bit-exactly; GEMM / MoE outputs within rtol 2e-2 /
atol 2e-2 (bf16 activations, fp32 accumulation).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from sglang_restomod_b200 import _lib, ops, synth
from sglang_restomod_b200.layer import block_size_for
from tests.conftest import assert_close


def wide_sample(tokens: int, n: int = 256, seed: int = 0) -> torch.Tensor:
    """n token indices: the first and last n/4 (the first and last route
    slots of every expert's run, so the first and last tcgen05 items) and n/2
    drawn from the rest."""
    if tokens <= n:
        return torch.arange(tokens)
    q = n // 4
    edge = torch.cat([torch.arange(q), torch.arange(tokens - q, tokens)])
    middle = q + torch.randperm(tokens - 2 * q, generator=torch.Generator().manual_seed(seed))[: n - 2 * q]
    return torch.cat([edge, middle]).sort().values

pytestmark = pytest.mark.gpu


def _dequant_fp8_bank(q, s, experts=None):
    ids = range(q.shape[0]) if experts is None else experts
    return {int(e): oracle.dequant_block_fp8(q[e].cpu(), s[e].cpu()) for e in ids}


def _dequant_nvfp4_bank(p, s, gs, experts=None):
    ids = range(p.shape[0]) if experts is None else experts
    return {int(e): oracle.dequant_nvfp4(p[e].cpu(), s[e].cpu(), float(gs[e])) for e in ids}


def _stack(d, n):
    first = next(iter(d.values()))
    out = torch.zeros(n, *first.shape)
    for e, w in d.items():
        out[e] = w
    return out


# ------------------------------------------------------------------ align
ALIGN_CASES = [
    (0, 4, 8),
    (1, 4, 8),
    (128, 16, 64),   # configuration 0: 32 tokens x top-4, block 64
    (40, 512, 8),    # a decode step of the reference's profile
    (2560, 512, 16),
    (10, 1, 8),
    (81920, 512, 64),  # configuration 2 prefill: 8192 tokens x top-10
    (4096 * 8, 256, 64),
    (3000, 1024, 16),  # the kernel's maximum expert count
    (20000, 1024, 64),
    (777, 1024, 5),
    # up to 32 routes: the one-warp align
    (11, 513, 8),    # a one-token config2 step with the shared route
    (32, 64, 16),
    (24, 8, 64),
    (32, 1024, 8),
    (17, 3, 4),
    (32, 2, 5),
    (33, 16, 8),     # one past it
]


@pytest.mark.parametrize("numel,experts,bs", ALIGN_CASES)
@pytest.mark.parametrize("drop", [False, True])
def test_moe_align_bit_exact(cuda_device, numel, experts, bs, drop):
    rng = np.random.default_rng(numel + experts + bs)
    ids = rng.integers(0, experts, size=numel).astype(np.int32)
    if drop and numel:
        ids[rng.random(numel) < 0.2] = -1
    t = torch.from_numpy(ids).to(cuda_device)
    sorted_ids, expert_ids, ntpp = ops.moe_align_block_size(t, bs, experts)
    want_sorted, want_experts, want_total = oracle.moe_align_block_size(ids, experts, bs)
    torch.cuda.synchronize()
    assert int(ntpp.item()) == want_total
    assert np.array_equal(sorted_ids.cpu().numpy(), want_sorted)
    assert np.array_equal(expert_ids.cpu().numpy(), want_experts)


def test_moe_align_all_one_expert_and_repeat(cuda_device):
    ids = torch.zeros(1000, dtype=torch.int32, device=cuda_device)
    a = [x.cpu() for x in ops.moe_align_block_size(ids, 16, 8)]
    b = [x.cpu() for x in ops.moe_align_block_size(ids, 16, 8)]
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    want_sorted, want_experts, total = oracle.moe_align_block_size(ids.cpu().numpy(), 8, 16)
    assert int(a[2]) == total == 1008
    assert np.array_equal(a[0].numpy(), want_sorted)


# --------------------------------------------------------------- combine
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_moe_sum_reduce(cuda_device, dtype):
    g = torch.Generator(device=cuda_device).manual_seed(3)
    x = torch.randn(37, 10, 2048, generator=g, device=cuda_device).to(dtype)
    out = torch.empty(37, 2048, dtype=dtype, device=cuda_device)
    ops.moe_sum_reduce(x, out, 2.5)
    want = oracle.moe_sum_reduce_ref(x.cpu(), 2.5)
    assert_close(out, want, rtol=1e-2, atol=1e-2, what="sum_reduce")


def test_moe_combine_skips_dropped_routes(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(4)
    routed = torch.randn(6 * 4, 256, generator=g, device=cuda_device).half()
    ids = torch.randint(0, 8, (6, 4), generator=g, device=cuda_device, dtype=torch.int32)
    ids[0, 1] = -1
    ids[5, :] = -1
    shared = torch.randn(6, 256, generator=g, device=cuda_device).bfloat16()
    out = ops.moe_combine(routed, ids, 8, 1.5, shared_out=shared)
    r = routed.float().cpu().view(6, 4, 256)
    mask = (ids.cpu() >= 0).float()[..., None]
    want = (r * mask).sum(1) * 1.5 + shared.float().cpu()
    assert_close(out, want, rtol=1e-2, atol=1e-2, what="combine")
    assert_close(out[5], shared[5], rtol=0, atol=0, what="all-dropped token")


# ----------------------------------------------------------- dense linear
DENSE_SMALL = [(1, 256, 384), (4, 512, 256), (16, 384, 512), (64, 256, 256), (13, 1024, 640),
               (100, 256, 384), (2, 640, 256), (8, 128, 384)]


@pytest.mark.parametrize("m,k,n", DENSE_SMALL)
@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16])
def test_fp8_linear_small(cuda_device, m, k, n, x_dtype):
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=m + k + n)
    x = synth.activations(m, k, cuda_device, seed=5, dtype=x_dtype)
    packed = ops.fp8_prepack(q[0], gated=False)
    y = ops.linear(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, scales=s[0])
    want = oracle.fp8_linear_ref(x.cpu(), q[0].cpu(), s[0].cpu())
    assert_close(y, want, what=f"fp8 linear m={m} k={k} n={n}")
    assert ops.workspace_status() == 0


@pytest.mark.parametrize("m", [1, 8, 33])
def test_fp8_linear_gated_fused(cuda_device, m):
    inter, k = 256, 512
    q, s = synth.fp8_bank(1, 2 * inter, k, cuda_device, seed=9)
    x = synth.activations(m, k, cuda_device, seed=6)
    packed = ops.fp8_prepack(q[0], gated=True)
    y = ops.linear(x, packed, 2 * inter, quant=_lib.QUANT_FP8_BLOCK, scales=s[0],
                   gated_mode=_lib.GATED_FUSED)
    want = oracle.fp8_linear_ref(x.cpu(), q[0].cpu(), s[0].cpu(), gated=True)
    assert_close(y, want, what="fused gate/up")
    ysplit = ops.linear(x, packed, 2 * inter, quant=_lib.QUANT_FP8_BLOCK, scales=s[0],
                        gated_mode=_lib.GATED_SPLIT)
    assert_close(ysplit, oracle.fp8_linear_ref(x.cpu(), q[0].cpu(), s[0].cpu()), what="split gate/up")


@pytest.mark.parametrize("k,n", [(5120, 25600), (25600, 5120)])
@pytest.mark.parametrize("m", [1, 4, 16, 64])
def test_fp8_linear_config1(cuda_device, k, n, m):
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=1)
    x = synth.activations(m, k, cuda_device, seed=2)
    packed = ops.fp8_prepack(q[0], gated=False)
    y = ops.linear(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, scales=s[0])
    # Check a fixed sample of 1024 output columns against the oracle.
    cols = torch.randperm(n, generator=torch.Generator().manual_seed(0))[:1024].sort().values
    w = oracle.dequant_block_fp8(q[0].cpu(), s[0].cpu())[cols]
    want = x.cpu().float() @ w.T
    assert_close(y.cpu()[:, cols], want, what=f"config1 m={m} k={k} n={n}")


def test_fp8_linear_lm_head_sampled(cuda_device):
    k, n, m = 5120, 152064, 4
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=3)
    x = synth.activations(m, k, cuda_device, seed=4)
    packed = ops.fp8_prepack(q[0], gated=False)
    y = ops.linear(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, scales=s[0])
    blocks = torch.tensor([0, 7, 600, 1187])  # first, middle, last 128-row blocks
    rows = (blocks[:, None] * 128 + torch.arange(128)).flatten()
    qs = q[0][rows.to(cuda_device)].cpu()
    ss = s[0][blocks.to(cuda_device)].cpu()
    want = x.cpu().float() @ oracle.dequant_block_fp8(qs, ss).T
    assert_close(y.cpu()[:, rows], want, what="lm_head")


# K = 384 and 640 leave a pipeline stage with fewer K-units than the others
@pytest.mark.parametrize("m,k,n", [(1, 256, 256), (8, 512, 384), (16, 1024, 256), (64, 256, 512),
                                   (4, 384, 256), (2, 640, 384), (16, 640, 128)])
def test_nvfp4_linear(cuda_device, m, k, n):
    p, s, gs = synth.nvfp4_bank(1, n, k, cuda_device, seed=m + n)
    x = synth.activations(m, k, cuda_device, seed=7)
    packed = ops.nvfp4_prepack(p[0], s[0], gated=False)
    y = ops.linear(x, packed, n, quant=_lib.QUANT_NVFP4, global_scale=gs[:1])
    want = oracle.nvfp4_linear_ref(x.cpu(), p[0].cpu(), s[0].cpu(), float(gs[0]))
    assert_close(y, want, what=f"nvfp4 linear m={m}")


def test_linear_cuda_graph_replay(cuda_device):
    """Capture once, replay with new inputs (graph-safe: no host sync, no allocation)."""
    m, k, n = 4, 512, 768
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=12)
    packed = ops.fp8_prepack(q[0], gated=False)
    x = synth.activations(m, k, cuda_device, seed=1)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_device)
    ops.linear(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, scales=s[0], out=y)  # warm-up sizes the workspace
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.linear(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, scales=s[0], out=y)
    for seed in (2, 3):
        x.copy_(synth.activations(m, k, cuda_device, seed=seed))
        graph.replay()
        torch.cuda.synchronize()
        assert_close(y, oracle.fp8_linear_ref(x.cpu(), q[0].cpu(), s[0].cpu()), what=f"replay {seed}")


# ----------------------------------------------------------- grouped GEMM
@pytest.mark.parametrize("quant", [_lib.QUANT_FP8_BLOCK, _lib.QUANT_NVFP4])
@pytest.mark.parametrize("block", [8, 16, 32, 64])
@pytest.mark.parametrize("gated_mode", [_lib.GATED_NONE, _lib.GATED_FUSED, _lib.GATED_SPLIT])
def test_moe_gemm(cuda_device, quant, block, gated_mode):
    experts, tokens, top_k, k = 6, 19, 3, 256
    n = 512
    ids, weights = synth.route(tokens, experts, top_k, cuda_device, seed=block)
    ids[0, 0] = -1  # an expert-parallel drop
    x = synth.activations(tokens, k, cuda_device, seed=8)
    gated = gated_mode != _lib.GATED_NONE
    if quant == _lib.QUANT_FP8_BLOCK:
        q, s = synth.fp8_bank(experts, n, k, cuda_device, seed=2)
        packed, scales, gs = ops.fp8_prepack(q, gated), s, None
        dense = _stack(_dequant_fp8_bank(q, s), experts)
    else:
        p, s8, gs = synth.nvfp4_bank(experts, n, k, cuda_device, seed=2)
        packed, scales = ops.nvfp4_prepack(p, s8, gated), None
        dense = _stack(_dequant_nvfp4_bank(p, s8, gs), experts)
    sorted_ids, expert_ids, ntpp = ops.moe_align_block_size(ids, block, experts)
    routes = tokens * top_k
    cols = n // 2 if gated_mode == _lib.GATED_FUSED else n
    c = torch.zeros(routes, cols, dtype=torch.bfloat16, device=cuda_device)
    mul = gated_mode == _lib.GATED_NONE
    ops.moe_gemm(x, packed, n, quant=quant, num_experts=experts, sorted_token_ids=sorted_ids,
                 expert_ids=expert_ids, num_tokens_post_pad=ntpp, block_size=block, top_k=top_k,
                 num_routes=routes, c=c, scales=scales, global_scale=gs, topk_weights=weights,
                 mul_topk_weights=mul, gated_mode=gated_mode)
    want, written = oracle.moe_gemm_ref(
        x.cpu(), dense, sorted_ids.cpu().numpy(), expert_ids.cpu().numpy(), int(ntpp.item()),
        block, top_k, routes, weights.cpu(), mul, 1 if gated_mode == _lib.GATED_FUSED else 0,
    )
    assert not bool(written[0])  # the dropped route is never computed
    assert_close(c.cpu()[written], want[written], what=f"moe_gemm q={quant} bs={block} g={gated_mode}")
    assert ops.workspace_status() == 0


# ------------------------------------------------------------ MoE layer
def _layer_inputs(shape, tokens, quant, device, seed=0):
    ids, weights = synth.route(tokens, shape.experts, shape.top_k, device, seed=seed + 1)
    x = synth.activations(tokens, shape.hidden, device, seed=seed)
    if quant == _lib.QUANT_FP8_BLOCK:
        q13, s13 = synth.fp8_bank(shape.experts, 2 * shape.inter, shape.hidden, device, seed=10)
        q2, s2 = synth.fp8_bank(shape.experts, shape.hidden, shape.inter, device, seed=11)
        bank = dict(w13=ops.fp8_prepack(q13, True), w2=ops.fp8_prepack(q2, False),
                    w13_scales=s13, w2_scales=s2)
        deq = lambda e: (oracle.dequant_block_fp8(q13[e].cpu(), s13[e].cpu()),  # noqa: E731
                         oracle.dequant_block_fp8(q2[e].cpu(), s2[e].cpu()))
    else:
        p13, s13, g13 = synth.nvfp4_bank(shape.experts, 2 * shape.inter, shape.hidden, device, seed=10)
        p2, s2, g2 = synth.nvfp4_bank(shape.experts, shape.hidden, shape.inter, device, seed=11)
        bank = dict(w13=ops.nvfp4_prepack(p13, s13, True), w2=ops.nvfp4_prepack(p2, s2, False),
                    w13_global=g13, w2_global=g2)
        deq = lambda e: (oracle.dequant_nvfp4(p13[e].cpu(), s13[e].cpu(), float(g13[e])),  # noqa: E731
                         oracle.dequant_nvfp4(p2[e].cpu(), s2[e].cpu(), float(g2[e])))
    return x, ids, weights, bank, deq


def _check_layer(shape, tokens, quant, device, block, sample_tokens=None, rsf=1.0):
    x, ids, weights, bank, deq = _layer_inputs(shape, tokens, quant, device)
    out = ops.moe_layer_forward(x, ids, weights, quant=quant, num_experts=shape.experts,
                                inter=shape.inter, block_size=block, routed_scaling_factor=rsf,
                                **bank)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0
    sel = torch.arange(tokens) if sample_tokens is None else sample_tokens
    ids_c = ids.cpu()[sel]
    # The touched experts are dequantized one at a time, inside the oracle.
    want = oracle.moe_layer_ref(x.cpu()[sel], ids_c, weights.cpu()[sel], deq, shape.experts,
                                routed_scaling_factor=rsf)
    assert_close(out.cpu()[sel], want, what=f"layer q={quant} T={tokens}")


@pytest.mark.parametrize("quant", [_lib.QUANT_FP8_BLOCK, _lib.QUANT_NVFP4])
def test_layer_config0(cuda_device, quant):
    _check_layer(synth.CONFIG0, 32, quant, cuda_device, block=64 if quant == 0 else 16, rsf=1.0)


@pytest.mark.parametrize("quant", [_lib.QUANT_FP8_BLOCK, _lib.QUANT_NVFP4])
@pytest.mark.parametrize("tokens", [1, 8, 64, 256])
def test_layer_config2_decode(cuda_device, quant, tokens):
    # every token checked; the layer's own block rule (8-slot groups up to 6
    # routes per expert, 16-slot above) and 16-slot groups for comparison
    for block in sorted({16, block_size_for(tokens * synth.CONFIG2.top_k, synth.CONFIG2.experts)}):
        _check_layer(synth.CONFIG2, tokens, quant, cuda_device, block=block, rsf=2.0)


# ------------------------------------------------- tcgen05 (prefill) path
@pytest.mark.parametrize("quant", [_lib.QUANT_FP8_BLOCK, _lib.QUANT_NVFP4])
@pytest.mark.parametrize("block", [64, 128, 256])
@pytest.mark.parametrize("gated_mode", [_lib.GATED_NONE, _lib.GATED_FUSED, _lib.GATED_SPLIT])
@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16])
def test_moe_gemm_tcgen05(cuda_device, quant, block, gated_mode, x_dtype):
    """Expert GEMM on the tensor-core path: many routes per expert."""
    experts, tokens, top_k, k, n = 5, 150, 3, 384, 512
    ids, weights = synth.route(tokens, experts, top_k, cuda_device, seed=block + gated_mode)
    ids[3, 1] = -1
    x = synth.activations(tokens, k, cuda_device, seed=9, dtype=x_dtype)
    gated = gated_mode != _lib.GATED_NONE
    if quant == _lib.QUANT_FP8_BLOCK:
        q, s = synth.fp8_bank(experts, n, k, cuda_device, seed=3)
        packed, scales, gs = ops.fp8_prepack(q, gated), s, None
        dense = _stack(_dequant_fp8_bank(q, s), experts)
    else:
        p4, s8, gs = synth.nvfp4_bank(experts, n, k, cuda_device, seed=3)
        packed, scales = ops.nvfp4_prepack(p4, s8, gated), None
        dense = _stack(_dequant_nvfp4_bank(p4, s8, gs), experts)
    sorted_ids, expert_ids, ntpp = ops.moe_align_block_size(ids, block, experts)
    routes = tokens * top_k
    cols = n // 2 if gated_mode == _lib.GATED_FUSED else n
    c = torch.zeros(routes, cols, dtype=x_dtype, device=cuda_device)
    mul = gated_mode == _lib.GATED_NONE
    ops.moe_gemm(x, packed, n, quant=quant, num_experts=experts,
                 sorted_token_ids=sorted_ids, expert_ids=expert_ids, num_tokens_post_pad=ntpp,
                 block_size=block, top_k=top_k, num_routes=routes, c=c, scales=scales,
                 global_scale=gs, topk_weights=weights, mul_topk_weights=mul,
                 gated_mode=gated_mode)
    want, written = oracle.moe_gemm_ref(
        x.cpu(), dense, sorted_ids.cpu().numpy(), expert_ids.cpu().numpy(), int(ntpp.item()),
        block, top_k, routes, weights.cpu(), mul, 1 if gated_mode == _lib.GATED_FUSED else 0,
    )
    assert_close(c.cpu()[written], want[written], what=f"tc moe_gemm q={quant} bs={block} g={gated_mode}")
    assert ops.workspace_status() == 0


@pytest.mark.parametrize("block", [64, 256])
@pytest.mark.parametrize("gated_mode", [_lib.GATED_NONE, _lib.GATED_FUSED])
def test_moe_gemm_tcgen05_long_runs(cuda_device, block, gated_mode):
    """Skewed routing: experts with thousands of routes (many 256-slot items
    per expert, runs cut mid-expert), more than 1024 groups (the plan's tile
    carry), an idle expert and dropped routes."""
    experts, tokens, top_k, k, n = 9, 20000, 4, 256, 256
    g = torch.Generator(device="cpu").manual_seed(11 + block)
    # Experts 0-2 take most routes, expert 5 none.
    p = torch.tensor([0.3, 0.25, 0.2, 0.05, 0.05, 0.0, 0.05, 0.05, 0.05])
    ids = torch.multinomial(p.expand(tokens, -1), top_k, replacement=False, generator=g)
    ids = ids.to(torch.int32)
    ids[::97, 2] = -1
    weights = torch.rand(tokens, top_k, generator=g)
    ids, weights = ids.to(cuda_device), weights.to(cuda_device)
    x = synth.activations(tokens, k, cuda_device, seed=21)
    q, s = synth.fp8_bank(experts, n, k, cuda_device, seed=5)
    packed = ops.fp8_prepack(q, gated_mode != _lib.GATED_NONE)
    dense = _stack(_dequant_fp8_bank(q, s), experts)
    sorted_ids, expert_ids, ntpp = ops.moe_align_block_size(ids, block, experts)
    assert int(ntpp.item()) // block > 1024 or block == 256
    routes = tokens * top_k
    cols = n // 2 if gated_mode == _lib.GATED_FUSED else n
    c = torch.zeros(routes, cols, dtype=torch.bfloat16, device=cuda_device)
    mul = gated_mode == _lib.GATED_NONE
    ops.moe_gemm(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, num_experts=experts,
                 sorted_token_ids=sorted_ids, expert_ids=expert_ids, num_tokens_post_pad=ntpp,
                 block_size=block, top_k=top_k, num_routes=routes, c=c, scales=s,
                 topk_weights=weights, mul_topk_weights=mul, gated_mode=gated_mode)
    want, written = oracle.moe_gemm_ref(
        x.cpu(), dense, sorted_ids.cpu().numpy(), expert_ids.cpu().numpy(), int(ntpp.item()),
        block, top_k, routes, weights.cpu(), mul, 1 if gated_mode == _lib.GATED_FUSED else 0,
    )
    assert int(written.sum()) == int((ids >= 0).sum())
    assert_close(c.cpu()[written], want[written], what=f"tc long runs bs={block} g={gated_mode}")
    assert ops.workspace_status() == 0


def test_fp8_linear_tcgen05_scale_spread(cuda_device):
    """Block scales spread over 2^-20..2^12 along K, and an all-zero row
    block: the per-row power of two keeps the f16 operands in range."""
    m, k, n = 96, 1024, 512
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=17)
    s = s.clone()
    spread = torch.tensor([2.0 ** -20, 1.0, 2.0 ** 12, 2.0 ** -6, 0.5, 2.0 ** 7, 1.0, 2.0 ** -12],
                          device=cuda_device)
    s[0] = s[0] * spread[None, :]
    s[0, 2] = 0.0
    x = synth.activations(m, k, cuda_device, seed=8)
    packed = ops.fp8_prepack(q[0], gated=False)
    y = ops.linear(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, scales=s[0])
    want = oracle.fp8_linear_ref(x.cpu(), q[0].cpu(), s[0].cpu(), gated=False)
    assert torch.isfinite(y.float()).all()
    # The 2^12 block dominates every output: compare at the outputs' scale.
    scale = float(want.abs().mean())
    assert_close(y.float().cpu() / scale, want / scale, what="tc linear scale spread")


@pytest.mark.parametrize("m", [33, 130, 300])
@pytest.mark.parametrize("gated_mode", [_lib.GATED_NONE, _lib.GATED_FUSED])
def test_nvfp4_linear_tcgen05(cuda_device, m, gated_mode):
    k, n = 768, 1024
    p4, s8, gs = synth.nvfp4_bank(1, n, k, cuda_device, seed=m)
    x = synth.activations(m, k, cuda_device, seed=5)
    packed = ops.nvfp4_prepack(p4[0], s8[0], gated=gated_mode != _lib.GATED_NONE)
    y = ops.linear(x, packed, n, quant=_lib.QUANT_NVFP4, global_scale=gs[:1], gated_mode=gated_mode)
    want = oracle.nvfp4_linear_ref(x.cpu(), p4[0].cpu(), s8[0].cpu(), float(gs[0]),
                                   gated=gated_mode == _lib.GATED_FUSED)
    assert_close(y, want, what=f"tc nvfp4 linear m={m} g={gated_mode}")


def test_layer_config3_prefill_sampled(cuda_device):
    """The NVFP4 layer (config-2 shapes, NVFP4 weights) at 4096 tokens on the
    tensor-core path; 256 tokens checked against the oracle."""
    sample = wide_sample(4096)
    _check_layer(synth.CONFIG2, 4096, _lib.QUANT_NVFP4, cuda_device, block=64,
                 sample_tokens=sample, rsf=1.0)


@pytest.mark.parametrize("m", [33, 64, 130, 300])
@pytest.mark.parametrize("gated_mode", [_lib.GATED_NONE, _lib.GATED_FUSED])
def test_fp8_linear_tcgen05(cuda_device, m, gated_mode):
    k, n = 768, 1024
    q, s = synth.fp8_bank(1, n, k, cuda_device, seed=m)
    x = synth.activations(m, k, cuda_device, seed=4)
    packed = ops.fp8_prepack(q[0], gated=gated_mode != _lib.GATED_NONE)
    y = ops.linear(x, packed, n, quant=_lib.QUANT_FP8_BLOCK, scales=s[0], gated_mode=gated_mode)
    want = oracle.fp8_linear_ref(x.cpu(), q[0].cpu(), s[0].cpu(), gated=gated_mode == _lib.GATED_FUSED)
    assert_close(y, want, what=f"tc linear m={m} g={gated_mode}")


@pytest.mark.parametrize("tokens,block", [(8192, 256), (2048, 64)])
def test_layer_config2_prefill(cuda_device, tokens, block):
    sample = wide_sample(tokens)
    _check_layer(synth.CONFIG2, tokens, _lib.QUANT_FP8_BLOCK, cuda_device, block=block,
                 sample_tokens=sample, rsf=1.0)


def test_layer_config4_prefill_sampled(cuda_device):
    """Expert-parallel layer shape (H=7168, I=2048, 256 experts, top-8) at 4096
    tokens on one GPU; 256 tokens checked against the oracle."""
    sample = wide_sample(4096)
    _check_layer(synth.CONFIG4, 4096, _lib.QUANT_FP8_BLOCK, cuda_device, block=256,
                 sample_tokens=sample, rsf=1.0)


# ------------------------------------------------ fused shared expert
@pytest.mark.parametrize("tokens,block", [(1, None), (8, None), (1, 64), (16, 64), (128, 64),
                                          (512, 64), (512, 128), (1024, 64)])
@pytest.mark.parametrize("rsf", [1.0, 2.5])
def test_fused_shared_expert_matches_separate(cuda_device, tokens, block, rsf):
    """Shared expert appended to the routed bank (one more route per token,
    weight 1 / rsf) gives the layer output of the separate dense MLP. Fusion
    is taken with blocks of 64+ (the tensor-core GEMM)."""
    from sglang_restomod_b200.layer import QuantMoELayer

    shape = synth.MoEShape(hidden=512, inter=256, experts=32, top_k=4, shared_inter=256)
    sep = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, cuda_device)
    fused = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, cuda_device, fuse_shared=True)
    assert fused.shared_fused and not sep.shared_fused
    sep.routed_scaling_factor = fused.routed_scaling_factor = rsf
    sep.block_size = fused.block_size = block
    x = synth.activations(tokens, shape.hidden, cuda_device, seed=21)
    ids, w = synth.route(tokens, shape.experts, shape.top_k, cuda_device, seed=22)
    # fused on the tensor-core path, or when the batch fits one stream group
    assert fused.fused_block_size(tokens) == (block or fused.fused_block_size(tokens))
    assert fused.fused_block_size(tokens) is not None
    got = fused.forward(x, ids, w)
    want = sep.forward(x, ids, w)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0
    assert_close(got, want, what=f"fused shared T={tokens} block={block} rsf={rsf}")
    # and against the CPU oracle: routed layer + the shared MLP as a 1-expert MoE
    q13, s13 = synth.fp8_bank(shape.experts, 2 * shape.inter, shape.hidden, cuda_device, 10)
    q2, s2 = synth.fp8_bank(shape.experts, shape.hidden, shape.inter, cuda_device, 11)
    d13 = torch.stack([oracle.dequant_block_fp8(q13[e].cpu(), s13[e].cpu()) for e in range(shape.experts)])
    d2 = torch.stack([oracle.dequant_block_fp8(q2[e].cpu(), s2[e].cpu()) for e in range(shape.experts)])
    sq13, ss13 = synth.fp8_bank(1, 2 * shape.shared_inter, shape.hidden, cuda_device, 12)
    sq2, ss2 = synth.fp8_bank(1, shape.hidden, shape.shared_inter, cuda_device, 13)
    sd13 = oracle.dequant_block_fp8(sq13[0].cpu(), ss13[0].cpu()).unsqueeze(0)
    sd2 = oracle.dequant_block_fp8(sq2[0].cpu(), ss2[0].cpu()).unsqueeze(0)
    xc = x.cpu()
    shared = oracle.moe_layer_ref(xc, torch.zeros(tokens, 1, dtype=torch.int32),
                                  torch.ones(tokens, 1), sd13, sd2)
    want_o = oracle.moe_layer_ref(xc, ids.cpu(), w.cpu(), d13, d2, routed_scaling_factor=rsf,
                                  shared_out=shared)
    assert_close(got, want_o, what=f"fused shared vs oracle T={tokens}")


@pytest.mark.parametrize("tokens,block,x_dtype", [(3, 8, torch.bfloat16), (3, 8, torch.float16),
                                                  (40, 64, torch.bfloat16), (900, 16, torch.bfloat16),
                                                  (1024, 64, torch.float16)])
def test_layer_forward_fused_shared_entry(cuda_device, tokens, block, x_dtype):
    """b200_moe_layer_forward_fused_shared returns the caller's routes plus
    (E, 1 / rsf) per token, and its output is bit-identical to
    b200_moe_layer_forward on those routes over the E + 1 expert bank: up to
    4095 routes through the one preparation kernel (append + align + bf16
    conversion), from 4096 through the append and the multi-CTA align."""
    from sglang_restomod_b200.layer import QuantMoELayer

    shape = synth.MoEShape(hidden=256, inter=128, experts=16, top_k=4, shared_inter=128)
    layer = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, cuda_device, fuse_shared=True)
    assert layer.shared_fused
    rsf = 2.5
    x = synth.activations(tokens, shape.hidden, cuda_device, seed=3, dtype=x_dtype)
    ids, w = synth.route(tokens, shape.experts, shape.top_k, cuda_device, seed=4)
    ids[0, 1] = -1  # an expert-parallel drop stays dropped
    kw = dict(quant=_lib.QUANT_FP8_BLOCK, inter=shape.inter, w13=layer.w13, w2=layer.w2,
              w13_scales=layer.w13_scales, w2_scales=layer.w2_scales, block_size=block,
              routed_scaling_factor=rsf)
    out, ids2, w2 = ops.moe_layer_forward_fused_shared(x, ids, w, num_experts=shape.experts, **kw)
    want_ids = torch.cat([ids, torch.full((tokens, 1), shape.experts, dtype=torch.int32,
                                          device=cuda_device)], 1)
    want_w = torch.cat([w, torch.full((tokens, 1), 1.0 / rsf, device=cuda_device)], 1)
    ref = ops.moe_layer_forward(x, want_ids, want_w, num_experts=shape.experts + 1, **kw)
    torch.cuda.synchronize()
    assert torch.equal(ids2, want_ids) and torch.equal(w2, want_w)
    assert torch.equal(out, ref)
    assert ops.workspace_status() == 0


def test_layer_empty_batch(cuda_device):
    """Zero tokens: nothing launched, an empty output."""
    from sglang_restomod_b200.layer import QuantMoELayer

    shape = synth.MoEShape(hidden=256, inter=128, experts=8, top_k=2, shared_inter=128)
    layer = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, cuda_device)
    x = torch.empty(0, shape.hidden, dtype=torch.bfloat16, device=cuda_device)
    ids = torch.empty(0, shape.top_k, dtype=torch.int32, device=cuda_device)
    w = torch.empty(0, shape.top_k, dtype=torch.float32, device=cuda_device)
    out = ops.moe_layer_forward(x, ids, w, quant=0, num_experts=shape.experts, inter=shape.inter,
                                w13=layer.w13, w2=layer.w2, w13_scales=layer.w13_scales,
                                w2_scales=layer.w2_scales)
    assert out.shape == (0, shape.hidden)
