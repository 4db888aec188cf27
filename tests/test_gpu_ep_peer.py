"""Expert-parallel peer-memory exchange (b200_ep_*) on one GPU.

One process stands in for ``world`` ranks: each rank gets its own exchange
region on the same GPU and its "peers" are those local buffers, so the
dispatch / expert / combine kernels move exactly the bytes they move across
NVLink, with the ranks' steps interleaved on one stream (every dispatch, then
every expert step, then every combine). No kernel ever waits for a kernel
that runs at the same time: each wait is satisfied by kernels that already
completed. Every rank's output must match the single-GPU layer holding all
experts, within the GEMM tolerance. A last test leaves a flag unset on
purpose and checks that the bounded wait reports it instead of hanging.
"""

from __future__ import annotations

import time

import pytest
import torch

import oracle
from tests.conftest import assert_close
from sglang_restomod_b200 import _lib, ops, synth
from sglang_restomod_b200.ep import ExpertParallelMoE, PeerExchange
from sglang_restomod_b200.layer import QuantMoELayer

pytestmark = pytest.mark.gpu

SHAPE = synth.MoEShape(hidden=256, inter=128, experts=16, top_k=4, shared_inter=128)


def _setup(world, max_tokens, quant, dev, block_size=None, shape=SHAPE, fused=False):
    full = QuantMoELayer.synthetic(shape, quant, dev)
    per = shape.experts // world
    routes_k = shape.top_k + (1 if fused else 0)
    nbytes = ops.ep_region_bytes(world, max_tokens, routes_k, shape.hidden)
    regions = [ops.aligned_zeros(nbytes, dev) for _ in range(world)]
    models = []
    for r in range(world):
        local = QuantMoELayer.synthetic(shape, quant, dev, first_expert=r * per, num_experts=per,
                                        fuse_shared=fused)
        assert local.shared_fused == fused
        local.block_size = block_size
        ex = PeerExchange(world, r, max_tokens, routes_k, shape.hidden, dev, regions=regions)
        models.append(ExpertParallelMoE(local, shape.experts, r, world, transport="peer",
                                        max_tokens=max_tokens, exchange=ex))
    return full, models


def _step(models, inputs):
    """One forward of every emulated rank, interleaved on the current stream.
    A fused shared expert travels as one more route per token."""
    routed = []
    for m, (x, ids, w) in zip(models, inputs):
        if m.fused:
            ids, w = m.local.fused_routes(ids, w, shared_id=m.num_experts)
        routed.append((ids, w))
        m.peer_dispatch(x, ids, w)
    for m in models:
        m.peer_experts()
    outs = []
    for m, (x, _, _), (ids, _) in zip(models, inputs, routed):
        shared = None
        if not m.fused and m.local.shared is not None and len(x):
            shared = m.local.shared.forward(x)
        outs.append(m.peer_combine(ids, shared, None, x.dtype))
    return outs


def _inputs(tokens, shape, dev, seed):
    x = synth.activations(tokens, shape.hidden, dev, seed=seed)
    ids, w = synth.route(tokens, shape.experts, shape.top_k, dev, seed=seed + 1)
    return x, ids, w


@pytest.mark.parametrize("quant", [_lib.QUANT_FP8_BLOCK, _lib.QUANT_NVFP4])
def test_peer_ep_world2_matches_single_gpu(cuda_device, quant):
    dev = cuda_device
    full, models = _setup(2, 24, quant, dev)
    for step in range(3):  # flags carry the step number; regions are reused
        inputs = [_inputs(24, SHAPE, dev, 100 * step + 10 * r) for r in range(2)]
        outs = _step(models, inputs)
        torch.cuda.synchronize()
        for r, ((x, ids, w), out) in enumerate(zip(inputs, outs)):
            want = full.forward(x, ids, w)
            assert_close(out, want, what=f"step {step} rank {r}")
    for m in models:
        assert m.exchange.status() == 0
    assert ops.workspace_status() == 0


def test_peer_ep_world2_against_oracle(cuda_device):
    dev = cuda_device
    shape = synth.MoEShape(hidden=256, inter=128, experts=8, top_k=2)
    full, models = _setup(2, 16, _lib.QUANT_FP8_BLOCK, dev, shape=shape)
    inputs = [_inputs(16, shape, dev, 7 + r) for r in range(2)]
    outs = _step(models, inputs)
    torch.cuda.synchronize()
    q13, s13 = synth.fp8_bank(shape.experts, 2 * shape.inter, shape.hidden, dev, 10)
    q2, s2 = synth.fp8_bank(shape.experts, shape.hidden, shape.inter, dev, 11)
    d13 = torch.stack([oracle.dequant_block_fp8(q13[e].cpu(), s13[e].cpu()) for e in range(shape.experts)])
    d2 = torch.stack([oracle.dequant_block_fp8(q2[e].cpu(), s2[e].cpu()) for e in range(shape.experts)])
    for r, ((x, ids, w), out) in enumerate(zip(inputs, outs)):
        want = oracle.moe_layer_ref(x.cpu(), ids.cpu(), w.cpu(), d13, d2)
        assert_close(out, want, what=f"rank {r} vs oracle")


def test_peer_ep_world4_ragged_tokens(cuda_device):
    """Ranks with fewer tokens than max_tokens, one with none at all."""
    dev = cuda_device
    full, models = _setup(4, 40, _lib.QUANT_FP8_BLOCK, dev)
    for step, counts in enumerate(((40, 7, 0, 33), (1, 40, 40, 0))):
        inputs = [_inputs(t, SHAPE, dev, 1000 + 17 * r + step) for r, t in enumerate(counts)]
        outs = _step(models, inputs)
        torch.cuda.synchronize()
        for r, ((x, ids, w), out) in enumerate(zip(inputs, outs)):
            assert out.shape == (counts[r], SHAPE.hidden)
            if counts[r]:
                assert_close(out, full.forward(x, ids, w), what=f"step {step} rank {r}")
    for m in models:
        assert m.exchange.status() == 0


def test_peer_ep_tensor_core_path(cuda_device):
    """Blocks of 64 route slots: the owner's GEMMs run on the tcgen05 kernel,
    whose epilogue stores through the destination-row table."""
    dev = cuda_device
    full, models = _setup(2, 128, _lib.QUANT_FP8_BLOCK, dev, block_size=64)
    inputs = [_inputs(128, SHAPE, dev, 55 + r) for r in range(2)]
    outs = _step(models, inputs)
    torch.cuda.synchronize()
    for r, ((x, ids, w), out) in enumerate(zip(inputs, outs)):
        assert_close(out, full.forward(x, ids, w), what=f"rank {r}")
    assert ops.workspace_status() == 0


@pytest.mark.parametrize("world,block", [(2, None), (4, None), (2, 64)])
def test_peer_ep_fused_shared_expert(cuda_device, world, block):
    """The shared expert as one more local route per token (kept on the source
    rank by the dispatch), stream and tcgen05 owner GEMMs."""
    dev = cuda_device
    full, models = _setup(world, 64, _lib.QUANT_FP8_BLOCK, dev, block_size=block, fused=True)
    assert all(m.fused for m in models)
    for step in range(2):
        inputs = [_inputs(64 - 9 * r * step, SHAPE, dev, 500 + 31 * r + step) for r in range(world)]
        outs = _step(models, inputs)
        torch.cuda.synchronize()
        for r, ((x, ids, w), out) in enumerate(zip(inputs, outs)):
            assert_close(out, full.forward(x, ids, w), what=f"fused w={world} step {step} rank {r}")
    for m in models:
        assert m.exchange.status() == 0
    assert ops.workspace_status() == 0


def test_peer_ep_graph_replay(cuda_device):
    """The three calls of every rank captured in one CUDA graph and replayed."""
    dev = cuda_device
    full, models = _setup(2, 24, _lib.QUANT_FP8_BLOCK, dev)
    inputs = [_inputs(24, SHAPE, dev, 300 + r) for r in range(2)]
    _step(models, inputs)  # warm-up (workspace sized before capture)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = _step(models, inputs)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    for r, ((x, ids, w), out) in enumerate(zip(inputs, outs)):
        assert_close(out, full.forward(x, ids, w), what=f"rank {r}")
    for m in models:
        assert m.exchange.status() == 0


def test_peer_ep_missing_rank_times_out_with_status(cuda_device):
    """Rank 1 never dispatches: rank 0's waits give up after their bound and
    report bit 8 in its region status; nothing hangs."""
    dev = cuda_device
    _, models = _setup(2, 8, _lib.QUANT_FP8_BLOCK, dev)
    x, ids, w = _inputs(8, SHAPE, dev, 5)
    m0 = models[0]
    t0 = time.time()
    m0.peer_dispatch(x, ids, w)
    m0.peer_experts()
    m0.peer_combine(ids, None, None, x.dtype)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert m0.exchange.status() & 8
    assert elapsed < 30, elapsed


def test_peer_ep_one_row_per_token_and_owner(cuda_device):
    """Deduplicated dispatch: each owner receives exactly one row per
    (source token, owner) pair, whatever the number of that token's routes it
    owns, and the output still matches the single-GPU layer."""
    dev = cuda_device
    world, tokens = 4, 32
    full, models = _setup(world, tokens, _lib.QUANT_FP8_BLOCK, dev)
    inputs = [_inputs(tokens, SHAPE, dev, 900 + r) for r in range(world)]
    outs = _step(models, inputs)
    torch.cuda.synchronize()
    per = SHAPE.experts // world
    for o, m in enumerate(models):
        want_rows = sum(int(((ids.long() // per) == o).any(1).sum()) for _, ids, _ in inputs)
        ids_r, _, _ = m.exchange.received()
        assert ids_r.shape == (world * tokens, SHAPE.top_k)
        live = int((ids_r >= 0).any(1).sum())
        assert live == want_rows, (o, live, want_rows)
        routes_here = sum(int(((ids.long() // per) == o).sum()) for _, ids, _ in inputs)
        assert int((ids_r >= 0).sum()) == routes_here
    for r, ((x, ids, w), out) in enumerate(zip(inputs, outs)):
        assert_close(out, full.forward(x, ids, w), what=f"rank {r}")
    for m in models:
        assert m.exchange.status() == 0

