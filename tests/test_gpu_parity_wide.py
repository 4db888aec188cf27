"""GPU parity on the benchmarked configurations themselves and on the
reference's own outputs.

* The default bench workload (config4 decode: H=7168, I=2048, 256 experts,
  top-8, shared expert I=2048, 128 tokens), built exactly as ``bench.py``
  builds it at N=1 - same seeds, the shared expert appended to the banks,
  the layer's own block-size rule (8-slot groups at 4 routes per expert) and
  the separate shared MLP that rule implies - with every token checked
  against the oracle.
* The golden fixtures made by running the reference's own code
  (``tests/golden/make_golden.py``): ``quant/sm70_fp8_moe/check.py``'s dense
  loop and ``SM70Fp8MoEMethod.apply`` (dense, EP clamp, EP compaction,
  empty, output scale). Their inputs go straight into
  ``b200_moe_layer_forward`` and the result is compared with the stored
  reference outputs, so the kernel -> reference link does not pass through
  the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from sglang_restomod_b200 import _lib, ops, synth
from sglang_restomod_b200.layer import QuantMoELayer, block_size_for
from tests.conftest import assert_close, load_golden

pytestmark = pytest.mark.gpu


def _fp8_fetch(q13, s13, q2, s2):
    """e -> (dequantized w13[e], w2[e]) on the CPU, one expert at a time."""

    def fetch(e):
        return (oracle.dequant_block_fp8(q13[e].cpu(), s13[e].cpu()),
                oracle.dequant_block_fp8(q2[e].cpu(), s2[e].cpu()))

    return fetch


def test_config4_decode_bench_workload_exact(cuda_device):
    """bench.py's default workload at N=1, every token against the oracle."""
    shape, tokens, seed = synth.CONFIG4, 128, 10
    # bench.MoEWorkload: QuantMoELayer.synthetic(..., fuse_shared=True), inputs
    # seeded 100 + rank / 200 + rank, forward through ExpertParallelMoE at world 1
    layer = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, cuda_device, first_expert=0,
                                    num_experts=shape.experts, fuse_shared=True)
    x = synth.activations(tokens, shape.hidden, cuda_device, seed=100)
    ids, w = synth.route(tokens, shape.experts, shape.top_k, cuda_device, seed=200)
    # the configuration bench times: 8-slot stream groups, shared expert as its own MLP
    assert block_size_for(tokens * shape.top_k, shape.experts) == 8
    assert layer.shared_fused and layer.fused_block_size(tokens) is None
    from sglang_restomod_b200.ep import ExpertParallelMoE

    model = ExpertParallelMoE(layer, shape.experts, 0, 1)
    out = torch.empty_like(x)
    model.forward(x, ids, w, out=out)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0

    q13, s13 = synth.fp8_bank(shape.experts, 2 * shape.inter, shape.hidden, cuda_device, seed)
    q2, s2 = synth.fp8_bank(shape.experts, shape.hidden, shape.inter, cuda_device, seed + 1)
    sq13, ss13 = synth.fp8_bank(1, 2 * shape.shared_inter, shape.hidden, cuda_device, seed + 2)
    sq2, ss2 = synth.fp8_bank(1, shape.hidden, shape.shared_inter, cuda_device, seed + 3)
    xc = x.cpu()
    shared = oracle.moe_layer_ref(xc, torch.zeros(tokens, 1, dtype=torch.int32),
                                  torch.ones(tokens, 1), _fp8_fetch(sq13, ss13, sq2, ss2), 1)
    want = oracle.moe_layer_ref(xc, ids.cpu(), w.cpu(), _fp8_fetch(q13, s13, q2, s2),
                                shape.experts, shared_out=shared)
    assert_close(out, want, what="config4 decode bench workload, all 128 tokens")


# -------------------------------------------- the reference's own outputs
def _f16(a, shape):
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.float16).reshape(shape)


def _e4m3(a):
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn)


def _golden_bank(g, device):
    q13 = _e4m3(g["w13"]).to(device)  # [E, 2I, H]
    q2 = _e4m3(g["w2"]).to(device)    # [E, H, I]
    s13 = torch.from_numpy(g["s13"]).to(device)
    s2 = torch.from_numpy(g["s2"]).to(device)
    return dict(w13=ops.fp8_prepack(q13, True), w2=ops.fp8_prepack(q2, False), w13_scales=s13,
                w2_scales=s2), int(q13.shape[0]), int(q13.shape[1]) // 2


@pytest.mark.parametrize("block", [8, 16, 64])
@pytest.mark.parametrize("ids_key,ref_key", [("ids", "ref"), ("ids_ep", "ref_ep")])
def test_kernels_match_reference_check_outputs(cuda_device, block, ids_key, ref_key):
    """quant/sm70_fp8_moe/check.py:34-48 (_reference): dense and EP-dropped routes."""
    g = load_golden("fp8_moe_check.npz")
    bank, experts, inter = _golden_bank(g, cuda_device)
    hidden = inter
    x = _f16(g["x"], (-1, hidden)).to(cuda_device)
    ids = torch.from_numpy(g[ids_key]).to(cuda_device).contiguous()
    w = torch.from_numpy(g["weights"]).to(cuda_device).contiguous()
    out = ops.moe_layer_forward(x, ids, w, quant=_lib.QUANT_FP8_BLOCK, num_experts=experts,
                                inter=inter, block_size=block, out=torch.empty_like(x), **bank)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0
    assert_close(out, torch.from_numpy(g[ref_key]), what=f"check.py {ids_key} block {block}")


@pytest.mark.parametrize("block", [8, 16, 64])
@pytest.mark.parametrize("case", ["dense", "ep_clamp", "ep_compact", "empty", "scaled"])
def test_kernels_match_reference_method_outputs(cuda_device, block, case):
    """SM70Fp8MoEMethod.apply (quant/sm70_fp8_moe/method.py:239-309) run by the
    reference on the CPU; its output_scale maps to routed_scaling_factor (no
    shared expert). The reference rounds to fp16 at every step, so the
    absolute tolerance is taken relative to the output's largest value."""
    g = load_golden("fp8_moe_method.npz")
    bank, experts, inter = _golden_bank(g, cuda_device)
    hidden = inter
    ids = torch.from_numpy(g[f"{case}__ids"]).to(cuda_device).contiguous()
    tokens = ids.shape[0]
    x = _f16(g[f"{case}__x"], (tokens, hidden)).to(cuda_device)
    w = torch.from_numpy(g[f"{case}__weights"]).to(cuda_device).contiguous()
    scale = float(g[f"{case}__output_scale"])
    out = ops.moe_layer_forward(x, ids, w, quant=_lib.QUANT_FP8_BLOCK, num_experts=experts,
                                inter=inter, block_size=block, routed_scaling_factor=scale,
                                out=torch.empty_like(x), **bank)
    torch.cuda.synchronize()
    assert ops.workspace_status() == 0
    want = _f16(g[f"{case}__out"], (tokens, hidden)).float()
    atol = 2e-2 * float(want.abs().max().clamp_min(1.0))
    assert_close(out, want, rtol=2e-2, atol=atol, what=f"method {case} block {block}")
    if case == "empty":
        assert int(torch.count_nonzero(out)) == 0
