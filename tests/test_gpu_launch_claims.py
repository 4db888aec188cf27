"""bench.py's ``gpu_launches`` claim at N=1 is ``launches_per_forward`` of the
layer (the separate shared MLP's launches included), which restates the
library's scheduling rules. These tests profile one forward and count the
kernels it actually launched, across the regimes the bench and its sweep use:
small decode batches (one preparation kernel, stream GEMMs), the default
decode shape (separate shared MLP with a K-split finishing kernel), the
tensor-core path (plan + slot-order copy) and the three-kernel align from
4096 routes on."""

from __future__ import annotations

import pytest
import torch
from torch.profiler import ProfilerActivity, profile

from sglang_restomod_b200 import _lib, synth
from sglang_restomod_b200.layer import QuantMoELayer

pytestmark = pytest.mark.gpu


def _count_kernels(fn) -> tuple[int, list[str]]:
    fn()  # warm-up: workspaces and plans allocated outside the count
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA
             and "memcpy" not in e.name.lower() and "memset" not in e.name.lower()]
    return len(names), sorted({n.split("(")[0] for n in names})


@pytest.mark.parametrize("tokens,fuse,block", [
    (1, True, None),      # one-token decode, shared route fused
    (8, False, None),     # small batch, separate shared MLP
    (128, False, None),   # the default bench shape's regime (8-slot groups)
    (128, False, 64),     # tensor-core GEMMs: plan + slot-order copy
    (600, False, None),   # >= 4096 routes: three-kernel align
])
def test_layer_launch_claim(cuda_device, tokens, fuse, block):
    dev = cuda_device
    shape = synth.MoEShape(hidden=512, inter=256, experts=32, top_k=8, shared_inter=256)
    layer = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, dev, fuse_shared=fuse)
    layer.block_size = block
    x = synth.activations(tokens, shape.hidden, dev, seed=3)
    ids, w = synth.route(tokens, shape.experts, shape.top_k, dev, seed=4)
    out = torch.empty_like(x)
    n, names = _count_kernels(lambda: layer.forward(x, ids, w, out=out))
    claim = layer.launches_per_forward(x.dtype, tokens)  # includes a separate shared MLP
    assert n == claim, (n, claim, names)
