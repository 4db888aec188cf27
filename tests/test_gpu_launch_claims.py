"""bench.py's ``gpu_launches`` claim at N=1 is ``launches_per_forward`` of the
layer (the separate shared MLP's launches included), which restates the
library's scheduling rules. These tests profile one forward and count the
kernels it actually launched, across the regimes the bench and its sweep use:
small decode batches (one preparation kernel, stream GEMMs), the default
decode shape (separate shared MLP with a K-split finishing kernel), the
tensor-core path (plan + slot-order copy) and the three-kernel align from
4096 routes on.

The counting runs in a fresh interpreter: a profiler session opened after
other profiler sessions of the same process missed kernels here."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
CASES = [
    (1, True, None),      # one-token decode, shared route fused
    (8, False, None),     # small batch, separate shared MLP
    (128, False, None),   # the default bench shape's regime (8-slot groups)
    (128, False, 64),     # tensor-core GEMMs: plan + slot-order copy
    (600, False, None),   # >= 4096 routes: three-kernel align
]

_SCRIPT = r"""
import json, sys, torch
sys.path[:0] = [sys.argv[1] + '/sglang-restomod_b200', sys.argv[1]]
from torch.profiler import ProfilerActivity, profile
from sglang_restomod_b200 import _lib, synth
from sglang_restomod_b200.layer import QuantMoELayer
dev = torch.device('cuda', 0)
shape = synth.MoEShape(hidden=512, inter=256, experts=32, top_k=8, shared_inter=256)
res = []
for tokens, fuse, block in json.loads(sys.argv[2]):
    layer = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, dev, fuse_shared=fuse)
    layer.block_size = block
    x = synth.activations(tokens, shape.hidden, dev, seed=3)
    ids, w = synth.route(tokens, shape.experts, shape.top_k, dev, seed=4)
    out = torch.empty_like(x)
    run = lambda: layer.forward(x, ids, w, out=out)
    run(); torch.cuda.synchronize()  # workspaces and plans allocated outside the count
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        run(); torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA
             and 'memcpy' not in e.name.lower() and 'memset' not in e.name.lower()]
    res.append([len(names), layer.launches_per_forward(x.dtype, tokens),
                sorted({n.split('(')[0] for n in names})])
print(json.dumps(res))
"""


@pytest.fixture(scope="module")
def counts(cuda_device):
    proc = subprocess.run([sys.executable, "-c", _SCRIPT, str(ROOT), json.dumps(CASES)],
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    return json.loads(proc.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("case", range(len(CASES)), ids=[str(c) for c in CASES])
def test_layer_launch_claim(counts, case):
    n, claim, names = counts[case]
    assert n == claim, (CASES[case], n, claim, names)  # the claim includes a separate shared MLP


_EP_SCRIPT = r"""
import json, sys, torch
sys.path[:0] = [sys.argv[1] + '/sglang-restomod_b200', sys.argv[1]]
from torch.profiler import ProfilerActivity, profile
from sglang_restomod_b200 import _lib
from tests.test_gpu_ep_peer import SHAPE, _inputs, _setup, _step
dev = torch.device('cuda', 0)
world = 2
res = []
for block in json.loads(sys.argv[2]):
    full, models = _setup(world, 24, _lib.QUANT_FP8_BLOCK, dev, block_size=block)
    inputs = [_inputs(24, SHAPE, dev, 77 + r) for r in range(world)]
    _step(models, inputs); torch.cuda.synchronize()  # workspaces allocated outside the count
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        _step(models, inputs); torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA
             and 'memcpy' not in e.name.lower() and 'memset' not in e.name.lower()]
    claim = sum(m.peer_launches_per_forward(inputs[0][0].dtype) for m in models)
    res.append([len(names), claim, sorted({n.split('(')[0] for n in names})])
print(json.dumps(res))
"""
EP_BLOCKS = [None, 64]


@pytest.fixture(scope="module")
def ep_counts(cuda_device):
    proc = subprocess.run([sys.executable, "-c", _EP_SCRIPT, str(ROOT), json.dumps(EP_BLOCKS)],
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    return json.loads(proc.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("case", range(len(EP_BLOCKS)), ids=[str(b) for b in EP_BLOCKS])
def test_peer_ep_launch_claim(ep_counts, case):
    """Two emulated ranks on one GPU: the kernels of one forward of each
    (dispatch ... combine, plus its shared MLP) against the bench's claim."""
    n, claim, names = ep_counts[case]
    assert n == claim, (EP_BLOCKS[case], n, claim, names)
