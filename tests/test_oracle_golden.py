"""Pin the CPU oracle against outputs of the reference's own code.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py,
which runs the sglang-restomod functions named there on the CPU.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle import align as oalign
from tests.conftest import load_golden


def _f16(a):
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.float16)


def _e4m3(a, shape=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn)
    return t.reshape(shape) if shape is not None else t


def test_fp8_block_quant_matches_reference():
    g = load_golden("fp8_quant.npz")
    w = _f16(g["w"]).reshape(256, 256)
    q, s = oracle.quant_block_fp8(w)
    assert np.array_equal(q.view(torch.uint8).numpy().reshape(-1), g["q"].reshape(-1))
    assert np.array_equal(s.numpy(), g["s"])
    deq = oracle.dequant_block_fp8(q, s)
    assert np.array_equal(deq.numpy(), g["deq"])


def test_fp8_lm_head_quant_matches_reference():
    g = load_golden("fp8_quant.npz")
    head = _f16(g["head"]).reshape(256, 256)
    q, s = oracle.quant_block_fp8_lm_head(head)
    assert np.array_equal(q.view(torch.uint8).numpy().reshape(-1), g["head_q"].reshape(-1))
    assert np.array_equal(s.numpy(), g["head_s"])


def _fp8_moe_inputs(g, ids_key):
    experts, hidden, inter = 4, 128, 128
    w13 = oracle.dequant_block_fp8  # alias for brevity below
    q13 = _e4m3(g["w13"], (experts, 2 * inter, hidden))
    q2 = _e4m3(g["w2"], (experts, hidden, inter))
    s13 = torch.from_numpy(g["s13"])
    s2 = torch.from_numpy(g["s2"])
    d13 = torch.stack([w13(q13[e], s13[e]) for e in range(experts)])
    d2 = torch.stack([w13(q2[e], s2[e]) for e in range(experts)])
    x = _f16(g["x"]).reshape(8, hidden)
    ids = torch.from_numpy(g[ids_key])
    weights = torch.from_numpy(g["weights"])
    return x, ids, weights, d13, d2


@pytest.mark.parametrize("ids_key,ref_key", [("ids", "ref"), ("ids_ep", "ref_ep")])
def test_fp8_moe_dense_reference(ids_key, ref_key):
    """The layer oracle equals check._reference (the reference's dense loop)."""
    g = load_golden("fp8_moe_check.npz")
    x, ids, weights, d13, d2 = _fp8_moe_inputs(g, ids_key)
    got = oracle.moe_layer_ref(x, ids, weights, d13, d2, inter_dtype=None)
    np.testing.assert_allclose(got.numpy(), g[ref_key], rtol=1e-5, atol=1e-5)


CASES = ["dense", "ep_clamp", "ep_compact", "empty", "scaled"]


@pytest.mark.parametrize("case", CASES)
def test_fp8_moe_method_semantics(case):
    """oracle.fp8_moe_method_ref agrees with SM70Fp8MoEMethod.apply run on the CPU.

    The reference rounds the gathered rows, both GEMM outputs, the router
    weights and the index_add_ accumulator to fp16; the oracle keeps fp32, so
    the comparison allows fp16-level differences.
    """
    g = load_golden("fp8_moe_method.npz")
    local, hidden, inter = 4, 128, 128
    q13 = _e4m3(g["w13"], (local, 2 * inter, hidden))
    q2 = _e4m3(g["w2"], (local, hidden, inter))
    s13, s2 = torch.from_numpy(g["s13"]), torch.from_numpy(g["s2"])
    d13 = torch.stack([oracle.dequant_block_fp8(q13[e], s13[e]) for e in range(local)])
    d2 = torch.stack([oracle.dequant_block_fp8(q2[e], s2[e]) for e in range(local)])
    ids = torch.from_numpy(g[f"{case}__ids"])
    tokens = ids.shape[0]
    x = _f16(g[f"{case}__x"]).reshape(tokens, hidden)
    weights = torch.from_numpy(g[f"{case}__weights"])
    scale = float(g[f"{case}__output_scale"])
    want = _f16(g[f"{case}__out"]).reshape(tokens, hidden).float()
    got = oracle.fp8_moe_method_ref(x, ids, weights, d13, d2, output_scale=scale)
    tol = 2e-2 * float(want.abs().max().clamp_min(1.0))
    np.testing.assert_allclose(got.numpy(), want.numpy(), rtol=2e-2, atol=tol)
    if case == "empty":
        assert int(torch.count_nonzero(want)) == 0


@pytest.mark.parametrize("case", ["dense", "ep_compact"])
def test_align_order_matches_reference_method_order(case):
    """The oracle's moe_align route order equals the order in which the
    reference's SM70Fp8MoEMethod.apply gathers rows (its stable argsort)."""
    g = load_golden("fp8_moe_method.npz")
    ids = g[f"{case}__ids"]
    tokens, top_k = ids.shape
    offsets = g[f"{case}__offsets"]
    gathered_tokens = g[f"{case}__order"].astype(np.int64)
    sorted_ids, expert_ids, total = oracle.moe_align_block_size(ids, 4, 1)
    assert total == int((ids >= 0).sum())
    for e in range(4):
        mine = [int(r) // top_k for r in sorted_ids[:total] if ids.reshape(-1)[int(r)] == e]
        theirs = gathered_tokens[offsets[e] : offsets[e + 1]].tolist()
        assert mine == theirs, f"expert {e}: {mine} != {theirs}"


def test_nvfp4_quant_and_dequant_match_reference():
    g = load_golden("nvfp4_quant.npz")
    w = _f16(g["w"]).reshape(128, 256)
    packed, scales = oracle.quantize_nvfp4(w)
    assert np.array_equal(packed.numpy(), g["packed"])
    assert np.array_equal(scales.view(torch.uint8).numpy().reshape(-1), g["scales"].reshape(-1))
    deq = oracle.dequant_nvfp4(packed, scales)
    want = _f16(g["deq"]).reshape(128, 256).float()
    assert torch.equal(deq, want)


def test_nvfp4_scale_encoder_golden_table():
    g = load_golden("nvfp4_scales.npz")
    table = _e4m3(g["table"], (1, 1, 8))
    got = oracle.encode_scales(table).reshape(-1).numpy()
    assert np.array_equal(got, g["enc_table"].reshape(-1))
    # The test file's own table, in the encoder's 0,2,1,3 pair order.
    want = [int(g["golden_byte"][i]) for i in (0, 2, 1, 3, 4, 6, 5, 7)]
    assert got.tolist() == want
    rnd = _e4m3(g["rnd"], (2, 3, 64))
    assert np.array_equal(oracle.encode_scales(rnd).reshape(-1).numpy(), g["enc_rnd"].reshape(-1))
    gs = torch.from_numpy(g["gs"])
    assert np.array_equal(oracle.encode_global_scale(gs).numpy(), g["enc_gs"])


def test_align_oracle_properties():
    rng = np.random.default_rng(0)
    for numel, experts, bs in [(0, 4, 8), (1, 4, 8), (128, 16, 64), (2560, 512, 16), (97, 7, 3)]:
        ids = rng.integers(-1, experts, size=numel).astype(np.int32)
        sorted_ids, expert_ids, total = oracle.moe_align_block_size(ids, experts, bs)
        cap = oalign.sorted_capacity(numel, experts, bs)
        assert sorted_ids.shape == (cap,)
        assert total % bs == 0 and total <= cap
        valid = [(i, e) for i, e in enumerate(ids.tolist()) if 0 <= e < experts]
        got = [int(r) for r in sorted_ids[:total] if r != numel]
        assert got == [i for i, _ in sorted(valid, key=lambda t: t[1])]  # stable expert-major
        for b in range(total // bs):
            block = sorted_ids[b * bs : (b + 1) * bs]
            real = [int(r) for r in block if r != numel]
            assert all(ids[r] == expert_ids[b] for r in real)
        assert (expert_ids[total // bs :] == -1).all()
        assert (sorted_ids[total:] == numel).all()


def test_grouped_router_oracle_known_case():
    """Group score by maximum vs by top-2 sum (biased grouped top-k)."""
    logits = torch.full((1, 16), -4.0)
    logits[0, 0] = 4.0
    logits[0, 4:6] = 3.0
    logits[0, 8:10] = 2.9
    ids, w = oracle.route_topk_grouped(logits, 2, 4, 1, scoring="sigmoid", bias=torch.zeros(16))
    assert ids[0].tolist() == [4, 5] and abs(float(w.sum()) - 1.0) < 1e-6
    ids, _ = oracle.route_topk_grouped(logits, 2, 4, 1, scoring="sigmoid")
    assert ids[0].tolist() == [0, 1]
    # with every group kept it is the plain top-k
    x = torch.randn(5, 32, generator=torch.Generator().manual_seed(1))
    a = oracle.route_topk_grouped(x, 4, 4, 4)
    b = oracle.route_topk_general(x, 4)
    assert torch.equal(a[0], b[0]) and torch.allclose(a[1], b[1])
