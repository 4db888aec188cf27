"""Host-side logic of the plugin surface, without a GPU (the reference's CPU
test strategy: registry, attestation, mode switches, shape guards)."""

from __future__ import annotations

import ctypes
import json
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from sglang_restomod_b200 import attest, plugins
from tests.conftest import load_golden


@pytest.fixture(autouse=True)
def _fresh_attest():
    attest.reset()
    yield
    attest.reset()


def test_selection_parses_dedups_and_refuses_unknown():
    env = {plugins.ENV_COMPONENTS: " fp8_moe, fp8_dense,fp8_moe ,, "}
    assert plugins.selection(env) == ["fp8_moe", "fp8_dense"]
    assert plugins.selection({}) == []
    with pytest.raises(ValueError, match="unknown component"):
        plugins.selection({plugins.ENV_COMPONENTS: "fp8_moe,bogus"})
    with pytest.raises(ValueError, match="not part of the B200 MoE/GEMV path"):
        plugins.selection({plugins.ENV_COMPONENTS: "attention_v100"})


def test_load_enabled_records_every_outcome(tmp_path, monkeypatch):
    # On a machine without a B200 each selected component registers but is inactive.
    monkeypatch.setenv(attest.ENV_ATTEST, str(tmp_path / "attest.json"))
    names = ["fp8_moe", "fp4_moe", "fp8_dense", "moe_align_sm70", "fp8_dense_quant", "fp4_dense"]
    loaded = plugins.load_enabled({plugins.ENV_COMPONENTS: ",".join(names)})
    assert loaded == names
    snap = json.loads((tmp_path / "attest.json").read_text())
    assert snap["selected"] == names
    assert sorted(snap["inactive"]) == sorted(names)
    assert snap["failed"] == [] and snap["missing"] == []
    assert "inactive" in snap["components"]["fp8_moe"]["detail"]


def test_forced_mode_on_a_non_b200_host_is_a_recorded_failure(monkeypatch):
    monkeypatch.setenv("SGLANG_B200_FP8_MOE", "on")
    loaded = plugins.load_enabled({plugins.ENV_COMPONENTS: "fp8_moe,fp8_dense"})
    snap = attest.snapshot()
    assert "fp8_moe" in snap["failed"] and "fp8_moe" not in loaded
    assert "requires a B200" in snap["components"]["fp8_moe"]["detail"]
    assert "fp8_dense" in loaded  # one failure does not take the others down


def test_unknown_mode_value_raises(monkeypatch):
    from sglang_restomod_b200._common import mode

    monkeypatch.setenv("SGLANG_B200_FP8_MOE", "maybe")
    with pytest.raises(ValueError, match="auto, on or off"):
        mode("SGLANG_B200_FP8_MOE")
    monkeypatch.setenv("SGLANG_B200_FP8_MOE", "OFF")
    assert mode("SGLANG_B200_FP8_MOE") == "off"


def test_attest_inactive_keeps_reason_after_record():
    attest.inactive("x", "why not")
    attest.record("x", True)
    snap = attest.snapshot()
    assert snap["components"]["x"]["detail"] == "registered, inactive: why not"
    assert snap["inactive"] == ["x"] and snap["loaded"] == ["x"]


def _cfg(**kw):
    base = dict(activation="silu", is_gated=True, swiglu_limit=None, gemm1_clamp_limit=None,
                gemm1_alpha=None, gemm1_beta=None, apply_router_weight_on_input=False,
                no_combine=False, wide_output_scale=1.0, gate_up_input_scale=1.0)
    base.update(kw)
    return SimpleNamespace(**base)


def test_fp8_moe_method_refuses_what_the_epilogue_cannot_do():
    from sglang_restomod_b200.quant.fp8_moe.method import B200Fp8MoEMethod

    check = B200Fp8MoEMethod._unsupported_reason
    assert check(_cfg()) is None
    assert "activation" in check(_cfg(activation="gelu"))
    assert check(_cfg(swiglu_limit=7.0)) == "clamped SwiGLU"
    assert check(_cfg(gemm1_alpha=1.7)) == "SwiGLU alpha/beta"
    assert "router weight" in check(_cfg(no_combine=True))
    assert check(_cfg(wide_output_scale=2.0)) == "FP8 range scaling"


def test_shape_guards():
    from sglang_restomod_b200.quant.fp4_moe.method import check_expert_shape
    from sglang_restomod_b200.quant.fp8_dense import _check_dense_weight_shape
    from sglang_restomod_b200.quant.fp8_moe import _check_gemm_shape

    with pytest.raises(RuntimeError, match="needs K a multiple of the 128-wide quantization group"):
        _check_gemm_shape(100, 256)
    with pytest.raises(RuntimeError, match="needs N a multiple of 256"):
        _check_gemm_shape(128, 384, gated=True)
    _check_gemm_shape(128, 384)
    with pytest.raises(RuntimeError, match="multiples of 128"):
        check_expert_shape(320, 2560)  # the reference's TP4 shard: not a 128-row multiple
    with pytest.raises(RuntimeError, match="positive"):
        _check_dense_weight_shape(0, 128)


def test_regroup_unsupported_block_sizes():
    from sglang_restomod_b200.quant.fp4_moe.method import _regroup

    sentinel = 99
    # block 48: two blocks (experts 3, 5) holding 2 and 1 real routes
    sorted_ids = torch.full((96,), sentinel, dtype=torch.int32)
    sorted_ids[0], sorted_ids[1], sorted_ids[48] = 4, 7, 2
    expert_ids = torch.tensor([3, 5], dtype=torch.int32)
    ntpp = torch.tensor([96], dtype=torch.int32)
    s2, e2, n2, block = _regroup(sorted_ids, expert_ids, ntpp, 48, sentinel)
    assert block == 64 and e2.tolist() == [3, 5] and int(n2) == 128
    assert s2[:2].tolist() == [4, 7] and int(s2[64]) == 2 and int((s2 != sentinel).sum()) == 3
    # block 128 splits into two 64-slot blocks of the same expert
    sorted_ids = torch.full((128,), sentinel, dtype=torch.int32)
    sorted_ids[0], sorted_ids[100] = 1, 0
    s3, e3, n3, block = _regroup(sorted_ids, torch.tensor([6], dtype=torch.int32),
                                 torch.tensor([128], dtype=torch.int32), 128, sentinel)
    assert block == 64 and e3.tolist() == [6, 6] and int(n3) == 128
    assert int(s3[0]) == 1 and int(s3[100]) == 0


def test_lm_head_quantizer_matches_reference_golden():
    from sglang_restomod_b200.quant.fp8_lm_head import _quantize

    g = load_golden("fp8_quant.npz")
    head = torch.from_numpy(np.ascontiguousarray(g["head"])).view(torch.float16).reshape(256, 256)
    q, s = _quantize(head)
    assert np.array_equal(q.view(torch.uint8).numpy().reshape(-1), g["head_q"].reshape(-1))
    assert np.array_equal(s.numpy(), g["head_s"])


def test_router_host_validation_without_a_gpu():
    """b200_topk_route refuses bad arguments before touching the device."""
    import ctypes

    from sglang_restomod_b200 import _lib

    lib = _lib.load()
    ids = (ctypes.c_int32 * 8)()
    w = (ctypes.c_float * 8)()
    logits = (ctypes.c_float * 64)()
    # top_k above 32
    assert lib.b200_topk_route(logits, 2, 1, 64, 33, 0, 1, None, ids, w, None) == _lib.ERR_INVALID
    # top_k above num_experts
    assert lib.b200_topk_route(logits, 2, 1, 4, 8, 0, 1, None, ids, w, None) == _lib.ERR_INVALID
    # correction bias with softmax scoring
    bias = (ctypes.c_float * 64)()
    assert lib.b200_topk_route(logits, 2, 1, 64, 8, 0, 1, bias, ids, w, None) == _lib.ERR_INVALID
    # too many experts, bad dtype, unknown scoring
    assert lib.b200_topk_route(logits, 2, 1, 2000, 8, 0, 1, None, ids, w, None) == _lib.ERR_UNSUPPORTED
    assert lib.b200_topk_route(logits, 7, 1, 64, 8, 0, 1, None, ids, w, None) == _lib.ERR_UNSUPPORTED
    assert lib.b200_topk_route(logits, 2, 1, 64, 8, 5, 1, None, ids, w, None) == _lib.ERR_INVALID
    # no tokens: nothing to do
    assert lib.b200_topk_route(None, 2, 0, 64, 8, 0, 1, None, None, None, None) == _lib.OK


def test_router_oracle_tie_order():
    import torch

    import oracle

    logits = torch.zeros(2, 8)
    logits[:, 5] = 1.0
    logits[:, 2] = 0.5
    logits[:, 6] = 0.5
    ids, w = oracle.route_topk_general(logits, 3)
    assert ids.tolist() == [[5, 2, 6], [5, 2, 6]]
    assert torch.allclose(w.sum(-1), torch.ones(2))


def test_block_size_rule_follows_the_measured_crossovers():
    """8-slot groups up to 6 routes per expert, 16-slot up to 16, then the
    tcgen05 blocks of 64 (the B200 measurements in block_size_for's doc)."""
    from sglang_restomod_b200.layer import block_size_for

    assert block_size_for(1024, 256) == 8      # config4 decode, 4 per expert
    assert block_size_for(2816, 513) == 8      # config2 T=256 with the shared route
    assert block_size_for(600, 100) == 8       # 6.0
    assert block_size_for(601, 100) == 16
    assert block_size_for(1024, 128) == 16     # 8 per expert
    assert block_size_for(1535, 128) == 16     # just under 12
    assert block_size_for(1536, 128) == 64     # 12 per expert
    assert block_size_for(1024, 64) == 64      # 16 per expert: the tensor-core GEMM
    assert block_size_for(1024, 32) == 64      # expert-parallel owner at 8 ranks
    assert block_size_for(0, 512) == 8


def test_dense_split_rule_matches_the_measured_choices():
    """The split-K choices b200_linear makes on 148 SMs for the shapes it was
    measured on (restated in layer.dense_k_parts for launch accounting)."""
    from sglang_restomod_b200.layer import dense_k_parts

    assert dense_k_parts(64, 25600, 5120, 148) == 1    # evening out waves: slower split
    assert dense_k_parts(33, 25600, 5120, 148) == 1
    assert dense_k_parts(128, 4096, 7168, 148) == 4    # shared expert gate/up: fills idle SMs
    assert dense_k_parts(128, 7168, 2048, 148) == 1    # shared expert down
    assert dense_k_parts(64, 5120, 25600, 148) == 7
    assert dense_k_parts(64, 152064, 5120, 148) == 1   # partials beyond the workspace


# ------------------------------------------------ fp8_dense_quant admission
def test_dense_quant_admission_reasons():
    from sglang_restomod_b200.quant.fp8_dense_quant import refusal

    class ReplicatedLinear(torch.nn.Linear):
        pass

    lin = torch.nn.Linear(256, 384, bias=False).to(torch.bfloat16)
    assert refusal("model.layers.0.mlp.down_proj", lin) is None
    assert refusal("", lin) == "unnamed"
    assert refusal("model.layers.0.mlp.experts.w2", lin) == "expert"
    assert refusal("model.layers.0.mlp.shared_experts.down_proj", lin) == "expert"
    assert refusal("lm_head", lin) == "lm_head"
    assert refusal("model.gate", ReplicatedLinear(256, 384).to(torch.bfloat16)) == "router"
    assert refusal("x", torch.nn.Linear(256, 384)) == "dtype"  # fp32
    assert refusal("x", torch.nn.Linear(200, 384).to(torch.bfloat16)) == "shape:384x200"
    assert refusal("x", torch.nn.LayerNorm(256).to(torch.bfloat16)) == "no-2d-weight"

    class EngineLinear(torch.nn.Module):  # duck-typed engine linear
        def __init__(self, method):
            super().__init__()
            self.weight = torch.nn.Parameter(torch.zeros(256, 256, dtype=torch.bfloat16))
            self.quant_method = method
            self.input_size_per_partition = 256

    class UnquantizedLinearMethod:
        pass

    class Fp8LinearMethod:
        pass

    assert refusal("a.b", EngineLinear(UnquantizedLinearMethod())) is None
    assert refusal("a.b", EngineLinear(Fp8LinearMethod())) == "quantized:Fp8LinearMethod"


def test_dense_quant_hooks_load_model_once():
    from sglang_restomod_b200.quant.fp8_dense_quant import hook_load_model

    seen = []

    class Runner:
        def load_model(self):
            self.model = "the model"
            return "loaded"

    assert hook_load_model(Runner, convert_all=lambda m: seen.append(m) or {"converted": 1})
    assert not hook_load_model(Runner, convert_all=lambda m: seen.append(("again", m)))
    assert Runner().load_model() == "loaded"
    assert seen == ["the model"]

    class Broken:
        def load_model(self):
            self.model = None

    hook_load_model(Broken, convert_all=lambda m: 1 / 0)
    Broken().load_model()  # a failing conversion leaves the server up


def test_rebind_reaches_modules_that_imported_the_name(monkeypatch):
    import sys
    import types

    from sglang_restomod_b200._common import rebind_everywhere

    def original():
        return "upstream"

    def replacement():
        return "b200"

    consumer = types.ModuleType("fake_consumer_of_align")
    consumer.moe_align_block_size = original
    monkeypatch.setitem(sys.modules, "fake_consumer_of_align", consumer)
    other = types.ModuleType("fake_unrelated")
    other.moe_align_block_size = lambda: "someone else's"
    monkeypatch.setitem(sys.modules, "fake_unrelated", other)
    assert rebind_everywhere("moe_align_block_size", original, replacement) == 1
    assert consumer.moe_align_block_size is replacement
    assert other.moe_align_block_size() == "someone else's"


def test_attest_failure_overrides_inactive_and_write_is_atomic(tmp_path):
    attest.set_selected(["a", "b", "c"])
    attest.inactive("a", "no GPU")
    attest.record("a", False, "RuntimeError: boom")
    attest.record("b", True)
    snap = attest.snapshot()
    assert snap["failed"] == ["a"] and snap["loaded"] == ["b"] and snap["missing"] == ["c"]
    assert snap["components"]["a"] == {"ok": False, "detail": "RuntimeError: boom"}
    path = tmp_path / "out.json"
    assert attest.write(str(path)) == str(path)
    assert json.loads(path.read_text())["selected"] == ["a", "b", "c"]
    assert [p.name for p in tmp_path.iterdir()] == ["out.json"]
    assert attest.write(str(tmp_path / "missing-dir" / "x.json")) is None


# ------------------------------------------------------- census and profile
def test_census_records_the_library_path_decision():
    from sglang_restomod_b200 import _lib, census

    lib = _lib.load()
    rows = ctypes.c_int32(0)
    parts = ctypes.c_int32(0)
    assert lib.b200_linear_path(1, 25600, 5120, ctypes.byref(rows), ctypes.byref(parts)) == \
        _lib.PATH_STREAM and rows.value == 8
    assert lib.b200_linear_path(64, 1024, 5120, ctypes.byref(rows), ctypes.byref(parts)) == \
        _lib.PATH_TCGEN05 and parts.value > 1
    assert lib.b200_moe_path(0, 8, 100, ctypes.byref(rows)) == _lib.PATH_STREAM and rows.value == 8
    assert lib.b200_moe_path(0, 64, 100, ctypes.byref(rows)) == _lib.PATH_TCGEN05
    census.reset()
    census.enable(True)
    try:
        census.note_linear("linear", 4, 25600, 5120)
        census.note_linear("linear", 4, 25600, 5120)
        census.note_moe("moe_layer", 0, 128, 1024, 256, 8, 200, 4096, 7168)
        line = census.report()
    finally:
        census.enable(False)
        census.reset()
    assert "linear stream/8rows m=4 n=25600 k=5120 x2" in line
    assert "moe_layer stream/8rows q=0 tokens=128 routes/expert=4.0 block=8" in line
    census.note_linear("linear", 4, 25600, 5120)  # disabled: nothing recorded
    assert census.tally() == {}


def test_profile_window_wraps_forward_once(monkeypatch, tmp_path):
    from sglang_restomod_b200 import census

    class FakeProfile:
        def __init__(self, activities):
            self.entered = False

        def __enter__(self):
            self.entered = True

        def __exit__(self, *a):
            pass

        def key_averages(self):
            return type("T", (), {"table": lambda self, **kw: "kernel table"})()

    monkeypatch.setattr(torch.profiler, "profile", FakeProfile)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda: None)
    out = tmp_path / "prof.txt"
    monkeypatch.setenv(census.ENV_PROFILE, "2")
    monkeypatch.setenv(census.ENV_PROFILE_OUT, str(out))

    class Runner:
        calls = 0

        def forward(self, x):
            Runner.calls += 1
            return x + 1

    assert census.install_profile(Runner)
    assert not census.install_profile(Runner)  # already wrapped
    r = Runner()
    for i in range(3):
        assert r.forward(i) == i + 1
        assert out.exists() == (i == 2)  # forwards 1 and 2 profiled, written after the second
    assert out.read_text() == "kernel table"
    monkeypatch.setenv(census.ENV_PROFILE, "zero")
    assert not census.install_profile(Runner)
