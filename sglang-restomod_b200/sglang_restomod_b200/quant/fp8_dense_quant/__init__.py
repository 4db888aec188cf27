"""Post-load block-FP8 quantization of bf16/fp16 dense linears (the
``fp8_dense_quant`` component; reference ``quant/sm70_fp8_dense_quant``).

A checkpoint that ships its dense projections in bf16 reads two bytes per
weight on every decode step; the B200 GEMV reads one byte plus a scale per
128x128 block. After ``ModelRunner.load_model`` returns, every admitted
linear is quantized with the LM-head rule (``scale = clamp(amax / 448,
1e-8)`` per 128x128 block, ``quant/sm70_fp8_lm_head/__init__.py:33-41``),
prepacked, and from then on served by ``b200_linear``.

Admission (:func:`refusal` returns None) follows the reference's rule set
(``quant/sm70_fp8_dense_quant/__init__.py:58-80``): a 2-D bf16/fp16 weight,
both sides multiples of 128, a plain ``nn.Linear`` or an engine linear whose
quantization method is the unquantized one, not an expert bank, not the LM
head (it has its own component) and not a ``ReplicatedLinear`` (the MoE
router). Everything else keeps its path. A layer whose conversion raises
keeps its original weights and is counted as failed; the server still
starts.
"""

from __future__ import annotations

import logging
import os
from collections import Counter

from ... import attest

logger = logging.getLogger(__name__)

BLOCK = 128
EXPERT_NAME_PART = "experts"
LM_HEAD_SUFFIX = "lm_head"
ROUTER_TYPE = "ReplicatedLinear"
ENV_DETAILS = "SGLANG_B200_FP8_DENSE_QUANT_DETAILS"
_HOOK_MARK = "_b200_fp8_dense_quant"


def _engine_linear_base():
    try:
        from sglang.srt.layers.linear import LinearBase
    except Exception:  # noqa: BLE001 - no engine: only duck-typed linears qualify
        return None
    return LinearBase


def _is_engine_linear(module) -> bool:
    base = _engine_linear_base()
    if base is not None and isinstance(module, base):
        return True
    return hasattr(module, "quant_method") and hasattr(module, "input_size_per_partition")


def refusal(name: str, module) -> str | None:
    """Why ``module`` is not converted, or None when it is admitted."""
    import torch

    if not name:
        return "unnamed"
    if EXPERT_NAME_PART in name:
        return "expert"
    if name.endswith(LM_HEAD_SUFFIX):
        return "lm_head"
    if type(module).__name__ == ROUTER_TYPE:
        return "router"
    weight = getattr(module, "weight", None)
    if not isinstance(weight, torch.Tensor) or weight.dim() != 2:
        return "no-2d-weight"
    if weight.dtype not in (torch.bfloat16, torch.float16):
        return "dtype"
    if getattr(module, "b200_fp8_packed", None) is not None:
        return "converted"
    engine = _is_engine_linear(module)
    if not engine and not isinstance(module, torch.nn.Linear):
        return "not-a-linear"
    if engine and "Unquantized" not in type(getattr(module, "quant_method", None)).__name__:
        return "quantized:" + type(module.quant_method).__name__
    n, k = weight.shape
    if n % BLOCK or k % BLOCK:
        return f"shape:{n}x{k}"
    return None


class B200DenseFp8Method:
    """Quantization method of a converted engine linear: serve it on the GEMV."""

    def process_weights_after_loading(self, layer) -> None:  # already prepacked
        return None

    def apply(self, layer, x, bias=None):
        from ..fp8_dense import apply_b200_fp8_linear

        return apply_b200_fp8_linear(layer, x, bias)


def _linear_forward(self, x):
    from ..fp8_dense import apply_b200_fp8_linear

    return apply_b200_fp8_linear(self, x, self.bias)


def convert(module) -> None:
    """Quantize an admitted module's weight in place and route its forward to
    the B200 GEMV; raises (leaving the module as it was) on failure."""
    import torch

    from ..fp8_dense import prepare_b200_fp8_linear
    from ..fp8_lm_head import _quantize

    weight = module.weight
    q, scale = _quantize(weight.data.to(torch.float16))
    holder = type("DenseWeights", (), {})()
    holder.weight, holder.weight_scale_inv = q, scale
    prepare_b200_fp8_linear(holder)
    # nothing on the module changes until every step above succeeded
    for attr in ("b200_fp8_packed", "b200_fp8_scales", "b200_fp8_in_features",
                 "b200_fp8_out_features", "b200_fp8_gated"):
        setattr(module, attr, getattr(holder, attr))
    module.weight = torch.nn.Parameter(torch.empty(0, dtype=weight.dtype, device=weight.device),
                                       requires_grad=False)
    if _is_engine_linear(module):
        module.quant_method = B200DenseFp8Method()
    else:
        module.forward = _linear_forward.__get__(module, type(module))


def quantize_dense_linears(model) -> Counter:
    """Convert every admitted linear of ``model``. Returns a count per
    outcome: ``converted``, ``failed`` and one key per refusal reason."""
    outcome: Counter = Counter()
    details = os.environ.get(ENV_DETAILS, "").strip().lower() in ("1", "true", "on", "yes")
    for name, module in list(model.named_modules()):
        if not hasattr(module, "weight"):
            continue
        reason = refusal(name, module)
        if reason is None:
            try:
                convert(module)
                reason = "converted"
            except Exception as exc:  # noqa: BLE001 - one layer must not stop the rest
                reason = "failed"
                logger.warning("b200 fp8_dense_quant: %s keeps its weights (%s)", name, exc)
        outcome[reason] += 1
        if details:
            logger.info("b200 fp8_dense_quant: %s %s", name, reason)
    return outcome


def hook_load_model(runner_cls, convert_all=quantize_dense_linears) -> bool:
    """Wrap ``runner_cls.load_model`` so the model's dense linears are
    converted once the weights are in. False when already wrapped."""
    original = runner_cls.load_model
    if getattr(original, _HOOK_MARK, False):
        return False

    def load_model(self, *args, **kwargs):
        result = original(self, *args, **kwargs)
        try:
            outcome = convert_all(self.model)
            logger.info("b200 fp8_dense_quant: %s", dict(outcome))
        except Exception as exc:  # noqa: BLE001 - a bf16 server beats a dead one
            logger.warning("b200 fp8_dense_quant: skipped (%s)", exc)
        return result

    setattr(load_model, _HOOK_MARK, True)
    runner_cls.load_model = load_model
    return True


def apply(module, x, bias=None):
    from ..fp8_dense import apply_b200_fp8_linear

    return apply_b200_fp8_linear(module, x, bias)


def install() -> bool:
    from ..._common import is_b200, library_loadable

    if not is_b200() or not library_loadable():
        attest.inactive("fp8_dense_quant", "no B200 or libb200moe.so not loadable")
        return False
    try:
        from sglang.srt.model_executor.model_runner import ModelRunner
    except Exception as exc:  # noqa: BLE001
        attest.inactive("fp8_dense_quant", f"ModelRunner not importable: {exc}")
        return False
    return hook_load_model(ModelRunner)


def register() -> None:
    install()
