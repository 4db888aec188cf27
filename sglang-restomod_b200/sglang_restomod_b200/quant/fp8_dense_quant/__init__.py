"""Post-load block-FP8 quantization of bf16/fp16 dense linears (the
``fp8_dense_quant`` component; reference ``quant/sm70_fp8_dense_quant``).

:func:`convert` quantizes one linear's weight with the LM-head rule and
prepacks it for the B200 GEMV; :func:`apply` then serves it.
"""

from __future__ import annotations

from ... import attest


def convert(module) -> bool:
    """Quantize ``module.weight`` ([N, K] bf16/fp16) in place; True when done."""
    import torch

    from ..fp8_dense import _check_dense_weight_shape, prepare_b200_fp8_linear
    from ..fp8_lm_head import _quantize

    weight = getattr(module, "weight", None)
    if weight is None or weight.dim() != 2 or weight.dtype not in (torch.float16, torch.bfloat16):
        return False
    n, k = weight.shape
    try:
        _check_dense_weight_shape(int(n), int(k))
    except RuntimeError:
        return False
    q, scale = _quantize(weight.data.to(torch.float16))
    holder = type("W", (), {})()
    holder.weight, holder.weight_scale_inv = q, scale
    prepare_b200_fp8_linear(holder)
    for name in ("b200_fp8_packed", "b200_fp8_scales", "b200_fp8_in_features",
                 "b200_fp8_out_features", "b200_fp8_gated"):
        setattr(module, name, getattr(holder, name))
    return True


def apply(module, x, bias=None):
    from ..fp8_dense import apply_b200_fp8_linear

    return apply_b200_fp8_linear(module, x, bias)


def register() -> None:
    attest.inactive("fp8_dense_quant", "conversion is explicit: call convert(module) after load")
