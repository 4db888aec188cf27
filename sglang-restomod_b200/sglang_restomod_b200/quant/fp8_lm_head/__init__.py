"""Block-FP8 LM head on B200 (the ``fp8_lm_head`` component).

After the model loads, the ``[vocab, hidden]`` head is quantized to block FP8
with the reference's rule (``quant/sm70_fp8_lm_head/__init__.py:33-41``:
scale = block amax / 448 clamped to 1e-8, computed in the weight's dtype) and
served by the dense B200 GEMV - the (5120, 152064) configuration of the
benchmark definition streams at over 90% of HBM bandwidth.
"""

from __future__ import annotations

import logging

from ... import attest

logger = logging.getLogger(__name__)

BLOCK = 128


def _quantize(weight):
    """(e4m3 [N, K], fp32 scale [N/128, K/128]); runs on the weight's device."""
    import torch

    n, k = weight.shape
    if n % BLOCK or k % BLOCK:
        raise ValueError(f"lm_head shape {tuple(weight.shape)} is not a multiple of {BLOCK}")
    wb = weight.view(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    scale = (wb.abs().amax(dim=(1, 3)) / 448.0).clamp(min=1e-8)
    q = (wb / scale[:, None, :, None]).to(torch.float8_e4m3fn).view(n, k)
    return q.contiguous(), scale.to(torch.float32).contiguous()


def quantize_lm_head(model) -> bool:
    """Quantize ``model.lm_head`` in place for the B200 GEMV; True when converted."""
    import torch

    from ..fp8_dense import prepare_b200_fp8_linear

    head = getattr(model, "lm_head", None)
    if head is None or not hasattr(head, "weight"):
        return False
    weight = head.weight.data
    if weight.dim() != 2 or weight.dtype not in (torch.float16, torch.bfloat16):
        return False
    q, scale = _quantize(weight.to(torch.float16))
    holder = type("HeadWeights", (), {})()
    holder.weight = q
    holder.weight_scale_inv = scale
    prepare_b200_fp8_linear(holder)
    for name in ("b200_fp8_packed", "b200_fp8_scales", "b200_fp8_in_features",
                 "b200_fp8_out_features", "b200_fp8_gated"):
        setattr(head, name, getattr(holder, name))
    head.weight = torch.nn.Parameter(torch.empty(0, dtype=weight.dtype, device=weight.device),
                                     requires_grad=False)
    logger.info("b200 fp8_lm_head: quantized %d x %d", q.shape[0], q.shape[1])
    return True


def install() -> bool:
    from ..._common import is_b200, library_loadable

    if not is_b200() or not library_loadable():
        attest.inactive("fp8_lm_head", "no B200 or libb200moe.so not loadable")
        return False
    from sglang.srt.model_executor.model_runner import ModelRunner

    original = ModelRunner.load_model
    if getattr(original, "_b200_fp8_lm_head", False):
        return False

    def load_model(self):
        result = original(self)
        try:
            quantize_lm_head(self.model)
        except Exception as exc:  # noqa: BLE001 - a slow head beats a dead server
            logger.warning("b200 fp8_lm_head: skipped (%s)", exc)
        return result

    load_model._b200_fp8_lm_head = True
    ModelRunner.load_model = load_model
    return True


def register() -> None:
    install()
