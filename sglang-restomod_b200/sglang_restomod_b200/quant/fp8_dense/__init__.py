"""Block-FP8 dense linear / decode GEMV on B200 (the ``fp8_dense`` component).

Replaces ``apply_sm70_turbomind_fp8_linear`` and its fused gate/up variant
(``sglang_restomod/quant/sm70_fp8_dense/_method.py:713-863``) behind
``Fp8LinearMethod``: W8A16 with ``[128, 128]`` block scales. After load the
weight is prepacked into the streamed layout; ``apply`` is one library call
for any M (up to 64 rows per weight pass). A gate/up projection prepared as
gated can also run with the fused SiLU*up epilogue
(:func:`apply_b200_fp8_fused_silu_and_mul`).
"""

from __future__ import annotations

import logging

from ... import attest
from ..._common import is_b200, library_loadable, mode

logger = logging.getLogger(__name__)

ENV_MODE = "SGLANG_B200_FP8_DENSE"
GROUP = 128


def _check_dense_weight_shape(n: int, k: int, group_size: int = GROUP, gated: bool = False) -> None:
    """Messages as in ``quant/sm70_fp8_dense/_method.py:64-80``."""
    if n <= 0 or k <= 0:
        raise RuntimeError(f"B200 FP8 dense needs positive N and K, got N={n} K={k}.")
    unit = 256 if gated else 128
    if n % unit:
        raise RuntimeError(f"B200 FP8 dense needs N a multiple of {unit}, got N={n}.")
    if k % group_size:
        raise RuntimeError(
            f"B200 FP8 dense needs K a multiple of the {group_size}-wide quantization group, got K={k}."
        )


def _check_activation_k(layer, x_2d) -> None:
    expected = getattr(layer, "b200_fp8_in_features", None)
    if expected is not None and x_2d.shape[-1] != expected:
        raise RuntimeError(
            "B200 FP8 dense: activation K disagrees with the prepared weight "
            f"(prepared K={expected}, got {x_2d.shape[-1]})."
        )


def prepare_b200_fp8_linear(layer, gated_silu: bool = False) -> None:
    """Prepack ``layer.weight`` ([N, K] e4m3, scales ``weight_scale_inv``)."""
    from ..._common import b200_ops

    w = layer.weight
    s = layer.weight_scale_inv
    n, k = (int(d) for d in w.shape)
    _check_dense_weight_shape(n, k, gated=gated_silu)
    if tuple(s.shape) != (n // GROUP, k // GROUP):
        raise RuntimeError(f"B200 FP8 dense scales must be [{n // GROUP}, {k // GROUP}], got {tuple(s.shape)}")
    layer.b200_fp8_packed = b200_ops().fp8_prepack(w.data.contiguous(), gated=gated_silu)
    layer.b200_fp8_scales = s.data.float().contiguous()
    layer.b200_fp8_in_features = k
    layer.b200_fp8_out_features = n
    layer.b200_fp8_gated = bool(gated_silu)


def apply_b200_fp8_linear(layer, x, bias=None):
    """``y = x . dequant(W)^T (+ bias)``; the ordinary linear contract (a gated
    bank still returns ``[gate | up]``)."""
    from ... import _lib
    from ..._common import b200_ops

    x_2d = x.reshape(-1, x.shape[-1])
    if x_2d.stride(-1) != 1 or not x_2d.is_contiguous():
        x_2d = x_2d.contiguous()
    _check_activation_k(layer, x_2d)
    n = layer.b200_fp8_out_features
    mode_ = _lib.GATED_SPLIT if layer.b200_fp8_gated else _lib.GATED_NONE
    out = b200_ops().linear(x_2d, layer.b200_fp8_packed, n, quant=_lib.QUANT_FP8_BLOCK,
                     scales=layer.b200_fp8_scales, gated_mode=mode_, out_dtype=x.dtype)
    if bias is not None:
        out.add_(bias)
    return out.reshape(*x.shape[:-1], n)


def apply_b200_fp8_fused_silu_and_mul(layer, x):
    """Gate/up projection and ``silu(gate) * up`` in one GEMM (None when the
    layer was not prepared gated)."""
    from ... import _lib
    from ..._common import b200_ops

    if not getattr(layer, "b200_fp8_gated", False):
        return None
    x_2d = x.reshape(-1, x.shape[-1]).contiguous()
    _check_activation_k(layer, x_2d)
    n = layer.b200_fp8_out_features
    out = b200_ops().linear(x_2d, layer.b200_fp8_packed, n, quant=_lib.QUANT_FP8_BLOCK,
                     scales=layer.b200_fp8_scales, gated_mode=_lib.GATED_FUSED, out_dtype=x.dtype)
    return out.reshape(*x.shape[:-1], n // 2)


def _is_block_fp8(method) -> bool:
    cfg = getattr(method, "quant_config", None)
    block = getattr(cfg, "weight_block_size", None)
    return block is not None and list(block) == [GROUP, GROUP]


_INSTALLED = False


def install() -> bool:
    """Hook ``Fp8LinearMethod`` (post-load prepack and apply) for block-FP8 layers."""
    global _INSTALLED
    if _INSTALLED:
        return True
    m = mode(ENV_MODE)
    if m == "off":
        return False
    if not is_b200() or not library_loadable():
        if m == "on":
            raise RuntimeError(f"{ENV_MODE}=on requires a B200 and a loadable libb200moe.so")
        attest.inactive("fp8_dense", "no B200 or libb200moe.so not loadable")
        return False
    from sglang.srt.layers.quantization.fp8 import Fp8LinearMethod

    original_pwal = Fp8LinearMethod.process_weights_after_loading
    original_apply = Fp8LinearMethod.apply

    def process_weights_after_loading(self, layer):
        original_pwal(self, layer)
        if _is_block_fp8(self):
            prepare_b200_fp8_linear(layer)

    def apply(self, layer, x, bias=None, *args, **kwargs):
        if getattr(layer, "b200_fp8_packed", None) is not None:
            return apply_b200_fp8_linear(layer, x, bias)
        return original_apply(self, layer, x, bias, *args, **kwargs)

    apply._b200 = True
    Fp8LinearMethod.process_weights_after_loading = process_weights_after_loading
    Fp8LinearMethod.apply = apply
    _INSTALLED = True
    return True


def register() -> None:
    install()
