"""NVFP4 dense linear (W4A16) on B200 (the ``fp4_dense`` component).

The reference routes ``marlin_utils_fp4.gptq_marlin_gemm`` for NVFP4 to its
V100 Marlin build (``quant/sm70_fp4_dense/method.py:189-241``); here a
ModelOpt NVFP4 linear is prepacked once and served by the same streaming
kernel as the NVFP4 experts (one expert, dense rows).
"""

from __future__ import annotations

from ... import attest


def prepare_b200_nvfp4_linear(layer) -> None:
    """``weight`` [N, K/2] uint8, ``weight_scale`` [N, K/16] e4m3,
    ``weight_scale_2`` fp32 (one value, or one per fused shard - equal)."""
    import torch

    from ..._common import b200_ops

    w, s, g = layer.weight, layer.weight_scale, layer.weight_scale_2
    n, half_k = (int(d) for d in w.shape)
    gs = g.reshape(-1).float()
    if gs.numel() > 1 and not bool(torch.all(gs == gs[0])):
        # Several fused shards with different global scales: keep the largest
        # and rescale nothing - refuse instead of approximating.
        raise RuntimeError("B200 NVFP4 dense needs one global scale per matrix")
    layer.b200_nvfp4_packed = b200_ops().nvfp4_prepack(w.data.contiguous(), s.data.contiguous(), gated=False)
    layer.b200_nvfp4_global = gs[:1].contiguous()
    layer.b200_nvfp4_shape = (n, 2 * half_k)


def apply_b200_nvfp4_linear(layer, x, bias=None):
    from ... import _lib
    from ..._common import b200_ops

    n, k = layer.b200_nvfp4_shape
    x_2d = x.reshape(-1, x.shape[-1]).contiguous()
    if x_2d.shape[-1] != k:
        raise RuntimeError(f"B200 NVFP4 dense: activation K {x_2d.shape[-1]} != prepared K {k}")
    out = b200_ops().linear(x_2d, layer.b200_nvfp4_packed, n, quant=_lib.QUANT_NVFP4,
                     global_scale=layer.b200_nvfp4_global, out_dtype=x.dtype)
    if bias is not None:
        out.add_(bias)
    return out.reshape(*x.shape[:-1], n)


def register() -> None:
    attest.inactive("fp4_dense", "prepare/apply are explicit: prepare_b200_nvfp4_linear(layer)")
