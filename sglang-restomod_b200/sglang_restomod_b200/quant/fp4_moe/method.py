"""NVFP4 MoE on B200 through the upstream Marlin-MoE hooks.

Replaces the same three upstream hooks as the reference
(``sglang_restomod/quant/sm70_fp4_moe/method.py:290-764``):

1. ``prepare_moe_nvfp4_layer_for_marlin`` -> :func:`prepare_moe_nvfp4`: the
   ModelOpt checkpoint (``[E, N, K/2]`` uint8, ``[E, N, K/16]`` E4M3 group
   scales, fp32 ``weight_scale_2``) is re-laid into the library's streamed
   units with the group scales inline; the global scale stays raw fp32 (the
   kernel rounds ``e4m3 * global`` to fp16 once, as the reference's QPN2 path
   does).
2. ``moe_wna16_marlin_gemm`` -> :func:`moe_wna16_marlin_gemm`: same 28
   arguments and routing semantics (route ``token * top_k + slot``,
   activation row ``route / top_k``, output row ``route``, optional
   ``mul_topk_weights``), on the B200 kernel. The gate/up call writes
   ``[gate | up]`` as upstream's SiLU-and-mul expects.
3. ``sgl_kernel.moe_sum_reduce`` is supplied when the installed build lacks
   it (:mod:`sglang_restomod_b200.moe.sum_reduce`).
"""

from __future__ import annotations

import logging

from ... import attest
from ..._common import is_b200, library_loadable, mode

logger = logging.getLogger(__name__)

ENV_MODE = "SGLANG_B200_FP4_MOE"
_SUPPORTED_BLOCKS = (8, 16, 32, 64)
_MARK = "_b200_nvfp4"


def check_expert_shape(size_n: int, size_k: int) -> None:
    """Reject an expert shard the kernel cannot cover (reachable without a GPU)."""
    if size_k % 128 or size_n % 128:
        raise RuntimeError(
            f"B200 NVFP4 MoE needs K and N multiples of 128, got N={size_n} K={size_k}"
        )


def _ep_size():
    try:
        from sglang.srt.runtime_context import get_parallel

        return int(get_parallel().moe_ep_size)
    except Exception:  # noqa: BLE001 - an unpublished context is not an error
        return None


def _rebind(layer, name, tensor):
    import torch

    try:
        from sglang.srt.layers.utils import copy_or_rebind_param

        copy_or_rebind_param(layer, name, tensor)
    except Exception:  # noqa: BLE001 - outside SGLang: plain attribute
        setattr(layer, name, torch.nn.Parameter(tensor, requires_grad=False))


def _global_scale(scales_2, what):
    import torch

    if scales_2.ndim == 2:
        if not torch.equal(scales_2[:, 0], scales_2[:, 1]):
            raise RuntimeError(f"Unequal NVFP4 gate/up global scales are unsupported ({what})")
        scales_2 = scales_2[:, 0]
    return scales_2.to(torch.float32).contiguous()


def prepare_moe_nvfp4(layer, group_size: int | None = None) -> None:
    """Replace the ModelOpt expert layout with the B200 streamed layout."""
    import torch

    from ..._common import b200_ops

    if getattr(layer, "params_dtype", torch.bfloat16) not in (torch.bfloat16, torch.float16):
        raise RuntimeError(f"B200 NVFP4 MoE needs bf16 or fp16 activations, got {layer.params_dtype}")
    ep = _ep_size()
    if ep is not None and ep != 1:
        raise RuntimeError(
            "B200 NVFP4 Marlin-hook path does not support expert parallelism; launch with "
            f"--ep-size 1 (got moe_ep_size={ep})"
        )
    if hasattr(layer, "moe_runner_config") and not layer.moe_runner_config.is_gated:
        raise RuntimeError("The B200 NVFP4 path requires gated MoE experts")
    if group_size is None:
        group_size = getattr(getattr(layer, "quant_config", None), "group_size", 16)
    if group_size != 16:
        raise RuntimeError(f"B200 NVFP4 MoE requires group_size=16, got {group_size}")
    if any(getattr(layer, n, None) is not None for n in ("w13_bias", "w2_bias")):
        raise RuntimeError("The B200 NVFP4 path does not support expert bias")

    for prefix, gated in (("w13", True), ("w2", False)):
        weight = getattr(layer, prefix + "_weight")
        scales = getattr(layer, prefix + "_weight_scale")
        if weight.dtype != torch.uint8 or weight.ndim != 3:
            raise RuntimeError(f"{prefix}: expected a packed [E, N, K/2] uint8 weight, got "
                               f"{tuple(weight.shape)} {weight.dtype}")
        experts, size_n, half_k = (int(d) for d in weight.shape)
        check_expert_shape(size_n, 2 * half_k)
        gs = _global_scale(getattr(layer, prefix + "_weight_scale_2"), prefix)
        packed = b200_ops().nvfp4_prepack(weight.data.contiguous(), scales.data.contiguous(), gated=gated)
        setattr(packed, _MARK, {"gated": gated, "n": size_n, "k": 2 * half_k, "experts": experts})
        _rebind(layer, prefix + "_weight", packed)
        getattr(layer, prefix + "_weight").__dict__[_MARK] = {
            "gated": gated, "n": size_n, "k": 2 * half_k, "experts": experts}
        # The scales now live inside the bank.
        _rebind(layer, prefix + "_weight_scale", torch.empty(0, dtype=scales.dtype, device=scales.device))
        _rebind(layer, prefix + "_weight_scale_2", gs)
        swizzled = prefix + "_blockscale_swizzled"
        if hasattr(layer, swizzled):
            setattr(layer, swizzled, None)


def _layout(b_q_weight):
    info = getattr(b_q_weight, _MARK, None)
    if info is None:
        info = getattr(b_q_weight, "__dict__", {}).get(_MARK)
    return info


def _regroup(sorted_token_ids, expert_ids, num_tokens_post_padded, block: int, sentinel: int):
    """Re-express align blocks of an unsupported size as blocks the kernel
    takes: each block of ``block`` slots becomes ceil(block/64) (or one padded)
    block(s) of a supported size, on the device (graph-safe)."""
    import torch

    target = next((b for b in _SUPPORTED_BLOCKS if b >= block), 64)
    per = -(-block // target)  # new blocks per old block
    nb = expert_ids.numel()
    flat = sorted_token_ids.reshape(-1)
    if flat.numel() < nb * block:
        flat = torch.cat([flat, torch.full((nb * block - flat.numel(),), sentinel,
                                           dtype=flat.dtype, device=flat.device)])
    slots = flat[: nb * block].view(nb, block)
    padded = torch.full((nb, per * target), sentinel, dtype=slots.dtype, device=slots.device)
    padded[:, :block] = slots
    new_sorted = padded.reshape(-1).contiguous()
    new_experts = expert_ids.repeat_interleave(per).contiguous()
    new_ntpp = (num_tokens_post_padded // block * per * target).to(torch.int32).contiguous()
    return new_sorted, new_experts, new_ntpp, target


def moe_wna16_marlin_gemm(
    a, c_or_none, b_q_weight, b_bias_or_none, b_scales, global_scale_or_none, b_zeros_or_none,
    g_idx_or_none, perm_or_none, workspace, sorted_token_ids, expert_ids,
    num_tokens_post_padded, topk_weights, moe_block_size, top_k, mul_topk_weights, is_ep,
    b_q_type, size_m, size_n, size_k, is_k_full=True, use_atomic_add=False,
    use_fp32_reduce=False, is_zp_float=False, expert_ids_are_sorted=False,
    zero_inactive_output=False, has_inactive_prefix_count=False,
):
    """Upstream's Marlin-MoE GEMM signature, served by the B200 NVFP4 kernel.

    ``workspace``, the launch hints and the sortedness hints are accepted and
    not needed (the B200 kernel uses its own zeroed workspace).
    """
    import torch

    from ... import _lib
    from ..._common import b200_ops

    if is_ep:
        raise RuntimeError(
            "B200 NVFP4 Marlin-hook path does not support expert parallelism; launch with --ep-size 1"
        )
    info = _layout(b_q_weight)
    if info is None:
        raise RuntimeError(
            "moe_wna16_marlin_gemm got a weight that prepare_moe_nvfp4 did not prepare for B200"
        )
    if any(t is not None for t in (b_bias_or_none, b_zeros_or_none, g_idx_or_none, perm_or_none)):
        raise RuntimeError("B200 NVFP4 MoE does not support bias, zero points, g_idx or perm")
    if global_scale_or_none is None:
        raise RuntimeError("B200 NVFP4 MoE needs the per-expert global scale")
    if info["n"] != size_n or info["k"] != size_k:
        raise RuntimeError(
            f"B200 NVFP4 MoE: size_n/size_k {size_n}/{size_k} disagree with the prepared bank "
            f"{info['n']}/{info['k']}"
        )
    routes = int(size_m) * int(top_k)
    if c_or_none is None:
        c = torch.zeros((routes, size_n), dtype=a.dtype, device=a.device)
    else:
        c = c_or_none
        if zero_inactive_output:
            c.zero_()
    sorted_ids = sorted_token_ids
    e_ids = expert_ids
    ntpp = num_tokens_post_padded
    block = int(moe_block_size)
    if block not in _SUPPORTED_BLOCKS:
        sorted_ids, e_ids, ntpp, block = _regroup(sorted_ids, e_ids, ntpp, block, routes)
    gated_mode = _lib.GATED_SPLIT if info["gated"] else _lib.GATED_NONE
    b200_ops().moe_gemm(a.contiguous(), b_q_weight, size_n, quant=_lib.QUANT_NVFP4,
                 num_experts=info["experts"], sorted_token_ids=sorted_ids.contiguous(),
                 expert_ids=e_ids.contiguous(), num_tokens_post_pad=ntpp.contiguous(),
                 block_size=block, top_k=int(top_k), num_routes=routes, c=c,
                 global_scale=global_scale_or_none.float().contiguous(),
                 topk_weights=topk_weights.reshape(-1).float().contiguous()
                 if topk_weights is not None else None,
                 mul_topk_weights=bool(mul_topk_weights), gated_mode=gated_mode)
    return c


_INSTALLED = False
_ORIGINALS: dict[str, object] = {}


def _patch(module, name, replacement) -> bool:
    original = getattr(module, name, None)
    if original is None:
        logger.warning("B200 NVFP4 MoE: %s.%s not found; the hook did not bind", module.__name__, name)
        return False
    _ORIGINALS[f"{module.__name__}.{name}"] = original
    setattr(module, name, replacement)
    return True


def install() -> bool:
    """Install the NVFP4 hooks; refuse at weight-load time when they cannot work."""
    global _INSTALLED
    if _INSTALLED:
        return True
    m = mode(ENV_MODE)
    if m == "off":
        return False
    if not is_b200():
        if m == "on":
            raise RuntimeError(f"{ENV_MODE}=on requires a B200 (sm_100) device")
        attest.inactive("fp4_moe", "not a B200 device")
        return False
    from sglang.srt.layers.quantization import marlin_utils_fp4, modelopt_quant

    if not library_loadable():
        def _refuse(*_a, **_k):
            raise RuntimeError(f"{ENV_MODE}={m} needs libb200moe.so; it cannot be loaded. "
                               f"Set {ENV_MODE}=off to disable the layer.")

        _patch(marlin_utils_fp4, "prepare_moe_nvfp4_layer_for_marlin", _refuse)
        _patch(modelopt_quant, "prepare_moe_nvfp4_layer_for_marlin", _refuse)
        attest.inactive("fp4_moe", "libb200moe.so cannot be loaded; weight loading will refuse")
        return False
    from ...moe import sum_reduce

    sum_reduce.install()
    from sglang.kernels.ops.moe import moe_wna16_marlin

    bound = {
        "marlin_utils_fp4.prepare_moe_nvfp4_layer_for_marlin":
            _patch(marlin_utils_fp4, "prepare_moe_nvfp4_layer_for_marlin", prepare_moe_nvfp4),
        "modelopt_quant.prepare_moe_nvfp4_layer_for_marlin":
            _patch(modelopt_quant, "prepare_moe_nvfp4_layer_for_marlin", prepare_moe_nvfp4),
        "moe_wna16_marlin.moe_wna16_marlin_gemm":
            _patch(moe_wna16_marlin, "moe_wna16_marlin_gemm", moe_wna16_marlin_gemm),
    }
    missing = sorted(k for k, ok in bound.items() if not ok)
    if missing:
        names = ", ".join(missing)

        def _refuse_binding(*_a, **_k):
            raise RuntimeError(f"B200 NVFP4 MoE: hook(s) did not bind: {names}")

        for module in (marlin_utils_fp4, modelopt_quant):
            _patch(module, "prepare_moe_nvfp4_layer_for_marlin", _refuse_binding)
        attest.inactive("fp4_moe", f"hook(s) did not bind: {names}")
        return False
    try:
        from sglang.srt.layers.moe.fused_moe_triton import fused_marlin_moe

        _patch(fused_marlin_moe, "moe_wna16_marlin_gemm", moe_wna16_marlin_gemm)
    except ImportError:
        pass
    _INSTALLED = True
    return True


def uninstall() -> None:
    global _INSTALLED
    import importlib

    for key, original in list(_ORIGINALS.items()):
        module_name, attr = key.rsplit(".", 1)
        setattr(importlib.import_module(module_name), attr, original)
    _ORIGINALS.clear()
    _INSTALLED = False
