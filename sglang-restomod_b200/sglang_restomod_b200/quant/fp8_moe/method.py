"""B200 block-FP8 fused-MoE method.

Replaces ``Fp8MoEMethod`` for ``[128, 128]`` block-FP8 ``FusedMoE`` layers, as
``SM70Fp8MoEMethod`` does on V100 (``sglang_restomod/quant/sm70_fp8_moe/
method.py:69-309``). ``apply`` is a single library call
(``b200_moe_layer_forward``): moe_align -> gate/up GEMM with the SiLU*up
epilogue -> down GEMM times the router weight -> top-k combine, times the
routed scaling factor. Under expert parallelism the dispatcher has mapped
global ids to local ones and marked foreign routes -1; those routes are
dropped inside the align kernel, so neither the reference's compaction (with
its host read) nor its clamp-onto-expert-0 is needed, and every shape stays
static for CUDA-graph capture.
"""

from __future__ import annotations

import logging

from ... import attest
from ..._common import combine_input, is_b200, library_loadable, mode

logger = logging.getLogger(__name__)

ENV_MODE = "SGLANG_B200_FP8_MOE"

try:  # the SGLang base class when the engine is importable
    from sglang.srt.layers.quantization.fp8 import Fp8MoEMethod as _Base
except Exception:  # noqa: BLE001 - host logic stays testable without SGLang
    _Base = object


class B200Fp8MoEMethod(_Base):
    """Block-FP8 experts on the B200 streaming kernels."""

    def __init__(self, quant_config=None):
        if _Base is not object:
            super().__init__(quant_config)
        self.quant_config = quant_config
        self.ready = False
        self.output_scale = 1.0

    @staticmethod
    def _unsupported_reason(cfg) -> str | None:
        """Configurations the fused epilogue does not cover (the checks of
        ``quant/sm70_fp8_moe/method.py:84-103``)."""
        if cfg.activation != "silu" or not cfg.is_gated:
            return f"activation={cfg.activation} is_gated={cfg.is_gated}"
        if getattr(cfg, "swiglu_limit", None) is not None or getattr(cfg, "gemm1_clamp_limit", None) is not None:
            return "clamped SwiGLU"
        if getattr(cfg, "gemm1_alpha", None) is not None or getattr(cfg, "gemm1_beta", None) is not None:
            return "SwiGLU alpha/beta"
        if getattr(cfg, "apply_router_weight_on_input", False) or getattr(cfg, "no_combine", False):
            return "router weight on input or no combine"
        if getattr(cfg, "wide_output_scale", 1.0) != 1.0 or getattr(cfg, "gate_up_input_scale", 1.0) != 1.0:
            return "FP8 range scaling"
        return None

    def process_weights_after_loading(self, layer) -> None:
        import torch

        from ... import _lib
        from ..._common import b200_ops
        from ...layer import QuantMoELayer
        from . import _check_gemm_shape

        cfg = self.moe_runner_config
        reason = self._unsupported_reason(cfg)
        if reason is not None:
            raise RuntimeError(f"B200 FP8 MoE does not support {reason}")
        w13, w2 = layer.w13_weight, layer.w2_weight
        s13 = getattr(layer, "w13_weight_scale_inv", None)
        s2 = getattr(layer, "w2_weight_scale_inv", None)
        if w13 is None or w2 is None or s13 is None or s2 is None:
            raise RuntimeError("FP8 MoE weights or scales are missing")
        experts, n13, hidden = (int(d) for d in w13.shape)
        inter = n13 // 2
        if n13 % 256 or hidden % 128 or inter % 128:
            raise RuntimeError(
                "block-128 FP8 MoE needs hidden and per-expert intermediate multiples of 128, "
                f"got {hidden}/{inter}"
            )
        _check_gemm_shape(hidden, n13, gated=True)
        _check_gemm_shape(inter, hidden)
        packed13 = b200_ops().fp8_prepack(w13.data.contiguous(), gated=True)
        packed2 = b200_ops().fp8_prepack(w2.data.contiguous(), gated=False)
        scales13 = s13.data.float().contiguous()
        scales2 = s2.data.float().contiguous()
        # Release the checkpoint layout through the parameters themselves (the
        # loader may hold the Parameter objects for the whole post-load pass).
        for param in (w13, w2, s13, s2):
            param.data = torch.empty(0, dtype=param.dtype, device=param.device)
        layer.w13_weight = None
        layer.w2_weight = None
        layer.w13_weight_scale_inv = None
        layer.w2_weight_scale_inv = None

        scale = getattr(cfg, "routed_scaling_factor", None)
        fuse = getattr(layer, "should_fuse_routed_scaling_factor_in_topk", False)
        self.output_scale = 1.0 if scale in (None, 1.0) or fuse else float(scale)
        layer.b200_moe = QuantMoELayer(
            quant=_lib.QUANT_FP8_BLOCK, hidden=hidden, inter=inter, num_experts=experts,
            top_k=int(cfg.top_k), w13=packed13, w2=packed2, w13_scales=scales13,
            w2_scales=scales2, routed_scaling_factor=self.output_scale,
        )
        self.ready = True
        logger.info("B200 FP8 MoE: experts=%d hidden=%d intermediate=%d topk=%d", experts,
                    hidden, inter, cfg.top_k)

    def apply(self, layer, dispatch_output):
        import torch

        if not self.ready:
            raise RuntimeError("B200 FP8 MoE was not prepared for this layer")
        x = dispatch_output.hidden_states
        topk = dispatch_output.topk_output
        moe = layer.b200_moe
        if x.shape[0] == 0:
            return combine_input(torch.zeros_like(x))
        ids = topk.topk_ids
        if ids.dtype != torch.int32:
            ids = ids.to(torch.int32)
        weights = topk.topk_weights
        if weights.dtype != torch.float32:
            weights = weights.float()
        out = moe.forward(x.contiguous(), ids.contiguous(), weights.contiguous())
        return combine_input(out)


_INSTALLED = False


def install() -> bool:
    """Route ``[128, 128]`` block-FP8 FusedMoE layers to :class:`B200Fp8MoEMethod`.

    ``SGLANG_B200_FP8_MOE=off`` keeps the upstream method; ``auto`` installs
    on a B200 with the library loadable; ``on`` requires both.
    """
    global _INSTALLED
    if _INSTALLED:
        return True
    m = mode(ENV_MODE)
    if m == "off":
        return False
    if not is_b200():
        if m == "on":
            raise RuntimeError(f"{ENV_MODE}=on requires a B200 (sm_100) device")
        attest.inactive("fp8_moe", "not a B200 device")
        return False
    if not library_loadable():
        if m == "on":
            raise RuntimeError(f"{ENV_MODE}=on but libb200moe.so cannot be loaded")
        attest.inactive("fp8_moe", "libb200moe.so cannot be loaded; the upstream method is in place")
        return False
    from sglang.srt.layers.moe.fused_moe_triton.layer import FusedMoE
    from sglang.srt.layers.quantization.fp8 import Fp8Config, Fp8MoEMethod

    original = Fp8Config.get_quant_method
    Fp8Config._b200_original_get_quant_method = original

    def get_quant_method(self, layer, prefix):
        method = original(self, layer, prefix)
        block = self.weight_block_size
        if (isinstance(layer, FusedMoE) and isinstance(method, Fp8MoEMethod)
                and block is not None and list(block) == [128, 128]):
            return B200Fp8MoEMethod(self)
        return method

    Fp8Config.get_quant_method = get_quant_method
    _INSTALLED = True
    return True


def uninstall() -> None:
    """Restore the upstream selection (tests)."""
    global _INSTALLED
    if not _INSTALLED:
        return
    from sglang.srt.layers.quantization.fp8 import Fp8Config

    original = getattr(Fp8Config, "_b200_original_get_quant_method", None)
    if original is not None:
        Fp8Config.get_quant_method = original
        del Fp8Config._b200_original_get_quant_method
    _INSTALLED = False
