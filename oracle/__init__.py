"""CPU oracle for the quantized MoE / decode-GEMM path. TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the sglang-restomod
reference for the path the B200 library implements. It exists to check the
CUDA kernels; it is never the thing measured and never a fallback:

* only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
  ``--impl reference`` legs of ``bench.py`` may import it;
* the product package (``sglang_restomod_b200``) never imports it.

Every function cites the reference file:line it restates (paths inside the
sglang-restomod tree). The restatement is pinned against golden vectors made
by running the reference's own CPU code (``tests/golden/make_golden.py``,
checked by ``tests/test_oracle_golden.py``):

* block-FP8 quantize / dequantize / dense MoE reference
  (``quant/sm70_fp8_moe/check.py:18-48``), the LM-head quantizer
  (``quant/sm70_fp8_lm_head/__init__.py:33-41``);
* the FP8 method's sort / gather / EP-drop / combine semantics, by running
  ``SM70Fp8MoEMethod.apply`` (``quant/sm70_fp8_moe/method.py:239-309``) on the
  CPU with the GEMM contract of ``quant/sm70_fp8_moe/README.md:23-58``;
* NVFP4 quantize / dequantize (``quant/sm70_fp4_moe/check.py:31-64``) and the
  scale byte encoder (``quant/sm70_fp4_moe/scales.py:20-56``) with the golden
  table of ``tests/test_sm70_fp4_scales.py:33-42``.

``moe_align_block_size`` lives upstream (sgl_kernel, not in the reference
tree); its restatement here is pinned to the reference's own stable
expert-major order (``method.py:285``) through the method fixture, and is
otherwise "parity unpinned" against upstream's kernel. The router
(softmax / sigmoid top-k) is upstream too: its restatement follows the
benchmark's definition (softmax -> top-k -> renormalise) and is parity
unpinned against upstream's fused top-k kernel.
"""

from .align import moe_align_block_size
from .fp8 import (
    dequant_block_fp8,
    fp8_linear_ref,
    quant_block_fp8,
    quant_block_fp8_lm_head,
)
from .moe import (
    fp8_moe_method_ref,
    moe_gemm_ref,
    moe_layer_ref,
    moe_sum_reduce_ref,
)
from .nvfp4 import (
    E2M1_GRID,
    dequant_nvfp4,
    encode_global_scale,
    encode_scales,
    nvfp4_linear_ref,
    quantize_nvfp4,
)
from .router import route_topk, route_topk_general, route_topk_grouped
from .w8a8 import act_dequant_fp8, act_quant_fp8, quantized_activations, w8a8_linear_ref

__all__ = [
    "act_dequant_fp8",
    "act_quant_fp8",
    "quantized_activations",
    "w8a8_linear_ref",
    "E2M1_GRID",
    "dequant_block_fp8",
    "dequant_nvfp4",
    "encode_global_scale",
    "encode_scales",
    "fp8_linear_ref",
    "fp8_moe_method_ref",
    "moe_align_block_size",
    "moe_gemm_ref",
    "moe_layer_ref",
    "moe_sum_reduce_ref",
    "nvfp4_linear_ref",
    "quant_block_fp8",
    "quant_block_fp8_lm_head",
    "quantize_nvfp4",
    "route_topk",
    "route_topk_general",
    "route_topk_grouped",
]
