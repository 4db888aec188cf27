"""``moe_sum_reduce`` on the B200 kernel.

Same contract as the reference's Triton replacement for the op missing from
``sgl_kernel`` (``sglang_restomod/quant/sm70_fp4_moe/sum_reduce.py:84-123``):
``output[t] = routed_scaling_factor * sum_k input[t, k]`` in fp32, stored in
the input dtype. Non-contiguous tensors are refused rather than silently
taking another path.
"""

from __future__ import annotations

import logging

logger = logging.getLogger(__name__)


def moe_sum_reduce(input_tensor, output_tensor, routed_scaling_factor=1.0):
    from .._common import b200_ops

    b200_ops().moe_sum_reduce(input_tensor, output_tensor, float(routed_scaling_factor))
    return output_tensor


def install() -> bool:
    """Bind the replacement wherever the installed sgl_kernel lacks the op,
    including modules that imported the name before this ran."""
    from .._common import rebind_everywhere

    try:
        import sgl_kernel
        import sgl_kernel.moe as sgl_moe
    except ImportError:
        return False
    original = getattr(sgl_moe, "moe_sum_reduce", None)
    sgl_kernel.moe_sum_reduce = moe_sum_reduce
    sgl_moe.moe_sum_reduce = moe_sum_reduce
    if original is not None:
        rebind_everywhere("moe_sum_reduce", original, moe_sum_reduce)
    return True
