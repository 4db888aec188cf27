"""moe_align_block_size on the B200 kernel (the ``moe_align_sm70`` component).

The reference only steers upstream's ``moe_align_block_size`` onto its CUDA
pair (``sglang_restomod/moe/align_sm70.py:35-55``). Here the op itself is the
library's single-kernel stable counting sort; :func:`register` points the
upstream module's function at it.
"""

from __future__ import annotations

import logging

from .. import attest
from .._common import is_b200, library_loadable

logger = logging.getLogger(__name__)


def moe_align_block_size(topk_ids, block_size: int, num_experts: int, expert_map=None,
                         pad_sorted_ids: bool = False):
    """(sorted_token_ids, expert_ids, num_tokens_post_pad), upstream's contract.

    Route ids outside ``[0, num_experts)`` are dropped. ``expert_map``
    (global -> local ids, -1 for foreign experts) is applied on the device
    first when given. ``pad_sorted_ids`` is accepted: the output is always
    padded to the worst case.
    """
    import torch

    from .._common import b200_ops

    ids = topk_ids
    if expert_map is not None:
        ids = expert_map[ids.long()]
    ids = ids.to(torch.int32).contiguous()
    return b200_ops().moe_align_block_size(ids, int(block_size), int(num_experts))


_ORIGINAL = None


def register() -> None:
    global _ORIGINAL
    if not is_b200():
        attest.inactive("moe_align_sm70", "not a B200 device")
        return
    if not library_loadable():
        attest.inactive("moe_align_sm70", "libb200moe.so cannot be loaded")
        return
    try:
        from sglang.srt.layers.moe.fused_moe_triton import moe_align_block_size as upstream
    except Exception as exc:  # noqa: BLE001
        attest.inactive("moe_align_sm70", f"upstream module not importable: {exc}")
        return
    if _ORIGINAL is None:
        from .._common import rebind_everywhere

        _ORIGINAL = upstream.moe_align_block_size
        upstream.moe_align_block_size = moe_align_block_size
        # modules that imported the function by name before this ran
        rebind_everywhere("moe_align_block_size", _ORIGINAL, moe_align_block_size)
