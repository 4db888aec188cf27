"""moe_align_block_size restated in numpy (test infrastructure only).

The op is upstream (sgl_kernel) and absent from the reference tree; the
reference pins the CUDA pair with ``sglang_restomod/moe/align_sm70.py:35-55``
and consumes its output in ``quant/sm70_fp4_moe/decode_gemv.py:226-260`` and
``csrc/decode_gemv_qpn2.cu:73-110``:

* ``sorted_token_ids`` holds route indices ``token * top_k + slot``; a padding
  slot holds the sentinel ``numel``;
* ``expert_ids[b]`` names the expert of block ``b``;
* ``num_tokens_post_pad`` is the padded total.

Within an expert, routes keep their index order: the stable expert-major
order of ``torch.argsort(flat_ids, stable=True)`` in
``quant/sm70_fp8_moe/method.py:285``. Ids outside ``[0, num_experts)`` (the
-1 of expert parallelism) are dropped. Every slot is defined: the tail holds
the sentinel, blocks past the total hold -1.
"""

from __future__ import annotations

import numpy as np


def sorted_capacity(numel: int, num_experts: int, block_size: int) -> int:
    """Worst-case padded slots: every busy expert wastes block_size - 1."""
    return numel + min(numel, num_experts) * (block_size - 1)


def moe_align_block_size(topk_ids, num_experts: int, block_size: int, capacity: int | None = None):
    """Return (sorted_token_ids int32[cap], expert_ids int32[ceil(cap/bs)], total)."""
    ids = np.asarray(topk_ids).astype(np.int64).reshape(-1)
    numel = int(ids.size)
    cap = sorted_capacity(numel, num_experts, block_size) if capacity is None else int(capacity)
    valid = (ids >= 0) & (ids < num_experts)
    counts = np.bincount(ids[valid], minlength=num_experts).astype(np.int64)
    padded = (counts + block_size - 1) // block_size * block_size
    offsets = np.concatenate([[0], np.cumsum(padded)]).astype(np.int64)
    total = int(offsets[-1])
    if total > cap:
        raise ValueError(f"capacity {cap} < padded total {total}")

    sorted_ids = np.full(cap, numel, dtype=np.int32)
    key = np.where(valid, ids, num_experts)
    order = np.argsort(key, kind="stable")
    start = 0
    for e in range(num_experts):
        c = int(counts[e])
        sorted_ids[offsets[e] : offsets[e] + c] = order[start : start + c]
        start += c

    blocks = (cap + block_size - 1) // block_size
    expert_ids = np.full(blocks, -1, dtype=np.int32)
    for e in range(num_experts):
        expert_ids[offsets[e] // block_size : offsets[e + 1] // block_size] = e
    return sorted_ids, expert_ids, total
