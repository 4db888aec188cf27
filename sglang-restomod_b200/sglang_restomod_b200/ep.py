"""Expert parallelism: experts split contiguously across ranks, tokens
dispatched to the ranks that own their experts and combined back.

The reference has no all-to-all: its expert parallelism is upstream SGLang's
dispatcher, which maps global ids to local ones and marks foreign routes -1
(``sglang_restomod/quant/sm70_fp8_moe/method.py:8-12, 253-283``), followed by
an all-reduce. Here each rank owns ``E / world`` experts and one forward is:

1. route -> destination rank; routes sorted stably by destination;
2. per-destination route counts exchanged (``all_to_all_single`` of ``world``
   ints over NCCL);
3. token rows and (local expert, weight) metadata sent to their owners
   (``all_to_all_single`` with the exchanged split sizes);
4. the owner runs its local experts on the received routes as one-slot
   tokens (``b200_moe_layer_forward`` with top_k = 1: the output rows come
   back already multiplied by their router weight);
5. rows returned with the reverse exchange and summed per token by the
   library's combine kernel, which also adds the shared expert (computed
   on the rank's own tokens) and applies ``routed_scaling_factor``.

The split sizes make one host read per forward (step 2); the collectives run
on the current stream.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops
from .layer import QuantMoELayer, block_size_for  # noqa: F401


class ExpertParallelMoE:
    """``local`` holds this rank's ``num_experts / world`` experts.

    ``local_fn(rows, local_ids[R,1], weights[R,1]) -> weighted rows`` and
    ``combine_fn(routed[T*k,H], topk_ids, shared) -> out`` default to the
    library (the local layer and its combine kernel); tests substitute CPU
    implementations to check the exchange itself over gloo.
    """

    def __init__(self, local: QuantMoELayer | None, num_experts: int, rank: int, world: int,
                 group=None, local_fn=None, combine_fn=None, shared_fn=None):
        if num_experts % world:
            raise ValueError(f"{num_experts} experts do not split over {world} ranks")
        if local is not None and local.num_experts != num_experts // world:
            raise ValueError("local layer must hold num_experts / world experts")
        self.local = local
        self.num_experts = num_experts
        self.rank = rank
        self.world = world
        self.group = group
        self.experts_per_rank = num_experts // world
        self.last_recv = None  # (rows, local ids, weights) of the last forward
        self._local_fn = local_fn
        self._combine_fn = combine_fn
        self._shared_fn = shared_fn

    def _run_local(self, rows, ids1, w1):
        if self._local_fn is not None:
            return self._local_fn(rows, ids1, w1)
        bs = self.local.block_size or block_size_for(rows.shape[0], self.local.num_experts)
        return self.local.forward(rows, ids1, w1, block_size=bs, use_shared=False)

    def _combine(self, routed, topk_ids, shared, out):
        if self._combine_fn is not None:
            return self._combine_fn(routed, topk_ids, shared)
        # every route was computed by its owner: no id is dropped here
        return ops.moe_combine(routed, topk_ids.clamp(min=0), self.num_experts, 1.0,
                               shared_out=shared, out=out, out_dtype=routed.dtype)

    def _shared(self, x):
        if self._shared_fn is not None:
            return self._shared_fn(x)
        if self.local is not None and self.local.shared is not None:
            return self.local.shared.forward(x)
        return None

    def dispatch_plan(self, topk_ids: torch.Tensor):
        """(order, send_counts): routes sorted stably by destination rank."""
        dest = (topk_ids.reshape(-1).long() // self.experts_per_rank).clamp_(0, self.world - 1)
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world)
        return order, dest, send_counts

    def forward(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        shared = self._shared(x)
        if self.world == 1 and self._local_fn is None:
            return self.local.forward(x, topk_ids, topk_weights, out=out, shared_out=shared)

        tokens, top_k = topk_ids.shape
        order, dest, send_counts = self.dispatch_plan(topk_ids)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        counts = torch.stack([send_counts, recv_counts]).to("cpu")
        send_split = counts[0].tolist()
        recv_split = counts[1].tolist()
        n_recv = int(sum(recv_split))

        flat_ids = topk_ids.reshape(-1)[order]
        local_ids = (flat_ids - dest[order].to(flat_ids.dtype) * self.experts_per_rank).to(torch.int32)
        meta = torch.stack([local_ids, topk_weights.reshape(-1)[order].view(torch.int32)], dim=1)
        rows = x.index_select(0, order // top_k)

        recv_rows = torch.empty(n_recv, x.shape[1], dtype=x.dtype, device=x.device)
        recv_meta = torch.empty(n_recv, 2, dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_rows, rows, recv_split, send_split, group=self.group)
        dist.all_to_all_single(recv_meta, meta, recv_split, send_split, group=self.group)

        if n_recv:
            ids1 = recv_meta[:, :1].contiguous()
            w1 = recv_meta[:, 1:].contiguous().view(torch.float32)
            done = self._run_local(recv_rows, ids1, w1).contiguous()
            self.last_recv = (recv_rows, ids1, w1)
        else:
            done = recv_rows
        back = torch.empty(tokens * top_k, x.shape[1], dtype=done.dtype, device=x.device)
        dist.all_to_all_single(back, done, send_split, recv_split, group=self.group)
        routed = torch.empty_like(back)
        routed.index_copy_(0, order, back)
        return self._combine(routed, topk_ids, shared, out)
