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
on the current stream. That is the NCCL transport (``transport="nccl"``).

The peer transport (``transport="peer"``, the default on GPUs) needs no host
read and no NCCL call per forward: every rank maps every other rank's
exchange region (:class:`PeerExchange`, CUDA IPC over NVLink) and one
forward is three library calls on the current stream -
``b200_ep_dispatch`` (rows stored straight into the owners' regions),
``b200_ep_expert_forward`` (the owner's experts; the down GEMM's epilogue
stores each weighted row into its source's region) and ``b200_ep_combine``.
Ranks synchronize through flags in the regions, so the forward can be
captured in a CUDA graph and replayed on every rank.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops
from .layer import B, QuantMoELayer, block_size_for  # noqa: F401


class PeerExchange:
    """This rank's exchange region, and every rank's region mapped here.

    ``region`` is a zero-filled buffer of ``b200_ep_region_bytes``; the CUDA IPC
    handles are exchanged once with ``all_gather_object`` over ``group``.
    ``peers`` (int64 [world], on the device) holds rank r's region address in
    this process. ``regions`` lets a single process stand in for ``world``
    ranks (tests): then no IPC is involved and every rank's peers are the
    given local buffers.
    """

    def __init__(self, world: int, rank: int, max_tokens: int, top_k: int, hidden: int,
                 device: torch.device, group=None, regions: list | None = None):
        self.world, self.rank = world, rank
        self.max_tokens, self.top_k, self.hidden = max_tokens, top_k, hidden
        self._opened: list[tuple[int, int]] = []
        nbytes = ops.ep_region_bytes(world, max_tokens, top_k, hidden)
        if regions is not None:
            self.region = regions[rank]
            ptrs = [int(r.data_ptr()) for r in regions]
        else:
            self.region = ops.aligned_zeros(nbytes, device)
            torch.cuda.synchronize(device)
            mine = ops.ipc_get_handle(self.region)
            gathered = [None] * world
            dist.all_gather_object(gathered, mine, group=group)
            ptrs = []
            for r, (handle, offset) in enumerate(gathered):
                if r == rank:
                    ptrs.append(int(self.region.data_ptr()))
                else:
                    addr = ops.ipc_open_handle(handle, offset)
                    self._opened.append((addr, offset))
                    ptrs.append(addr)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        if regions is None:
            torch.cuda.synchronize(device)
            dist.barrier(group=group)

    def received(self):
        """Views of what the last expert step received: (local ids int32
        [slots, 1], -1 = empty; router weights fp32 [slots, 1]; rows f16
        [slots, hidden]), slots = world * max_tokens * top_k."""
        lay = ops.ep_region_layout(self.world, self.max_tokens, self.top_k, self.hidden)
        slots = self.world * self.max_tokens * self.top_k
        reg = self.region
        ids = reg[lay["ids"] : lay["ids"] + 4 * slots].view(torch.int32).view(slots, 1)
        w = reg[lay["weights"] : lay["weights"] + 4 * slots].view(torch.float32).view(slots, 1)
        rows = reg[lay["recv"] : lay["recv"] + 2 * slots * self.hidden].view(torch.float16)
        return ids, w, rows.view(slots, self.hidden)

    def status(self, reset: bool = True) -> int:
        return ops.region_status(self.region, reset)

    def close(self) -> None:
        for addr, offset in self._opened:
            ops.ipc_close_handle(addr, offset)
        self._opened = []


class ExpertParallelMoE:
    """``local`` holds this rank's ``num_experts / world`` experts.

    ``local_fn(rows, local_ids[R,1], weights[R,1]) -> weighted rows`` and
    ``combine_fn(routed[T*k,H], topk_ids, shared) -> out`` default to the
    library (the local layer and its combine kernel); tests substitute CPU
    implementations to check the exchange itself over gloo.
    """

    def __init__(self, local: QuantMoELayer | None, num_experts: int, rank: int, world: int,
                 group=None, local_fn=None, combine_fn=None, shared_fn=None,
                 transport: str = "nccl", max_tokens: int | None = None,
                 exchange: PeerExchange | None = None):
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
        if transport not in ("nccl", "peer"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self.exchange = exchange
        self.fused = False
        if transport == "peer":
            if local is None or max_tokens is None:
                raise ValueError("the peer transport needs the local layer and max_tokens")
            # A fused shared expert travels as one more route per token, kept
            # on the source rank (its local expert num_experts / world); used
            # when the owner's GEMMs run on the tensor-core path (blocks of 64+).
            fbs = local.block_size or block_size_for(max_tokens * (local.top_k + 1),
                                                     local.num_experts + 1)
            self.fused = local.shared_fused and (fbs >= 64 or max_tokens <= fbs)
            routes_k = local.top_k + (1 if self.fused else 0)
            if exchange is not None and exchange.top_k != routes_k:
                raise ValueError(f"exchange sized for {exchange.top_k} routes per token, "
                                 f"this layer sends {routes_k}")
            if exchange is None:
                self.exchange = PeerExchange(world, rank, max_tokens, routes_k, local.hidden,
                                             local.w13.device, group=group)
            # Each owner receives about max_tokens * top_k routes per step.
            self.peer_block_size = local.block_size or block_size_for(
                max_tokens * routes_k, local.num_experts + (1 if self.fused else 0))

    def _run_local(self, rows, ids1, w1):
        if self._local_fn is not None:
            return self._local_fn(rows, ids1, w1)
        bs = self.local.block_size or block_size_for(rows.shape[0], self.local.num_experts)
        return self.local.forward(rows, ids1, w1, block_size=bs, use_shared=False)

    def _combine(self, routed, topk_ids, shared, out):
        if self._combine_fn is not None:
            return self._combine_fn(routed, topk_ids, shared)
        # every route was computed by its owner: no id is dropped here
        y = B.moe_combine(routed, topk_ids.clamp(min=0), self.num_experts, 1.0, shared,
                          routed.dtype)
        if out is None:
            return y
        out.copy_(y)
        return out

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
        if self.transport == "peer" and self.fused:
            ids, w = self.local.fused_routes(topk_ids, topk_weights, shared_id=self.num_experts)
            return self._forward_peer(x, ids, w, None, out)
        if self.world == 1 and self._local_fn is None and self.transport != "peer":
            # all experts are local: one layer forward (shared expert inside)
            return self.local.forward(x, topk_ids, topk_weights, out=out)
        shared = self._shared(x)
        if self.transport == "peer":
            return self._forward_peer(x, topk_ids, topk_weights, shared, out)

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

    def _forward_peer(self, x, topk_ids, topk_weights, shared, out):
        self.peer_dispatch(x, topk_ids, topk_weights)
        self.peer_experts()
        return self.peer_combine(topk_ids, shared, out, x.dtype)

    def peer_launches_per_forward(self, x_dtype=torch.bfloat16) -> int:
        """Kernels of one peer-transport forward: dispatch, receive, align (3
        kernels from 4096 receive slots on), [tcgen05 plan], gate/up, down,
        signal, combine, + the shared expert's."""
        layer = self.local
        slots = self.world * self.exchange.max_tokens * self.exchange.top_k
        n = 1 + 1 + (3 if slots >= 4096 else 1) + (1 if self.peer_block_size >= 64 else 0) + 4
        if self.fused:
            n += 1 + (1 if self.peer_block_size >= 64 else 0)  # route append, permute
        elif layer.shared is not None:
            n += layer.shared.launches(self.exchange.max_tokens, layer.hidden, x_dtype)
            n += 1 if self.peer_block_size >= 64 else 0  # permute
        else:
            n += 1 if self.peer_block_size >= 64 else 0
        return n

    # The three steps of a peer-transport forward; every rank runs them in this
    # order. (A single process standing in for several ranks interleaves them
    # rank by rank: all dispatches, then all expert steps, then all combines.)
    def peer_dispatch(self, x, topk_ids, topk_weights):
        """topk_ids / topk_weights: [T, k], or [T, k + 1] with the shared
        route appended when the layer's shared expert is fused."""
        ex = self.exchange
        B.ep_dispatch(x, topk_ids, topk_weights, self.num_experts, self.rank, self.world,
                      ex.peers, ex.region, ex.max_tokens, self.fused)

    def peer_experts(self):
        ex, layer = self.exchange, self.local
        B.ep_expert_forward(
            layer.quant, layer.hidden, layer.inter, layer.num_experts + (1 if self.fused else 0),
            layer.w13, layer.w2, layer.w13_scales, layer.w2_scales, layer.w13_global,
            layer.w2_global, self.peer_block_size, self.rank, self.world, ex.peers, ex.region,
            ex.max_tokens, ex.top_k)

    def peer_combine(self, topk_ids, shared=None, out=None, out_dtype=torch.bfloat16):
        ex, layer = self.exchange, self.local
        if out is None:
            out = torch.empty(topk_ids.shape[0], layer.hidden, dtype=out_dtype,
                              device=topk_ids.device)
        B.ep_combine(topk_ids, layer.hidden, self.num_experts + (1 if self.fused else 0),
                     self.world, ex.region, ex.max_tokens, layer.routed_scaling_factor, shared, out)
        return out
