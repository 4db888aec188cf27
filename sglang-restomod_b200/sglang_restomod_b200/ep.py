"""Expert parallelism: experts split contiguously across ranks, tokens
dispatched to the ranks that own their experts and combined back.

The reference has no all-to-all: its expert parallelism is upstream SGLang's
dispatcher, which maps global ids to local ones and marks foreign routes -1
(``sglang_restomod/quant/sm70_fp8_moe/method.py:8-12, 253-283``), followed by
an all-reduce. Here each rank owns ``E / world`` experts and one forward is:

1. per token, the set of owner ranks its routes go to; one (token, owner)
   pair per owner, pairs sorted stably by owner;
2. per-owner pair counts exchanged (``all_to_all_single`` of ``world`` ints
   over NCCL);
3. each pair's token row, once, with the token's top_k route slots (local
   expert id, -1 for the routes owned elsewhere, and router weight) sent to
   the owner (``all_to_all_single`` with the exchanged split sizes);
4. the owner runs its local experts on the received rows as tokens with
   top_k slots (``b200_moe_layer_forward``, foreign slots skipped): each
   output row is already the weighted sum over the owner's routes of that
   token, times ``routed_scaling_factor``;
5. one row per pair returned with the reverse exchange; the source adds its
   token's returned rows (one per owner) and the shared expert (computed on
   the rank's own tokens).

A token crosses the network once per distinct owner each way, not once per
route (top-8 over 8 ranks: ~5.3 times for uniform routing).

The split sizes make one host read per forward (step 2); the collectives run
on the current stream. That is the NCCL transport (``transport="nccl"``).

The peer transport (``transport="peer"``, the default on GPUs) needs no host
read and no NCCL call per forward: every rank maps every other rank's
exchange region (:class:`PeerExchange`, CUDA IPC over NVLink) and one
forward is three library calls on the current stream -
``b200_ep_dispatch`` (one row per (token, owner) stored straight into the
owners' regions), ``b200_ep_expert_forward`` (the owner's experts, then one
summed row per received row stored into its source's region) and
``b200_ep_combine``.
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
        [rows, top_k], -1 = not on this rank or empty; router weights fp32
        [rows, top_k]; activation rows f16 [rows, hidden]),
        rows = world * max_tokens."""
        lay = ops.ep_region_layout(self.world, self.max_tokens, self.top_k, self.hidden)
        rows = self.world * self.max_tokens
        slots = rows * self.top_k
        reg = self.region
        ids = reg[lay["ids"] : lay["ids"] + 4 * slots].view(torch.int32).view(rows, self.top_k)
        w = reg[lay["weights"] : lay["weights"] + 4 * slots].view(torch.float32).view(rows, self.top_k)
        x = reg[lay["recv"] : lay["recv"] + 2 * rows * self.hidden].view(torch.float16)
        return ids, w, x.view(rows, self.hidden)

    def status(self, reset: bool = True) -> int:
        return ops.region_status(self.region, reset)

    def close(self) -> None:
        for addr, offset in self._opened:
            ops.ipc_close_handle(addr, offset)
        self._opened = []


class ExpertParallelMoE:
    """``local`` holds this rank's ``num_experts / world`` experts.

    ``local_fn(rows[R,H], local_ids[R,k], weights[R,k]) -> summed rows[R,H]``
    (slots with id -1 belong to other ranks) and ``combine_fn(returned[P,H],
    pair_token[P], topk_ids, shared) -> out`` default to the library (the local
    layer, and a sum of each token's returned rows plus the shared expert);
    tests substitute CPU implementations to check the exchange itself over
    gloo.
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
        self.last_recv = None  # (rows, local ids [R, k], weights [R, k]) of the last forward
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

    def _run_local(self, rows, ids, w):
        if self._local_fn is not None:
            return self._local_fn(rows, ids, w)
        bs = self.local.block_size or block_size_for(int((ids >= 0).sum()), self.local.num_experts)
        return self.local.forward(rows, ids, w, block_size=bs, use_shared=False)

    def _combine(self, returned, pair_token, topk_ids, shared, out):
        if self._combine_fn is not None:
            return self._combine_fn(returned, pair_token, topk_ids, shared)
        tokens = topk_ids.shape[0]
        acc = torch.zeros(tokens, returned.shape[1], dtype=torch.float32, device=returned.device)
        acc.index_add_(0, pair_token, returned.float())
        if shared is not None:
            acc += shared.float()
        if out is None:
            return acc.to(returned.dtype)
        out.copy_(acc)
        return out

    def _shared(self, x):
        if self._shared_fn is not None:
            return self._shared_fn(x)
        if self.local is not None and self.local.shared is not None:
            return self.local.shared.forward(x)
        return None

    def dispatch_plan(self, topk_ids: torch.Tensor):
        """(pair_token, pair_owner, send_counts): one (token, owner) pair per
        distinct owner of a token's valid routes, sorted stably by owner."""
        tokens = topk_ids.shape[0]
        ids = topk_ids.long()
        valid = (ids >= 0) & (ids < self.num_experts)
        dest = torch.where(valid, ids // self.experts_per_rank, torch.zeros_like(ids))
        owned = torch.zeros(tokens, self.world, dtype=torch.bool, device=ids.device)
        owned.scatter_(1, dest, valid)
        # nonzero walks token-major; a stable sort by owner keeps token order
        pair_token, pair_owner = owned.nonzero(as_tuple=True)
        order = torch.argsort(pair_owner, stable=True)
        pair_token, pair_owner = pair_token[order], pair_owner[order]
        send_counts = torch.bincount(pair_owner, minlength=self.world)
        return pair_token, pair_owner, send_counts

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
        pair_token, pair_owner, send_counts = self.dispatch_plan(topk_ids)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        counts = torch.stack([send_counts, recv_counts]).to("cpu")
        send_split = counts[0].tolist()
        recv_split = counts[1].tolist()
        n_recv = int(sum(recv_split))

        # Each pair carries its token's top_k slots: the local expert where the
        # route belongs to the pair's owner, -1 elsewhere.
        ids = topk_ids.long()[pair_token]
        valid = (ids >= 0) & (ids < self.num_experts)
        mine = valid & (ids // self.experts_per_rank == pair_owner[:, None])
        local_ids = torch.where(mine, ids - pair_owner[:, None] * self.experts_per_rank,
                                torch.full_like(ids, -1)).to(torch.int32)
        meta = torch.cat([local_ids, topk_weights[pair_token].float().view(torch.int32)], dim=1)
        rows = x.index_select(0, pair_token)

        recv_rows = torch.empty(n_recv, x.shape[1], dtype=x.dtype, device=x.device)
        recv_meta = torch.empty(n_recv, 2 * top_k, dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_rows, rows, recv_split, send_split, group=self.group)
        dist.all_to_all_single(recv_meta, meta, recv_split, send_split, group=self.group)

        if n_recv:
            ids_r = recv_meta[:, :top_k].contiguous()
            w_r = recv_meta[:, top_k:].contiguous().view(torch.float32)
            done = self._run_local(recv_rows, ids_r, w_r).contiguous()
            self.last_recv = (recv_rows, ids_r, w_r)
        else:
            done = recv_rows
        back = torch.empty(pair_token.numel(), x.shape[1], dtype=done.dtype, device=x.device)
        dist.all_to_all_single(back, done, send_split, recv_split, group=self.group)
        return self._combine(back, pair_token, topk_ids, shared, out)

    def _forward_peer(self, x, topk_ids, topk_weights, shared, out):
        self.peer_dispatch(x, topk_ids, topk_weights)
        self.peer_experts()
        return self.peer_combine(topk_ids, shared, out, x.dtype)

    def peer_launches_per_forward(self, x_dtype=torch.bfloat16) -> int:
        """Kernels of one peer-transport forward: dispatch, receive, align (3
        kernels from 4096 receive slots on), [tcgen05 plan], gate/up, down,
        pre-sum, signal, combine, + the shared expert's."""
        layer = self.local
        slots = self.world * self.exchange.max_tokens * self.exchange.top_k
        n = 1 + 1 + (3 if slots >= 4096 else 1) + (1 if self.peer_block_size >= 64 else 0) + 5
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
