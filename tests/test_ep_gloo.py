"""Expert-parallel dispatch / combine over world_size 2 (gloo, CPU).

Each rank owns half of the experts; the exchange (counts, rows, metadata,
returned rows) runs through torch.distributed exactly as on NCCL, with the
expert compute and the combine done by the CPU oracle. Every rank's output
must equal the single-process oracle over all experts. A second test makes
one rank fail before the exchange and checks that its peer gets an error
(from a short process-group timeout) instead of hanging.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from sglang_restomod_b200.ep import ExpertParallelMoE

E, H, I, K, T = 8, 128, 128, 3, 10


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bank():
    g = torch.Generator().manual_seed(5)
    w13, w2 = [], []
    for _ in range(E):
        q, s = oracle.quant_block_fp8(torch.randn(2 * I, H, generator=g) * 0.05)
        w13.append(oracle.dequant_block_fp8(q, s))
        q, s = oracle.quant_block_fp8(torch.randn(H, I, generator=g) * 0.05)
        w2.append(oracle.dequant_block_fp8(q, s))
    return torch.stack(w13), torch.stack(w2)


def _inputs(rank):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(T, H, generator=g).bfloat16()
    ids, w = oracle.route_topk(torch.randn(T, E, generator=g), K)
    return x, ids, w


def _worker(rank, world, port, mode, results):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        w13, w2 = _bank()
        per = E // world
        mine = slice(rank * per, (rank + 1) * per)

        def local_fn(rows, ids_r, w_r):
            # one row per (token, this owner); slots of other owners are -1
            assert ids_r.shape == w_r.shape == (rows.shape[0], K)
            out = oracle.moe_layer_ref(rows, ids_r, w_r, w13[mine], w2[mine], inter_dtype=None)
            return out.to(rows.dtype)

        def combine_fn(returned, pair_token, topk_ids, shared):
            # exactly one returned row per (token, distinct owner of its routes)
            owners = [len({int(e) // per for e in row}) for row in topk_ids.tolist()]
            assert returned.shape[0] == pair_token.numel() == sum(owners)
            assert torch.bincount(pair_token, minlength=len(owners)).tolist() == owners
            acc = torch.zeros(topk_ids.shape[0], returned.shape[1])
            return acc.index_add_(0, pair_token, returned.float())

        ep = ExpertParallelMoE(None, E, rank, world, local_fn=local_fn, combine_fn=combine_fn)
        x, ids, w = _inputs(rank)
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure before the exchange")
        out = ep.forward(x, ids, w)
        want = oracle.moe_layer_ref(x, ids, w, w13, w2, inter_dtype=None)
        err = float((out - want).abs().max())
        results[rank] = ("ok", err)
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        results[rank] = ("error", f"{type(exc).__name__}: {exc}")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(mode):
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("an EP rank did not finish")
    return dict(results)


def test_ep_dispatch_combine_world2():
    res = _run("ok")
    for rank in range(2):
        status, value = res[rank]
        assert status == "ok", value
        assert value < 2e-2, f"rank {rank} max error {value}"


def test_ep_rank_failure_is_an_error_not_a_hang():
    res = _run("fail")
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error"  # the surviving rank's collective timed out or saw the peer leave
