"""Expert parallelism across real GPUs (2 ranks, one process per GPU).

Each rank maps the other's exchange region through CUDA IPC and runs the
peer-memory forward (b200_ep_dispatch / expert_forward / combine: P2P stores
over NVLink, flags in peer memory), eagerly and replayed from a CUDA graph,
and the NCCL all-to-all transport; every output must match the single-GPU
layer that holds all experts. Skipped on boxes with fewer than 2 GPUs.
NVLS is off (NCCL_NVLS_ENABLE=0) and no kernel uses multicast.
"""

from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, results):
    try:
        from datetime import timedelta

        import torch.distributed as dist

        from sglang_restomod_b200 import _lib, ops, synth
        from sglang_restomod_b200.ep import ExpertParallelMoE
        from sglang_restomod_b200.layer import QuantMoELayer
        from tests.conftest import assert_close

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60),
                                device_id=dev)
        shape = synth.MoEShape(hidden=256, inter=128, experts=16, top_k=4, shared_inter=128)
        per = shape.experts // WORLD
        full = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, dev)
        local = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, dev, first_expert=rank * per,
                                        num_experts=per)
        max_tokens = 32
        peer = ExpertParallelMoE(local, shape.experts, rank, WORLD, transport="peer",
                                 max_tokens=max_tokens)
        fused_local = QuantMoELayer.synthetic(shape, _lib.QUANT_FP8_BLOCK, dev,
                                              first_expert=rank * per, num_experts=per,
                                              fuse_shared=True)
        fused_local.block_size = 64  # the tensor-core owner path, where fusion applies
        peer_fused = ExpertParallelMoE(fused_local, shape.experts, rank, WORLD, transport="peer",
                                       max_tokens=max_tokens)
        assert peer_fused.fused
        nccl = ExpertParallelMoE(local, shape.experts, rank, WORLD, transport="nccl")
        errors = []
        for step in range(3):
            t = max_tokens - 5 * step * rank
            x = synth.activations(t, shape.hidden, dev, seed=50 + 10 * step + rank)
            ids, w = synth.route(t, shape.experts, shape.top_k, dev, seed=80 + 10 * step + rank)
            want = full.forward(x, ids, w)
            got = peer.forward(x, ids, w)
            got_nccl = nccl.forward(x, ids, w)
            got_fused = peer_fused.forward(x, ids, w)
            torch.cuda.synchronize()
            assert_close(got, want, what=f"peer step {step}")
            assert_close(got_fused, want, what=f"peer fused-shared step {step}")
            assert_close(got_nccl, want, what=f"nccl step {step}")
        # CUDA graph of the peer forward, replayed in lockstep on both ranks.
        x = synth.activations(max_tokens, shape.hidden, dev, seed=7 + rank)
        ids, w = synth.route(max_tokens, shape.experts, shape.top_k, dev, seed=9 + rank)
        out = torch.empty_like(x)
        peer.forward(x, ids, w, out=out)
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            peer.forward(x, ids, w, out=out)
        for _ in range(5):
            graph.replay()
        torch.cuda.synchronize()
        assert_close(out, full.forward(x, ids, w), what="graph replay")
        status = peer.exchange.status()
        assert status == 0, f"region status {status}"
        assert ops.workspace_status() == 0
        dist.barrier()
        del graph
        peer.exchange.close()
        peer_fused.exchange.close()
        results[rank] = ("ok", "")
    except Exception:  # noqa: BLE001 - reported to the parent
        results[rank] = ("error", traceback.format_exc())
    finally:
        try:
            import torch.distributed as dist

            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def test_peer_ep_two_gpus(cuda_device):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "an EP rank did not finish"
    for r in range(WORLD):
        status, msg = results.get(r, ("missing", "no result"))
        assert status == "ok", f"rank {r}: {msg}"
