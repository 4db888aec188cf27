"""Benchmark of the B200 quantized-MoE path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]

Default workload ("config4-decode"): the expert-parallel block-FP8 MoE layer
of the benchmark definition - H=7168, I=2048, 256 routed experts, top-8, one
shared expert (I=2048), 128 tokens per rank - on N GPUs of one node, one
process per GPU (torchrun), experts split E/N per rank, tokens dispatched
and combined with NCCL all-to-all. Per-rank work is fixed as N grows
(weak scaling); ``value`` is the tokens of all ranks divided by the slowest
rank's device time. Other workloads (``--workload``) are the single-GPU
configurations: config2-T<t> / config3-T<t> (E=512 FP8 / NVFP4 MoE layer)
and config1-<K>x<N>-M<m> (dense FP8 GEMV).

Inputs are seeded synthetic tensors (no dataset): activations N(0,1),
router logits N(0,1) -> softmax -> top-k -> renormalised, weights N(0,0.02)
quantized to block FP8 (or NVFP4). Weights read per step exceed the 126 MB
L2 in the default workload. A workload whose step reads less than L2 (one-
token decode, configuration 0) is built several times over, each copy with
its own weights, and the timed steps rotate over the copies, so a copy's
weights are evicted from L2 before its next step (the config says how many).

``--impl reference`` times the reference's CPU torch arithmetic (the
oracle port of sglang-restomod's dequantize-then-matmul MoE path) on the
host cores, rank 0 only, on a bounded sample of tokens per step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

L2_BYTES = 126 * 1000 * 1000  # B200 L2

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "sglang-restomod_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer & GEMV tokens/s per B200 + % HBM/tensor roofline; EP 1/2/4/8 tokens/s"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


# ------------------------------------------------------------------ helpers
def torch_empty_like(t):
    import torch

    return torch.empty_like(t)


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        0x4: "sw_power_cap",
        0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown",
        0x2: "applications_clocks_setting",
    }

    def __init__(self, device_index: int, period: float = 0.01):
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            import torch

            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode() if isinstance(uuid, str) else uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # noqa: BLE001 - clocks are reported, not required
            self._nvml = None
            self.error = str(exc)
        self.period = period

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                try:
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    reasons = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.samples.append((mhz, int(reasons)))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def start(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = statistics.median(s[0] for s in self.samples)
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = [name for bit, name in self.REASONS.items() if bits & bit]
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


def dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local_rank)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local_rank


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


class PipelinedIO:
    """Double-buffered end-to-end I/O around one workload step.

    Step i computes on device buffer i % 2 while a copy stream returns step
    i-1's result to pinned host memory and brings step i+1's inputs to the
    device (the copy engines run beside the kernels). Every step's input copy
    and result copy still happen inside the timed region: the first inputs
    are copied before the first step, the last result after the last one.
    """

    def __init__(self, host_inputs, device_out, compute):
        import torch

        self.h_in = list(host_inputs)
        self.d_in = [[torch.empty_like(t, device=device_out.device) for t in self.h_in]
                     for _ in range(2)]
        self.d_out = [device_out, torch.empty_like(device_out)]
        self.h_out = [torch.empty_like(device_out, device="cpu").pin_memory() for _ in range(2)]
        self.copy = torch.cuda.Stream(device=device_out.device)
        self.compute = compute

    def load_first(self):
        for d, h in zip(self.d_in[0], self.h_in):
            d.copy_(h, non_blocking=True)

    def step(self, p: int):
        import torch

        main = torch.cuda.current_stream()
        self.copy.wait_stream(main)
        with torch.cuda.stream(self.copy):
            self.h_out[1 - p].copy_(self.d_out[1 - p], non_blocking=True)
            for d, h in zip(self.d_in[1 - p], self.h_in):
                d.copy_(h, non_blocking=True)
        self.compute(self.d_in[p], self.d_out[p])
        main.wait_stream(self.copy)

    def drain(self, p: int):
        self.h_out[p].copy_(self.d_out[p], non_blocking=True)


# ---------------------------------------------------------------- workloads
def parse_workload(name: str):
    from sglang_restomod_b200 import synth

    if name in ("config4-decode", "config4-prefill"):
        return dict(kind="ep", shape=synth.CONFIG4, tokens=128 if name.endswith("decode") else 4096,
                    quant=0)
    if name.startswith("config2-T") or name.startswith("config3-T"):
        return dict(kind="moe", shape=synth.CONFIG2, tokens=int(name.split("-T")[1]),
                    quant=0 if name.startswith("config2") else 1)
    if name.startswith("config0"):
        return dict(kind="moe", shape=synth.CONFIG0, tokens=32, quant=0)
    if name.startswith("config1-"):
        kn, m = name[len("config1-"):].split("-M")
        k, n = (int(v) for v in kn.split("x"))
        return dict(kind="dense", k=k, n=n, m=int(m))
    raise SystemExit(f"unknown workload {name}")


class MoEWorkload:
    """One MoE layer forward per step on this rank's tokens."""

    def __init__(self, spec, rank, world, device, layer=None):
        import torch

        from sglang_restomod_b200 import synth
        from sglang_restomod_b200.ep import ExpertParallelMoE
        from sglang_restomod_b200.layer import QuantMoELayer

        shape = spec["shape"]
        self.shape = shape
        self.tokens = spec["tokens"]
        self.quant = spec["quant"]
        self.world = world
        e_local = shape.experts // world
        # The shared expert rides in the routed GEMMs (one more expert) when its
        # shapes and quantization match the routed experts'. ``layer`` reuses
        # an already built layer of the same shape (the sweep's prefill point).
        self.layer = layer if layer is not None else QuantMoELayer.synthetic(
            shape, self.quant, device, first_expert=rank * e_local, num_experts=e_local,
            fuse_shared=spec.get("fuse_shared", True))
        # N > 1: the peer-memory exchange (NVLink P2P stores, no host sync) by
        # default; --transport nccl selects the all-to-all baseline.
        self.transport = spec.get("transport", "peer") if world > 1 else "local"
        if self.transport == "peer":
            self.model = ExpertParallelMoE(self.layer, shape.experts, rank, world,
                                           transport="peer", max_tokens=self.tokens)
        else:
            self.model = ExpertParallelMoE(self.layer, shape.experts, rank, world)
        # Each rank's tokens are its own seeded batch.
        self.x = synth.activations(self.tokens, shape.hidden, device, seed=100 + rank)
        self.ids, self.w = synth.route(self.tokens, shape.experts, shape.top_k, device, seed=200 + rank)
        self.out = torch.empty_like(self.x)
        # pinned host copies for the end-to-end leg
        self.h_x = self.x.cpu().pin_memory()
        self.h_ids = self.ids.cpu().pin_memory()
        self.h_w = self.w.cpu().pin_memory()
        self.h_out = torch.empty_like(self.h_x).pin_memory()
        self.d_out = torch.empty_like(self.x)

    def replica(self):
        """This workload on its own copy of the layer's weights (same inputs
        and routing, own output buffers); single GPU."""
        import copy

        import torch

        from sglang_restomod_b200.ep import ExpertParallelMoE

        assert self.world == 1

        def cloned(obj):
            c = copy.copy(obj)
            for k, v in vars(obj).items():
                if isinstance(v, torch.Tensor) and v.is_cuda:
                    setattr(c, k, v.clone())
            return c

        r = copy.copy(self)
        r.layer = cloned(self.layer)
        if self.layer.shared is not None:
            r.layer.shared = cloned(self.layer.shared)
        r.model = ExpertParallelMoE(r.layer, self.shape.experts, 0, 1)
        r.out = torch.empty_like(self.out)
        r.d_out = torch.empty_like(self.d_out)
        return r

    def step(self):
        self.model.forward(self.x, self.ids, self.w, out=self.out)

    def e2e_io(self):
        return PipelinedIO([self.h_x, self.h_ids, self.h_w], self.d_out,
                           lambda d, out: self.model.forward(d[0], d[1], d[2], out=out))

    def io_bytes(self):
        h2d = self.h_x.numel() * 2 + self.h_ids.numel() * 4 + self.h_w.numel() * 4
        return h2d, self.h_out.numel() * 2

    def launches_per_step(self):
        if self.transport == "peer":
            return self.model.peer_launches_per_forward(self.x.dtype)
        # local layer (+ shared); under EP one more combine of returned rows
        return (self.layer.launches_per_forward(self.x.dtype, self.tokens)
                + (1 if self.world > 1 else 0))

    def algorithmic(self):
        """(bytes, flops) of one step on this rank (realized routing)."""
        import torch

        layer = self.layer
        shape = self.shape
        ids = self.ids.reshape(-1).long()
        if self.world > 1:
            # experts this rank owns that any rank's routing touches is not
            # known locally; count the local experts (all are touched at
            # these token counts) - checked by the routing stats below.
            touched = layer.num_experts
        else:
            touched = int(torch.unique(ids).numel())
        wbytes = touched * layer.weight_bytes_per_expert()
        if layer.shared is not None:
            wbytes += 3 * shape.hidden * shape.shared_inter
        act = self.tokens * shape.hidden * 2 * 2
        routes = self.tokens * shape.top_k
        flops = 2 * routes * 3 * shape.hidden * shape.inter
        if layer.shared is not None:
            flops += 2 * self.tokens * 3 * shape.hidden * shape.shared_inter
        return wbytes + act, flops, touched

    def dominant(self, loads_only: bool = False):
        """Closure timing the gate/up expert GEMM alone (the largest kernel);
        ``loads_only``: its data-movement floor (same copies, no math)."""
        import torch

        from sglang_restomod_b200 import _lib, ops
        from sglang_restomod_b200.layer import block_size_for

        layer = self.layer
        if self.world == 1:
            ids, x = self.ids, self.x
        elif self.transport == "peer":
            # the owner's gate/up GEMM on the routes its region received
            ids, _, x = self.model.exchange.received()
        else:
            if self.model.last_recv is None:
                return None
            x, ids, _ = self.model.last_recv
        if self.transport == "peer":
            bs = self.model.peer_block_size
        else:
            bs = block_size_for(ids.numel(), layer.num_experts)
        sorted_ids, expert_ids, ntpp = ops.moe_align_block_size(ids, bs, layer.num_experts)
        x16 = x if x.dtype == torch.float16 else x.half()
        routes = ids.numel()
        c = torch.empty(routes, layer.inter, dtype=torch.float16, device=self.x.device)

        def run():
            ops.moe_gemm(x16, layer.w13, 2 * layer.inter, quant=layer.quant,
                         num_experts=layer.num_experts, sorted_token_ids=sorted_ids,
                         expert_ids=expert_ids, num_tokens_post_pad=ntpp, block_size=bs,
                         top_k=ids.shape[1], num_routes=routes, c=c, scales=layer.w13_scales,
                         global_scale=layer.w13_global, gated_mode=_lib.GATED_FUSED,
                         loads_only=loads_only)

        valid = ids[(ids >= 0) & (ids < layer.num_experts)]
        touched = int(torch.unique(valid).numel())
        if layer.quant == 0:
            per_expert = 2 * layer.inter * layer.hidden + (2 * layer.inter // 128) * (layer.hidden // 128) * 4
        else:
            per_expert = 2 * layer.inter * layer.hidden // 2 + 2 * layer.inter * layer.hidden // 16
        nvalid = int(valid.numel())
        if self.transport == "peer":  # only received slots are read and written
            nbytes = touched * per_expert + nvalid * layer.hidden * 2 + nvalid * layer.inter * 2
        else:
            nbytes = touched * per_expert + x.shape[0] * layer.hidden * 2 + routes * layer.inter * 2
        flops = 2 * nvalid * 2 * layer.inter * layer.hidden
        name = ("tc_gemm_kernel (gate/up, gated SiLU epilogue)" if bs >= 64 else
                "stream_gemm_kernel (gate/up, gated SiLU epilogue)")
        return run, nbytes, name, flops


class DenseWorkload:
    def __init__(self, spec, device):
        import torch

        from sglang_restomod_b200 import ops, synth

        self.k, self.n, self.m = spec["k"], spec["n"], spec["m"]
        self.tokens = self.m
        q, s = synth.fp8_bank(1, self.n, self.k, device, seed=1)
        self.packed = ops.fp8_prepack(q[0], gated=False)
        self.scales = s[0]
        del q
        self.x = synth.activations(self.m, self.k, device, seed=2)
        self.out = torch.empty(self.m, self.n, dtype=torch.bfloat16, device=device)
        self.h_x = self.x.cpu().pin_memory()
        self.h_out = torch.empty(self.m, self.n, dtype=torch.bfloat16).pin_memory()

    def _run(self, x, out=None, loads_only=False):
        from sglang_restomod_b200 import _lib, ops

        ops.linear(x, self.packed, self.n, quant=_lib.QUANT_FP8_BLOCK, scales=self.scales,
                   out=self.out if out is None else out, loads_only=loads_only)

    def step(self):
        self._run(self.x)

    def e2e_io(self):
        return PipelinedIO([self.h_x], torch_empty_like(self.out),
                           lambda d, out: self._run(d[0], out))

    def io_bytes(self):
        return self.h_x.numel() * 2, self.h_out.numel() * 2

    def launches_per_step(self):
        """bf16 -> f16 conversion and the GEMM (stream GEMM up to 32 rows;
        tcgen05 beyond, plus its finishing kernel when K is split)."""
        from sglang_restomod_b200 import ops
        from sglang_restomod_b200.layer import dense_k_parts

        split = self.m >= 33 and dense_k_parts(self.m, self.n, self.k, ops.num_sms()) > 1
        return 3 if split else 2

    def algorithmic(self):
        wbytes = self.n * self.k + (self.n // 128) * (self.k // 128) * 4
        return wbytes + self.m * (self.k + self.n) * 2, 2 * self.m * self.n * self.k, 1

    def dominant(self, loads_only: bool = False):
        # b200_linear runs 33+ rows on the tcgen05 GEMM, fewer on the stream GEMM
        name = "tc_gemm_kernel (dense)" if self.m >= 33 else "stream_gemm_kernel (dense)"
        run = (lambda: self._run(self.x, loads_only=True)) if loads_only else self.step
        return run, self.algorithmic()[0], name, 2 * self.m * self.n * self.k


# -------------------------------------------------------------- CPU legs
def cpu_reference_step(spec, threads: int):
    """One step of the reference's CPU arithmetic on the GPU arm's own batch.

    The oracle port of sglang-restomod's dequantize-then-matmul path (the
    reference's CPU torch path; its kernels are closed V100 binaries) on the
    same seeded inputs rank 0 of the GPU arm runs: the same tokens, routing
    and weights (generated with the same seeds; on the GPU when one is
    present, where the GPU arm generates them, then moved to host memory).
    Inside the step every touched expert - and the shared expert - is
    dequantized from its checkpoint format and applied, as the reference's
    CPU path does. Returns (step, tokens, description).
    """
    import torch

    import oracle
    from sglang_restomod_b200 import synth

    torch.set_num_threads(threads)
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
    if spec["kind"] == "dense":
        k, n, m = spec["k"], spec["n"], spec["m"]
        q, s = synth.fp8_bank(1, n, k, dev, seed=1)
        q, s = q[0].cpu(), s[0].cpu()
        x = synth.activations(m, k, dev, seed=2).cpu()

        def step():
            return oracle.fp8_linear_ref(x, q, s)

        return step, m, f"{m} rows x [{n}, {k}] block-FP8 weight, dequantized inside the step"

    shape, tokens, quant = spec["shape"], spec["tokens"], spec["quant"]
    h, i, e_all, top_k = shape.hidden, shape.inter, shape.experts, shape.top_k
    x = synth.activations(tokens, h, dev, seed=100).cpu()
    ids, wts = synth.route(tokens, e_all, top_k, dev, seed=200)
    ids, wts = ids.cpu(), wts.cpu()
    seed = 10  # QuantMoELayer.synthetic's default
    bank = {}
    for e in torch.unique(ids).tolist():
        if quant == 0:
            q13, s13 = synth.fp8_bank(1, 2 * i, h, dev, seed, e)
            q2, s2 = synth.fp8_bank(1, h, i, dev, seed + 1, e)
            bank[e] = ((q13[0].cpu(), s13[0].cpu()), (q2[0].cpu(), s2[0].cpu()))
        else:
            p13, s13, g13 = synth.nvfp4_bank(1, 2 * i, h, dev, seed, e)
            p2, s2, g2 = synth.nvfp4_bank(1, h, i, dev, seed + 1, e)
            bank[e] = ((p13[0].cpu(), s13[0].cpu(), float(g13[0])),
                       (p2[0].cpu(), s2[0].cpu(), float(g2[0])))
    shared = None
    if shape.shared_inter:
        si = shape.shared_inter
        sq13, ss13 = synth.fp8_bank(1, 2 * si, h, dev, seed + 2, 0)
        sq2, ss2 = synth.fp8_bank(1, h, si, dev, seed + 3, 0)
        shared = ((sq13[0].cpu(), ss13[0].cpu()), (sq2[0].cpu(), ss2[0].cpu()))

    def deq(item, fp8):
        return oracle.dequant_block_fp8(*item) if fp8 else oracle.dequant_nvfp4(*item)

    def fetch(e):  # dequantized inside the timed step, one expert at a time
        a, b = bank[e]
        return deq(a, quant == 0), deq(b, quant == 0)

    ones_ids = torch.zeros(tokens, 1, dtype=torch.int32)
    ones_w = torch.ones(tokens, 1)

    def step():
        out = oracle.moe_layer_ref(x, ids, wts, fetch, e_all)
        if shared is not None:
            out = out + oracle.moe_layer_ref(
                x, ones_ids, ones_w, lambda _e: (deq(shared[0], True), deq(shared[1], True)), 1)
        return out

    extra = " + the shared expert" if shared is not None else ""
    return step, tokens, (
        f"the full {tokens}-token batch x top-{top_k} ({len(bank)} touched experts{extra} "
        f"dequantized and applied per step): oracle port of the reference's CPU "
        f"dequantize-then-matmul path"
    )


def reference_arm(args, rank, world):
    """--impl reference: the reference's CPU torch path on host cores, rank 0 only.

    Each step is the GPU arm's whole per-rank batch (same workload, same
    inputs) through the oracle port, on every host thread. One untimed
    warm-up step; then up to K timed steps, stopping early once 150 s of CPU
    time have passed (the line's ``steps`` says how many ran).
    """
    if rank != 0:
        return
    spec = parse_workload(args.workload)
    threads = os.cpu_count() or 1
    step, tokens, desc = cpu_reference_step(spec, threads)
    step()  # warm-up
    times = []
    budget = time.perf_counter() + 150.0
    for _ in range(max(1, args.steps)):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > budget:
            break
    mean_s = sum(times) / len(times)
    value = tokens / mean_s
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": len(times), "warmup": 1, "ms_per_step": 1000.0 * mean_s,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (dequantized weights) x bf16", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": args.workload, "tokens_per_step": tokens},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------- sweep and EP check
SWEEP = (
    "config1-5120x25600-M1", "config1-5120x25600-M64", "config1-25600x5120-M64",
    "config1-5120x152064-M1", "config2-T1", "config2-T64", "config2-T8192", "config3-T1",
    "config3-T128", "config3-T4096", "config4-prefill",
)


def weight_copies(wl, step_bytes: int, world: int) -> int:
    """Steps that read less than twice the L2 rotate over copies of the
    workload (own weights, same inputs), enough that the copies together
    read at least twice the L2: a copy's weights are evicted before its next
    step."""
    if world == 1 and step_bytes < 2 * L2_BYTES and hasattr(wl, "replica"):
        return int(min(16, max(2, -(-2 * L2_BYTES // step_bytes))))
    return 1


def sweep_point(name, args, device, hbm_gbs, bf16_tflops, reuse=None):
    """One configuration on one GPU: step time (CUDA graph replay, CUDA
    events) and its dominant kernel's time and roofline fractions."""
    import torch

    spec = parse_workload(name)
    spec["transport"] = "local"
    spec["fuse_shared"] = True
    if spec["kind"] == "dense":
        wl = DenseWorkload(spec, device)
    else:
        wl = MoEWorkload(spec, 0, 1, device, layer=reuse)
    step_bytes, step_flops, touched = wl.algorithmic()
    copies = weight_copies(wl, step_bytes, 1)
    wls = [wl] + [wl.replica() for _ in range(copies - 1)]
    stream = torch.cuda.current_stream()
    for _ in range(3):
        for w in wls:
            w.step()
    torch.cuda.synchronize()
    graphs, fns = [], []
    for w in wls:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            w.step()
        graphs.append(g)
        fns.append(g.replay)
    doms = [w.dominant() for w in wls]
    dom_fns = []
    for run, _, _, _ in doms:
        run()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run()
        graphs.append(g)
        dom_fns.append(g.replay)
    for f in fns + dom_fns:
        f()
    torch.cuda.synchronize()
    reps = max(20, min(args.steps, 200))
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(reps):
        fns[i % copies]()
    end.record(stream)
    torch.cuda.synchronize()
    step_ms = start.elapsed_time(end) / reps
    start.record(stream)
    for i in range(reps):
        dom_fns[i % copies]()
    end.record(stream)
    torch.cuda.synchronize()
    dom_ms = start.elapsed_time(end) / reps
    _, dom_bytes, dom_name, dom_flops = doms[0]
    # the same kernel's loads-only twin: the floor set by moving its bytes
    floor_run = wls[0].dominant(loads_only=True)[0]
    floor_ms = None
    if floor_run is not None:
        floor_run()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            floor_run()
        graphs.append(g)
        g.replay()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(reps):
            g.replay()
        end.record(stream)
        torch.cuda.synchronize()
        floor_ms = start.elapsed_time(end) / reps
    hbm_frac = dom_bytes / (dom_ms * 1e-3) / 1e9 / hbm_gbs
    tensor_frac = dom_flops / (dom_ms * 1e-3) / 1e12 / bf16_tflops
    prefill = wl.tokens >= 2048
    point = {
        "ms_per_step": step_ms, "tokens_per_s": wl.tokens / (step_ms * 1e-3),
        "layer_hbm_frac": step_bytes / (step_ms * 1e-3) / 1e9 / hbm_gbs,
        "layer_tensor_frac": step_flops / (step_ms * 1e-3) / 1e12 / bf16_tflops,
        "dominant": dom_name, "dominant_us": dom_ms * 1e3,
        "bound": "tensor" if prefill else "hbm",
        "frac": tensor_frac if prefill else hbm_frac,
        "dominant_hbm_frac": hbm_frac, "dominant_tensor_frac": tensor_frac,
        "weight_copies": copies,
        "dominant_loads_only_us": None if floor_ms is None else floor_ms * 1e3,
    }
    del graphs, fns, dom_fns, doms, wls, wl
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return point


def measure_fp8_peak(device) -> float:
    """Dense FP8 tensor peak on this GPU: cuBLASLt e4m3 GEMM (torch._scaled_mm)
    at 8192^3, best of 10, CUDA events (TFLOP/s)."""
    import torch

    n = 8192
    a = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
    one = torch.ones((), device=device)
    for _ in range(3):
        torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    best = float("inf")
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    for _ in range(10):
        start.record()
        torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        end.record()
        torch.cuda.synchronize()
        best = min(best, start.elapsed_time(end))
    del a, b
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def w8a8_points(args, device, fp8_tflops, bf16_tflops):
    """The opt-in W8A8 block-FP8 GEMMs (quantized activations) at prefill
    shapes: the config-2 gate/up expert GEMM at 8192 tokens (blocks of 64) and
    a dense 8192 x 7168 x 4096 GEMM; kernel time per call including the
    activation quantization, CUDA graph replay, CUDA events."""
    import torch

    from sglang_restomod_b200 import _lib, ops, synth

    out = {}
    stream = torch.cuda.current_stream()

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(reps):
            g.replay()
        end.record(stream)
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / reps
        del g
        return ms

    reps = max(20, min(args.steps, 100))
    shape = synth.CONFIG2
    tokens = 8192
    ids, _ = synth.route(tokens, shape.experts, shape.top_k, device, seed=200)
    x = synth.activations(tokens, shape.hidden, device, seed=100)
    q, s = synth.fp8_bank(shape.experts, 2 * shape.inter, shape.hidden, device, seed=10)
    sorted_ids, expert_ids, ntpp = ops.moe_align_block_size(ids, 64, shape.experts)
    routes = tokens * shape.top_k
    c = torch.empty(routes, shape.inter, dtype=torch.float16, device=device)

    def moe():
        ops.w8a8_moe_gemm(x, q, s, num_experts=shape.experts, sorted_token_ids=sorted_ids,
                          expert_ids=expert_ids, num_tokens_post_pad=ntpp, block_size=64,
                          top_k=shape.top_k, num_routes=routes, c=c,
                          gated_mode=_lib.GATED_FUSED)

    ms = timed(moe, reps)
    flops = 2 * routes * 2 * shape.inter * shape.hidden
    out["config2-T8192-gateup"] = {
        "us": ms * 1e3, "tflops": flops / (ms * 1e-3) / 1e12,
        "fp8_frac": flops / (ms * 1e-3) / 1e12 / fp8_tflops,
        "bf16_frac": flops / (ms * 1e-3) / 1e12 / bf16_tflops}
    del q, s, c, x
    m, k, n = 8192, 7168, 4096
    qd, sd = synth.fp8_bank(1, n, k, device, seed=3)
    xd = synth.activations(m, k, device, seed=4)
    yd = torch.empty(m, n // 2, dtype=torch.bfloat16, device=device)

    def dense():
        ops.w8a8_linear(xd, qd[0], sd[0], gated_mode=_lib.GATED_FUSED, out=yd)

    ms = timed(dense, reps)
    flops = 2 * m * n * k
    out["dense-8192x7168x4096-gated"] = {
        "us": ms * 1e3, "tflops": flops / (ms * 1e-3) / 1e12,
        "fp8_frac": flops / (ms * 1e-3) / 1e12 / fp8_tflops,
        "bf16_frac": flops / (ms * 1e-3) / 1e12 / bf16_tflops}
    del qd, sd, xd, yd
    torch.cuda.empty_cache()
    return out


def run_sweep(args, device, hbm_gbs, bf16_tflops, reuse_config4=None):
    """The headline configurations besides the main workload, each measured
    the same way (prefill points against the bf16 tensor burst peak, decode
    points against HBM)."""
    out = {}
    for name in SWEEP:
        if name == args.workload:
            continue
        reuse = reuse_config4 if name.startswith("config4") else None
        try:
            out[name] = sweep_point(name, args, device, hbm_gbs, bf16_tflops, reuse)
        except Exception as exc:  # noqa: BLE001 - a failed point is reported, not fatal
            out[name] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    try:
        fp8 = measure_fp8_peak(device)
        out["w8a8"] = {"fp8_peak_tflops": fp8, "fp8_peak_source": "torch._scaled_mm 8192^3 here",
                       **w8a8_points(args, device, fp8, bf16_tflops)}
    except Exception as exc:  # noqa: BLE001
        out["w8a8"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    return out


def ep_check(wl, device, world):
    """This rank's last output of the expert-parallel step against the same
    tokens through a single-GPU layer holding all experts (built from the
    same per-expert seeds); every token, rtol / atol 2e-2. Max over ranks."""
    import torch

    from sglang_restomod_b200.layer import QuantMoELayer

    full = QuantMoELayer.synthetic(wl.shape, wl.quant, device, first_expert=0,
                                   num_experts=wl.shape.experts, fuse_shared=False)
    want = full.forward(wl.x, wl.ids, wl.w).float()
    got = wl.out.float()
    torch.cuda.synchronize()
    err = (got - want).abs()
    bad = int((err > 2e-2 + 2e-2 * want.abs()).sum())
    stats = torch.tensor([float(err.max()), float(bad)], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    del full
    torch.cuda.empty_cache()
    return {"tokens": int(wl.tokens), "ranks": world, "max_err": float(stats[0]),
            "bad_elements_max_rank": int(stats[1]), "rtol": 2e-2, "atol": 2e-2,
            "ok": int(stats[1]) == 0}


def dist_teardown(world):
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# -------------------------------------------------------------------- main
def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config4-decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="no CUDA graph replay")
    ap.add_argument("--transport", default="peer", choices=["peer", "nccl"],
                    help="expert-parallel exchange at N > 1")
    ap.add_argument("--separate-shared", action="store_true",
                    help="run the shared expert as its own dense MLP instead of fused")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the other configurations' points (N=1)")
    ap.add_argument("--no-ep-check", action="store_true",
                    help="skip the untimed expert-parallel correctness pass (N>1)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")

    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        reference_arm(args, rank, world_env)
        return 0

    import torch

    rank, world, local_rank = dist_setup()
    device = torch.device("cuda", torch.cuda.current_device())
    spec = parse_workload(args.workload)
    spec["transport"] = args.transport
    spec["fuse_shared"] = not args.separate_shared

    if spec["kind"] == "dense":
        wl = DenseWorkload(spec, device)
    else:
        wl = MoEWorkload(spec, rank, world, device)
    step_bytes = wl.algorithmic()[0]
    copies = weight_copies(wl, step_bytes, world)
    wls = [wl] + [wl.replica() for _ in range(copies - 1)]
    torch.cuda.synchronize()

    from sglang_restomod_b200 import ops

    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        for w in wls:
            w.step()
    torch.cuda.synchronize()
    # One process per GPU replays the step as a CUDA graph, as a serving
    # engine does at decode. Under expert parallelism the peer transport has
    # no host sync and is replayed too (every rank in lockstep); the NCCL
    # transport reads its all-to-all split sizes on the host and runs eagerly.
    use_graph = not args.eager and (world == 1 or args.transport == "peer")
    ios = [w.e2e_io() for w in wls]
    graphs = []
    step_fns = [w.step for w in wls]
    e2e_fns = [[(lambda io=io, p=p: io.step(p)) for p in range(2)] for io in ios]
    if use_graph:
        for io in ios:
            io.load_first()
            for i in range(2):
                io.step(i)
        torch.cuda.synchronize()
        step_fns, e2e_fns, graphs = [], [], []
        for w, io in zip(wls, ios):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                w.step()
            graphs.append(g)
            step_fns.append(g.replay)
            pair = []
            for i in range(2):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    io.step(i)
                graphs.append(g)
                pair.append(g.replay)
            e2e_fns.append(pair)
        for _ in range(args.warmup):
            for f in step_fns:
                f()
        torch.cuda.synchronize()

    # clocks sampled over the whole timed phase: device-timed, e2e and
    # dominant-kernel legs
    sampler = ClockSampler(device.index)
    sampler.start()
    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("bench_timed")
    start.record(stream)
    for i in range(args.steps):
        step_fns[i % copies]()
    end.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world)

    # end-to-end: pinned host inputs in, result out, every step (double
    # buffered: copies of step i+1's inputs and step i-1's result overlap
    # step i's kernels; the first inputs and the last result are copied inside
    # the timed region too)
    # (with copies, step i runs copy i % copies on its buffer (i // copies) % 2)
    def e2e_run(steps):
        for io in ios[:min(copies, steps)]:
            io.load_first()
        for i in range(steps):
            e2e_fns[i % copies][(i // copies) % 2]()
        for r in range(min(copies, steps)):
            last = r + (steps - 1 - r) // copies * copies
            ios[r].drain((last // copies) % 2)

    e2e_run(4 * copies)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start.record(stream)
    e2e_run(args.steps)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(start.elapsed_time(end), world)

    # dominant kernel alone, CUDA events on its launch stream
    doms = [w.dominant() for w in wls]
    roofline = None
    runs = []
    hbm_gbs, bf16_tflops, peak_kind = measured_peaks()
    if doms[0] is not None:
        _, dom_bytes, dom_name, _ = doms[0]
        runs = []
        for run, _, _, _ in doms:
            for _ in range(3):
                run()
            torch.cuda.synchronize()
            if use_graph:
                g_dom = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g_dom):
                    run()
                graphs.append(g_dom)
                run = g_dom.replay
                run()
                torch.cuda.synchronize()
            runs.append(run)
        reps = max(args.steps, 20)
        start.record(stream)
        for i in range(reps):
            runs[i % copies]()
        end.record(stream)
        torch.cuda.synchronize()
        dom_ms = start.elapsed_time(end) / reps
        achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
        traffic = None
        tfile = ROOT / "profiles" / "traffic.json"
        if tfile.is_file() and world == 1:
            traffic = json.loads(tfile.read_text()).get(args.workload)
        roofline = {"bound": "hbm", "kernel": dom_name, "achieved": achieved, "peak": hbm_gbs,
                    "unit": "GB/s", "frac": achieved / hbm_gbs, "traffic": traffic,
                    "peak_source": peak_kind, "algorithmic_bytes": dom_bytes,
                    "launch_us": dom_ms * 1e3}
    sampler.stop()

    status = ops.workspace_status()
    if status != 0:
        raise SystemExit(f"kernels reported device error bits {status}")

    # Untimed correctness pass under expert parallelism: this rank's tokens
    # through one GPU's full-bank layer, compared with what the exchange gave.
    ep_result = None
    if world > 1 and spec["kind"] != "dense" and not args.no_ep_check:
        ep_result = ep_check(wl, device, world)
    # release every CUDA graph (and the closures replaying them)
    del graphs, step_fns, e2e_fns, runs
    if ep_result is not None and not ep_result["ok"]:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "error": "ep_check failed", "ep_check": ep_result}),
                  flush=True)
        dist_teardown(world)
        return 1

    sweep = None
    if world == 1 and not args.no_sweep:
        reuse = wl.layer if args.workload == "config4-decode" else None
        del wls, ios, doms
        sweep = run_sweep(args, device, hbm_gbs, bf16_tflops, reuse)

    alg_bytes, alg_flops, touched = wl.algorithmic()
    total_tokens = wl.tokens * world
    value = total_tokens / (elapsed_ms * 1e-3 / args.steps)
    e2e_value = total_tokens / (e2e_ms * 1e-3 / args.steps)
    step_s = elapsed_ms * 1e-3 / args.steps
    h2d, d2h = wl.io_bytes()

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        cpu_step, cpu_tokens, desc = cpu_reference_step(spec, threads)
        t0 = time.perf_counter()
        cpu_step()
        cpu_s = time.perf_counter() - t0
        cpu_baseline = {"value": cpu_tokens / cpu_s, "unit": "tokens/s", "cores": threads,
                        "kind": "port", "sample": "one step: " + desc}

    if rank == 0:
        if copies == 1:
            l2_note = "weights read per step exceed the 126 MB L2; no flush"
        else:
            l2_note = (f"weights read per step ({step_bytes / 1e6:.1f} MB) fit the 126 MB L2: "
                       f"{copies} copies of the layer's weights, rotated every step")
        config = {"workload": args.workload, "l2": l2_note, "weight_copies": copies}
        if spec["kind"] != "dense":
            s = spec["shape"]
            config.update({"hidden": s.hidden, "inter": s.inter, "experts": s.experts,
                           "top_k": s.top_k, "shared_inter": s.shared_inter,
                           "tokens_per_rank": wl.tokens,
                           "quant": "block-fp8" if spec["quant"] == 0 else "nvfp4",
                           "parallelism": f"ep{world}", "experts_touched_per_rank": touched})
        else:
            config.update({"K": spec["k"], "N": spec["n"], "M": spec["m"], "quant": "block-fp8"})
        config["layer_hbm_frac"] = (alg_bytes / step_s / 1e9) / hbm_gbs
        config["layer_algorithmic_bytes"] = alg_bytes
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3*f16->f32" if spec.get("quant", 0) == 0 else "e2m1*f16->f32",
            "data": "synthetic", "config": config, "roofline": roofline,
            "cpu_baseline": cpu_baseline,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world},
            "clocks": sampler.summary(),
            "cuda_graph": use_graph,
            "gpu_launches": wl.launches_per_step() * args.steps,
        }
        if ep_result is not None:
            line["ep_check"] = ep_result
        if sweep is not None:
            line["sweep"] = sweep
        print(json.dumps(line), flush=True)
    dist_teardown(world)
    return 0


if __name__ == "__main__":
    sys.exit(main())
