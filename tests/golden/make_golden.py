"""Generate the golden fixtures in this directory from the reference itself.

    PYTHONPATH=<sglang-restomod checkout> python tests/golden/make_golden.py

Runs the reference's own CPU code (it must be importable; sglang is not
needed) and stores inputs and outputs as small .npz files. The tests read
only the .npz files, so they run anywhere - this script is the only thing
that needs the reference, and it is not run by the test suite.

Reference functions exercised (paths inside the sglang-restomod tree):
* quant/sm70_fp8_moe/check.py: _quant_block, _dequant, _reference
* quant/sm70_fp8_lm_head/__init__.py: _quantize
* quant/sm70_fp8_moe/method.py: SM70Fp8MoEMethod.apply, run on the CPU with
  the sglang base classes faked (the pattern of the reference's own tests,
  e.g. tests/test_moe_align_sm70.py:13-17) and the expert GEMM replaced by a
  CPU implementation of its documented contract
  (quant/sm70_fp8_moe/README.md:23-58)
* quant/sm70_fp4_moe/check.py: _quantize, _dequant
* quant/sm70_fp4_moe/scales.py: encode_scales, encode_global_scale, with the
  golden table of tests/test_sm70_fp4_scales.py:33-42
"""

from __future__ import annotations

import sys
import types
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _u8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy().copy()


def _install_fake_sglang() -> None:
    names = [
        "sglang",
        "sglang.srt",
        "sglang.srt.layers",
        "sglang.srt.layers.moe",
        "sglang.srt.layers.moe.token_dispatcher",
        "sglang.srt.layers.quantization",
        "sglang.srt.layers.quantization.fp8",
    ]
    for name in names:
        sys.modules.setdefault(name, types.ModuleType(name))

    class StandardCombineInput:
        def __init__(self, hidden_states):
            self.hidden_states = hidden_states

    class Fp8MoEMethod:
        def __init__(self, quant_config):
            self.quant_config = quant_config

    sys.modules["sglang.srt.layers.moe.token_dispatcher"].StandardCombineInput = StandardCombineInput
    sys.modules["sglang.srt.layers.quantization.fp8"].Fp8MoEMethod = Fp8MoEMethod


def fp8_quant() -> None:
    from sglang_restomod.quant.sm70_fp8_lm_head import _quantize
    from sglang_restomod.quant.sm70_fp8_moe import check as c8

    torch.manual_seed(11)
    w = (torch.randn(256, 256) * 0.2).half()
    w[:128, :128] *= 40.0  # a block with a different scale
    q, s = c8._quant_block(w)
    deq = c8._dequant(q, s)
    torch.manual_seed(12)
    head = (torch.randn(256, 256) * 0.05).half()
    hq, hs = _quantize(head)
    np.savez_compressed(
        OUT / "fp8_quant.npz",
        w=_u8(w), q=_u8(q), s=s.numpy(), deq=deq.numpy(),
        head=_u8(head), head_q=_u8(hq), head_s=hs.numpy(),
    )


def _fp8_bank(experts, n, k, seed):
    from sglang_restomod.quant.sm70_fp8_moe import check as c8

    torch.manual_seed(seed)
    qs, ss = [], []
    for _ in range(experts):
        q, s = c8._quant_block((torch.randn(n, k) * 0.2).half())
        qs.append(q)
        ss.append(s)
    return torch.stack(qs), torch.stack(ss)


def fp8_moe_check() -> None:
    from sglang_restomod.quant.sm70_fp8_moe import check as c8

    experts, hidden, inter, top_k, tokens = 4, 128, 128, 3, 8
    w13, s13 = _fp8_bank(experts, 2 * inter, hidden, 1)
    w2, s2 = _fp8_bank(experts, hidden, inter, 2)
    torch.manual_seed(7)
    x = (torch.randn(tokens, hidden) * 0.5).half()
    ids = torch.randint(0, experts, (tokens, top_k), dtype=torch.int32)
    weights = torch.rand(tokens, top_k, dtype=torch.float32)
    ids_ep = ids.clone()
    ids_ep[0, 0] = -1
    ids_ep[1, -1] = -1
    ref = c8._reference(x, ids, weights, w13, s13, w2, s2)
    ref_ep = c8._reference(x, ids_ep, weights, w13, s13, w2, s2)
    np.savez_compressed(
        OUT / "fp8_moe_check.npz",
        x=_u8(x), ids=ids.numpy(), ids_ep=ids_ep.numpy(), weights=weights.numpy(),
        w13=_u8(w13), s13=s13.numpy(), w2=_u8(w2), s2=s2.numpy(),
        ref=ref.numpy(), ref_ep=ref_ep.numpy(),
    )


def fp8_moe_method() -> None:
    """Run the reference's SM70Fp8MoEMethod.apply on the CPU."""
    _install_fake_sglang()
    from sglang_restomod.quant.sm70_fp8_moe import check as c8
    from sglang_restomod.quant.sm70_fp8_moe import method as m8

    record = {}

    def fake_gemm(out, sorted_input, offsets, experts, *, gated_silu=True):
        if gated_silu:
            record["offsets"] = offsets.clone()
            record["first_col"] = sorted_input[:, 0].float().clone()
        for e in range(experts.q.shape[0]):
            lo, hi = int(offsets[e]), int(offsets[e + 1])
            if hi <= lo:
                continue
            y = sorted_input[lo:hi].float() @ c8._dequant(experts.q[e], experts.s[e]).T
            if gated_silu:
                half = y.shape[1] // 2
                y = torch.nn.functional.silu(y[:, :half]) * y[:, half:]
            out[lo:hi] = y.to(out.dtype)

    m8.fp8_apply = fake_gemm

    local, hidden, inter, top_k = 4, 128, 128, 3
    w13, s13 = _fp8_bank(local, 2 * inter, hidden, 3)
    w2, s2 = _fp8_bank(local, hidden, inter, 4)

    def run(tokens, global_experts, drop, output_scale, seed):
        meth = object.__new__(m8.SM70Fp8MoEMethod)
        meth.use_turbomind = True
        meth.output_scale = output_scale
        meth.moe_runner_config = SimpleNamespace(num_experts=global_experts)
        layer = SimpleNamespace(
            sm70_num_experts=local,
            sm70_hidden_size=hidden,
            sm70_intermediate_size=inter,
            sm70_top_k=top_k,
            w13_tm_weight=torch.empty(0),
            w13_quant=SimpleNamespace(q=w13, s=s13),
            w2_quant=SimpleNamespace(q=w2, s=s2),
        )
        m8.SM70Fp8MoEMethod._allocate_buffers(layer, 32)
        gen = torch.Generator().manual_seed(seed)
        x = (torch.randn(tokens, hidden, generator=gen) * 0.5).half()
        x[:, 0] = torch.arange(tokens).half()  # recovers the gather order
        ids = torch.stack(
            [torch.randperm(local, generator=gen)[:top_k] for _ in range(tokens)]
        ).to(torch.int32)
        if drop == "some":
            mask = torch.rand(tokens, top_k, generator=gen) < 0.3
            ids[mask] = -1
        elif drop == "all":
            ids[:] = -1
        weights = torch.rand(tokens, top_k, generator=gen, dtype=torch.float32)
        record.clear()
        out = meth.apply(
            layer,
            SimpleNamespace(
                hidden_states=x,
                topk_output=SimpleNamespace(topk_ids=ids, topk_weights=weights),
            ),
        ).hidden_states
        offsets = record.get("offsets", torch.zeros(local + 1, dtype=torch.int32))
        order = record.get("first_col", torch.zeros(0))
        return dict(
            x=_u8(x), ids=ids.numpy(), weights=weights.numpy(), out=_u8(out),
            offsets=offsets.numpy(), order=order.numpy(),
            output_scale=np.float32(output_scale if output_scale is not None else 1.0),
        )

    cases = {
        "dense": run(8, local, None, None, 21),
        "ep_clamp": run(8, 2 * local, "some", None, 22),
        "ep_compact": run(80, 2 * local, "some", None, 23),
        "empty": run(3, 2 * local, "all", None, 24),
        "scaled": run(8, local, None, 2.5, 25),
    }
    flat = {f"{case}__{key}": value for case, d in cases.items() for key, value in d.items()}
    np.savez_compressed(
        OUT / "fp8_moe_method.npz",
        w13=_u8(w13), s13=s13.numpy(), w2=_u8(w2), s2=s2.numpy(), **flat,
    )


def nvfp4_quant() -> None:
    from sglang_restomod.quant.sm70_fp4_moe import check as c4

    torch.manual_seed(5)
    w = torch.randn(128, 256).half()
    w[3] *= 0.01  # small groups exercise small e4m3 scales
    packed, scales, codes = c4._quantize(w)
    deq = c4._dequant(packed, scales)
    np.savez_compressed(
        OUT / "nvfp4_quant.npz",
        w=_u8(w), packed=packed.numpy(), scales=_u8(scales), codes=codes.numpy().astype(np.int8),
        deq=_u8(deq),
    )


def nvfp4_scales() -> None:
    from sglang_restomod.quant.sm70_fp4_moe.scales import encode_global_scale, encode_scales

    # (scale, byte) golden table of tests/test_sm70_fp4_scales.py:33-42
    golden = [(1.0, 176), (0.5, 168), (2.0, 184), (3.0, 188), (0.25, 160), (448.0, 246),
              (0.0, 0), (6.0, 196)]
    values = torch.tensor([v for v, _ in golden], dtype=torch.float32)
    table = values.to(torch.float8_e4m3fn).reshape(1, 1, len(golden))
    enc_table, _ = encode_scales(table, torch.float16)
    torch.manual_seed(0)
    rnd = (torch.rand(2, 3, 64) * 400).to(torch.float8_e4m3fn)
    enc_rnd, _ = encode_scales(rnd, torch.float16)
    gs = torch.tensor([1.0, 0.5, 2.0, 0.0123], dtype=torch.float32)
    np.savez_compressed(
        OUT / "nvfp4_scales.npz",
        golden_scale=values.numpy(), golden_byte=np.array([b for _, b in golden], np.uint8),
        table=_u8(table), enc_table=_u8(enc_table), rnd=_u8(rnd), enc_rnd=_u8(enc_rnd),
        gs=gs.numpy(), enc_gs=encode_global_scale(gs, torch.float16).numpy(),
    )


def main() -> None:
    fp8_quant()
    fp8_moe_check()
    fp8_moe_method()
    nvfp4_quant()
    nvfp4_scales()
    for path in sorted(OUT.glob("*.npz")):
        print(f"{path.name}: {path.stat().st_size} bytes")


if __name__ == "__main__":
    main()
