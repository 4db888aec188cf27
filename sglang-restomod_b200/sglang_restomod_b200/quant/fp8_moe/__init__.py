"""Block-FP8 expert GEMM on B200 (the ``fp8_moe`` component).

Same surface as the reference's ``sglang_restomod/quant/sm70_fp8_moe/__init__.py``
(``prepare_experts`` / ``gemm`` / ``apply`` over expert-sorted rows and
``offsets[E+1]``), on the library's streaming kernel instead of the closed
TurboMind binary:

* weights per expert ``[N, K]`` e4m3 with ``[N/128, K/128]`` fp32 scales;
* ``prepare_experts(..., interleave_gated_silu=True)`` lays a ``[2I, K]``
  gate/up bank out so the GEMM writes ``silu(y[:, :I]) * y[:, I:]``
  (``quant/sm70_fp8_moe/README.md:53-56``);
* ``gemm`` consumes rows already sorted by expert. Graph-safe: the offsets
  are turned into routing blocks on the device.
"""

from __future__ import annotations

from dataclasses import dataclass

GROUP = 128


def _check_gemm_shape(k: int, n: int, group_size: int = GROUP, gated: bool = False) -> None:
    """Reject an expert GEMM the kernel cannot represent (messages as in
    ``quant/sm70_fp8_moe/__init__.py:48-62``; the B200 unit is 128 rows)."""
    if k <= 0 or n <= 0:
        raise RuntimeError(f"B200 FP8 MoE needs positive K and N, got K={k} N={n}.")
    if group_size != GROUP:
        raise RuntimeError(f"B200 FP8 MoE needs [128, 128] weight blocks, got {group_size}.")
    if k % group_size:
        raise RuntimeError(
            f"B200 FP8 MoE needs K a multiple of the {group_size}-wide quantization group, got K={k}."
        )
    unit = 256 if gated else 128
    if n % unit:
        raise RuntimeError(f"B200 FP8 MoE needs N a multiple of {unit}, got N={n}.")


@dataclass(frozen=True)
class Experts:
    """Prepared expert bank: streamed weights + the checkpoint's block scales."""

    packed: object
    scales: object
    num_experts: int
    k: int
    n: int
    group_size: int
    gated: bool


def prepare_experts(weights, scales, *, group_size: int = GROUP,
                    interleave_gated_silu: bool = True) -> Experts:
    """``weights`` ``[E, N, K]`` e4m3, ``scales`` ``[E, N/128, K/128]`` fp32."""
    from ..._common import b200_ops

    experts, n, k = (int(d) for d in weights.shape)
    _check_gemm_shape(k, n, group_size, gated=interleave_gated_silu)
    if tuple(scales.shape) != (experts, n // group_size, k // group_size):
        raise RuntimeError(
            f"B200 FP8 MoE scales must be [{experts}, {n // group_size}, {k // group_size}], "
            f"got {tuple(scales.shape)}"
        )
    packed = b200_ops().fp8_prepack(weights.contiguous(), gated=interleave_gated_silu)
    return Experts(packed=packed, scales=scales.float().contiguous(), num_experts=experts, k=k,
                   n=n, group_size=group_size, gated=interleave_gated_silu)


def _check_call_matches_prepared(k: int, n: int, experts: Experts) -> None:
    if k != experts.k or n != experts.n:
        raise RuntimeError(
            "B200 FP8 MoE: gemm K/N disagree with the prepared experts "
            f"(prepared K={experts.k} N={experts.n}, got K={k} N={n})."
        )


def gemm(out, sorted_input, expert_offsets, experts: Experts, *, k, n, gated_silu=True,
         block_size: int = 16):
    """Expert GEMM over expert-sorted rows into ``out`` (sorted order)."""
    import torch

    from ... import _lib
    from ..._common import b200_ops

    k, n = int(k), int(n)
    _check_gemm_shape(k, n, experts.group_size, gated=gated_silu)
    _check_call_matches_prepared(k, n, experts)
    if bool(gated_silu) != experts.gated:
        raise RuntimeError("gated_silu must match the interleave the experts were prepared with")
    rows = int(sorted_input.shape[0])
    if rows == 0:
        return out
    # Row r belongs to the expert e with offsets[e] <= r < offsets[e+1].
    offsets = expert_offsets.to(torch.int32)
    row_expert = torch.searchsorted(offsets[1:].contiguous(),
                                    torch.arange(rows, device=offsets.device, dtype=torch.int32),
                                    right=True).to(torch.int32)
    sorted_ids, expert_ids, ntpp = b200_ops().moe_align_block_size(row_expert, block_size,
                                                            experts.num_experts)
    b200_ops().moe_gemm(sorted_input.contiguous(), experts.packed, n, quant=_lib.QUANT_FP8_BLOCK,
                 num_experts=experts.num_experts, sorted_token_ids=sorted_ids,
                 expert_ids=expert_ids, num_tokens_post_pad=ntpp, block_size=block_size, top_k=1,
                 num_routes=rows, c=out, scales=experts.scales,
                 gated_mode=_lib.GATED_FUSED if gated_silu else _lib.GATED_NONE)
    return out


def apply(out, sorted_input, expert_offsets, experts: Experts, *, gated_silu=True):
    """Like :func:`gemm`, inferring ``k`` and ``n`` from the tensors."""
    k = int(sorted_input.shape[1])
    n = int(out.shape[1] * 2 if gated_silu else out.shape[1])
    return gemm(out, sorted_input, expert_offsets, experts, k=k, n=n, gated_silu=gated_silu)


def register() -> None:
    """Component entry point: route block-FP8 FusedMoE layers to the B200 method."""
    from .method import install

    install()
