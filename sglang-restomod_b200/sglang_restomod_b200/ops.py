"""Torch-facing wrappers of the libb200moe C ABI.

Every function here takes CUDA tensors, validates what the C ABI cannot see
(dtype, device, contiguity), and calls the library on the current CUDA stream.
Outputs are allocated here unless the caller passes them (the reference's
``Tensor(a!) out`` convention, ``quant/sm70_fp8_moe/shim.cpp:50-56``).

Workspaces are cached per device, sized once and zero-filled; a call that
needs a larger one grows it, except during CUDA-graph capture, where growing
would be an allocation inside the capture and raises instead (size them up
front with :func:`reserve_workspace`, as the reference sizes its decode
workspace for the largest capture batch, ``decode_gemv.py:170-180``).
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

_DTYPE_CODE = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}
_WS_LOCK = threading.Lock()
_WORKSPACES: dict[int, torch.Tensor] = {}


def _vp(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _code(t: torch.Tensor, what: str) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise TypeError(f"{what} must be bf16 or f16, got {t.dtype}") from None


def _cuda(t: torch.Tensor, what: str) -> None:
    if not (isinstance(t, torch.Tensor) and t.is_cuda):
        raise ValueError(f"{what} must be a CUDA tensor")


def _contig(t: torch.Tensor, what: str) -> None:
    _cuda(t, what)
    if not t.is_contiguous():
        raise ValueError(f"{what} must be contiguous")


def lib():
    return _lib.load()


def num_sms() -> int:
    return int(lib().b200_num_sms())


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Per-device zero-filled workspace of at least ``nbytes`` bytes."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    with _WS_LOCK:
        ws = _WORKSPACES.get(index)
        if ws is not None and ws.numel() >= nbytes:
            return ws
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                f"b200 workspace needs {nbytes} bytes during CUDA-graph capture; "
                "call reserve_workspace() before capturing"
            )
        size = max(nbytes, 0 if ws is None else ws.numel())
        ws = torch.zeros(size + 256, dtype=torch.uint8, device=torch.device("cuda", index))
        # The library wants a 256-byte aligned base.
        offset = (-ws.data_ptr()) % 256
        ws = ws[offset : offset + size]
        _WORKSPACES[index] = ws
        return ws


def reserve_workspace(nbytes: int, device: torch.device | None = None) -> torch.Tensor:
    return workspace(nbytes, device or torch.device("cuda", torch.cuda.current_device()))


def workspace_status(device: torch.device | None = None, reset: bool = True) -> int:
    """Device error bits recorded by the kernels (0 = none). Synchronizes."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    ws = _WORKSPACES.get(device.index if device.index is not None else torch.cuda.current_device())
    if ws is None:
        return 0
    bits = ctypes.c_int32(0)
    _lib.check(lib().b200_workspace_status(_vp(ws), ctypes.byref(bits), int(reset), _stream(ws.device)))
    return int(bits.value)


# ----------------------------------------------------------------- routing
def align_capacity(numel: int, num_experts: int, block_size: int) -> tuple[int, int]:
    cap = numel + min(numel, num_experts) * (block_size - 1)
    return cap, (cap + block_size - 1) // block_size


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int, out=None):
    """(sorted_token_ids, expert_ids, num_tokens_post_pad) for ``topk_ids``."""
    _contig(topk_ids, "topk_ids")
    if topk_ids.dtype != torch.int32:
        raise TypeError(f"topk_ids must be int32, got {topk_ids.dtype}")
    numel = topk_ids.numel()
    cap, blocks = align_capacity(numel, num_experts, block_size)
    if out is None:
        dev = topk_ids.device
        sorted_ids = torch.empty(cap, dtype=torch.int32, device=dev)
        expert_ids = torch.empty(blocks, dtype=torch.int32, device=dev)
        ntpp = torch.empty(1, dtype=torch.int32, device=dev)
    else:
        sorted_ids, expert_ids, ntpp = out
    _lib.check(
        lib().b200_moe_align_block_size(
            _vp(topk_ids), numel, num_experts, block_size, _vp(sorted_ids), sorted_ids.numel(),
            _vp(expert_ids), expert_ids.numel(), _vp(ntpp), _stream(topk_ids.device),
        )
    )
    return sorted_ids, expert_ids, ntpp


# ----------------------------------------------------------------- combine
_LOGIT_CODE = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16,
               torch.float32: _lib.DTYPE_F32}


def topk_route(router_logits: torch.Tensor, top_k: int, *, scoring: int = _lib.SCORING_SOFTMAX,
               renormalize: bool = True, correction_bias: torch.Tensor | None = None,
               out: tuple[torch.Tensor, torch.Tensor] | None = None):
    """(topk_ids int32 [T, k], topk_weights fp32 [T, k]) from router logits [T, E]."""
    _contig(router_logits, "router_logits")
    try:
        code = _LOGIT_CODE[router_logits.dtype]
    except KeyError:
        raise TypeError(f"router_logits must be bf16, f16 or f32, got {router_logits.dtype}") from None
    tokens, experts = (int(d) for d in router_logits.shape)
    if correction_bias is not None:
        _contig(correction_bias, "correction_bias")
        if correction_bias.dtype != torch.float32 or correction_bias.numel() != experts:
            raise ValueError("correction_bias must be fp32 [num_experts]")
    if out is None:
        ids = torch.empty(tokens, top_k, dtype=torch.int32, device=router_logits.device)
        w = torch.empty(tokens, top_k, dtype=torch.float32, device=router_logits.device)
    else:
        ids, w = out
    _lib.check(
        lib().b200_topk_route(
            _vp(router_logits), code, tokens, experts, top_k, scoring, int(renormalize),
            _vp(correction_bias), _vp(ids), _vp(w), _stream(router_logits.device),
        )
    )
    return ids, w


def topk_route_grouped(router_logits: torch.Tensor, top_k: int, num_expert_group: int,
                       topk_group: int, *, scoring: int = _lib.SCORING_SOFTMAX,
                       renormalize: bool = True, correction_bias: torch.Tensor | None = None):
    """Grouped top-k (upstream grouped_topk / biased_grouped_topk): only the
    ``topk_group`` best of ``num_expert_group`` expert groups are selectable."""
    _contig(router_logits, "router_logits")
    try:
        code = _LOGIT_CODE[router_logits.dtype]
    except KeyError:
        raise TypeError(f"router_logits must be bf16, f16 or f32, got {router_logits.dtype}") from None
    tokens, experts = (int(d) for d in router_logits.shape)
    if correction_bias is not None:
        _contig(correction_bias, "correction_bias")
        if correction_bias.dtype != torch.float32 or correction_bias.numel() != experts:
            raise ValueError("correction_bias must be fp32 [num_experts]")
    ids = torch.empty(tokens, top_k, dtype=torch.int32, device=router_logits.device)
    w = torch.empty(tokens, top_k, dtype=torch.float32, device=router_logits.device)
    _lib.check(
        lib().b200_topk_route_grouped(
            _vp(router_logits), code, tokens, experts, top_k, scoring, int(renormalize),
            _vp(correction_bias), int(num_expert_group), int(topk_group), _vp(ids), _vp(w),
            _stream(router_logits.device),
        )
    )
    return ids, w


def append_shared_route(topk_ids: torch.Tensor, topk_weights: torch.Tensor, shared_id: int,
                        shared_weight: float = 1.0):
    """[T, k] routes -> [T, k + 1] with one route per token to ``shared_id``."""
    _contig(topk_ids, "topk_ids")
    _contig(topk_weights, "topk_weights")
    tokens, top_k = (int(d) for d in topk_ids.shape)
    ids = torch.empty(tokens, top_k + 1, dtype=torch.int32, device=topk_ids.device)
    w = torch.empty(tokens, top_k + 1, dtype=torch.float32, device=topk_ids.device)
    _lib.check(
        lib().b200_append_shared_route(_vp(topk_ids), _vp(topk_weights), tokens, top_k, shared_id,
                                       float(shared_weight), _vp(ids), _vp(w),
                                       _stream(topk_ids.device))
    )
    return ids, w


def moe_sum_reduce(input_tensor: torch.Tensor, output_tensor: torch.Tensor,
                   routed_scaling_factor: float = 1.0) -> torch.Tensor:
    """``out[t] = rsf * sum_k in[t, k]`` (``quant/sm70_fp4_moe/sum_reduce.py:84-123``)."""
    _contig(input_tensor, "input")
    _contig(output_tensor, "output")
    if input_tensor.dtype != output_tensor.dtype:
        raise ValueError(
            f"moe_sum_reduce dtype mismatch: input {input_tensor.dtype}, output {output_tensor.dtype}"
        )
    tokens, top_k, hidden = input_tensor.shape
    if tuple(output_tensor.shape) != (tokens, hidden):
        raise ValueError(f"output must be [{tokens}, {hidden}], got {tuple(output_tensor.shape)}")
    _lib.check(
        lib().b200_moe_sum_reduce(
            _vp(input_tensor), _vp(output_tensor), tokens, top_k, hidden,
            _code(input_tensor, "input"), float(routed_scaling_factor), _stream(input_tensor.device),
        )
    )
    return output_tensor


def moe_combine(routed: torch.Tensor, topk_ids: torch.Tensor | None, num_experts: int,
                routed_scaling_factor: float = 1.0, shared_out: torch.Tensor | None = None,
                out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16):
    """Sum weighted per-route rows ``routed [T*k, H]`` over valid slots."""
    _contig(routed, "routed")
    if topk_ids is None:
        raise ValueError("topk_ids is required to know top_k")
    _contig(topk_ids, "topk_ids")
    tokens, top_k = topk_ids.shape
    hidden = routed.shape[-1]
    if out is None:
        out = torch.empty(tokens, hidden, dtype=out_dtype, device=routed.device)
    if shared_out is not None:
        _contig(shared_out, "shared_out")
    _lib.check(
        lib().b200_moe_combine(
            _vp(routed), _code(routed, "routed"), _vp(topk_ids), num_experts, tokens, top_k, hidden,
            float(routed_scaling_factor), _vp(shared_out),
            _code(shared_out, "shared_out") if shared_out is not None else 0,
            _vp(out), _code(out, "out"), _stream(routed.device),
        )
    )
    return out


# ----------------------------------------------------------------- prepack
def fp8_prepack(w: torch.Tensor, gated: bool) -> torch.Tensor:
    """e4m3 ``[E, N, K]`` (or ``[N, K]``) -> streamed bank ``[E, N*K]`` uint8."""
    _contig(w, "weight")
    if w.dtype != torch.float8_e4m3fn:
        raise TypeError(f"weight must be float8_e4m3fn, got {w.dtype}")
    w3 = w.unsqueeze(0) if w.dim() == 2 else w
    e, n, k = (int(d) for d in w3.shape)
    nbytes = int(lib().b200_fp8_packed_bytes(e, n, k))
    out = torch.empty(e, nbytes // e, dtype=torch.uint8, device=w.device)
    _lib.check(lib().b200_fp8_prepack(_vp(w3), e, n, k, int(gated), _vp(out), _stream(w.device)))
    return out


def nvfp4_prepack(w: torch.Tensor, scales: torch.Tensor, gated: bool) -> torch.Tensor:
    """ModelOpt ``[E, N, K/2]`` uint8 + ``[E, N, K/16]`` e4m3 -> streamed bank."""
    _contig(w, "weight")
    _contig(scales, "scales")
    if w.dtype != torch.uint8:
        raise TypeError(f"packed NVFP4 weight must be uint8, got {w.dtype}")
    if scales.dtype != torch.float8_e4m3fn:
        raise TypeError(f"NVFP4 scales must be float8_e4m3fn, got {scales.dtype}")
    w3 = w.unsqueeze(0) if w.dim() == 2 else w
    s3 = scales.unsqueeze(0) if scales.dim() == 2 else scales
    e, n, half_k = (int(d) for d in w3.shape)
    k = 2 * half_k
    if tuple(s3.shape) != (e, n, k // 16):
        raise ValueError(f"scales must be [{e}, {n}, {k // 16}], got {tuple(s3.shape)}")
    nbytes = int(lib().b200_nvfp4_packed_bytes(e, n, k))
    if nbytes < 0:
        raise ValueError(f"NVFP4 bank needs N and K multiples of 128, got N={n} K={k}")
    out = torch.empty(e, nbytes // e, dtype=torch.uint8, device=w.device)
    _lib.check(
        lib().b200_nvfp4_prepack(_vp(w3), _vp(s3), e, n, k, int(gated), _vp(out), _stream(w.device))
    )
    return out


# ------------------------------------------------------------------- GEMMs
def gemm_workspace_bytes(convert_elems: int) -> int:
    return int(lib().b200_gemm_workspace_bytes(int(convert_elems)))


def linear(x: torch.Tensor, packed: torch.Tensor, n: int, *, quant: int,
           scales: torch.Tensor | None = None, global_scale: torch.Tensor | None = None,
           gated_mode: int = _lib.GATED_NONE, out: torch.Tensor | None = None,
           out_dtype: torch.dtype | None = None, loads_only: bool = False) -> torch.Tensor:
    """Dense ``y = x . dequant(W)^T`` on a prepacked bank (one expert).
    ``loads_only``: the call's data-movement floor (no math, ``out`` untouched)."""
    _contig(x, "x")
    x2 = x.reshape(-1, x.shape[-1])
    m, k = (int(d) for d in x2.shape)
    cols = n // 2 if gated_mode == _lib.GATED_FUSED else n
    if out is None:
        out = torch.empty(m, cols, dtype=out_dtype or x.dtype, device=x.device)
    ws = workspace(gemm_workspace_bytes(m * k if x.dtype == torch.bfloat16 else 0), x.device)
    fn = lib().b200_linear_loads_only if loads_only else lib().b200_linear
    _lib.check(
        fn(
            quant, _vp(x2), _code(x2, "x"), m, k, _vp(packed), _vp(scales), _vp(global_scale), n,
            gated_mode, _vp(out), _code(out, "out"), _vp(ws), ws.numel(), _stream(x.device),
        )
    )
    return out.reshape(*x.shape[:-1], cols)


def moe_gemm(a: torch.Tensor, packed: torch.Tensor, n: int, *, quant: int, num_experts: int,
             sorted_token_ids: torch.Tensor, expert_ids: torch.Tensor,
             num_tokens_post_pad: torch.Tensor, block_size: int, top_k: int, num_routes: int,
             c: torch.Tensor, scales: torch.Tensor | None = None,
             global_scale: torch.Tensor | None = None, topk_weights: torch.Tensor | None = None,
             mul_topk_weights: bool = False, gated_mode: int = _lib.GATED_NONE,
             loads_only: bool = False) -> torch.Tensor:
    """Grouped expert GEMM with ``moe_wna16_marlin_gemm`` routing semantics.
    ``loads_only``: the call's data-movement floor (no math, ``c`` untouched)."""
    _contig(a, "a")
    _contig(c, "c")
    a_rows, k = (int(d) for d in a.reshape(-1, a.shape[-1]).shape)
    if topk_weights is not None:
        _contig(topk_weights, "topk_weights")
        if topk_weights.dtype != torch.float32:
            topk_weights = topk_weights.float().contiguous()
    if c.shape[0] < num_routes:
        raise ValueError(f"c has {c.shape[0]} rows, the routes need {num_routes}")
    if mul_topk_weights and (topk_weights is None or topk_weights.numel() < num_routes):
        raise ValueError("mul_topk_weights needs one topk weight per route")
    groups = min(expert_ids.numel(), sorted_token_ids.numel() // block_size)
    ws = workspace(gemm_workspace_bytes(a_rows * k if a.dtype == torch.bfloat16 else 0), a.device)
    fn = lib().b200_moe_gemm_loads_only if loads_only else lib().b200_moe_gemm
    _lib.check(
        fn(
            quant, _vp(a), _code(a, "a"), a_rows, k, _vp(packed), _vp(scales), _vp(global_scale),
            num_experts, n, gated_mode, _vp(sorted_token_ids), _vp(expert_ids), groups,
            _vp(num_tokens_post_pad), block_size, top_k, num_routes, _vp(topk_weights),
            int(mul_topk_weights), _vp(c), _code(c, "c"), c.shape[-1], _vp(ws), ws.numel(),
            _stream(a.device),
        )
    )
    return c


def moe_layer_workspace_bytes(tokens: int, hidden: int, inter: int, num_experts: int,
                              top_k: int, block_size: int) -> int:
    return int(lib().b200_moe_layer_workspace_bytes(tokens, hidden, inter, num_experts, top_k, block_size))


def moe_layer_forward(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, *,
                      quant: int, num_experts: int, inter: int, w13: torch.Tensor,
                      w2: torch.Tensor, w13_scales: torch.Tensor | None = None,
                      w2_scales: torch.Tensor | None = None,
                      w13_global: torch.Tensor | None = None,
                      w2_global: torch.Tensor | None = None, block_size: int = 16,
                      routed_scaling_factor: float = 1.0, shared_out: torch.Tensor | None = None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """align -> gate_up(+SiLU*up) -> down(x weight) -> combine, one library call."""
    _contig(x, "x")
    _contig(topk_ids, "topk_ids")
    _contig(topk_weights, "topk_weights")
    if topk_ids.dtype != torch.int32:
        raise TypeError(f"topk_ids must be int32, got {topk_ids.dtype}")
    if topk_weights.dtype != torch.float32:
        raise TypeError(f"topk_weights must be float32, got {topk_weights.dtype}")
    tokens, hidden = (int(d) for d in x.shape)
    top_k = int(topk_ids.shape[1])
    if out is None:
        out = torch.empty(tokens, hidden, dtype=x.dtype, device=x.device)
    if shared_out is not None:
        _contig(shared_out, "shared_out")
    ws = workspace(
        moe_layer_workspace_bytes(tokens, hidden, inter, num_experts, top_k, block_size), x.device
    )
    _lib.check(
        lib().b200_moe_layer_forward(
            quant, _vp(x), _code(x, "x"), tokens, hidden, inter, _vp(topk_ids), _vp(topk_weights),
            top_k, num_experts, _vp(w13), _vp(w13_scales), _vp(w13_global), _vp(w2),
            _vp(w2_scales), _vp(w2_global), block_size, float(routed_scaling_factor),
            _vp(shared_out), _code(shared_out, "shared_out") if shared_out is not None else 0,
            _vp(out), _code(out, "out"), _vp(ws), ws.numel(), _stream(x.device),
        )
    )
    return out


def moe_layer_forward_fused_shared(x: torch.Tensor, topk_ids: torch.Tensor,
                                   topk_weights: torch.Tensor, *, quant: int, num_experts: int,
                                   inter: int, w13: torch.Tensor, w2: torch.Tensor,
                                   w13_scales: torch.Tensor | None = None,
                                   w2_scales: torch.Tensor | None = None, block_size: int = 16,
                                   routed_scaling_factor: float = 1.0,
                                   shared_route_weight: float | None = None,
                                   out: torch.Tensor | None = None):
    """The layer with the shared expert as the banks' last expert (index
    ``num_experts``, the routed count): one more route per token, appended
    inside the call. Returns (out, extended ids, extended weights), the
    routes [T, top_k + 1] the layer ran on."""
    _contig(x, "x")
    _contig(topk_ids, "topk_ids")
    _contig(topk_weights, "topk_weights")
    if topk_ids.dtype != torch.int32:
        raise TypeError(f"topk_ids must be int32, got {topk_ids.dtype}")
    if topk_weights.dtype != torch.float32:
        raise TypeError(f"topk_weights must be float32, got {topk_weights.dtype}")
    tokens, hidden = (int(d) for d in x.shape)
    top_k = int(topk_ids.shape[1])
    if shared_route_weight is None:
        shared_route_weight = 1.0 / routed_scaling_factor
    ids = torch.empty(tokens, top_k + 1, dtype=torch.int32, device=x.device)
    w = torch.empty(tokens, top_k + 1, dtype=torch.float32, device=x.device)
    if out is None:
        out = torch.empty(tokens, hidden, dtype=x.dtype, device=x.device)
    ws = workspace(
        moe_layer_workspace_bytes(tokens, hidden, inter, num_experts + 1, top_k + 1, block_size),
        x.device,
    )
    _lib.check(
        lib().b200_moe_layer_forward_fused_shared(
            quant, _vp(x), _code(x, "x"), tokens, hidden, inter, _vp(topk_ids), _vp(topk_weights),
            top_k, num_experts, float(shared_route_weight), _vp(ids), _vp(w), _vp(w13),
            _vp(w13_scales), None, _vp(w2), _vp(w2_scales), None, block_size,
            float(routed_scaling_factor), _vp(out), _code(out, "out"), _vp(ws), ws.numel(),
            _stream(x.device),
        )
    )
    return out, ids, w


def moe_layer_forward_logits(x: torch.Tensor, router_logits: torch.Tensor, top_k: int, *,
                             quant: int, num_experts: int, inter: int, w13: torch.Tensor,
                             w2: torch.Tensor, w13_scales=None, w2_scales=None, w13_global=None,
                             w2_global=None, block_size: int = 16,
                             routed_scaling_factor: float = 1.0,
                             shared_out: torch.Tensor | None = None,
                             scoring: int = _lib.SCORING_SOFTMAX, renormalize: bool = True,
                             correction_bias: torch.Tensor | None = None,
                             out: torch.Tensor | None = None):
    """Router top-k + layer in one library call: (out, topk_ids, topk_weights)."""
    _contig(x, "x")
    _contig(router_logits, "router_logits")
    try:
        lcode = _LOGIT_CODE[router_logits.dtype]
    except KeyError:
        raise TypeError(f"router_logits must be bf16, f16 or f32, got {router_logits.dtype}") from None
    tokens, hidden = (int(d) for d in x.shape)
    if correction_bias is not None:
        _contig(correction_bias, "correction_bias")
    ids = torch.empty(tokens, top_k, dtype=torch.int32, device=x.device)
    w = torch.empty(tokens, top_k, dtype=torch.float32, device=x.device)
    if out is None:
        out = torch.empty(tokens, hidden, dtype=x.dtype, device=x.device)
    if shared_out is not None:
        _contig(shared_out, "shared_out")
    ws = workspace(
        moe_layer_workspace_bytes(tokens, hidden, inter, num_experts, top_k, block_size), x.device
    )
    _lib.check(
        lib().b200_moe_layer_forward_logits(
            quant, _vp(x), _code(x, "x"), tokens, hidden, inter, _vp(router_logits), lcode,
            scoring, int(renormalize), _vp(correction_bias), top_k, num_experts, _vp(ids), _vp(w),
            _vp(w13), _vp(w13_scales), _vp(w13_global), _vp(w2), _vp(w2_scales), _vp(w2_global),
            block_size, float(routed_scaling_factor), _vp(shared_out),
            _code(shared_out, "shared_out") if shared_out is not None else 0, _vp(out),
            _code(out, "out"), _vp(ws), ws.numel(), _stream(x.device),
        )
    )
    return out, ids, w


# ------------------------------------------------------ expert parallelism
# Peer-memory exchange (b200_ep_*): see ep.PeerExchange for the set-up of the
# per-rank regions and their mapping into every peer.
def ep_region_bytes(world: int, max_tokens: int, top_k: int, hidden: int) -> int:
    n = int(lib().b200_ep_region_bytes(world, max_tokens, top_k, hidden))
    if n < 0:
        raise ValueError("bad expert-parallel region shape")
    return n


def ep_region_layout(world: int, max_tokens: int, top_k: int, hidden: int) -> dict:
    """Byte offsets of a region's arrays (see b200_ep_region_layout)."""
    arr = (ctypes.c_int64 * 7)()
    _lib.check(lib().b200_ep_region_layout(world, max_tokens, top_k, hidden, arr))
    keys = ("ids", "weights", "orig", "rows", "recv", "comb", "total")
    return dict(zip(keys, (int(v) for v in arr)))


def aligned_zeros(nbytes: int, device: torch.device) -> torch.Tensor:
    """Zero-filled uint8 buffer of ``nbytes`` whose base is 256-byte aligned."""
    raw = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
    offset = (-raw.data_ptr()) % 256
    return raw[offset : offset + nbytes]


def ipc_get_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of t's allocation, t's offset inside it)."""
    _cuda(t, "buffer")
    handle = ctypes.create_string_buffer(64)
    offset = ctypes.c_int64(0)
    _lib.check(lib().b200_ipc_get_handle(_vp(t), handle, ctypes.byref(offset)))
    return handle.raw, int(offset.value)


def ipc_open_handle(handle: bytes, offset: int) -> int:
    """Maps a peer's allocation; returns the device address of its buffer."""
    if len(handle) != 64:
        raise ValueError("an IPC handle is 64 bytes")
    ptr = ctypes.c_void_p(0)
    _lib.check(lib().b200_ipc_open_handle(ctypes.create_string_buffer(handle, 64), int(offset),
                                          ctypes.byref(ptr)))
    return int(ptr.value)


def ipc_close_handle(address: int, offset: int) -> None:
    _lib.check(lib().b200_ipc_close_handle(ctypes.c_void_p(address), int(offset)))


def _peers_arg(peers: torch.Tensor, world: int):
    _contig(peers, "peer_regions")
    if peers.dtype != torch.int64 or peers.numel() != world:
        raise ValueError(f"peer_regions must be int64[{world}] on the device")
    return _vp(peers)


def ep_dispatch(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, *,
                num_experts: int, rank: int, world: int, peers: torch.Tensor,
                region: torch.Tensor, max_tokens: int, shared_expert: bool = False) -> None:
    """Source side: this rank's routes (rows + routing) into their owners' regions."""
    _contig(x, "x")
    _contig(topk_ids, "topk_ids")
    _contig(topk_weights, "topk_weights")
    _contig(region, "region")
    if topk_ids.dtype != torch.int32 or topk_weights.dtype != torch.float32:
        raise TypeError("topk_ids must be int32 and topk_weights float32")
    tokens, hidden = (int(d) for d in x.shape)
    _lib.check(
        lib().b200_ep_dispatch(
            _vp(x), _code(x, "x"), tokens, hidden, _vp(topk_ids), _vp(topk_weights),
            int(topk_ids.shape[1]), num_experts, int(shared_expert), rank, world,
            _peers_arg(peers, world), _vp(region), max_tokens, _stream(x.device),
        )
    )


def ep_expert_workspace_bytes(world: int, max_tokens: int, top_k: int, hidden: int, inter: int,
                              local_experts: int, block_size: int) -> int:
    return int(lib().b200_ep_expert_workspace_bytes(world, max_tokens, top_k, hidden, inter,
                                                    local_experts, block_size))


def ep_expert_forward(*, quant: int, hidden: int, inter: int, local_experts: int,
                      w13: torch.Tensor, w2: torch.Tensor, w13_scales=None, w2_scales=None,
                      w13_global=None, w2_global=None, block_size: int, rank: int, world: int,
                      peers: torch.Tensor, region: torch.Tensor, max_tokens: int,
                      top_k: int) -> None:
    """Owner side: wait for every source, run this rank's experts on what
    arrived, store each weighted row into its source's region."""
    _contig(region, "region")
    ws = workspace(
        ep_expert_workspace_bytes(world, max_tokens, top_k, hidden, inter, local_experts,
                                  block_size),
        region.device,
    )
    _lib.check(
        lib().b200_ep_expert_forward(
            quant, hidden, inter, local_experts, _vp(w13), _vp(w13_scales), _vp(w13_global),
            _vp(w2), _vp(w2_scales), _vp(w2_global), block_size, rank, world,
            _peers_arg(peers, world), _vp(region), max_tokens, top_k, _vp(ws), ws.numel(),
            _stream(region.device),
        )
    )


def ep_combine(topk_ids: torch.Tensor, *, hidden: int, num_experts: int, world: int,
               region: torch.Tensor, max_tokens: int, routed_scaling_factor: float = 1.0,
               shared_out: torch.Tensor | None = None, out: torch.Tensor | None = None,
               out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Source side: wait for every owner, sum each token's returned rows."""
    _contig(topk_ids, "topk_ids")
    _contig(region, "region")
    tokens, top_k = (int(d) for d in topk_ids.shape)
    if out is None:
        out = torch.empty(tokens, hidden, dtype=out_dtype, device=topk_ids.device)
    _contig(out, "out")
    if shared_out is not None:
        _contig(shared_out, "shared_out")
    _lib.check(
        lib().b200_ep_combine(
            tokens, hidden, _vp(topk_ids), top_k, num_experts, float(routed_scaling_factor),
            _vp(shared_out), _code(shared_out, "shared_out") if shared_out is not None else 0,
            _vp(out), _code(out, "out"), world, _vp(region), max_tokens, _stream(out.device),
        )
    )
    return out


def region_status(region: torch.Tensor, reset: bool = True) -> int:
    """Error bits of an expert-parallel region (8 = a wait on a peer timed out). Synchronizes."""
    bits = ctypes.c_int32(0)
    _lib.check(lib().b200_workspace_status(_vp(region), ctypes.byref(bits), int(reset),
                                           _stream(region.device)))
    return int(bits.value)


# ------------------------------------------- W8A8 block FP8 (opt-in path)
# FP8 x FP8 on the tensor cores; the activations are quantized per (row,
# 128-K group), so results differ from the W8A16 ops above. Weights are the
# checkpoint's row-major e4m3 [E, N, K] with fp32 scales [E, N/128, K/128].
def w8a8_workspace_bytes(slots: int, k: int) -> int:
    n = int(lib().b200_w8a8_workspace_bytes(int(slots), int(k)))
    if n < 0:
        raise ValueError(f"bad W8A8 workspace shape slots={slots} k={k}")
    return n


def fp8_act_quant(x: torch.Tensor, scales_ld: int | None = None):
    """(q e4m3 [rows, K], scales fp32 [K/128, scales_ld]) of bf16/f16 ``x``:
    scale = max(amax / 448, 1e-8) per (row, 128-K group)."""
    _contig(x, "x")
    rows, k = (int(d) for d in x.shape)
    ld = rows if scales_ld is None else int(scales_ld)
    q = torch.empty(rows, k, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(k // 128, ld, dtype=torch.float32, device=x.device)
    _lib.check(lib().b200_fp8_act_quant(_vp(x), _code(x, "x"), rows, k, _vp(q), _vp(s), ld,
                                        _stream(x.device)))
    return q, s


def _w8_weights(w: torch.Tensor, w_scales: torch.Tensor):
    _contig(w, "weight")
    _contig(w_scales, "weight scales")
    if w.dtype != torch.float8_e4m3fn:
        raise TypeError(f"W8A8 weights must be float8_e4m3fn, got {w.dtype}")
    if w_scales.dtype != torch.float32:
        raise TypeError(f"W8A8 weight scales must be float32, got {w_scales.dtype}")


def w8a8_linear(x: torch.Tensor, w: torch.Tensor, w_scales: torch.Tensor, *,
                gated_mode: int = _lib.GATED_NONE, out: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``y = W8A8(x, W)`` with W row-major e4m3 ``[N, K]`` and scales ``[N/128, K/128]``."""
    _contig(x, "x")
    _w8_weights(w, w_scales)
    x2 = x.reshape(-1, x.shape[-1])
    m, k = (int(d) for d in x2.shape)
    n = int(w.shape[-2])
    cols = n // 2 if gated_mode == _lib.GATED_FUSED else n
    if out is None:
        out = torch.empty(m, cols, dtype=out_dtype or x.dtype, device=x.device)
    ws = workspace(w8a8_workspace_bytes(m, k), x.device)
    _lib.check(
        lib().b200_w8a8_linear(_vp(x2), _code(x2, "x"), m, k, _vp(w), _vp(w_scales), n, gated_mode,
                               _vp(out), _code(out, "out"), _vp(ws), ws.numel(), _stream(x.device))
    )
    return out.reshape(*x.shape[:-1], cols)


def w8a8_moe_gemm(a: torch.Tensor, w: torch.Tensor, w_scales: torch.Tensor, *, num_experts: int,
                  sorted_token_ids: torch.Tensor, expert_ids: torch.Tensor,
                  num_tokens_post_pad: torch.Tensor, block_size: int, top_k: int, num_routes: int,
                  c: torch.Tensor, topk_weights: torch.Tensor | None = None,
                  mul_topk_weights: bool = False, gated_mode: int = _lib.GATED_NONE) -> torch.Tensor:
    """Grouped W8A8 expert GEMM with ``moe_wna16_marlin_gemm`` routing semantics;
    ``w`` e4m3 ``[E, N, K]`` row-major, ``w_scales`` ``[E, N/128, K/128]``."""
    _contig(a, "a")
    _contig(c, "c")
    _w8_weights(w, w_scales)
    a_rows, k = (int(d) for d in a.reshape(-1, a.shape[-1]).shape)
    n = int(w.shape[-2])
    if topk_weights is not None:
        topk_weights = topk_weights.reshape(-1).float().contiguous()
    if c.shape[0] < num_routes:
        raise ValueError(f"c has {c.shape[0]} rows, the routes need {num_routes}")
    if mul_topk_weights and (topk_weights is None or topk_weights.numel() < num_routes):
        raise ValueError("mul_topk_weights needs one topk weight per route")
    groups = min(expert_ids.numel(), sorted_token_ids.numel() // block_size)
    ws = workspace(w8a8_workspace_bytes(groups * block_size, k), a.device)
    _lib.check(
        lib().b200_w8a8_moe_gemm(
            _vp(a), _code(a, "a"), a_rows, k, _vp(w), _vp(w_scales), num_experts, n, gated_mode,
            _vp(sorted_token_ids), _vp(expert_ids), groups, _vp(num_tokens_post_pad), block_size,
            top_k, num_routes, _vp(topk_weights), int(mul_topk_weights), _vp(c), _code(c, "c"),
            c.shape[-1], _vp(ws), ws.numel(), _stream(a.device),
        )
    )
    return c
