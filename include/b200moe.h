/*
 * libb200moe - B200 (sm_100a) kernels for the quantized MoE and decode-GEMM
 * path of sglang-restomod, behind a plain C ABI.
 *
 * Every entry point takes raw device pointers, element counts and a CUDA
 * stream (as void*; NULL is the legacy default stream, which breaks graph
 * capture, so pass the caller's current stream). Nothing here allocates
 * device memory: outputs and workspaces belong to the caller. Every function
 * validates its arguments on the host first and returns a status:
 *   0  B200_OK
 *   1  B200_ERR_INVALID      bad argument (message in b200_last_error())
 *   2  B200_ERR_UNSUPPORTED  a valid call this build declines (shape/dtype)
 *   3  B200_ERR_CUDA         a CUDA runtime error while launching
 * No function throws, traps on the device, or reads the environment.
 *
 * Workspaces: functions taking (workspace, workspace_bytes) need a buffer of
 * at least the size the matching *_workspace_bytes() function returns, zero
 * filled before its first use. The kernels return every counter and partial
 * sum they touch to zero, so one workspace serves any number of calls - but
 * calls that share a workspace must be ordered (same stream, or joined by
 * events); two calls running at once on one workspace race.
 *
 * Dtype codes: 0 = bf16, 1 = f16, 2 = f32.
 *
 * Reference interfaces replaced are cited as path:line inside the
 * sglang-restomod source tree.
 */
#ifndef B200MOE_H_
#define B200MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_OK 0
#define B200_ERR_INVALID 1
#define B200_ERR_UNSUPPORTED 2
#define B200_ERR_CUDA 3

#define B200_DTYPE_BF16 0
#define B200_DTYPE_F16 1
#define B200_DTYPE_F32 2

#define B200_QUANT_FP8_BLOCK 0 /* e4m3 weights, fp32 scales per 128x128 block */
#define B200_QUANT_NVFP4 1     /* e2m1 weights, e4m3 scales per 16 K, fp32 global */

#define B200_GATED_NONE 0  /* plain rows: out[.., N] */
#define B200_GATED_FUSED 1 /* gate/up bank: out[.., N/2] = silu(gate) * up */
#define B200_GATED_SPLIT 2 /* gate/up bank: out[.., N] = gate | up (no activation) */

/* ABI version of this header; bumped on any signature change. */
int b200_abi_version(void);

/* Message of the last non-zero status returned on this thread. */
const char* b200_last_error(void);

/* SMs of the current device (the stream GEMM's persistent grid is a multiple). */
int b200_num_sms(void);

/*
 * Device-side error bits recorded in a workspace (1 = a pipeline wait timed
 * out, 2 = an expert id >= E reached a GEMM, 4 = a route pointed past the
 * activation rows) or an expert-parallel region (8 = a wait on another rank
 * timed out). Synchronizes `stream`; clears the bits when reset != 0.
 */
int b200_workspace_status(void* workspace, int32_t* bits, int32_t reset, void* stream);

/* ---------------------------------------------------------------- routing */

/*
 * moe_align_block_size. Replaces upstream sgl_kernel's moe_align_block_size
 * as pinned by sglang_restomod/moe/align_sm70.py:35-55 (its consumers:
 * quant/sm70_fp4_moe/decode_gemv.py:226-260, csrc/decode_gemv_qpn2.cu:73-110),
 * with the stable expert-major order of quant/sm70_fp8_moe/method.py:285.
 *
 * topk_ids[numel] (numel = tokens * top_k) -> sorted_token_ids holds route
 * indices grouped by expert in route order, each expert padded to a multiple
 * of block_size with the sentinel `numel`; expert_ids[b] is block b's expert
 * (-1 past the end); num_tokens_post_pad[0] is the padded total. Ids outside
 * [0, num_experts) are dropped. Needs sorted_capacity >= numel +
 * min(numel, num_experts) * (block_size - 1) and expert_capacity >=
 * ceil(sorted_capacity / block_size); every slot of both arrays is written.
 * num_experts <= 1024.
 */
int b200_moe_align_block_size(const int32_t* topk_ids, int64_t numel, int32_t num_experts,
                              int32_t block_size, int32_t* sorted_token_ids,
                              int64_t sorted_capacity, int32_t* expert_ids,
                              int64_t expert_capacity, int32_t* num_tokens_post_pad,
                              void* stream);

/*
 * Router top-k: router_logits [tokens, num_experts] (bf16 / f16 / f32) ->
 * topk_ids [tokens, top_k] int32 and topk_weights fp32, in descending order
 * of the selection key. Replaces upstream SGLang's select_experts / fused
 * top-k softmax, whose output (StandardTopKOutput: topk_weights, topk_ids)
 * the quant methods consume (quant/sm70_fp8_moe/check.py:106-114; the
 * benchmark's routing: softmax -> top-k -> renormalise).
 * scoring B200_SCORING_SOFTMAX: weights = softmax probabilities of the chosen
 * experts; B200_SCORING_SIGMOID: weights = sigmoid(logit), chosen by
 * sigmoid(logit) + correction_bias[e] when correction_bias is given (fp32
 * [num_experts]; softmax takes none). renormalize != 0 divides the chosen
 * weights by their sum. Ties go to the lower expert id. num_experts <= 1024,
 * top_k <= min(32, num_experts).
 */
#define B200_SCORING_SOFTMAX 0
#define B200_SCORING_SIGMOID 1
int b200_topk_route(const void* router_logits, int32_t logits_dtype, int64_t tokens,
                    int32_t num_experts, int32_t top_k, int32_t scoring, int32_t renormalize,
                    const float* correction_bias, int32_t* topk_ids, float* topk_weights,
                    void* stream);

/*
 * Grouped router top-k: b200_topk_route restricted to the topk_group best of
 * num_expert_group contiguous expert groups, as upstream SGLang's
 * grouped_topk / biased_grouped_topk (select_experts with num_expert_group /
 * topk_group), whose StandardTopKOutput the quant methods consume
 * (quant/sm70_fp8_moe/check.py:106-114). A group's score is its largest
 * selection key (softmax: logit; sigmoid: sigmoid(logit)), or with a
 * correction_bias the sum of its two largest sigmoid(logit) + bias keys;
 * ties go to the lower group and the lower expert. Weights as in
 * b200_topk_route (unbiased scores, renormalised on request).
 * num_experts % num_expert_group == 0, num_expert_group <= 32,
 * top_k <= topk_group * num_experts / num_expert_group.
 */
int b200_topk_route_grouped(const void* router_logits, int32_t logits_dtype, int64_t tokens,
                            int32_t num_experts, int32_t top_k, int32_t scoring,
                            int32_t renormalize, const float* correction_bias,
                            int32_t num_expert_group, int32_t topk_group, int32_t* topk_ids,
                            float* topk_weights, void* stream);

/*
 * Shared-expert fusion: ids_out / weights_out [tokens, top_k + 1] = the
 * routes of topk_ids / topk_weights [tokens, top_k] plus one route per token
 * to shared_id with shared_weight. With the shared expert's weights stored
 * as expert shared_id of the routed bank (same shapes and quantization), one
 * routed layer forward then computes the shared expert too (use
 * shared_weight = 1 / routed_scaling_factor, since the combine scales every
 * route). Replaces the shared expert's separate dense MLP (upstream's
 * always-on shared expert, which the FP8 checkpoint keeps as a dense
 * linear: docs/quantization-dispatch.md:112, 125-126).
 */
int b200_append_shared_route(const int32_t* topk_ids, const float* topk_weights, int64_t tokens,
                             int32_t top_k, int32_t shared_id, float shared_weight,
                             int32_t* ids_out, float* weights_out, void* stream);

/* ---------------------------------------------------------------- combine */

/*
 * moe_sum_reduce: output[t, :] = routed_scaling_factor * sum_k input[t, k, :]
 * (fp32 sum, stored in the input dtype). Replaces
 * quant/sm70_fp4_moe/sum_reduce.py:84-123. hidden % 8 == 0; contiguous.
 */
int b200_moe_sum_reduce(const void* input, void* output, int64_t tokens, int32_t top_k,
                        int64_t hidden, int32_t dtype, float routed_scaling_factor, void* stream);

/*
 * Top-k combine of rows already multiplied by their router weight
 * (quant/sm70_fp8_moe/method.py:305-309): out[t] = rsf * sum over k with
 * 0 <= topk_ids[t, k] < num_experts of routed[t * top_k + k] (+ shared[t]).
 * topk_ids may be NULL (every route counts); shared_out may be NULL.
 */
int b200_moe_combine(const void* routed, int32_t routed_dtype, const int32_t* topk_ids,
                     int32_t num_experts, int64_t tokens, int32_t top_k, int64_t hidden,
                     float routed_scaling_factor, const void* shared_out, int32_t shared_dtype,
                     void* out, int32_t out_dtype, void* stream);

/* ---------------------------------------------------------------- prepack */

/*
 * Block-FP8 weights [experts, n, k] e4m3 (row-major) -> this library's
 * streamed layout. Replaces the load-time prepare of
 * quant/sm70_fp8_moe/__init__.py:161-205 (fp8_prepare with
 * interleave_gated_silu) and quant/sm70_fp8_dense/_method.py:314-329
 * (_qpn8_prepack). gated != 0 interleaves the two halves of a [2I, K]
 * gate/up bank. n % 128 == 0, k % 128 == 0 (gated: n % 256 == 0).
 */
int64_t b200_fp8_packed_bytes(int64_t experts, int64_t n, int64_t k);
int b200_fp8_prepack(const uint8_t* w_e4m3, int64_t experts, int64_t n, int64_t k, int32_t gated,
                     uint8_t* out, void* stream);

/*
 * NVFP4 ModelOpt checkpoint [experts, n, k/2] uint8 (low nibble = even K) and
 * [experts, n, k/16] e4m3 group scales -> streamed layout (scales inline).
 * Replaces prepare_moe_nvfp4 / qpn2.pack_expert
 * (quant/sm70_fp4_moe/method.py:290-382, qpn2.py:65-110). The fp32 global
 * scale stays a separate [experts] array.
 */
int64_t b200_nvfp4_packed_bytes(int64_t experts, int64_t n, int64_t k);
int b200_nvfp4_prepack(const uint8_t* w_packed, const uint8_t* scales_e4m3, int64_t experts,
                       int64_t n, int64_t k, int32_t gated, uint8_t* out, void* stream);

/* ------------------------------------------------------------------ GEMMs */

/* Workspace for b200_linear / b200_moe_gemm; `convert_elems` is the number of
 * bf16 activation elements the call converts (0 for f16 activations). */
int64_t b200_gemm_workspace_bytes(int64_t convert_elems);

/*
 * Dense W8A16 / W4A16 linear, y[m, :] = x[m, :k] . dequant(W)^T.
 * Replaces apply_sm70_turbomind_fp8_linear (quant/sm70_fp8_dense/_method.py:
 * 713-784; its QPN8 decode kernel csrc/sm70_fp8_qpn8_decode.cu:60-149) and,
 * with gated_mode = B200_GATED_FUSED on a gated bank,
 * apply_sm70_turbomind_fp8_fused_silu_and_mul (_method.py:787-863,
 * csrc/sm70_fp8_qpn8_decode.cu:156-246).
 * quant: B200_QUANT_FP8_BLOCK (w_scales = [n/128, k/128] fp32) or
 * B200_QUANT_NVFP4 (global_scale = one fp32). x: bf16 or f16, rows of k.
 * m > 32 runs on the tcgen05 tensor-core GEMM (row groups of up to 192);
 * smaller m streams the weights once (decode GEMV).
 */
int b200_linear(int32_t quant, const void* x, int32_t x_dtype, int64_t m, int64_t k,
                const uint8_t* w_packed, const float* w_scales, const float* global_scale,
                int64_t n, int32_t gated_mode, void* y, int32_t y_dtype, void* workspace,
                int64_t workspace_bytes, void* stream);

/*
 * b200_linear for callers that cannot allocate device memory (an engine that
 * reserved all of it for its own pool before loading this library, a binding
 * with no access to the device allocator). No counterpart in the reference:
 * this entry point exists only for such callers. Same arguments and result
 * as b200_linear, without the workspace: it uses a 16 MiB array compiled
 * into the library (held on every device that loads it, until exit). The
 * array holds the fixed workspace, b200_gemm_workspace_bytes(0) on the
 * current device, and room for
 * (b200_linear_noalloc_scratch_bytes() - b200_gemm_workspace_bytes(0)) / 2
 * bf16 activation elements (M*K) to convert: 3,405,568 on a 148-SM B200.
 * Larger bf16 calls are refused with B200_ERR_INVALID (f16 activations need
 * no conversion room). The array is shared: calls on one device must not
 * overlap on the GPU. The first call on each device looks up the array's
 * address (cudaGetSymbolAddress) and clears it; make that call before any
 * stream capture. cudaDeviceReset after it is not supported. Calls no
 * cudaMalloc / cudaFree.
 */
int64_t b200_linear_noalloc_scratch_bytes(void);
int b200_linear_noalloc(int32_t quant, const void* x, int32_t x_dtype, int64_t m, int64_t k,
                        const uint8_t* w_packed, const float* w_scales, const float* global_scale,
                        int64_t n, int32_t gated_mode, void* y, int32_t y_dtype, void* stream);

/*
 * Device-side error bits of b200_linear_noalloc calls on the current device
 * (the bits of b200_workspace_status, kept in the static array, which the
 * caller cannot address). The bits are sticky across calls until read with
 * reset != 0, which also clears the array's partial sums when bits were set.
 * Synchronizes `stream`. No counterpart in the reference.
 */
int b200_linear_noalloc_status(int32_t* bits, int32_t reset, void* stream);

/*
 * The data-movement floor of b200_linear / b200_moe_gemm, for measurement:
 * the same arguments and launches, every weight and activation copy and
 * every pipeline barrier hand-off, but no conversion, MMA or store (y / c
 * are left untouched). The reference keeps the same instrument as a
 * kCompute=false instantiation of its NVFP4 decode GEMV
 * (quant/sm70_fp4_moe/csrc/decode_gemv_qpn2.cu:63-200); timing a call
 * against its loads-only twin separates the cost of moving the bytes from
 * the cost of the math.
 */
int b200_linear_loads_only(int32_t quant, const void* x, int32_t x_dtype, int64_t m, int64_t k,
                           const uint8_t* w_packed, const float* w_scales,
                           const float* global_scale, int64_t n, int32_t gated_mode, void* y,
                           int32_t y_dtype, void* workspace, int64_t workspace_bytes,
                           void* stream);
int b200_moe_gemm_loads_only(int32_t quant, const void* a, int32_t a_dtype, int64_t a_rows,
                             int64_t k, const uint8_t* w_packed, const float* w_scales,
                             const float* global_scale, int32_t num_experts, int64_t n,
                             int32_t gated_mode, const int32_t* sorted_token_ids,
                             const int32_t* expert_ids, int64_t expert_capacity,
                             const int32_t* num_tokens_post_pad, int32_t block_size,
                             int32_t top_k, int64_t num_routes, const float* topk_weights,
                             int32_t mul_topk_weights, void* c, int32_t c_dtype, int64_t ldc,
                             void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Which kernel a call takes (for census and profiling; no counterpart in the
 * reference, whose dispatcher decides the same question in Python,
 * quant/sm70_fp4_moe/decode_gemv.py:183-219). Returns B200_PATH_STREAM (the
 * weight-streaming decode GEMM; *tile_rows = rows per weight pass) or
 * B200_PATH_TCGEN05 (the tensor-core GEMM; *tile_rows = 192, *k_parts = K
 * split of a dense call), or an error status (negative never; check > 10).
 * b200_linear_path: b200_linear with m rows of [n, k]. b200_moe_path:
 * b200_moe_gemm / the layer forward with this block size and group count.
 */
#define B200_PATH_STREAM 16
#define B200_PATH_TCGEN05 17
int b200_linear_path(int64_t m, int64_t n, int64_t k, int32_t* tile_rows, int32_t* k_parts);
int b200_moe_path(int32_t quant, int32_t block_size, int64_t expert_capacity, int32_t* tile_rows);

/*
 * Grouped expert GEMM routed by moe_align_block_size output, with the
 * semantics of moe_wna16_marlin_gemm (quant/sm70_fp4_moe/method.py:385-564):
 * route slot p of block b multiplies activation row sorted_token_ids[p] /
 * top_k by expert expert_ids[b] and writes output row sorted_token_ids[p]
 * (times topk_weights[route] when mul_topk_weights). a: [a_rows, k];
 * c: rows of ldc elements. block_size in {8, 16, 32, 64, 128, 256}; blocks
 * of 64 and more run on the tcgen05 tensor-core GEMM (f16 operands; bf16
 * activations are converted in the workspace), smaller blocks on the
 * weight-streaming GEMM.
 * At most expert_capacity blocks are read, so sorted_token_ids must hold
 * expert_capacity * block_size entries (pass floor(sorted_len / block_size)
 * when the align output is shorter). topk_weights and c need num_routes rows.
 */
int b200_moe_gemm(int32_t quant, const void* a, int32_t a_dtype, int64_t a_rows, int64_t k,
                  const uint8_t* w_packed, const float* w_scales, const float* global_scale,
                  int32_t num_experts, int64_t n, int32_t gated_mode,
                  const int32_t* sorted_token_ids, const int32_t* expert_ids,
                  int64_t expert_capacity, const int32_t* num_tokens_post_pad,
                  int32_t block_size, int32_t top_k, int64_t num_routes,
                  const float* topk_weights, int32_t mul_topk_weights, void* c, int32_t c_dtype,
                  int64_t ldc, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * One fused-MoE layer forward (SM70Fp8MoEMethod.apply,
 * quant/sm70_fp8_moe/method.py:239-309; the NVFP4 fused_marlin_moe chain of
 * quant/sm70_fp4_moe/method.py:385-564 + sum_reduce.py:84-123):
 * align -> gate_up (+SiLU*up) -> down (x router weight) -> combine
 * (x routed_scaling_factor, + shared_out when given).
 * x [tokens, hidden] bf16/f16; topk_ids/topk_weights [tokens, top_k];
 * w13: gated bank [E, 2*inter, hidden]; w2: [E, hidden, inter].
 * Ids outside [0, E) contribute nothing (expert-parallel drops).
 */
int64_t b200_moe_layer_workspace_bytes(int64_t tokens, int64_t hidden, int64_t inter,
                                       int32_t num_experts, int32_t top_k, int32_t block_size);
int b200_moe_layer_forward(int32_t quant, const void* x, int32_t x_dtype, int64_t tokens,
                           int64_t hidden, int64_t inter, const int32_t* topk_ids,
                           const float* topk_weights, int32_t top_k, int32_t num_experts,
                           const uint8_t* w13_packed, const float* w13_scales,
                           const float* w13_global, const uint8_t* w2_packed,
                           const float* w2_scales, const float* w2_global, int32_t block_size,
                           float routed_scaling_factor, const void* shared_out,
                           int32_t shared_dtype, void* out, int32_t out_dtype, void* workspace,
                           int64_t workspace_bytes, void* stream);

/*
 * b200_moe_layer_forward with the shared expert fused into the routed bank
 * (upstream SGLang's always-on shared MLP beside the routed experts, which
 * the reference runs as a separate dense layer): w13 / w2 hold
 * num_experts + 1 experts, the last being the shared expert (its shapes and
 * block-FP8 weights match the routed ones). Every token gets one more route,
 * id num_experts, weight shared_route_weight (1 / routed_scaling_factor
 * leaves the shared output unscaled), written with the caller's routes to
 * topk_ids_out / topk_weights_out [tokens, top_k + 1] (distinct from the
 * inputs). For up to 4095 extended routes the append, moe_align and the
 * bf16 -> f16 activation conversion run as one kernel. Workspace:
 * b200_moe_layer_workspace_bytes(tokens, hidden, inter, num_experts + 1,
 * top_k + 1, block_size).
 */
int b200_moe_layer_forward_fused_shared(
    int32_t quant, const void* x, int32_t x_dtype, int64_t tokens, int64_t hidden, int64_t inter,
    const int32_t* topk_ids, const float* topk_weights, int32_t top_k, int32_t num_experts,
    float shared_route_weight, int32_t* topk_ids_out, float* topk_weights_out,
    const uint8_t* w13_packed, const float* w13_scales, const float* w13_global,
    const uint8_t* w2_packed, const float* w2_scales, const float* w2_global, int32_t block_size,
    float routed_scaling_factor, void* out, int32_t out_dtype, void* workspace,
    int64_t workspace_bytes, void* stream);

/*
 * b200_moe_layer_forward from router logits: the routing of b200_topk_route
 * (written to topk_ids_out / topk_weights_out [tokens, top_k], which the
 * caller keeps) followed by the layer. For up to 32 tokens the router and
 * moe_align run as one kernel. Replaces the select_experts ->
 * StandardTopKOutput -> quant method apply chain
 * (quant/sm70_fp8_moe/check.py:106-114, method.py:239-309).
 */
int b200_moe_layer_forward_logits(int32_t quant, const void* x, int32_t x_dtype, int64_t tokens,
                                  int64_t hidden, int64_t inter, const void* router_logits,
                                  int32_t logits_dtype, int32_t scoring, int32_t renormalize,
                                  const float* correction_bias, int32_t top_k,
                                  int32_t num_experts, int32_t* topk_ids_out,
                                  float* topk_weights_out, const uint8_t* w13_packed,
                                  const float* w13_scales, const float* w13_global,
                                  const uint8_t* w2_packed, const float* w2_scales,
                                  const float* w2_global, int32_t block_size,
                                  float routed_scaling_factor, const void* shared_out,
                                  int32_t shared_dtype, void* out, int32_t out_dtype,
                                  void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------- W8A8 block FP8 (opt-in path) */

/*
 * FP8 x FP8 prefill GEMMs on the tcgen05 tensor cores (kind::f8f6f4). The
 * reference has no such path (its FP8 linears and experts are W8A16:
 * quant/sm70_fp8_dense/_method.py:713-863 and the TurboMind expert GEMM of
 * quant/sm70_fp8_moe/method.py:303-304); this is upstream SGLang's
 * block-FP8 W8A8 arithmetic: activations quantized per (row, 128-K group) to
 * e4m3 with scale = max(amax / 448, 1e-8) (the block rule of
 * quant/sm70_fp8_lm_head/__init__.py:33-41), the checkpoint's e4m3 weights
 * with fp32 scales per 128x128 block, y = sum over 128-K blocks of
 * sa * sw * (qa . qw), fp32 accumulation. Quantizing the activations changes
 * results against the W8A16 entry points, so these are separate calls.
 * Weights are the checkpoint's ROW-MAJOR e4m3 [E][N][K] (no prepack); a
 * gate/up bank keeps its [gate | up] row order and gated_mode
 * B200_GATED_FUSED yields silu(gate) * up, N / 2 wide (B200_GATED_SPLIT and
 * B200_GATED_NONE both give all N rows). K % 128 == 0, N % 128 == 0.
 */

/* Workspace of b200_w8a8_linear (slots = M) or b200_w8a8_moe_gemm (slots =
 * expert_capacity * block_size); zero-filled before first use. */
int64_t b200_w8a8_workspace_bytes(int64_t slots, int64_t k);

/* Per-(row, 128-K group) quantization of x [rows, k] (bf16 / f16): q [rows, k]
 * e4m3, scales[(k / 128) * scales_ld] fp32 with scale of (row r, group g) at
 * g * scales_ld + r ("column-major" scales, scales_ld >= rows). Replaces
 * upstream SGLang's per_token_group_quant_fp8 (group 128). */
int b200_fp8_act_quant(const void* x, int32_t x_dtype, int64_t rows, int64_t k, uint8_t* q,
                       float* scales, int64_t scales_ld, void* stream);

/* Dense y [m, n or n/2] = W8A8(x [m, k], w). Replaces, opt-in, the W8A16
 * apply_sm70_turbomind_fp8_linear (quant/sm70_fp8_dense/_method.py:713-784). */
int b200_w8a8_linear(const void* x, int32_t x_dtype, int64_t m, int64_t k, const uint8_t* w_e4m3,
                     const float* w_scales, int64_t n, int32_t gated_mode, void* y,
                     int32_t y_dtype, void* workspace, int64_t workspace_bytes, void* stream);

/* Grouped expert GEMM with the routing of b200_moe_gemm
 * (moe_wna16_marlin_gemm semantics: slot p of block b multiplies activation
 * row sorted_token_ids[p] / top_k by expert expert_ids[b] and writes output
 * row sorted_token_ids[p], times topk_weights when mul_topk_weights), W8A8:
 * the activations are quantized straight into slot order first. Replaces,
 * opt-in, the W8A16 TurboMind expert GEMM (quant/sm70_fp8_moe/method.py:
 * 303-304). */
int b200_w8a8_moe_gemm(const void* a, int32_t a_dtype, int64_t a_rows, int64_t k,
                       const uint8_t* w_e4m3, const float* w_scales, int32_t num_experts,
                       int64_t n, int32_t gated_mode, const int32_t* sorted_token_ids,
                       const int32_t* expert_ids, int64_t expert_capacity,
                       const int32_t* num_tokens_post_pad, int32_t block_size, int32_t top_k,
                       int64_t num_routes, const float* topk_weights, int32_t mul_topk_weights,
                       void* c, int32_t c_dtype, int64_t ldc, void* workspace,
                       int64_t workspace_bytes, void* stream);

/* ---------------------------------------- expert parallelism (peer memory) */

/*
 * Expert-parallel token exchange over NVLink peer memory, replacing the
 * all-to-all around the expert compute. The reference's expert parallelism
 * is upstream SGLang's dispatcher (global -> local expert ids, foreign routes
 * -1: quant/sm70_fp8_moe/method.py:8-12, 253-283) plus the method's combine
 * (method.py:305-309); these entry points give the same layer output with
 * experts split contiguously, num_experts / world per rank.
 *
 * Every rank owns one exchange region of b200_ep_region_bytes() (zero-filled
 * before first use, 256-byte aligned, identical arguments on every rank) and
 * maps every peer's region (b200_ipc_get_handle / b200_ipc_open_handle, the
 * handles exchanged by the caller). peer_regions is a DEVICE array of `world`
 * 64-bit addresses: entry r = rank r's region as mapped in this process (its
 * own entry = its own region). One layer forward on every rank, in this order
 * on one stream:
 *   b200_ep_dispatch        each token's row once per owner of one of its
 *                           experts, with its top_k route slots (P2P stores)
 *   b200_ep_expert_forward  wait for every source, align, gate/up + down GEMMs
 *                           over the received rows, then one summed row per
 *                           received row stored into its source's region
 *   b200_ep_combine         wait for every owner, sum each token's returned
 *                           rows (one per owner) + shared_out, times
 *                           routed_scaling_factor
 * NVLink bytes scale with the distinct owners per token, not with top_k.
 * No host synchronization: the three calls can be captured in a CUDA graph.
 * Waits on other ranks are bounded (2 s) and set bit 8 in the region's status
 * word (read it with b200_workspace_status(region, ...)). Every rank must run
 * the same sequence of calls; calls on one region must not overlap.
 */
int64_t b200_ep_region_bytes(int32_t world, int64_t max_tokens, int32_t top_k, int64_t hidden);

/* Byte offsets inside a region, for inspection: offsets[0..6] = received
 * route slots' local expert ids (int32 [world * max_tokens][top_k], -1 = not
 * on this rank or empty once received), their router weights (fp32, same
 * shape), each received row's source token (int32 [world * max_tokens]), each
 * row's return address (u64, 0 = empty), received rows (f16
 * [world * max_tokens][hidden]), returned rows (f16 [max_tokens * world]
 * [hidden], token t from owner o at t * world + o), total bytes. top_k <= 32. */
int b200_ep_region_layout(int32_t world, int64_t max_tokens, int32_t top_k, int64_t hidden,
                          int64_t* offsets);

/* CUDA IPC of the allocation holding dev_ptr: a 64-byte handle plus the
 * pointer's offset inside it; open maps a peer's allocation, close unmaps. */
int b200_ipc_get_handle(const void* dev_ptr, void* handle, int64_t* offset);
int b200_ipc_open_handle(const void* handle, int64_t offset, void** dev_ptr);
int b200_ipc_close_handle(void* dev_ptr, int64_t offset);

/* Source side: x [tokens, hidden] bf16/f16, topk_ids / topk_weights
 * [tokens, top_k] (global expert ids; ids outside [0, num_experts) are not
 * sent), tokens <= max_tokens. shared_expert != 0: id num_experts is a shared
 * expert held by every rank (appended by b200_append_shared_route); those
 * routes stay on this rank as its local expert num_experts / world. */
int b200_ep_dispatch(const void* x, int32_t x_dtype, int64_t tokens, int64_t hidden,
                     const int32_t* topk_ids, const float* topk_weights, int32_t top_k,
                     int32_t num_experts, int32_t shared_expert, int32_t rank, int32_t world,
                     const uint64_t* peer_regions, void* region, int64_t max_tokens,
                     void* stream);

/* Owner side: this rank's local_experts experts (w13: gated bank
 * [local_experts, 2*inter, hidden], w2: [local_experts, hidden, inter], as for
 * b200_moe_layer_forward). block_size as for b200_moe_layer_forward, sized
 * for about max_tokens * top_k routes per rank. */
int64_t b200_ep_expert_workspace_bytes(int32_t world, int64_t max_tokens, int32_t top_k,
                                       int64_t hidden, int64_t inter, int32_t local_experts,
                                       int32_t block_size);
int b200_ep_expert_forward(int32_t quant, int64_t hidden, int64_t inter, int32_t local_experts,
                           const uint8_t* w13_packed, const float* w13_scales,
                           const float* w13_global, const uint8_t* w2_packed,
                           const float* w2_scales, const float* w2_global, int32_t block_size,
                           int32_t rank, int32_t world, const uint64_t* peer_regions, void* region,
                           int64_t max_tokens, int32_t top_k, void* workspace,
                           int64_t workspace_bytes, void* stream);

/* Source side: out [tokens, hidden] = rsf * sum over the owners of token t's
 * routes of the row each returned (its experts' weighted outputs, summed) +
 * shared_out[t] (optional). tokens and topk_ids as given to b200_ep_dispatch. */
int b200_ep_combine(int64_t tokens, int64_t hidden, const int32_t* topk_ids, int32_t top_k,
                    int32_t num_experts, float routed_scaling_factor, const void* shared_out,
                    int32_t shared_dtype, void* out, int32_t out_dtype, int32_t world, void* region,
                    int64_t max_tokens, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200MOE_H_ */
