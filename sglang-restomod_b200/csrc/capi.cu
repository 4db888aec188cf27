// C ABI of libb200moe: host-side validation, workspace carving and launch
// orchestration. The signatures are declared (with the reference interface
// each one replaces) in include/b200moe.h.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/b200moe.h"
#include "internal.h"

namespace b200 {

int device_sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
      sms = 148;
    cached[dev] = sms;
  }
  return cached[dev];
}

}  // namespace b200

namespace {

using namespace b200;

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return B200_OK;
  return fail(B200_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int64_t kAlign = 256;
int64_t align_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Workspace layout: [status int | pad] [counters, kMaxSlots ints] [tcgen05
// GEMM plan] [partials, slots x kWsSlotFloats fp32] [scratch ...]
constexpr int64_t kStatusBytes = 256;
constexpr int kMaxSlots = 1024;
constexpr int64_t kCounterBytes = kMaxSlots * 4;
constexpr int kTcPlanCap = 32768;  // route-slot groups the tcgen05 path plans for
int64_t plan_region_bytes() { return align_up(tc_plan_bytes(kTcPlanCap)); }

int max_grid_slots() {
  int g = stream_gemm_ctas_per_sm(1) * device_sm_count();
  return g > kMaxSlots ? kMaxSlots : g;
}

int64_t stream_ws_bytes() {
  return kStatusBytes + kCounterBytes + plan_region_bytes() +
         (int64_t)max_grid_slots() * kWsSlotFloats * 4;
}

struct WsView {
  int* status;
  int* counters;
  void* plan;
  float* partials;
  uint8_t* scratch;
  int64_t scratch_bytes;
};

bool carve(void* ws, int64_t bytes, WsView& v) {
  const int64_t fixed = stream_ws_bytes();
  if (ws == nullptr || bytes < fixed || (reinterpret_cast<uintptr_t>(ws) % kAlign) != 0) return false;
  uint8_t* base = reinterpret_cast<uint8_t*>(ws);
  v.status = reinterpret_cast<int*>(base);
  v.counters = reinterpret_cast<int*>(base + kStatusBytes);
  v.plan = base + kStatusBytes + kCounterBytes;
  v.partials = reinterpret_cast<float*>(base + kStatusBytes + kCounterBytes + plan_region_bytes());
  v.scratch = base + fixed;
  v.scratch_bytes = bytes - fixed;
  return true;
}

int nt_for_rows(int64_t rows) {
  if (rows <= 8) return 1;
  if (rows <= 16) return 2;
  if (rows <= 32) return 4;
  return 8;
}

bool valid_dtype16(int32_t d) { return d == B200_DTYPE_BF16 || d == B200_DTYPE_F16; }

// Converts bf16 activations into the f16 operand the stream GEMM reads.
int stage_activations(const void* a, int32_t a_dtype, int64_t elems, WsView& ws, int64_t& used,
                      const __half** out, cudaStream_t stream) {
  if (a_dtype == B200_DTYPE_F16) {
    *out = reinterpret_cast<const __half*>(a);
    return B200_OK;
  }
  const int64_t need = align_up(elems * 2);
  if (used + need > ws.scratch_bytes)
    return fail(B200_ERR_INVALID, "workspace too small for %lld converted activations",
                (long long)elems);
  __half* dst = reinterpret_cast<__half*>(ws.scratch + used);
  used += need;
  int rc = check_cuda(launch_bf16_to_f16(a, dst, elems, stream), "bf16->f16 conversion");
  if (rc) return rc;
  *out = dst;
  return B200_OK;
}

int check_weight_shape(int32_t quant, int64_t n, int64_t k, int32_t gated_mode) {
  if (quant != B200_QUANT_FP8_BLOCK && quant != B200_QUANT_NVFP4)
    return fail(B200_ERR_INVALID, "unknown quant %d", quant);
  if (n <= 0 || k <= 0) return fail(B200_ERR_INVALID, "needs positive N and K, got N=%lld K=%lld",
                                    (long long)n, (long long)k);
  // The reference refuses partial quantization groups the same way
  // (quant/sm70_fp8_moe/__init__.py:48-73).
  if (k % 128)
    return fail(B200_ERR_INVALID,
                "needs K a multiple of the 128-wide quantization group, got K=%lld", (long long)k);
  if (n % 128)
    return fail(B200_ERR_INVALID, "needs N a multiple of 128, got N=%lld", (long long)n);
  if (gated_mode != B200_GATED_NONE && gated_mode != B200_GATED_FUSED &&
      gated_mode != B200_GATED_SPLIT)
    return fail(B200_ERR_INVALID, "unknown gated mode %d", gated_mode);
  if (gated_mode != B200_GATED_NONE && n % 256)
    return fail(B200_ERR_INVALID, "a gate/up bank needs N a multiple of 256, got N=%lld",
                (long long)n);
  if (n > (1ll << 30) || k > (1ll << 30)) return fail(B200_ERR_INVALID, "N or K too large");
  return B200_OK;
}

int run_stream(int32_t quant, int nt, StreamParams& p, long long max_units, WsView& ws,
               cudaStream_t stream) {
  p.ws = ws.partials;
  p.ws_cnt = ws.counters;
  p.status = ws.status;
  long long grid = (long long)max_grid_slots();
  if (nt >= 4) grid = (long long)stream_gemm_ctas_per_sm(nt) * device_sm_count();
  // A few short (group, row block) pairs - at most one per SM, each of at
  // most the whole-pair stage count - stream one pair per CTA; then one CTA
  // per SM with a deeper ring keeps more of each pair's bytes in flight.
  const int sms = device_sm_count();
  const long long kch = p.K / 128;
  const long long kcs = (kch + stream_gemm_stage_units(quant) - 1) / stream_gemm_stage_units(quant);
  const long long max_pairs = max_units / (kch > 0 ? kch : 1);
  const bool solo = nt <= 2 && max_pairs <= sms && kcs <= stream_gemm_whole_pair_max_stages();
  if (solo) grid = sms;
  if (grid > max_units) grid = max_units;
  if (grid < 1) grid = 1;
  return check_cuda(launch_stream_gemm(quant, nt, p, (int)grid, stream, solo),
                    "stream GEMM launch");
}

// tcgen05 GEMM; in moe mode the plan is built first unless `planned` (the
// layer's second GEMM reuses the first one's plan).
int run_tc(int32_t quant, StreamParams& p, WsView& ws, bool planned, cudaStream_t stream,
           bool narrow = false) {
  p.ws = ws.partials;
  p.ws_cnt = ws.counters;
  p.status = ws.status;
  if (p.sorted_ids != nullptr && !planned) {
    int rc = check_cuda(narrow ? launch_tc_plan_slots(p, ws.plan, kTcPlanCap, tc_narrow_slots(),
                                                      stream)
                               : launch_tc_plan(p, ws.plan, kTcPlanCap, stream),
                        "tcgen05 plan launch");
    if (rc) return rc;
  }
  return check_cuda(launch_tc_gemm(quant == B200_QUANT_NVFP4 ? kQuantNvfp4 : kQuantFp8Block, p,
                                   ws.plan, device_sm_count(), stream, narrow),
                    "tcgen05 GEMM launch");
}

// The narrow tcgen05 configuration (items of at most 64 slots, a deeper
// weight ring) for blocks of 64 with few routes per expert: each expert's
// routes then fit one or two such items anyway, and the wide configuration's
// 192-row activation ring only takes shared memory from the weights in
// flight. Measured on the expert-parallel owner shape (H=7168, I=2048, ~32
// routes per expert): its loads-only twin took 256 of its 286 us there.
bool narrow_moe(int32_t block_size, int64_t routes, int64_t experts) {
  return block_size == 64 && routes <= 40 * experts;
}

// Route count from which the layer aligns with the multi-CTA kernels.
constexpr int64_t kAlignMultiMin = 4096;

// Dense calls use the tcgen05 GEMM once M exceeds the decode range: measured
// faster than the stream GEMM's 64-row tile even when its items (192-row
// chunks x 128-row weight blocks) cover only a quarter of the SMs.
constexpr int64_t kTcDenseMinRows = 33;
bool use_tc_dense(int64_t m, int64_t n) {
  (void)n;
  return m >= kTcDenseMinRows;
}

// K parts of a dense tcgen05 call. Items (192-row chunk x 128-row weight
// block) are dealt round-robin over the SMs, each streaming its K range.
// Split K (parts summed in fp32 in the workspace, then a finishing kernel)
// when that cuts the busiest SM's 128-K unit count by a quarter or more, each
// part charged for its m*n fp32 atomic adds at 3x the time of streaming the
// same bytes of weights. Measured on B200: a split that only evens out waves
// is slower (64 x 25600 x 5120: 64 us unsplit, 87 us in two parts), one that
// fills idle SMs is faster (128 x 4096 x 7168: 43 us in three parts, 35 us in
// four; 64 x 5120 x 25600: 64 us in three, 60 us in seven).
int dense_k_parts(int64_t m, int64_t n, int64_t k) {
  const int64_t kch = k / 128, sms = device_sm_count();
  const int64_t items = (m + 191) / 192 * (n / 128);
  if (m * n > (int64_t)max_grid_slots() * kWsSlotFloats) return 1;
  const double part_cost = 3.0 * (double)m * (double)n * 4.0 / 16384.0 / (double)sms;
  const double whole = (double)((items + sms - 1) / sms * kch);
  double best = whole;
  int best_parts = 1;
  for (int64_t ks = 2; ks <= 16 && ks <= kch; ++ks) {
    const int64_t kpart = (kch + ks - 1) / ks;
    const int64_t parts = (kch + kpart - 1) / kpart;
    const double cost =
        (double)((items * parts + sms - 1) / sms * kpart) + part_cost * (double)parts;
    if (cost < best) {
      best = cost;
      best_parts = (int)parts;
    }
  }
  return best < 0.75 * whole ? best_parts : 1;
}

// Moe calls take the tcgen05 GEMM for blocks of B200_TC_MOE_MIN_BLOCK (64)
// and more (the prefill regime) when every group fits the plan.
#ifndef B200_TC_MOE_MIN_BLOCK
#define B200_TC_MOE_MIN_BLOCK 64
#endif
bool use_tc_moe(int32_t quant, int32_t block_size, int64_t groups) {
  return (quant == B200_QUANT_FP8_BLOCK || quant == B200_QUANT_NVFP4) &&
         block_size >= B200_TC_MOE_MIN_BLOCK &&
         tc_gemm_supported(block_size) &&
         groups * tc_plan_slots_per_group(block_size) <= kTcPlanCap;
}

}  // namespace

int b200::set_last_error(int code, const char* message) {
  g_last_error = message;
  return code;
}

int64_t b200::ws_head_bytes() { return kStatusBytes + kCounterBytes; }
int64_t b200::ws_fixed_bytes() { return stream_ws_bytes(); }

extern "C" {

int b200_abi_version(void) { return 1; }

const char* b200_last_error(void) { return g_last_error.c_str(); }

int b200_num_sms(void) { return device_sm_count(); }

int b200_workspace_status(void* workspace, int32_t* bits, int32_t reset, void* stream) {
  if (workspace == nullptr || bits == nullptr) return fail(B200_ERR_INVALID, "null argument");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int host = 0;
  int rc = check_cuda(cudaMemcpyAsync(&host, workspace, sizeof(int), cudaMemcpyDeviceToHost, st),
                      "status read");
  if (rc) return rc;
  rc = check_cuda(cudaStreamSynchronize(st), "status sync");
  if (rc) return rc;
  *bits = host;
  if (reset && host != 0) {
    rc = check_cuda(cudaMemsetAsync(workspace, 0, sizeof(int), st), "status reset");
    if (rc) return rc;
  }
  return B200_OK;
}

int b200_moe_align_block_size(const int32_t* topk_ids, int64_t numel, int32_t num_experts,
                              int32_t block_size, int32_t* sorted_token_ids,
                              int64_t sorted_capacity, int32_t* expert_ids,
                              int64_t expert_capacity, int32_t* num_tokens_post_pad,
                              void* stream) {
  if (numel < 0 || numel >= (1ll << 31)) return fail(B200_ERR_INVALID, "bad numel %lld", (long long)numel);
  if (num_experts <= 0 || num_experts > moe_align_max_experts())
    return fail(B200_ERR_UNSUPPORTED, "num_experts must be in [1, %d], got %d",
                moe_align_max_experts(), num_experts);
  if (block_size <= 0 || block_size > 4096)
    return fail(B200_ERR_INVALID, "bad block_size %d", block_size);
  // Zero-length arrays may be null (an empty torch tensor has no storage).
  if ((numel > 0 && topk_ids == nullptr) || (sorted_capacity > 0 && sorted_token_ids == nullptr) ||
      (expert_capacity > 0 && expert_ids == nullptr) || num_tokens_post_pad == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  const int64_t busy = numel < num_experts ? numel : num_experts;
  const int64_t need = numel + busy * (block_size - 1);
  if (sorted_capacity < need)
    return fail(B200_ERR_INVALID, "sorted_token_ids holds %lld slots, needs %lld",
                (long long)sorted_capacity, (long long)need);
  if (expert_capacity < (need + block_size - 1) / block_size)
    return fail(B200_ERR_INVALID, "expert_ids holds %lld blocks, needs %lld",
                (long long)expert_capacity, (long long)((need + block_size - 1) / block_size));
  if (sorted_capacity >= (1ll << 31)) return fail(B200_ERR_INVALID, "sorted_capacity too large");
  return check_cuda(launch_moe_align(topk_ids, numel, num_experts, block_size, sorted_token_ids,
                                     sorted_capacity, expert_ids, expert_capacity,
                                     num_tokens_post_pad,
                                     reinterpret_cast<cudaStream_t>(stream)),
                    "moe_align launch");
}

int b200_topk_route(const void* router_logits, int32_t logits_dtype, int64_t tokens,
                    int32_t num_experts, int32_t top_k, int32_t scoring, int32_t renormalize,
                    const float* correction_bias, int32_t* topk_ids, float* topk_weights,
                    void* stream) {
  if (logits_dtype != B200_DTYPE_BF16 && logits_dtype != B200_DTYPE_F16 &&
      logits_dtype != B200_DTYPE_F32)
    return fail(B200_ERR_UNSUPPORTED, "router logits must be bf16, f16 or f32");
  if (tokens < 0) return fail(B200_ERR_INVALID, "bad tokens %lld", (long long)tokens);
  if (num_experts <= 0 || num_experts > router_max_experts())
    return fail(B200_ERR_UNSUPPORTED, "num_experts must be in [1, %d], got %d",
                router_max_experts(), num_experts);
  if (top_k <= 0 || top_k > 32 || top_k > num_experts)
    return fail(B200_ERR_INVALID, "top_k must be in [1, min(32, num_experts)], got %d", top_k);
  if (scoring != B200_SCORING_SOFTMAX && scoring != B200_SCORING_SIGMOID)
    return fail(B200_ERR_INVALID, "unknown scoring %d", scoring);
  if (correction_bias != nullptr && scoring != B200_SCORING_SIGMOID)
    return fail(B200_ERR_INVALID, "a correction bias needs sigmoid scoring");
  if (tokens == 0) return B200_OK;
  if (router_logits == nullptr || topk_ids == nullptr || topk_weights == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  return check_cuda(launch_topk_route(router_logits, logits_dtype, tokens, num_experts, top_k,
                                      scoring, renormalize != 0, correction_bias, topk_ids,
                                      topk_weights, reinterpret_cast<cudaStream_t>(stream)),
                    "router launch");
}

int b200_topk_route_grouped(const void* router_logits, int32_t logits_dtype, int64_t tokens,
                            int32_t num_experts, int32_t top_k, int32_t scoring,
                            int32_t renormalize, const float* correction_bias,
                            int32_t num_expert_group, int32_t topk_group, int32_t* topk_ids,
                            float* topk_weights, void* stream) {
  if (num_expert_group <= 0 || num_expert_group > 32 || num_experts % num_expert_group)
    return fail(B200_ERR_INVALID,
                "num_expert_group must divide num_experts and be in [1, 32], got %d for %d experts",
                num_expert_group, num_experts);
  if (topk_group <= 0 || topk_group > num_expert_group)
    return fail(B200_ERR_INVALID, "topk_group must be in [1, num_expert_group], got %d", topk_group);
  const int32_t per_group = num_experts / num_expert_group;
  if (top_k > topk_group * per_group)
    return fail(B200_ERR_INVALID, "top_k %d exceeds the %d experts of the kept groups", top_k,
                topk_group * per_group);
  if (correction_bias != nullptr && per_group < 2)
    return fail(B200_ERR_INVALID, "biased grouped top-k needs two experts per group");
  if (logits_dtype != B200_DTYPE_BF16 && logits_dtype != B200_DTYPE_F16 &&
      logits_dtype != B200_DTYPE_F32)
    return fail(B200_ERR_UNSUPPORTED, "router logits must be bf16, f16 or f32");
  if (tokens < 0) return fail(B200_ERR_INVALID, "bad tokens %lld", (long long)tokens);
  if (num_experts <= 0 || num_experts > router_max_experts())
    return fail(B200_ERR_UNSUPPORTED, "num_experts must be in [1, %d], got %d",
                router_max_experts(), num_experts);
  if (top_k <= 0 || top_k > 32 || top_k > num_experts)
    return fail(B200_ERR_INVALID, "top_k must be in [1, min(32, num_experts)], got %d", top_k);
  if (scoring != B200_SCORING_SOFTMAX && scoring != B200_SCORING_SIGMOID)
    return fail(B200_ERR_INVALID, "unknown scoring %d", scoring);
  if (correction_bias != nullptr && scoring != B200_SCORING_SIGMOID)
    return fail(B200_ERR_INVALID, "a correction bias needs sigmoid scoring");
  if (tokens == 0) return B200_OK;
  if (router_logits == nullptr || topk_ids == nullptr || topk_weights == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  return check_cuda(launch_topk_route(router_logits, logits_dtype, tokens, num_experts, top_k,
                                      scoring, renormalize != 0, correction_bias, topk_ids,
                                      topk_weights, reinterpret_cast<cudaStream_t>(stream),
                                      num_expert_group, topk_group),
                    "grouped router launch");
}

int b200_append_shared_route(const int32_t* topk_ids, const float* topk_weights, int64_t tokens,
                             int32_t top_k, int32_t shared_id, float shared_weight,
                             int32_t* ids_out, float* weights_out, void* stream) {
  if (tokens < 0 || top_k <= 0) return fail(B200_ERR_INVALID, "bad tokens/top_k");
  if (tokens == 0) return B200_OK;
  if (topk_ids == nullptr || topk_weights == nullptr || ids_out == nullptr || weights_out == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  return check_cuda(launch_append_shared_route(topk_ids, topk_weights, tokens, top_k, shared_id,
                                               shared_weight, ids_out, weights_out,
                                               reinterpret_cast<cudaStream_t>(stream)),
                    "append shared route launch");
}

int b200_moe_sum_reduce(const void* input, void* output, int64_t tokens, int32_t top_k,
                        int64_t hidden, int32_t dtype, float routed_scaling_factor, void* stream) {
  if (!valid_dtype16(dtype)) return fail(B200_ERR_UNSUPPORTED, "dtype must be bf16 or f16");
  if (tokens < 0 || top_k <= 0 || hidden <= 0 || hidden % 8)
    return fail(B200_ERR_INVALID, "bad shape tokens=%lld top_k=%d hidden=%lld (hidden %% 8 == 0)",
                (long long)tokens, top_k, (long long)hidden);
  if (tokens == 0) return B200_OK;
  if (!aligned16(input) || !aligned16(output))
    return fail(B200_ERR_INVALID, "input and output must be 16-byte aligned");
  return check_cuda(launch_moe_sum_reduce(input, output, tokens, top_k, hidden,
                                          dtype == B200_DTYPE_F16, routed_scaling_factor,
                                          reinterpret_cast<cudaStream_t>(stream)),
                    "moe_sum_reduce launch");
}

int b200_moe_combine(const void* routed, int32_t routed_dtype, const int32_t* topk_ids,
                     int32_t num_experts, int64_t tokens, int32_t top_k, int64_t hidden,
                     float routed_scaling_factor, const void* shared_out, int32_t shared_dtype,
                     void* out, int32_t out_dtype, void* stream) {
  if (!valid_dtype16(routed_dtype) || !valid_dtype16(out_dtype) ||
      (shared_out != nullptr && !valid_dtype16(shared_dtype)))
    return fail(B200_ERR_UNSUPPORTED, "dtypes must be bf16 or f16");
  if (tokens < 0 || top_k <= 0 || hidden <= 0 || hidden % 8)
    return fail(B200_ERR_INVALID, "bad shape tokens=%lld top_k=%d hidden=%lld",
                (long long)tokens, top_k, (long long)hidden);
  if (tokens == 0) return B200_OK;
  if (!aligned16(routed) || !aligned16(out) || (shared_out && !aligned16(shared_out)))
    return fail(B200_ERR_INVALID, "buffers must be 16-byte aligned");
  return check_cuda(launch_moe_combine(routed, routed_dtype == B200_DTYPE_F16, topk_ids,
                                       num_experts, tokens, top_k, hidden, routed_scaling_factor,
                                       shared_out, shared_dtype == B200_DTYPE_F16, out,
                                       out_dtype == B200_DTYPE_F16,
                                       reinterpret_cast<cudaStream_t>(stream)),
                    "moe_combine launch");
}

int64_t b200_fp8_packed_bytes(int64_t experts, int64_t n, int64_t k) {
  if (experts <= 0 || n <= 0 || k <= 0) return -1;
  return experts * n * k;
}

int b200_fp8_prepack(const uint8_t* w_e4m3, int64_t experts, int64_t n, int64_t k, int32_t gated,
                     uint8_t* out, void* stream) {
  int rc = check_weight_shape(B200_QUANT_FP8_BLOCK, n, k, gated ? B200_GATED_FUSED : B200_GATED_NONE);
  if (rc) return rc;
  if (experts <= 0) return fail(B200_ERR_INVALID, "experts must be positive");
  if (w_e4m3 == nullptr || out == nullptr) return fail(B200_ERR_INVALID, "null pointer argument");
  if (!aligned16(w_e4m3) || !aligned16(out))
    return fail(B200_ERR_INVALID, "weights must be 16-byte aligned");
  return check_cuda(launch_prepack_fp8(w_e4m3, experts, (int)n, (int)k, gated != 0, out,
                                       reinterpret_cast<cudaStream_t>(stream)),
                    "fp8 prepack launch");
}

int64_t b200_nvfp4_packed_bytes(int64_t experts, int64_t n, int64_t k) {
  if (experts <= 0 || n <= 0 || k <= 0 || n % 128 || k % 128) return -1;
  return experts * (n / 128) * (k / 128) * (int64_t)kFp4UnitBytes;
}

int b200_nvfp4_prepack(const uint8_t* w_packed, const uint8_t* scales_e4m3, int64_t experts,
                       int64_t n, int64_t k, int32_t gated, uint8_t* out, void* stream) {
  int rc = check_weight_shape(B200_QUANT_NVFP4, n, k, gated ? B200_GATED_FUSED : B200_GATED_NONE);
  if (rc) return rc;
  if (experts <= 0) return fail(B200_ERR_INVALID, "experts must be positive");
  if (w_packed == nullptr || scales_e4m3 == nullptr || out == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (!aligned16(w_packed) || !aligned16(out))
    return fail(B200_ERR_INVALID, "weights must be 16-byte aligned");
  return check_cuda(launch_prepack_nvfp4(w_packed, scales_e4m3, experts, (int)n, (int)k,
                                         gated != 0, out, reinterpret_cast<cudaStream_t>(stream)),
                    "nvfp4 prepack launch");
}

int64_t b200_gemm_workspace_bytes(int64_t convert_elems) {
  if (convert_elems < 0) return -1;
  return stream_ws_bytes() + align_up(convert_elems * 2);
}

}  // extern "C"

namespace {

int linear_impl(int32_t quant, const void* x, int32_t x_dtype, int64_t m, int64_t k,
                const uint8_t* w_packed, const float* w_scales, const float* global_scale,
                int64_t n, int32_t gated_mode, void* y, int32_t y_dtype, void* workspace,
                int64_t workspace_bytes, void* stream, bool loads_only) {
  int rc = check_weight_shape(quant, n, k, gated_mode);
  if (rc) return rc;
  if (!valid_dtype16(x_dtype) || !valid_dtype16(y_dtype))
    return fail(B200_ERR_UNSUPPORTED, "activations and output must be bf16 or f16");
  if (m < 0 || m >= (1ll << 31)) return fail(B200_ERR_INVALID, "bad M %lld", (long long)m);
  if (m == 0) return B200_OK;
  if (x == nullptr || w_packed == nullptr || y == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (quant == B200_QUANT_FP8_BLOCK && w_scales == nullptr)
    return fail(B200_ERR_INVALID, "FP8 weights need their block scales");
  if (quant == B200_QUANT_NVFP4 && global_scale == nullptr)
    return fail(B200_ERR_INVALID, "NVFP4 weights need their global scale");
  if (!aligned16(x) || !aligned16(w_packed))
    return fail(B200_ERR_INVALID, "x and weights must be 16-byte aligned");
  WsView ws;
  if (!carve(workspace, workspace_bytes, ws))
    return fail(B200_ERR_INVALID, "workspace missing, misaligned or smaller than %lld bytes",
                (long long)stream_ws_bytes());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (use_tc_dense(m, n)) {
    // Prefill-sized batch: tcgen05 tensor cores.
    int64_t used_tc = 0;
    const __half* xh = nullptr;
    rc = stage_activations(x, x_dtype, m * k, ws, used_tc, &xh, st);
    if (rc) return rc;
    StreamParams p{};
    p.wq = w_packed;
    p.wscale = w_scales;
    p.gscale = global_scale;
    p.x = xh;
    p.ldx = k;
    p.x_rows = m;
    p.xs = xh;  // contiguous rows: B tiles by TMA
    p.xs_rows = m;
    p.sorted_ids = nullptr;
    p.dense_m = (int)m;
    p.E = 1;
    p.N = (int)n;
    p.K = (int)k;
    p.gated = gated_mode != B200_GATED_NONE;
    p.fuse_act = gated_mode == B200_GATED_FUSED;
    p.out = y;
    p.ldo = gated_mode == B200_GATED_FUSED ? n / 2 : n;
    p.out_f16 = y_dtype == B200_DTYPE_F16;
    // Items (192-row chunk x 128-row weight block) are dealt round-robin over
    // the SMs, each streaming its K range. Split K (parts summed in fp32 in
    // the workspace, then a finishing kernel) when that cuts the busiest SM's
    // 128-K unit count by a quarter or more, each part charged for its m*n
    // fp32 atomic adds at 3x the time of streaming the same bytes of weights.
    // Measured on B200: a split that only evens out waves is slower
    // (64 x 25600 x 5120: 64 us unsplit, 87 us in two parts), one that fills
    // idle SMs is faster (128 x 4096 x 7168: 43 us in three parts, 35 us in
    // four; 64 x 5120 x 25600: 64 us in three, 60 us in seven).
    p.ksplit = dense_k_parts(m, n, k);
    p.loads_only = loads_only ? 1 : 0;
    rc = run_tc(quant, p, ws, false, st, m <= tc_narrow_slots());
    if (rc || p.ksplit <= 1 || loads_only) return rc;
    return check_cuda(launch_tc_split_finish(p, st), "split-K finish launch");
  }
  int64_t used = 0;
  const __half* x16 = nullptr;
  rc = stage_activations(x, x_dtype, m * k, ws, used, &x16, st);
  if (rc) return rc;

  StreamParams p{};
  p.wq = w_packed;
  p.wscale = w_scales;
  p.gscale = global_scale;
  p.x = x16;
  p.ldx = k;
  p.x_rows = m;
  p.sorted_ids = nullptr;
  p.E = 1;
  p.N = (int)n;
  p.K = (int)k;
  p.gated = gated_mode != B200_GATED_NONE;
  p.fuse_act = gated_mode == B200_GATED_FUSED;
  p.mul_w = 0;
  p.out = y;
  p.ldo = gated_mode == B200_GATED_FUSED ? n / 2 : n;
  p.out_f16 = y_dtype == B200_DTYPE_F16;
  const int nt = nt_for_rows(m);
  p.dense_m = (int)m;
  p.loads_only = loads_only ? 1 : 0;
  const long long groups = (m + 8 * nt - 1) / (8 * nt);
  const long long units = groups * (n / 128) * (k / 128);
  return run_stream(quant, nt, p, units, ws, st);
}

}  // namespace

extern "C" {

int b200_linear(int32_t quant, const void* x, int32_t x_dtype, int64_t m, int64_t k,
                const uint8_t* w_packed, const float* w_scales, const float* global_scale,
                int64_t n, int32_t gated_mode, void* y, int32_t y_dtype, void* workspace,
                int64_t workspace_bytes, void* stream) {
  return linear_impl(quant, x, x_dtype, m, k, w_packed, w_scales, global_scale, n, gated_mode, y,
                     y_dtype, workspace, workspace_bytes, stream, false);
}

int b200_linear_loads_only(int32_t quant, const void* x, int32_t x_dtype, int64_t m, int64_t k,
                           const uint8_t* w_packed, const float* w_scales,
                           const float* global_scale, int64_t n, int32_t gated_mode, void* y,
                           int32_t y_dtype, void* workspace, int64_t workspace_bytes,
                           void* stream) {
  return linear_impl(quant, x, x_dtype, m, k, w_packed, w_scales, global_scale, n, gated_mode, y,
                     y_dtype, workspace, workspace_bytes, stream, true);
}

int b200_linear_path(int64_t m, int64_t n, int64_t k, int32_t* tile_rows, int32_t* k_parts) {
  if (m <= 0 || n <= 0 || k <= 0 || n % 128 || k % 128)
    return fail(B200_ERR_INVALID, "bad shape m=%lld n=%lld k=%lld", (long long)m, (long long)n,
                (long long)k);
  int32_t rows = 0, parts = 1;
  int path = B200_PATH_STREAM;
  if (use_tc_dense(m, n)) {
    path = B200_PATH_TCGEN05;
    rows = 192;
    parts = dense_k_parts(m, n, k);
  } else {
    rows = 8 * nt_for_rows(m);
  }
  if (tile_rows) *tile_rows = rows;
  if (k_parts) *k_parts = parts;
  return path;
}

int b200_moe_path(int32_t quant, int32_t block_size, int64_t expert_capacity, int32_t* tile_rows) {
  if (quant != B200_QUANT_FP8_BLOCK && quant != B200_QUANT_NVFP4)
    return fail(B200_ERR_INVALID, "unknown quant %d", quant);
  if (block_size <= 0 || expert_capacity < 0) return fail(B200_ERR_INVALID, "bad block size");
  if (use_tc_moe(quant, block_size, expert_capacity)) {
    if (tile_rows) *tile_rows = 192;
    return B200_PATH_TCGEN05;
  }
  if (tile_rows) *tile_rows = block_size;
  return B200_PATH_STREAM;
}

}  // extern "C"

namespace {

int moe_gemm_impl(int32_t quant, const void* a, int32_t a_dtype, int64_t a_rows, int64_t k,
                  const uint8_t* w_packed, const float* w_scales, const float* global_scale,
                  int32_t num_experts, int64_t n, int32_t gated_mode,
                  const int32_t* sorted_token_ids, const int32_t* expert_ids,
                  int64_t expert_capacity, const int32_t* num_tokens_post_pad,
                  int32_t block_size, int32_t top_k, int64_t num_routes,
                  const float* topk_weights, int32_t mul_topk_weights, void* c, int32_t c_dtype,
                  int64_t ldc, void* workspace, int64_t workspace_bytes, void* stream,
                  bool loads_only) {
  int rc = check_weight_shape(quant, n, k, gated_mode);
  if (rc) return rc;
  if (!valid_dtype16(a_dtype) || !valid_dtype16(c_dtype))
    return fail(B200_ERR_UNSUPPORTED, "activations and output must be bf16 or f16");
  const bool tc = use_tc_moe(quant, block_size, expert_capacity);
  if (!tc && block_size != 8 && block_size != 16 && block_size != 32 && block_size != 64)
    return fail(B200_ERR_UNSUPPORTED,
                "block_size must be 8, 16, 32, 64, 128 or 256, got %d", block_size);
  if (num_experts <= 0 || num_experts >= (1 << 23))
    return fail(B200_ERR_INVALID, "num_experts must be in [1, 2^23)");
  if (top_k <= 0) return fail(B200_ERR_INVALID, "top_k must be positive");
  if (a_rows < 0 || num_routes < 0 || num_routes >= (1ll << 31) || expert_capacity < 0)
    return fail(B200_ERR_INVALID, "bad row counts");
  const int64_t out_cols = gated_mode == B200_GATED_FUSED ? n / 2 : n;
  if (ldc < out_cols) return fail(B200_ERR_INVALID, "ldc %lld < output width %lld",
                                  (long long)ldc, (long long)out_cols);
  if (expert_capacity == 0 || num_routes == 0 || a_rows == 0) return B200_OK;
  if (a == nullptr || w_packed == nullptr || c == nullptr || sorted_token_ids == nullptr ||
      expert_ids == nullptr || num_tokens_post_pad == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (mul_topk_weights && topk_weights == nullptr)
    return fail(B200_ERR_INVALID, "mul_topk_weights needs topk_weights");
  if (quant == B200_QUANT_FP8_BLOCK && w_scales == nullptr)
    return fail(B200_ERR_INVALID, "FP8 weights need their block scales");
  if (quant == B200_QUANT_NVFP4 && global_scale == nullptr)
    return fail(B200_ERR_INVALID, "NVFP4 weights need their global scale");
  if (!aligned16(a) || !aligned16(w_packed))
    return fail(B200_ERR_INVALID, "activations and weights must be 16-byte aligned");
  WsView ws;
  if (!carve(workspace, workspace_bytes, ws))
    return fail(B200_ERR_INVALID, "workspace missing, misaligned or smaller than %lld bytes",
                (long long)stream_ws_bytes());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int64_t used = 0;
  const __half* a16 = nullptr;
  rc = stage_activations(a, a_dtype, a_rows * k, ws, used, &a16, st);
  if (rc) return rc;

  StreamParams p{};
  p.wq = w_packed;
  p.wscale = w_scales;
  p.gscale = global_scale;
  p.x = a16;
  p.ldx = k;
  p.x_rows = a_rows;
  p.sorted_ids = sorted_token_ids;
  p.expert_ids = expert_ids;
  p.ntpp = num_tokens_post_pad;
  p.block_m = block_size;
  p.max_groups = expert_capacity;
  p.top_k = top_k;
  p.num_routes = (int)num_routes;
  p.topk_w = topk_weights;
  p.E = num_experts;
  p.N = (int)n;
  p.K = (int)k;
  p.gated = gated_mode != B200_GATED_NONE;
  p.fuse_act = gated_mode == B200_GATED_FUSED;
  p.mul_w = mul_topk_weights != 0;
  p.out = c;
  p.ldo = ldc;
  p.out_f16 = c_dtype == B200_DTYPE_F16;
  p.loads_only = loads_only ? 1 : 0;
  if (tc) return run_tc(quant, p, ws, false, st, narrow_moe(block_size, num_routes, num_experts));
  const long long units = (long long)expert_capacity * (n / 128) * (k / 128);
  return run_stream(quant, block_size / 8, p, units, ws, st);
}

}  // namespace

extern "C" {

int b200_moe_gemm(int32_t quant, const void* a, int32_t a_dtype, int64_t a_rows, int64_t k,
                  const uint8_t* w_packed, const float* w_scales, const float* global_scale,
                  int32_t num_experts, int64_t n, int32_t gated_mode,
                  const int32_t* sorted_token_ids, const int32_t* expert_ids,
                  int64_t expert_capacity, const int32_t* num_tokens_post_pad,
                  int32_t block_size, int32_t top_k, int64_t num_routes,
                  const float* topk_weights, int32_t mul_topk_weights, void* c, int32_t c_dtype,
                  int64_t ldc, void* workspace, int64_t workspace_bytes, void* stream) {
  return moe_gemm_impl(quant, a, a_dtype, a_rows, k, w_packed, w_scales, global_scale,
                       num_experts, n, gated_mode, sorted_token_ids, expert_ids, expert_capacity,
                       num_tokens_post_pad, block_size, top_k, num_routes, topk_weights,
                       mul_topk_weights, c, c_dtype, ldc, workspace, workspace_bytes, stream,
                       false);
}

int b200_moe_gemm_loads_only(int32_t quant, const void* a, int32_t a_dtype, int64_t a_rows,
                             int64_t k, const uint8_t* w_packed, const float* w_scales,
                             const float* global_scale, int32_t num_experts, int64_t n,
                             int32_t gated_mode, const int32_t* sorted_token_ids,
                             const int32_t* expert_ids, int64_t expert_capacity,
                             const int32_t* num_tokens_post_pad, int32_t block_size,
                             int32_t top_k, int64_t num_routes, const float* topk_weights,
                             int32_t mul_topk_weights, void* c, int32_t c_dtype, int64_t ldc,
                             void* workspace, int64_t workspace_bytes, void* stream) {
  return moe_gemm_impl(quant, a, a_dtype, a_rows, k, w_packed, w_scales, global_scale,
                       num_experts, n, gated_mode, sorted_token_ids, expert_ids, expert_capacity,
                       num_tokens_post_pad, block_size, top_k, num_routes, topk_weights,
                       mul_topk_weights, c, c_dtype, ldc, workspace, workspace_bytes, stream,
                       true);
}

int64_t b200_moe_layer_workspace_bytes(int64_t tokens, int64_t hidden, int64_t inter,
                                       int32_t num_experts, int32_t top_k, int32_t block_size) {
  if (tokens < 0 || hidden <= 0 || inter <= 0 || num_experts <= 0 || top_k <= 0 || block_size <= 0)
    return -1;
  const int64_t numel = tokens * top_k;
  const int64_t busy = numel < num_experts ? numel : num_experts;
  const int64_t cap = numel + busy * (block_size - 1);
  const int64_t blocks = (cap + block_size - 1) / block_size;
  // Streaming path: f16 activations + gate_up output per route. tcgen05
  // path (blocks of 64+): both operands in slot order, one row per slot.
  const int64_t stream_ops = align_up(tokens * hidden * 2) + align_up(numel * inter * 2);
  const int64_t tc_ops = block_size >= 64 ? align_up(cap * hidden * 2) + align_up(cap * inter * 2) : 0;
  return stream_ws_bytes() + (stream_ops > tc_ops ? stream_ops : tc_ops)  // operands
         + align_up(cap * 4) + align_up(blocks * 4) + align_up(4)           // routing
         + align_up(numel * hidden * 2);                                     // per-route down output
}

}  // extern "C"

namespace {

// Routing from router logits (b200_moe_layer_forward_logits): the chosen
// routes go to the caller's ids / weights buffers.
struct RouterArgs {
  const void* logits;
  int32_t dtype, scoring, renormalize;
  const float* bias;
  int32_t* ids_out;
  float* weights_out;
};

// The shared expert fused into the routed bank as its last expert
// (b200_moe_layer_forward_fused_shared): one more route per token, id
// num_experts (the routed count), weight `weight`, written with the routed
// ones to the caller's [tokens, top_k + 1] buffers.
struct SharedRoute {
  float weight;
  int32_t* ids_out;
  float* weights_out;
};

int layer_forward(int32_t quant, const void* x, int32_t x_dtype, int64_t tokens, int64_t hidden,
                  int64_t inter, const int32_t* topk_ids, const float* topk_weights, int32_t top_k,
                  int32_t num_experts, const uint8_t* w13_packed, const float* w13_scales,
                  const float* w13_global, const uint8_t* w2_packed, const float* w2_scales,
                  const float* w2_global, int32_t block_size, float routed_scaling_factor,
                  const void* shared_out, int32_t shared_dtype, void* out, int32_t out_dtype,
                  void* workspace, int64_t workspace_bytes, void* stream, const RouterArgs* router,
                  const SharedRoute* shared_route = nullptr) {
  int rc = check_weight_shape(quant, 2 * inter, hidden, B200_GATED_FUSED);
  if (rc) return rc;
  rc = check_weight_shape(quant, hidden, inter, B200_GATED_NONE);
  if (rc) return rc;
  if (!valid_dtype16(x_dtype) || !valid_dtype16(out_dtype))
    return fail(B200_ERR_UNSUPPORTED, "activations and output must be bf16 or f16");
  if (tokens < 0 || top_k <= 0 || num_experts <= 0)
    return fail(B200_ERR_INVALID, "bad tokens/top_k/num_experts");
  if (tokens == 0) return B200_OK;
  if (num_experts >= (1 << 23)) return fail(B200_ERR_INVALID, "num_experts must be below 2^23");
  const bool tc_block = block_size >= 64 && tc_gemm_supported(block_size);
  if (!tc_block && block_size != 8 && block_size != 16 && block_size != 32 && block_size != 64)
    return fail(B200_ERR_UNSUPPORTED,
                "block_size must be 8, 16, 32, 64, 128 or 256, got %d", block_size);
  if (router != nullptr) {
    topk_ids = router->ids_out;
    topk_weights = router->weights_out;
  }
  // The caller's routes; with a fused shared expert the layer runs on the
  // extended routes (one more per token, one more expert).
  const int32_t* in_ids = topk_ids;
  const float* in_w = topk_weights;
  const int32_t in_k = top_k;
  if (shared_route != nullptr) {
    if (router != nullptr) return fail(B200_ERR_INVALID, "router and shared route are exclusive");
    if (shared_route->ids_out == nullptr || shared_route->weights_out == nullptr)
      return fail(B200_ERR_INVALID, "null pointer argument");
    topk_ids = shared_route->ids_out;
    topk_weights = shared_route->weights_out;
    top_k += 1;
    num_experts += 1;
  }
  if (x == nullptr || in_ids == nullptr || in_w == nullptr || w13_packed == nullptr ||
      w2_packed == nullptr || out == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  const int64_t need = b200_moe_layer_workspace_bytes(tokens, hidden, inter, num_experts, top_k,
                                                      block_size);
  if (workspace_bytes < need)
    return fail(B200_ERR_INVALID, "workspace holds %lld bytes, needs %lld",
                (long long)workspace_bytes, (long long)need);
  WsView ws;
  if (!carve(workspace, workspace_bytes, ws))
    return fail(B200_ERR_INVALID, "workspace missing or misaligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  const int64_t numel = tokens * top_k;
  const int64_t busy = numel < num_experts ? numel : num_experts;
  const int64_t cap = numel + busy * (block_size - 1);
  const int64_t blocks = (cap + block_size - 1) / block_size;
  const bool tc = use_tc_moe(quant, block_size, blocks);
  int64_t used = 0;
  const __half* x16 = nullptr;
  __half* x16_conv = nullptr;  // bf16 activations converted for the stream GEMM
  __half* xs = nullptr;  // tcgen05: activations in slot order
  __half* inter_out = nullptr;
  if (tc) {
    xs = reinterpret_cast<__half*>(ws.scratch + used);
    used += align_up(cap * hidden * 2);
    inter_out = reinterpret_cast<__half*>(ws.scratch + used);  // slot order
    used += align_up(cap * inter * 2);
    const int64_t stream_ops = align_up(tokens * hidden * 2) + align_up(numel * inter * 2);
    if (used < stream_ops) used = stream_ops;
  } else {
    // f16 operand of the weight-streaming GEMM: the caller's rows, or a
    // converted copy written below (by the preparation kernel when it runs)
    if (x_dtype == B200_DTYPE_F16) {
      x16 = reinterpret_cast<const __half*>(x);
    } else {
      x16_conv = reinterpret_cast<__half*>(ws.scratch + used);
      x16 = x16_conv;
    }
    used += align_up(tokens * hidden * 2);
    inter_out = reinterpret_cast<__half*>(ws.scratch + used);  // route order
    used += align_up(numel * inter * 2);
    const int64_t tc_ops =
        block_size >= 64 ? align_up(cap * hidden * 2) + align_up(cap * inter * 2) : 0;
    if (used < tc_ops) used = tc_ops;
  }
  int32_t* sorted = reinterpret_cast<int32_t*>(ws.scratch + used);
  used += align_up(cap * 4);
  int32_t* eids = reinterpret_cast<int32_t*>(ws.scratch + used);
  used += align_up(blocks * 4);
  int32_t* ntpp = reinterpret_cast<int32_t*>(ws.scratch + used);
  used += align_up(4);
  __half* routed = reinterpret_cast<__half*>(ws.scratch + used);
  used += align_up(numel * hidden * 2);

  if (num_experts > moe_align_max_experts())
    return fail(B200_ERR_UNSUPPORTED, "num_experts must be in [1, %d], got %d",
                moe_align_max_experts(), num_experts);
  bool converted = x16_conv == nullptr;
  if (router != nullptr && tokens <= 32 && numel < kAlignMultiMin) {
    // Up to one token per warp: route and align in one launch. (Measured no
    // faster than the two kernels, which programmatic dependent launch
    // already overlaps; with more tokens the single CTA's routing is slower.)
    rc = check_cuda(launch_route_align(router->logits, router->dtype, tokens, num_experts, top_k,
                                       router->scoring, router->renormalize, router->bias,
                                       router->ids_out, router->weights_out, block_size, sorted,
                                       cap, eids, blocks, ntpp, st),
                    "route + align launch");
  } else if (numel >= kAlignMultiMin) {
    if (router != nullptr) {
      rc = check_cuda(launch_topk_route(router->logits, router->dtype, tokens, num_experts, top_k,
                                        router->scoring, router->renormalize, router->bias,
                                        router->ids_out, router->weights_out, st),
                      "router launch");
      if (rc) return rc;
    }
    if (shared_route != nullptr) {
      rc = check_cuda(launch_append_shared_route(in_ids, in_w, tokens, in_k, num_experts - 1,
                                                 shared_route->weight, shared_route->ids_out,
                                                 shared_route->weights_out, st),
                      "append shared route launch");
      if (rc) return rc;
    }
    // Many routes: the multi-CTA align, its per-segment histograms in the
    // routed-output buffer (written only later, by the down GEMM).
    rc = check_cuda(launch_moe_align_multi(topk_ids, numel, num_experts, block_size, sorted, cap,
                                           eids, blocks, ntpp, reinterpret_cast<int*>(routed), st),
                    "moe_align launch");
  } else {
    if (router != nullptr) {
      rc = check_cuda(launch_topk_route(router->logits, router->dtype, tokens, num_experts, top_k,
                                        router->scoring, router->renormalize, router->bias,
                                        router->ids_out, router->weights_out, st),
                      "router launch");
      if (rc) return rc;
    }
    // Small batches: the shared-route append, the align and the activation
    // conversion share one launch (each is a few microseconds of latency in
    // a decode step's chain of dependent kernels).
    rc = check_cuda(launch_moe_prep(in_ids, in_w, tokens, in_k, num_experts,
                                    shared_route != nullptr ? 1 : 0,
                                    shared_route != nullptr ? shared_route->weight : 0.f,
                                    shared_route != nullptr ? shared_route->ids_out : nullptr,
                                    shared_route != nullptr ? shared_route->weights_out : nullptr,
                                    block_size, sorted, cap, eids, blocks, ntpp,
                                    converted ? nullptr : x, x16_conv, tokens * hidden, st),
                    "moe_prep launch");
    converted = true;
  }
  if (rc) return rc;
  if (!converted) {
    rc = check_cuda(launch_bf16_to_f16(x, x16_conv, tokens * hidden, st), "bf16->f16 conversion");
    if (rc) return rc;
  }
  if (tc) {
    // One slot-ordered f16 copy of the routed rows (bf16 converted on the
    // way): the GEMM reads it as TMA tiles instead of gathering per route.
    rc = check_cuda(launch_permute_rows(x, x_dtype == B200_DTYPE_F16, hidden, tokens, hidden,
                                        sorted, ntpp, cap, top_k, numel, xs, st),
                    "permute launch");
    if (rc) return rc;
  }

  StreamParams p{};
  p.wq = w13_packed;
  p.wscale = w13_scales;
  p.gscale = w13_global;
  p.x = x16;
  p.ldx = hidden;
  p.x_rows = tokens;
  p.xs = xs;
  p.xs_rows = cap;
  p.out_by_slot = tc ? 1 : 0;
  p.sorted_ids = sorted;
  p.expert_ids = eids;
  p.ntpp = ntpp;
  p.block_m = block_size;
  p.max_groups = cap / block_size;
  p.top_k = top_k;
  p.num_routes = (int)numel;
  p.topk_w = topk_weights;
  p.E = num_experts;
  p.N = (int)(2 * inter);
  p.K = (int)hidden;
  p.gated = 1;
  p.fuse_act = 1;
  p.mul_w = 0;
  p.out = inter_out;
  p.ldo = inter;
  p.out_f16 = 1;
  const int nt = block_size / 8;
  if (tc)
    rc = run_tc(quant, p, ws, false, st, narrow_moe(block_size, numel, num_experts));
  else
    rc = run_stream(quant, nt, p, blocks * (2 * inter / 128) * (hidden / 128), ws, st);
  if (rc) return rc;

  StreamParams q = p;
  q.wq = w2_packed;
  q.wscale = w2_scales;
  q.gscale = w2_global;
  q.x = inter_out;
  q.ldx = inter;
  q.x_rows = numel;
  q.xs = tc ? inter_out : nullptr;  // written in slot order by the gate/up epilogue
  q.xs_rows = cap;
  q.out_by_slot = 0;
  q.top_k = 1;
  q.N = (int)hidden;
  q.K = (int)inter;
  q.gated = 0;
  q.fuse_act = 0;
  q.mul_w = 1;
  q.out = routed;
  q.ldo = hidden;
  q.out_f16 = 1;
  if (tc)
    rc = run_tc(quant, q, ws, true, st, narrow_moe(block_size, numel, num_experts));
  else
    rc = run_stream(quant, nt, q, blocks * (hidden / 128) * (inter / 128), ws, st);
  if (rc) return rc;

  return b200_moe_combine(routed, B200_DTYPE_F16, topk_ids, num_experts, tokens, top_k, hidden,
                          routed_scaling_factor, shared_out, shared_dtype, out, out_dtype, stream);
}

}  // namespace

extern "C" {

int b200_moe_layer_forward(int32_t quant, const void* x, int32_t x_dtype, int64_t tokens,
                           int64_t hidden, int64_t inter, const int32_t* topk_ids,
                           const float* topk_weights, int32_t top_k, int32_t num_experts,
                           const uint8_t* w13_packed, const float* w13_scales,
                           const float* w13_global, const uint8_t* w2_packed,
                           const float* w2_scales, const float* w2_global, int32_t block_size,
                           float routed_scaling_factor, const void* shared_out,
                           int32_t shared_dtype, void* out, int32_t out_dtype, void* workspace,
                           int64_t workspace_bytes, void* stream) {
  return layer_forward(quant, x, x_dtype, tokens, hidden, inter, topk_ids, topk_weights, top_k,
                       num_experts, w13_packed, w13_scales, w13_global, w2_packed, w2_scales,
                       w2_global, block_size, routed_scaling_factor, shared_out, shared_dtype, out,
                       out_dtype, workspace, workspace_bytes, stream, nullptr);
}

int b200_moe_layer_forward_fused_shared(
    int32_t quant, const void* x, int32_t x_dtype, int64_t tokens, int64_t hidden, int64_t inter,
    const int32_t* topk_ids, const float* topk_weights, int32_t top_k, int32_t num_experts,
    float shared_route_weight, int32_t* topk_ids_out, float* topk_weights_out,
    const uint8_t* w13_packed, const float* w13_scales, const float* w13_global,
    const uint8_t* w2_packed, const float* w2_scales, const float* w2_global, int32_t block_size,
    float routed_scaling_factor, void* out, int32_t out_dtype, void* workspace,
    int64_t workspace_bytes, void* stream) {
  if (tokens > 0 && (topk_ids_out == nullptr || topk_weights_out == nullptr))
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (tokens > 0 && (topk_ids_out == topk_ids ||
                     (const void*)topk_weights_out == (const void*)topk_weights))
    return fail(B200_ERR_INVALID, "the extended routes must not overwrite the input routes");
  const SharedRoute sr{shared_route_weight, topk_ids_out, topk_weights_out};
  return layer_forward(quant, x, x_dtype, tokens, hidden, inter, topk_ids, topk_weights, top_k,
                       num_experts, w13_packed, w13_scales, w13_global, w2_packed, w2_scales,
                       w2_global, block_size, routed_scaling_factor, nullptr, x_dtype, out,
                       out_dtype, workspace, workspace_bytes, stream, nullptr, &sr);
}

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
                                  void* workspace, int64_t workspace_bytes, void* stream) {
  if (logits_dtype != B200_DTYPE_BF16 && logits_dtype != B200_DTYPE_F16 &&
      logits_dtype != B200_DTYPE_F32)
    return fail(B200_ERR_UNSUPPORTED, "router logits must be bf16, f16 or f32");
  if (num_experts <= 0 || num_experts > router_max_experts() ||
      num_experts > moe_align_max_experts())
    return fail(B200_ERR_UNSUPPORTED, "num_experts must be in [1, %d], got %d",
                router_max_experts(), num_experts);
  if (top_k <= 0 || top_k > 32 || top_k > num_experts)
    return fail(B200_ERR_INVALID, "top_k must be in [1, min(32, num_experts)], got %d", top_k);
  if (scoring != B200_SCORING_SOFTMAX && scoring != B200_SCORING_SIGMOID)
    return fail(B200_ERR_INVALID, "unknown scoring %d", scoring);
  if (correction_bias != nullptr && scoring != B200_SCORING_SIGMOID)
    return fail(B200_ERR_INVALID, "a correction bias needs sigmoid scoring");
  if (tokens > 0 && (router_logits == nullptr || topk_ids_out == nullptr ||
                     topk_weights_out == nullptr))
    return fail(B200_ERR_INVALID, "null pointer argument");
  const RouterArgs r{router_logits, logits_dtype, scoring, renormalize != 0, correction_bias,
                     topk_ids_out, topk_weights_out};
  return layer_forward(quant, x, x_dtype, tokens, hidden, inter, nullptr, nullptr, top_k,
                       num_experts, w13_packed, w13_scales, w13_global, w2_packed, w2_scales,
                       w2_global, block_size, routed_scaling_factor, shared_out, shared_dtype, out,
                       out_dtype, workspace, workspace_bytes, stream, &r);
}

}  // extern "C"

// ------------------------------------------------------ expert parallelism

namespace {

using CuMemGetAddressRange = int (*)(unsigned long long*, size_t*, unsigned long long);

CuMemGetAddressRange get_address_range_fn() {
  static CuMemGetAddressRange fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CuMemGetAddressRange>(ptr);
  }
  return fn;
}

int check_ep_common(int32_t rank, int32_t world, int64_t max_tokens, int32_t top_k, int64_t hidden,
                    const void* region, const uint64_t* peers) {
  if (world < 1 || world > kEpMaxWorld)
    return fail(B200_ERR_INVALID, "world must be in [1, %d], got %d", kEpMaxWorld, world);
  if (rank < 0 || rank >= world) return fail(B200_ERR_INVALID, "rank %d outside [0, %d)", rank, world);
  if (max_tokens <= 0 || top_k <= 0 || top_k > 32 || hidden <= 0 || hidden % 128)
    return fail(B200_ERR_INVALID,
                "bad max_tokens=%lld top_k=%d hidden=%lld (top_k <= 32, hidden %% 128 == 0)",
                (long long)max_tokens, top_k, (long long)hidden);
  if ((int64_t)world * max_tokens * top_k >= (1ll << 31))
    return fail(B200_ERR_INVALID, "world * max_tokens * top_k must stay below 2^31");
  if (region == nullptr || (reinterpret_cast<uintptr_t>(region) % kAlign) != 0)
    return fail(B200_ERR_INVALID, "region missing or not 256-byte aligned");
  if (peers != nullptr && (reinterpret_cast<uintptr_t>(peers) & 7u))
    return fail(B200_ERR_INVALID, "peer_regions must be 8-byte aligned");
  return B200_OK;
}

// Expert-parallel owner workspace: fixed part, routing, align scratch, the
// gate_up output for every received route slot, and the down GEMM's weighted
// route rows that the pre-sum adds up per received row.
struct EpWs {
  int64_t numel, cap_a, blocks, total;
};
EpWs ep_ws(int32_t world, int64_t max_tokens, int32_t top_k, int64_t hidden, int64_t inter,
           int32_t local_experts, int32_t block_size) {
  EpWs w;
  w.numel = (int64_t)world * max_tokens * top_k;
  const int64_t busy = w.numel < local_experts ? w.numel : local_experts;
  w.cap_a = w.numel + busy * (block_size - 1);
  w.blocks = (w.cap_a + block_size - 1) / block_size;
  // gate_up output per route (streaming path) or, for blocks of 64+, both
  // tcgen05 operands in slot order (received rows + gate_up output).
  const int64_t stream_ops = align_up(w.numel * inter * 2);
  const int64_t tc_ops =
      block_size >= 64 ? align_up(w.cap_a * hidden * 2) + align_up(w.cap_a * inter * 2) : 0;
  w.total = stream_ws_bytes() + align_up(w.cap_a * 4) + align_up(w.blocks * 4) + align_up(4) +
            align_up(moe_align_scratch_ints(w.numel, local_experts) * 4) +
            (stream_ops > tc_ops ? stream_ops : tc_ops) + align_up(w.numel * hidden * 2);
  return w;
}

}  // namespace

extern "C" {

int64_t b200_ep_region_bytes(int32_t world, int64_t max_tokens, int32_t top_k, int64_t hidden) {
  if (world < 1 || world > kEpMaxWorld || max_tokens <= 0 || top_k <= 0 || hidden <= 0) return -1;
  return ep_layout(world, max_tokens, top_k, hidden).total;
}

int b200_ep_region_layout(int32_t world, int64_t max_tokens, int32_t top_k, int64_t hidden,
                          int64_t* offsets) {
  if (world < 1 || world > kEpMaxWorld || max_tokens <= 0 || top_k <= 0 || hidden <= 0 ||
      offsets == nullptr)
    return fail(B200_ERR_INVALID, "bad region shape");
  const EpLayout L = ep_layout(world, max_tokens, top_k, hidden);
  const int64_t v[7] = {L.off_ids, L.off_w, L.off_orig, L.off_rows, L.off_recv, L.off_comb, L.total};
  for (int i = 0; i < 7; ++i) offsets[i] = v[i];
  return B200_OK;
}

int b200_ipc_get_handle(const void* dev_ptr, void* handle, int64_t* offset) {
  if (dev_ptr == nullptr || handle == nullptr || offset == nullptr)
    return fail(B200_ERR_INVALID, "null argument");
  CuMemGetAddressRange range = get_address_range_fn();
  if (range == nullptr) return fail(B200_ERR_CUDA, "cuMemGetAddressRange is not available");
  unsigned long long base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<unsigned long long>(dev_ptr)) != 0)
    return fail(B200_ERR_INVALID, "pointer is not device memory of this process");
  cudaIpcMemHandle_t h;
  int rc = check_cuda(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  if (rc) return rc;
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<unsigned long long>(dev_ptr) - base);
  return B200_OK;
}

int b200_ipc_open_handle(const void* handle, int64_t offset, void** dev_ptr) {
  if (handle == nullptr || dev_ptr == nullptr || offset < 0)
    return fail(B200_ERR_INVALID, "bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  int rc = check_cuda(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess),
                      "cudaIpcOpenMemHandle");
  if (rc) return rc;
  *dev_ptr = static_cast<uint8_t*>(base) + offset;
  return B200_OK;
}

int b200_ipc_close_handle(void* dev_ptr, int64_t offset) {
  if (dev_ptr == nullptr || offset < 0) return fail(B200_ERR_INVALID, "bad argument");
  return check_cuda(cudaIpcCloseMemHandle(static_cast<uint8_t*>(dev_ptr) - offset),
                    "cudaIpcCloseMemHandle");
}

int b200_ep_dispatch(const void* x, int32_t x_dtype, int64_t tokens, int64_t hidden,
                     const int32_t* topk_ids, const float* topk_weights, int32_t top_k,
                     int32_t num_experts, int32_t shared_expert, int32_t rank, int32_t world,
                     const uint64_t* peer_regions, void* region, int64_t max_tokens,
                     void* stream) {
  int rc = check_ep_common(rank, world, max_tokens, top_k, hidden, region, peer_regions);
  if (rc) return rc;
  if (!valid_dtype16(x_dtype)) return fail(B200_ERR_UNSUPPORTED, "activations must be bf16 or f16");
  if (tokens < 0 || tokens > max_tokens)
    return fail(B200_ERR_INVALID, "tokens %lld outside [0, max_tokens=%lld]", (long long)tokens,
                (long long)max_tokens);
  if (num_experts <= 0 || num_experts % world)
    return fail(B200_ERR_INVALID, "%d experts do not split over %d ranks", num_experts, world);
  if (peer_regions == nullptr) return fail(B200_ERR_INVALID, "null peer_regions");
  if (tokens > 0 && (x == nullptr || topk_ids == nullptr || topk_weights == nullptr))
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (tokens > 0 && !aligned16(x)) return fail(B200_ERR_INVALID, "x must be 16-byte aligned");
  if ((int64_t)ep_dispatch_chunk(tokens > 0 ? tokens : 1) * world * 4 > 48 * 1024)
    return fail(B200_ERR_UNSUPPORTED, "too many tokens for one dispatch");
  const EpLayout L = ep_layout(world, max_tokens, top_k, hidden);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return check_cuda(launch_ep_dispatch(x, x_dtype == B200_DTYPE_F16, tokens, hidden, topk_ids,
                                       topk_weights, top_k, num_experts, shared_expert != 0,
                                       num_experts / world, rank, world,
                                       reinterpret_cast<const unsigned long long*>(peer_regions),
                                       region, L, st),
                    "ep dispatch launch");
}

int64_t b200_ep_expert_workspace_bytes(int32_t world, int64_t max_tokens, int32_t top_k,
                                       int64_t hidden, int64_t inter, int32_t local_experts,
                                       int32_t block_size) {
  if (world < 1 || max_tokens <= 0 || top_k <= 0 || hidden <= 0 || inter <= 0 ||
      local_experts <= 0 || block_size <= 0)
    return -1;
  return ep_ws(world, max_tokens, top_k, hidden, inter, local_experts, block_size).total;
}

int b200_ep_expert_forward(int32_t quant, int64_t hidden, int64_t inter, int32_t local_experts,
                           const uint8_t* w13_packed, const float* w13_scales,
                           const float* w13_global, const uint8_t* w2_packed,
                           const float* w2_scales, const float* w2_global, int32_t block_size,
                           int32_t rank, int32_t world, const uint64_t* peer_regions, void* region,
                           int64_t max_tokens, int32_t top_k, void* workspace,
                           int64_t workspace_bytes, void* stream) {
  int rc = check_ep_common(rank, world, max_tokens, top_k, hidden, region, peer_regions);
  if (rc) return rc;
  rc = check_weight_shape(quant, 2 * inter, hidden, B200_GATED_FUSED);
  if (rc) return rc;
  rc = check_weight_shape(quant, hidden, inter, B200_GATED_NONE);
  if (rc) return rc;
  if (peer_regions == nullptr || w13_packed == nullptr || w2_packed == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (local_experts <= 0 || local_experts > moe_align_max_experts())
    return fail(B200_ERR_UNSUPPORTED, "local_experts must be in [1, %d]", moe_align_max_experts());
  const bool tc_block = block_size >= 64 && tc_gemm_supported(block_size);
  if (!tc_block && block_size != 8 && block_size != 16 && block_size != 32 && block_size != 64)
    return fail(B200_ERR_UNSUPPORTED, "block_size must be 8, 16, 32, 64, 128 or 256, got %d",
                block_size);
  const EpWs w = ep_ws(world, max_tokens, top_k, hidden, inter, local_experts, block_size);
  if (workspace_bytes < w.total)
    return fail(B200_ERR_INVALID, "workspace holds %lld bytes, needs %lld",
                (long long)workspace_bytes, (long long)w.total);
  WsView ws;
  if (!carve(workspace, workspace_bytes, ws))
    return fail(B200_ERR_INVALID, "workspace missing or misaligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const EpLayout L = ep_layout(world, max_tokens, top_k, hidden);
  const unsigned long long* peers = reinterpret_cast<const unsigned long long*>(peer_regions);
  uint8_t* reg = static_cast<uint8_t*>(region);

  rc = check_cuda(launch_ep_receive(region, peers, rank, world, L, local_experts, st),
                  "ep receive launch");
  if (rc) return rc;

  // The received rows are the layer's tokens, each with top_k route slots.
  const int64_t numel = w.numel;
  const int64_t rows = (int64_t)world * max_tokens;
  int64_t used = 0;
  int32_t* sorted = reinterpret_cast<int32_t*>(ws.scratch + used);
  used += align_up(w.cap_a * 4);
  int32_t* eids = reinterpret_cast<int32_t*>(ws.scratch + used);
  used += align_up(w.blocks * 4);
  int32_t* ntpp = reinterpret_cast<int32_t*>(ws.scratch + used);
  used += align_up(4);
  int* align_scratch = reinterpret_cast<int*>(ws.scratch + used);
  used += align_up(moe_align_scratch_ints(numel, local_experts) * 4);
  const bool tc = use_tc_moe(quant, block_size, w.blocks);
  __half* xs = nullptr;  // tcgen05: received rows in slot order
  __half* inter_out = reinterpret_cast<__half*>(ws.scratch + used);
  if (tc) {
    xs = inter_out;
    inter_out = reinterpret_cast<__half*>(ws.scratch + used + align_up(w.cap_a * hidden * 2));
  }

  const int32_t* ids = reinterpret_cast<const int32_t*>(reg + L.off_ids);
  if (numel >= kAlignMultiMin) {
    rc = check_cuda(launch_moe_align_multi(ids, numel, local_experts, block_size, sorted, w.cap_a,
                                           eids, w.blocks, ntpp, align_scratch, st),
                    "moe_align launch");
  } else {
    rc = check_cuda(launch_moe_align(ids, numel, local_experts, block_size, sorted, w.cap_a, eids,
                                     w.blocks, ntpp, st),
                    "moe_align launch");
  }
  if (rc) return rc;
  const __half* recv = reinterpret_cast<const __half*>(reg + L.off_recv);
  if (tc) {
    rc = check_cuda(launch_permute_rows(recv, 1, hidden, rows, hidden, sorted, ntpp, w.cap_a, top_k,
                                        numel, xs, st),
                    "permute launch");
    if (rc) return rc;
  }
  // The down GEMM's weighted route rows (after the GEMM operands, as sized by
  // ep_ws), summed per received row by the pre-sum.
  const int64_t stream_ops = align_up(numel * inter * 2);
  const int64_t tc_ops =
      block_size >= 64 ? align_up(w.cap_a * hidden * 2) + align_up(w.cap_a * inter * 2) : 0;
  __half* routed = reinterpret_cast<__half*>(ws.scratch + used +
                                             (stream_ops > tc_ops ? stream_ops : tc_ops));

  StreamParams p{};
  p.wq = w13_packed;
  p.wscale = w13_scales;
  p.gscale = w13_global;
  p.x = recv;
  p.ldx = hidden;
  p.x_rows = rows;
  p.xs = xs;
  p.xs_rows = w.cap_a;
  p.out_by_slot = tc ? 1 : 0;
  p.sorted_ids = sorted;
  p.expert_ids = eids;
  p.ntpp = ntpp;
  p.block_m = block_size;
  p.max_groups = w.cap_a / block_size;
  p.top_k = top_k;
  p.num_routes = (int)numel;
  p.topk_w = reinterpret_cast<const float*>(reg + L.off_w);
  p.E = local_experts;
  p.N = (int)(2 * inter);
  p.K = (int)hidden;
  p.gated = 1;
  p.fuse_act = 1;
  p.mul_w = 0;
  p.out = inter_out;
  p.ldo = inter;
  p.out_f16 = 1;
  const int nt = block_size / 8;
  if (tc)
    rc = run_tc(quant, p, ws, false, st,
                narrow_moe(block_size, max_tokens * top_k, local_experts));
  else
    rc = run_stream(quant, nt, p, w.blocks * (2 * inter / 128) * (hidden / 128), ws, st);
  if (rc) return rc;

  StreamParams q = p;
  q.wq = w2_packed;
  q.wscale = w2_scales;
  q.gscale = w2_global;
  q.x = inter_out;
  q.ldx = inter;
  q.x_rows = numel;  // the intermediate has one row per route
  q.top_k = 1;
  q.xs = tc ? inter_out : nullptr;  // written in slot order by the gate/up epilogue
  q.xs_rows = w.cap_a;
  q.out_by_slot = 0;
  q.N = (int)hidden;
  q.K = (int)inter;
  q.gated = 0;
  q.fuse_act = 0;
  q.mul_w = 1;
  q.out = routed;
  q.out_rows = nullptr;
  q.ldo = hidden;
  q.out_f16 = 1;
  if (tc)
    rc = run_tc(quant, q, ws, true, st,
                narrow_moe(block_size, max_tokens * top_k, local_experts));
  else
    rc = run_stream(quant, nt, q, w.blocks * (hidden / 128) * (inter / 128), ws, st);
  if (rc) return rc;
  rc = check_cuda(launch_ep_presum(region, routed, world, L, st), "ep pre-sum launch");
  if (rc) return rc;
  return check_cuda(launch_ep_signal(region, peers, rank, world, L, st), "ep signal launch");
}

int b200_ep_combine(int64_t tokens, int64_t hidden, const int32_t* topk_ids, int32_t top_k,
                    int32_t num_experts, float routed_scaling_factor, const void* shared_out,
                    int32_t shared_dtype, void* out, int32_t out_dtype, int32_t world, void* region,
                    int64_t max_tokens, void* stream) {
  int rc = check_ep_common(0, world, max_tokens, top_k, hidden, region, nullptr);
  if (rc) return rc;
  if (!valid_dtype16(out_dtype) || (shared_out != nullptr && !valid_dtype16(shared_dtype)))
    return fail(B200_ERR_UNSUPPORTED, "dtypes must be bf16 or f16");
  if (tokens < 0 || tokens > max_tokens)
    return fail(B200_ERR_INVALID, "tokens %lld outside [0, max_tokens=%lld]", (long long)tokens,
                (long long)max_tokens);
  if (num_experts <= 0) return fail(B200_ERR_INVALID, "bad num_experts");
  if (tokens > 0 && (topk_ids == nullptr || out == nullptr))
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (!aligned16(out) || (shared_out && !aligned16(shared_out)))
    return fail(B200_ERR_INVALID, "buffers must be 16-byte aligned");
  const EpLayout L = ep_layout(world, max_tokens, top_k, hidden);
  return check_cuda(launch_ep_combine(region, L, world, tokens, routed_scaling_factor, shared_out,
                                      shared_dtype == B200_DTYPE_F16, out,
                                      out_dtype == B200_DTYPE_F16,
                                      reinterpret_cast<cudaStream_t>(stream)),
                    "ep combine launch");
}

}  // extern "C"

// ------------------------------------------------- W8A8 block FP8 (opt-in)

namespace {

// Scale rows per 128-K group: the activation rows (or slots) rounded up to 4
// (16-byte aligned bulk copies) plus one item of slack (a 128-row copy that
// starts at the last slot).
int64_t w8_scale_ld(int64_t slots) { return (slots + 3) / 4 * 4 + 128; }

struct W8Ws {
  uint8_t* q;
  float* scales;
  int64_t ld;
};

bool carve_w8(WsView& ws, int64_t slots, int64_t k, W8Ws& out) {
  const int64_t ld = w8_scale_ld(slots);
  const int64_t need = align_up(slots * k) + align_up((k / 128) * ld * 4);
  if (need > ws.scratch_bytes) return false;
  out.q = ws.scratch;
  out.scales = reinterpret_cast<float*>(ws.scratch + align_up(slots * k));
  out.ld = ld;
  return true;
}

int check_w8_weights(int64_t n, int64_t k, int32_t gated_mode) {
  int rc = check_weight_shape(B200_QUANT_FP8_BLOCK, n, k, gated_mode);
  if (rc) return rc;
  return B200_OK;
}

}  // namespace

extern "C" {

int64_t b200_w8a8_workspace_bytes(int64_t slots, int64_t k) {
  if (slots < 0 || k <= 0 || k % 128) return -1;
  return stream_ws_bytes() + align_up(slots * k) + align_up((k / 128) * w8_scale_ld(slots) * 4);
}

int b200_fp8_act_quant(const void* x, int32_t x_dtype, int64_t rows, int64_t k, uint8_t* q,
                       float* scales, int64_t scales_ld, void* stream) {
  if (!valid_dtype16(x_dtype)) return fail(B200_ERR_UNSUPPORTED, "x must be bf16 or f16");
  if (rows < 0 || rows >= (1ll << 31) || k <= 0 || k % 128 || k >= (1ll << 31))
    return fail(B200_ERR_INVALID, "needs K a multiple of the 128-wide quantization group, got K=%lld",
                (long long)k);
  if (scales_ld < rows) return fail(B200_ERR_INVALID, "scales_ld %lld < rows %lld",
                                    (long long)scales_ld, (long long)rows);
  if (rows == 0) return B200_OK;
  if (x == nullptr || q == nullptr || scales == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u) ||
      (reinterpret_cast<uintptr_t>(scales) & 3u))
    return fail(B200_ERR_INVALID, "x must be 16-byte aligned, q 8-byte and scales 4-byte aligned");
  return check_cuda(launch_fp8_act_quant(x, x_dtype == B200_DTYPE_F16, rows, (int)k, nullptr, 1,
                                         0, rows, q, scales, scales_ld, nullptr,
                                         reinterpret_cast<cudaStream_t>(stream)),
                    "activation quantization launch");
}

int b200_w8a8_linear(const void* x, int32_t x_dtype, int64_t m, int64_t k, const uint8_t* w_e4m3,
                     const float* w_scales, int64_t n, int32_t gated_mode, void* y,
                     int32_t y_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_w8_weights(n, k, gated_mode);
  if (rc) return rc;
  if (!valid_dtype16(x_dtype) || !valid_dtype16(y_dtype))
    return fail(B200_ERR_UNSUPPORTED, "activations and output must be bf16 or f16");
  if (m < 0 || m >= (1ll << 31)) return fail(B200_ERR_INVALID, "bad M %lld", (long long)m);
  if (m == 0) return B200_OK;
  if (x == nullptr || w_e4m3 == nullptr || w_scales == nullptr || y == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (!aligned16(x) || !aligned16(w_e4m3))
    return fail(B200_ERR_INVALID, "x and weights must be 16-byte aligned");
  WsView ws;
  W8Ws w8;
  if (!carve(workspace, workspace_bytes, ws) || !carve_w8(ws, m, k, w8))
    return fail(B200_ERR_INVALID, "workspace smaller than b200_w8a8_workspace_bytes(%lld, %lld)",
                (long long)m, (long long)k);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = check_cuda(launch_fp8_act_quant(x, x_dtype == B200_DTYPE_F16, m, (int)k, nullptr, 1, 0, m,
                                       w8.q, w8.scales, w8.ld, ws.status, st),
                  "activation quantization launch");
  if (rc) return rc;
  W8Launch L{};
  L.w = w_e4m3;
  L.wscale = w_scales;
  L.xq = w8.q;
  L.xscale = w8.scales;
  L.xs_ld = w8.ld;
  L.rows = m;
  L.E = 1;
  L.N = (int)n;
  L.K = (int)k;
  L.gated = gated_mode == B200_GATED_FUSED;
  L.out = y;
  L.ldo = gated_mode == B200_GATED_FUSED ? n / 2 : n;
  L.out_f16 = y_dtype == B200_DTYPE_F16;
  L.status = ws.status;
  return check_cuda(launch_w8a8_gemm(L, st), "W8A8 GEMM launch");
}

int b200_w8a8_moe_gemm(const void* a, int32_t a_dtype, int64_t a_rows, int64_t k,
                       const uint8_t* w_e4m3, const float* w_scales, int32_t num_experts,
                       int64_t n, int32_t gated_mode, const int32_t* sorted_token_ids,
                       const int32_t* expert_ids, int64_t expert_capacity,
                       const int32_t* num_tokens_post_pad, int32_t block_size, int32_t top_k,
                       int64_t num_routes, const float* topk_weights, int32_t mul_topk_weights,
                       void* c, int32_t c_dtype, int64_t ldc, void* workspace,
                       int64_t workspace_bytes, void* stream) {
  int rc = check_w8_weights(n, k, gated_mode);
  if (rc) return rc;
  if (!valid_dtype16(a_dtype) || !valid_dtype16(c_dtype))
    return fail(B200_ERR_UNSUPPORTED, "activations and output must be bf16 or f16");
  if (block_size != 8 && block_size != 16 && block_size != 32 && block_size != 64 &&
      block_size != 128 && block_size != 256)
    return fail(B200_ERR_UNSUPPORTED, "block_size must be 8, 16, 32, 64, 128 or 256, got %d",
                block_size);
  if (num_experts <= 0 || num_experts >= (1 << 23))
    return fail(B200_ERR_INVALID, "num_experts must be in [1, 2^23)");
  if (top_k <= 0) return fail(B200_ERR_INVALID, "top_k must be positive");
  if (a_rows < 0 || num_routes < 0 || num_routes >= (1ll << 31) || expert_capacity < 0)
    return fail(B200_ERR_INVALID, "bad row counts");
  const int64_t out_cols = gated_mode == B200_GATED_FUSED ? n / 2 : n;
  if (ldc < out_cols) return fail(B200_ERR_INVALID, "ldc %lld < output width %lld",
                                  (long long)ldc, (long long)out_cols);
  if (expert_capacity == 0 || num_routes == 0 || a_rows == 0) return B200_OK;
  if (a == nullptr || w_e4m3 == nullptr || w_scales == nullptr || c == nullptr ||
      sorted_token_ids == nullptr || expert_ids == nullptr || num_tokens_post_pad == nullptr)
    return fail(B200_ERR_INVALID, "null pointer argument");
  if (mul_topk_weights && topk_weights == nullptr)
    return fail(B200_ERR_INVALID, "mul_topk_weights needs topk_weights");
  if (!aligned16(a) || !aligned16(w_e4m3))
    return fail(B200_ERR_INVALID, "activations and weights must be 16-byte aligned");
  const int64_t slots = expert_capacity * block_size;
  if (slots >= (1ll << 31)) return fail(B200_ERR_INVALID, "too many route slots");
  const int plan_per_group = block_size > w8a8_item_slots() ? 2 : 1;
  if (expert_capacity * plan_per_group > kTcPlanCap)
    return fail(B200_ERR_UNSUPPORTED, "more than %d route-slot groups", kTcPlanCap / plan_per_group);
  WsView ws;
  W8Ws w8;
  if (!carve(workspace, workspace_bytes, ws) || !carve_w8(ws, slots, k, w8))
    return fail(B200_ERR_INVALID, "workspace smaller than b200_w8a8_workspace_bytes(%lld, %lld)",
                (long long)slots, (long long)k);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Activations quantized straight into slot order (padding slots zero).
  rc = check_cuda(launch_fp8_act_quant(a, a_dtype == B200_DTYPE_F16, a_rows, (int)k,
                                       sorted_token_ids, top_k, num_routes, slots, w8.q,
                                       w8.scales, w8.ld, ws.status, st),
                  "activation quantization launch");
  if (rc) return rc;
  StreamParams pp{};
  pp.expert_ids = expert_ids;
  pp.ntpp = num_tokens_post_pad;
  pp.block_m = block_size;
  pp.max_groups = expert_capacity;
  pp.E = num_experts;
  rc = check_cuda(launch_tc_plan_slots(pp, ws.plan, kTcPlanCap, w8a8_item_slots(), st),
                  "W8A8 plan launch");
  if (rc) return rc;
  W8Launch L{};
  L.w = w_e4m3;
  L.wscale = w_scales;
  L.xq = w8.q;
  L.xscale = w8.scales;
  L.xs_ld = w8.ld;
  L.rows = slots;
  L.sorted_ids = sorted_token_ids;
  L.ntpp = num_tokens_post_pad;
  L.num_routes = (int)num_routes;
  L.topk_w = topk_weights;
  L.mul_w = mul_topk_weights != 0;
  L.E = num_experts;
  L.N = (int)n;
  L.K = (int)k;
  L.gated = gated_mode == B200_GATED_FUSED;
  L.out = c;
  L.ldo = ldc;
  L.out_f16 = c_dtype == B200_DTYPE_F16;
  L.status = ws.status;
  L.plan_buf = ws.plan;
  L.plan_cap = (int)(expert_capacity * plan_per_group);
  return check_cuda(launch_w8a8_gemm(L, st), "W8A8 GEMM launch");
}

}  // extern "C"
