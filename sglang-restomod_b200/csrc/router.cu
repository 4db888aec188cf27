// Router top-k: router logits -> (topk_ids, topk_weights), one launch.
//
// Replaces upstream SGLang's select_experts / fused top-k softmax that feeds
// the quant methods (the StandardTopKOutput that
// sglang_restomod/quant/sm70_fp8_moe/check.py:106-114 builds: topk_weights,
// topk_ids) with the benchmark's routing: fp32 softmax over the experts,
// the top k, weights renormalised to sum 1. Also covers sigmoid scoring with
// an optional per-expert correction bias that only steers the selection
// (the weights stay the unbiased scores), and no renormalisation.
//
// One warp per token; lane l holds experts l, l + 32, ... in registers
// (num_experts <= 32 * kMaxPerLane). Selection runs on the selection key
// (the logit for softmax - exp is monotonic, so the order is the order of
// the probabilities - or sigmoid(logit) + bias), k rounds of a warp arg-max
// with ties to the lower expert id. Outputs are in descending key order, as
// torch.topk returns them.
#include "common.cuh"
#include "internal.h"
#include "route_topk.cuh"

namespace b200 {
namespace {

constexpr int kRouterWarps = 8;

template <int PER>
__global__ void __launch_bounds__(kRouterWarps * 32) topk_route_kernel(
    const void* __restrict__ logits, int dtype, long long tokens, int num_experts, int top_k,
    int scoring, int renormalize, const float* __restrict__ bias, int* __restrict__ topk_ids,
    float* __restrict__ topk_w, int groups, int topk_group) {
  griddep_wait();
  const long long warps = (long long)gridDim.x * kRouterWarps;
  for (long long t = blockIdx.x * (long long)kRouterWarps + (threadIdx.x >> 5); t < tokens;
       t += warps)
    route::route_token<PER>(logits, dtype, t, num_experts, top_k, scoring, renormalize, bias,
                            topk_ids, topk_w, groups, topk_group);
  griddep_launch_dependents();
}

}  // namespace

int router_max_experts() { return 32 * route::kMaxPerLane; }

cudaError_t launch_topk_route(const void* logits, int dtype, long long tokens, int num_experts,
                              int top_k, int scoring, int renormalize, const float* bias,
                              int* topk_ids, float* topk_w, cudaStream_t stream, int groups,
                              int topk_group) {
  if (tokens <= 0) return cudaSuccess;
  long long blocks = (tokens + kRouterWarps - 1) / kRouterWarps;
  const long long cap = (long long)device_sm_count() * 16;
  if (blocks > cap) blocks = cap;
  const dim3 grid((unsigned)blocks), block(kRouterWarps * 32);
  const int per = (num_experts + 31) / 32;
  if (per <= 1)
    return launch_pdl(topk_route_kernel<1>, grid, block, 0, stream, logits, dtype, tokens,
                      num_experts, top_k, scoring, renormalize, bias, topk_ids, topk_w, groups,
                      topk_group);
  if (per <= 4)
    return launch_pdl(topk_route_kernel<4>, grid, block, 0, stream, logits, dtype, tokens,
                      num_experts, top_k, scoring, renormalize, bias, topk_ids, topk_w, groups,
                      topk_group);
  if (per <= 8)
    return launch_pdl(topk_route_kernel<8>, grid, block, 0, stream, logits, dtype, tokens,
                      num_experts, top_k, scoring, renormalize, bias, topk_ids, topk_w, groups,
                      topk_group);
  if (per <= 16)
    return launch_pdl(topk_route_kernel<16>, grid, block, 0, stream, logits, dtype, tokens,
                      num_experts, top_k, scoring, renormalize, bias, topk_ids, topk_w, groups,
                      topk_group);
  return launch_pdl(topk_route_kernel<32>, grid, block, 0, stream, logits, dtype, tokens,
                    num_experts, top_k, scoring, renormalize, bias, topk_ids, topk_w, groups,
                      topk_group);
}

}  // namespace b200
