// Router top-k device code shared by the router kernel (router.cu) and the
// fused route + align kernel (moe_align.cu). See router.cu for the contract.
#pragma once

#include "common.cuh"

namespace b200 {
namespace route {

constexpr int kMaxPerLane = 32;  // up to 1024 experts

__device__ __forceinline__ float load_logit(const void* p, long long idx, int dtype) {
  if (dtype == 2) return reinterpret_cast<const float*>(p)[idx];
  const uint16_t b = reinterpret_cast<const uint16_t*>(p)[idx];
  if (dtype == 1) return __half2float(__ushort_as_half(b));
  return __bfloat162float(__ushort_as_bfloat16(b));
}

// (key, expert) arg-max over the warp; ties to the lower expert id.
__device__ __forceinline__ void warp_argmax(float& key, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float k2 = __shfl_xor_sync(0xffffffffu, key, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    if (k2 > key || (k2 == key && i2 < idx)) {
      key = k2;
      idx = i2;
    }
  }
}

// Expert-group restriction (upstream SGLang's grouped_topk /
// biased_grouped_topk): the experts form `groups` contiguous groups; a
// group's score is the largest selection key in it (no bias), or the sum of
// its two largest keys (with a correction bias); the topk_group best groups
// (ties to the lower group) stay selectable. Returns bit j set when this
// lane's expert lane + 32 j is in a kept group. groups <= 32.
template <int PER>
__device__ __forceinline__ uint32_t group_allowed(const float (&key)[PER], int num_experts,
                                                  int groups, int topk_group, bool top2) {
  const int lane = threadIdx.x & 31;
  const int gsz = num_experts / groups;
  float mine = -INFINITY;  // lane g < groups: score of group g
  for (int g = 0; g < groups; ++g) {
    float b1 = -INFINITY;
    int i1 = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < num_experts && e / gsz == g && (key[j] > b1 || (key[j] == b1 && e < i1))) {
        b1 = key[j];
        i1 = e;
      }
    }
    warp_argmax(b1, i1);
    float score = b1;
    if (top2) {
      float b2 = -INFINITY;
      int i2 = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int e = lane + 32 * j;
        if (e < num_experts && e / gsz == g && e != i1 && (key[j] > b2 || (key[j] == b2 && e < i2))) {
          b2 = key[j];
          i2 = e;
        }
      }
      warp_argmax(b2, i2);
      score = b1 + b2;
    }
    if (lane == g) mine = score;
  }
  uint32_t kept = 0;  // bit g: group g kept
  float k = lane < groups ? mine : -INFINITY;
  for (int r = 0; r < topk_group; ++r) {
    float kk = k;
    int ii = lane < groups ? lane : 0x7fffffff;
    if (k == -INFINITY && lane < groups) ii = 0x7ffffffe;  // retired groups never win
    warp_argmax(kk, ii);
    if (ii >= 0 && ii < groups) {
      kept |= 1u << ii;
      if (lane == ii) k = -INFINITY;
    }
  }
  uint32_t allow = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    if (e < num_experts && ((kept >> (e / gsz)) & 1u)) allow |= 1u << j;
  }
  return allow;
}

// Routes token t with one warp (lane l holds experts l, l + 32, ...): writes
// topk_ids[t, 0..k) and topk_w[t, 0..k). groups > 0 restricts the choice to
// the topk_group best expert groups (group_allowed).
template <int PER>
__device__ __forceinline__ void route_token(const void* __restrict__ logits, int dtype, long long t,
                                            int num_experts, int top_k, int scoring,
                                            int renormalize, const float* __restrict__ bias,
                                            int* __restrict__ topk_ids, float* __restrict__ topk_w,
                                            int groups = 0, int topk_group = 0) {
  const int lane = threadIdx.x & 31;
  float logit[PER], key[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    logit[j] = e < num_experts ? load_logit(logits, t * num_experts + e, dtype) : -INFINITY;
    mx = fmaxf(mx, logit[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  // Scores: softmax numerators exp(l - max) (the denominator is applied
  // below) or sigmoid(l). Selection keys: the logit, or sigmoid + bias.
  float score[PER];
  float denom = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    if (scoring == 0) {
      score[j] = e < num_experts ? expf(logit[j] - mx) : 0.f;
      denom += score[j];
      key[j] = logit[j];
    } else {
      score[j] = e < num_experts ? 1.f / (1.f + expf(-logit[j])) : 0.f;
      key[j] = e < num_experts ? score[j] + (bias != nullptr ? __ldg(bias + e) : 0.f) : -INFINITY;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) denom += __shfl_xor_sync(0xffffffffu, denom, o);
  float sel_w = 0.f;  // lane i < top_k keeps the i-th choice
  int sel_e = -1;
  float sel_sum = 0.f;
  uint32_t taken = 0;  // bit j: expert lane + 32 j already chosen (or not selectable)
  if (groups > 0) taken = ~group_allowed<PER>(key, num_experts, groups, topk_group, bias != nullptr);
  for (int i = 0; i < top_k; ++i) {
    float bk = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      const bool free = e < num_experts && !((taken >> j) & 1u);
      if (free && (key[j] > bk || (key[j] == bk && e < be))) {
        bk = key[j];
        be = e;
      }
    }
    warp_argmax(bk, be);
    // The owner of the winner reads its score and retires it.
    float sc = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      if (lane + 32 * j == be) {
        sc = score[j];
        taken |= 1u << j;
      }
    }
    sc = __shfl_sync(0xffffffffu, sc, be & 31);
    if (scoring == 0) sc = sc / denom;  // the softmax probability
    if (lane == i) {
      sel_w = sc;
      sel_e = be;
    }
    sel_sum += sc;
  }
  if (lane < top_k) {
    const float w = renormalize ? sel_w / sel_sum : sel_w;
    topk_ids[t * top_k + lane] = sel_e;
    topk_w[t * top_k + lane] = w;
  }
}

}  // namespace route
}  // namespace b200
