// moe_align_block_size for B200: bucket routes by expert, pad each bucket to
// block_size, emit the expert of every block.
//
// Contract (the one the reference's kernels consume; the align op itself is
// upstream sgl_kernel, forced onto its CUDA pair by
// sglang_restomod/moe/align_sm70.py:35-55, and read by
// quant/sm70_fp4_moe/csrc/decode_gemv_qpn2.cu:73-110 and
// quant/sm70_fp4_moe/decode_gemv.py:226-260):
//   * sorted_ids[p] holds a route index (token * top_k + slot) or the
//     sentinel numel for a padding slot;
//   * expert_ids[b] is the expert of block b (block b = slots [b*bs, b*bs+bs));
//   * num_tokens_post_pad[0] = sum over experts of ceil(count / bs) * bs.
// Order inside an expert is the route index order: the stable expert-major
// order of SM70Fp8MoEMethod.apply's torch.argsort(flat_ids, stable=True)
// (quant/sm70_fp8_moe/method.py:285). Route ids outside [0, E) (the -1 that
// expert parallelism writes for routes owned elsewhere) are dropped. The
// whole output is written: slots past the padded total hold the sentinel and
// blocks past it hold expert -1, so the result is bit-reproducible.
//
// One CTA of 32 warps; each warp owns a contiguous segment of routes:
//   1. per-warp per-expert counts (warp match_any aggregates equal ids);
//   2. per-expert exclusive scan over warps, then a block scan of the padded
//      counts gives every expert's first slot;
//   3. each warp re-reads its segment in order and scatters route indices at
//      offset + (earlier warps' count) + (rank among equal ids so far).
// Up to 32 routes (one- to three-token decode steps) one warp does the same
// with warp shuffles alone (align_warp below).
#include "common.cuh"
#include "internal.h"
#include "route_topk.cuh"

namespace b200 {
namespace {

constexpr int kWarps = 32;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxExperts = 1024;
constexpr int kBatch = 8;  // loads in flight per lane

// Route ids as written by an earlier kernel (read-only path) or by this
// kernel's own threads before a block barrier (plain coherent loads).
template <bool kReadOnly>
__device__ __forceinline__ int load_id(const int* p) {
  if constexpr (kReadOnly) return __ldg(p);
  return *p;
}

// The same result for at most 32 routes (decode steps of one to three
// tokens) from one warp, without the shared-memory histogram: lane i holds
// route i; equal experts are found with match_any, an expert's first slot is
// the sum of the padded counts of the smaller experts present, and a route's
// place inside its expert is its rank among the equal lanes below it. The
// whole block first writes the sentinels and the -1 blocks, then warp 0 the
// routes and the experts' blocks.
template <bool kReadOnly>
__device__ __forceinline__ void align_warp(const int* __restrict__ topk_ids, int numel, int E,
                                           int bs, int* __restrict__ sorted_ids,
                                           long long sorted_cap, int* __restrict__ expert_ids,
                                           long long expert_cap, int* __restrict__ ntpp) {
  const int tid = threadIdx.x;
  for (long long p = tid; p < sorted_cap; p += kThreads) sorted_ids[p] = numel;
  for (long long b = tid; b < expert_cap; b += kThreads) expert_ids[b] = -1;
  __syncthreads();  // orders the fills before warp 0's writes (same block)
  if (tid >= 32) return;
  const int lane = tid;
  const int e = lane < numel ? load_id<kReadOnly>(topk_ids + lane) : -1;
  const bool valid = e >= 0 && e < E;
  const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -1);
  const bool leader = valid && lane == __ffs(peers) - 1;
  const int pad = leader ? (__popc(peers) + bs - 1) / bs * bs : 0;
  int off = 0, total = 0;
#pragma unroll 4
  for (int j = 0; j < 32; ++j) {
    const int pj = __shfl_sync(0xffffffffu, pad, j);
    const int ej = __shfl_sync(0xffffffffu, e, j);
    total += pj;
    if (pj > 0 && ej < e) off += pj;
  }
  if (valid) {
    const long long pos = (long long)off + __popc(peers & ((1u << lane) - 1u));
    if (pos < sorted_cap) sorted_ids[pos] = lane;
  }
  if (leader)
    for (int b = off / bs; b < (off + pad) / bs && b < expert_cap; ++b) expert_ids[b] = e;
  if (lane == 0) ntpp[0] = total;
}

// The single-CTA align (steps 1-3 above) on `sm` (kWarps * E + 2 * E + 1 +
// kWarps ints). The caller zeroes the per-warp counts sm[0, kWarps * E)
// and synchronises the block first.
template <bool kReadOnly>
__device__ __forceinline__ void align_cta(const int* __restrict__ topk_ids, long long numel, int E,
                                          int bs, int* __restrict__ sorted_ids, long long sorted_cap,
                                          int* __restrict__ expert_ids, long long expert_cap,
                                          int* __restrict__ ntpp, int* sm) {
  int* cnt = sm;                  // [kWarps][E] per-warp counts, then running bases
  int* off = cnt + kWarps * E;    // [E + 1] first padded slot of each expert
  int* tot = off + E + 1;         // [E] routes per expert
  int* wsum = tot + E;            // [kWarps] scan scratch

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const long long seg = (numel + kWarps - 1) / kWarps;
  const long long s0 = (long long)warp * seg;
  const long long s1 = (s0 + seg < numel) ? s0 + seg : numel;

  // 1. histogram
  for (long long base = s0; base < s1; base += 32 * kBatch) {
    int ids[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const long long idx = base + b * 32 + lane;
      ids[b] = (idx < s1) ? load_id<kReadOnly>(topk_ids + idx) : -1;
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int e = ids[b];
      const bool valid = e >= 0 && e < E;
      const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -1);
      if (valid && lane == __ffs(peers) - 1) cnt[warp * E + e] += __popc(peers);
    }
  }
  __syncthreads();

  // 2a. per-expert exclusive scan over warps
  for (int e = tid; e < E; e += kThreads) {
    int run = 0;
    for (int w = 0; w < kWarps; ++w) {
      const int c = cnt[w * E + e];
      cnt[w * E + e] = run;
      run += c;
    }
    tot[e] = run;
  }
  __syncthreads();

  // 2b. exclusive block scan of the padded counts (E <= kThreads)
  const int pad = (tid < E) ? (tot[tid] + bs - 1) / bs * bs : 0;
  int x = pad;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int v = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    wsum[lane] = v;
  }
  __syncthreads();
  const int excl = x - pad + (warp > 0 ? wsum[warp - 1] : 0);
  if (tid < E) off[tid] = excl;
  if (tid == E - 1) off[E] = excl + pad;
  __syncthreads();

  const int total = off[E];
  if (tid == 0) ntpp[0] = total;

  // Block -> expert map; blocks past the total get -1.
  for (long long b = tid; b < expert_cap; b += kThreads) {
    const long long slot = b * bs;
    int v = -1;
    if (slot < total) {
      int lo = 0, hi = E - 1;  // last e with off[e] <= slot
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off[mid] <= slot) lo = mid; else hi = mid - 1;
      }
      v = lo;
    }
    expert_ids[b] = v;
  }
  // Padding slots inside each expert's range, and the tail.
  for (int e = tid; e < E; e += kThreads) {
    for (int p = off[e] + tot[e]; p < off[e + 1]; ++p)
      if (p < sorted_cap) sorted_ids[p] = (int)numel;
  }
  for (long long p = total + tid; p < sorted_cap; p += kThreads) sorted_ids[p] = (int)numel;

  // 3. stable scatter
  for (long long base = s0; base < s1; base += 32 * kBatch) {
    int ids[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const long long idx = base + b * 32 + lane;
      ids[b] = (idx < s1) ? load_id<kReadOnly>(topk_ids + idx) : -1;
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const long long idx = base + b * 32 + lane;
      const int e = ids[b];
      const bool valid = idx < s1 && e >= 0 && e < E;
      const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -1);
      if (valid) {
        const int rank = __popc(peers & ((1u << lane) - 1u));
        const long long pos = (long long)off[e] + cnt[warp * E + e] + rank;
        if (pos < sorted_cap) sorted_ids[pos] = (int)idx;
      }
      __syncwarp();
      if (valid && lane == __ffs(peers) - 1) cnt[warp * E + e] += __popc(peers);
      __syncwarp();
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    moe_align_kernel(const int* __restrict__ topk_ids, long long numel, int E, int bs,
                     int* __restrict__ sorted_ids, long long sorted_cap,
                     int* __restrict__ expert_ids, long long expert_cap, int* __restrict__ ntpp) {
  extern __shared__ int sm[];
  if (numel <= 32) {
    griddep_wait();  // topk_ids may come from the previous kernel
    if (threadIdx.x == 0) griddep_launch_dependents();
    align_warp<true>(topk_ids, (int)numel, E, bs, sorted_ids, sorted_cap, expert_ids, expert_cap,
                     ntpp);
    return;
  }
  for (int i = threadIdx.x; i < kWarps * E; i += kThreads) sm[i] = 0;
  griddep_wait();  // topk_ids may come from the previous kernel
  if (threadIdx.x == 0) griddep_launch_dependents();
  __syncthreads();
  align_cta<true>(topk_ids, numel, E, bs, sorted_ids, sorted_cap, expert_ids, expert_cap, ntpp, sm);
}

// Router + align in one launch (decode batches): each warp routes tokens
// warp, warp + 32, ... (route::route_token, the router kernel's code), then
// the block aligns the ids it just wrote.
template <int PER>
__global__ void __launch_bounds__(kThreads, 1) route_align_kernel(
    const void* __restrict__ logits, int dtype, long long tokens, int E, int top_k, int scoring,
    int renormalize, const float* __restrict__ bias, int* __restrict__ topk_ids,
    float* __restrict__ topk_w, int bs, int* __restrict__ sorted_ids, long long sorted_cap,
    int* __restrict__ expert_ids, long long expert_cap, int* __restrict__ ntpp) {
  extern __shared__ int sm[];
  for (int i = threadIdx.x; i < kWarps * E; i += kThreads) sm[i] = 0;
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();
  for (long long t = threadIdx.x >> 5; t < tokens; t += kWarps)
    route::route_token<PER>(logits, dtype, t, E, top_k, scoring, renormalize, bias, topk_ids,
                            topk_w);
  __syncthreads();
  align_cta<false>(topk_ids, tokens * top_k, E, bs, sorted_ids, sorted_cap, expert_ids,
                   expert_cap, ntpp, sm);
}

// Everything a small batch needs before its GEMMs, in one launch. Block 0
// optionally appends one shared-expert route per token (id E - 1, weight
// shared_w; the extended routes go to ids_out / w_out, [tokens, top_k + 1])
// and aligns the routes; blocks 1.. optionally convert the bf16 activations
// to the f16 operand of the weight-streaming GEMM (n8 groups of 8).
__global__ void __launch_bounds__(kThreads, 1) moe_prep_kernel(
    const int* __restrict__ topk_ids, const float* __restrict__ topk_w, long long tokens,
    int top_k, int E, int shared, float shared_w, int* __restrict__ ids_out,
    float* __restrict__ w_out, int bs, int* __restrict__ sorted_ids, long long sorted_cap,
    int* __restrict__ expert_ids, long long expert_cap, int* __restrict__ ntpp,
    const uint4* __restrict__ conv_in, uint4* __restrict__ conv_out, long long n8) {
  extern __shared__ int sm[];
  if (blockIdx.x > 0) {
    griddep_wait();  // the activations may come from the previous kernel
    if (threadIdx.x == 0) griddep_launch_dependents();
    const long long stride = (long long)(gridDim.x - 1) * kThreads;
    for (long long i = (long long)(blockIdx.x - 1) * kThreads + threadIdx.x; i < n8; i += stride)
      conv_out[i] = bf16x8_to_f16x8(conv_in[i]);
    return;
  }
  const long long numel = tokens * (top_k + (shared ? 1 : 0));
  if (numel > 32)
    for (int i = threadIdx.x; i < kWarps * E; i += kThreads) sm[i] = 0;
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();
  if (shared) {
    const int k1 = top_k + 1;
    for (long long i = threadIdx.x; i < tokens * k1; i += kThreads) {
      const long long t = i / k1;
      const int j = (int)(i - t * k1);
      ids_out[i] = j < top_k ? __ldg(topk_ids + t * top_k + j) : E - 1;
      w_out[i] = j < top_k ? __ldg(topk_w + t * top_k + j) : shared_w;
    }
    __syncthreads();  // also publishes ids_out to the whole block
    if (numel <= 32)
      align_warp<false>(ids_out, (int)numel, E, bs, sorted_ids, sorted_cap, expert_ids,
                        expert_cap, ntpp);
    else
      align_cta<false>(ids_out, numel, E, bs, sorted_ids, sorted_cap, expert_ids, expert_cap,
                       ntpp, sm);
  } else {
    __syncthreads();
    if (numel <= 32)
      align_warp<true>(topk_ids, (int)numel, E, bs, sorted_ids, sorted_cap, expert_ids,
                       expert_cap, ntpp);
    else
      align_cta<true>(topk_ids, numel, E, bs, sorted_ids, sorted_cap, expert_ids, expert_cap,
                      ntpp, sm);
  }
}

// ------------------------------------------------------------ multi-CTA
// The same contract for large route counts, in three launches over
// segments of kSeg routes (route order = segment order, so the result is
// identical): per-segment expert histograms into `hist[segments][E]`, one
// CTA turning them into per-segment exclusive counts plus the padded expert
// offsets `off[E + 1]` (stored after hist), expert_ids and padding, then a
// stable scatter per segment at off[e] + hist[segment][e] + rank.
constexpr int kSeg = 1024;
constexpr int kSegThreads = 256;
constexpr int kSegWarps = kSegThreads / 32;

__global__ void __launch_bounds__(kSegThreads)
    align_hist_kernel(const int* __restrict__ topk_ids, long long numel, int E,
                      int* __restrict__ hist) {
  extern __shared__ int hsm[];  // [E]
  for (int e = threadIdx.x; e < E; e += kSegThreads) hsm[e] = 0;
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();
  __syncthreads();
  const long long s0 = (long long)blockIdx.x * kSeg;
  for (int i = threadIdx.x; i < kSeg; i += kSegThreads) {
    const long long idx = s0 + i;
    if (idx < numel) {
      const int e = __ldg(topk_ids + idx);
      if (e >= 0 && e < E) atomicAdd(&hsm[e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kSegThreads)
    hist[(long long)blockIdx.x * E + e] = hsm[e];
}

__global__ void __launch_bounds__(kThreads, 1)
    align_scan_kernel(int* __restrict__ hist, int segments, long long numel, int E, int bs,
                      int* __restrict__ sorted_ids, long long sorted_cap,
                      int* __restrict__ expert_ids, long long expert_cap, int* __restrict__ ntpp) {
  extern __shared__ int ssm[];
  int* off = ssm;           // [E + 1]
  int* tot = off + E + 1;   // [E]
  int* wsum = tot + E;      // [kWarps]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  griddep_wait();
  if (tid == 0) griddep_launch_dependents();
  // Per expert: exclusive scan over segments (in place) and the total,
  // eight segments' loads in flight at a time.
  for (int e = tid; e < E; e += kThreads) {
    int run = 0;
    for (int c0 = 0; c0 < segments; c0 += 8) {
      int v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = c0 + j < segments ? hist[(long long)(c0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (c0 + j < segments) hist[(long long)(c0 + j) * E + e] = run;
        run += v[j];
      }
    }
    tot[e] = run;
  }
  __syncthreads();
  const int pad = (tid < E) ? (tot[tid] + bs - 1) / bs * bs : 0;
  int x = pad;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int v = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    wsum[lane] = v;
  }
  __syncthreads();
  const int excl = x - pad + (warp > 0 ? wsum[warp - 1] : 0);
  if (tid < E) off[tid] = excl;
  if (tid == E - 1) off[E] = excl + pad;
  __syncthreads();
  const int total = off[E];
  if (tid == 0) ntpp[0] = total;
  int* goff = hist + (long long)segments * E;
  for (int e = tid; e <= E; e += kThreads) goff[e] = off[e];
  for (long long b = tid; b < expert_cap; b += kThreads) {
    const long long slot = b * bs;
    int v = -1;
    if (slot < total) {
      int lo = 0, hi = E - 1;  // last e with off[e] <= slot
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off[mid] <= slot) lo = mid; else hi = mid - 1;
      }
      v = lo;
    }
    expert_ids[b] = v;
  }
  for (int e = tid; e < E; e += kThreads) {
    for (int p = off[e] + tot[e]; p < off[e + 1]; ++p)
      if (p < sorted_cap) sorted_ids[p] = (int)numel;
  }
  for (long long p = total + tid; p < sorted_cap; p += kThreads) sorted_ids[p] = (int)numel;
}

__global__ void __launch_bounds__(kSegThreads)
    align_scatter_kernel(const int* __restrict__ topk_ids, long long numel, int E,
                         const int* __restrict__ base, int segments, int* __restrict__ sorted_ids,
                         long long sorted_cap) {
  extern __shared__ int csm[];  // [kSegWarps][E] per-warp running positions
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < kSegWarps * E; i += kSegThreads) csm[i] = 0;
  griddep_wait();
  if (tid == 0) griddep_launch_dependents();
  __syncthreads();
  // Warp w owns routes s0 + w*128 .. +127 of the segment.
  const long long s0 = (long long)blockIdx.x * kSeg + warp * (kSeg / kSegWarps);
  int ids[kSeg / kSegWarps / 32];
#pragma unroll
  for (int b = 0; b < kSeg / kSegWarps / 32; ++b) {
    const long long idx = s0 + b * 32 + lane;
    ids[b] = idx < numel ? __ldg(topk_ids + idx) : -1;
  }
#pragma unroll
  for (int b = 0; b < kSeg / kSegWarps / 32; ++b) {
    const int e = ids[b];
    const bool valid = e >= 0 && e < E;
    const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -1);
    if (valid && lane == __ffs(peers) - 1) csm[warp * E + e] += __popc(peers);
  }
  __syncthreads();
  // Exclusive scan over the warps, offset by the segment's first slot.
  for (int e = tid; e < E; e += kSegThreads) {
    int run = base[(long long)segments * E + e] + base[(long long)blockIdx.x * E + e];
    for (int w = 0; w < kSegWarps; ++w) {
      const int c = csm[w * E + e];
      csm[w * E + e] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int b = 0; b < kSeg / kSegWarps / 32; ++b) {
    const long long idx = s0 + b * 32 + lane;
    const int e = ids[b];
    const bool valid = e >= 0 && e < E;
    const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -1);
    if (valid) {
      const int rank = __popc(peers & ((1u << lane) - 1u));
      const long long pos = (long long)csm[warp * E + e] + rank;
      if (pos < sorted_cap) sorted_ids[pos] = (int)idx;
    }
    __syncwarp();
    if (valid && lane == __ffs(peers) - 1) csm[warp * E + e] += __popc(peers);
    __syncwarp();
  }
}

}  // namespace

int moe_align_max_experts() { return kMaxExperts; }

long long moe_align_scratch_ints(long long numel, int num_experts) {
  return ((numel + kSeg - 1) / kSeg + 1) * (long long)num_experts + 1;
}

cudaError_t launch_moe_align_multi(const int* topk_ids, long long numel, int num_experts,
                                   int block_size, int* sorted_ids, long long sorted_cap,
                                   int* expert_ids, long long expert_cap, int* ntpp, int* scratch,
                                   cudaStream_t stream) {
  const int segments = (int)((numel + kSeg - 1) / kSeg);
  if (segments < 1) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(align_scatter_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)(sizeof(int) * kSegWarps * kMaxExperts));
    if (err != cudaSuccess) return err;
    configured[dev] = true;
  }
  const int E = num_experts;
  cudaError_t err = launch_pdl(align_hist_kernel, dim3(segments), dim3(kSegThreads),
                               sizeof(int) * E, stream, topk_ids, numel, E, scratch);
  if (err != cudaSuccess) return err;
  err = launch_pdl(align_scan_kernel, dim3(1), dim3(kThreads),
                   sizeof(int) * (2 * (size_t)E + 1 + kWarps), stream, scratch, segments, numel, E,
                   block_size, sorted_ids, sorted_cap, expert_ids, expert_cap, ntpp);
  if (err != cudaSuccess) return err;
  return launch_pdl(align_scatter_kernel, dim3(segments), dim3(kSegThreads),
                    sizeof(int) * kSegWarps * E, stream, topk_ids, numel, E,
                    (const int*)scratch, segments, sorted_ids, sorted_cap);
}

namespace {

template <int PER>
cudaError_t launch_route_align_t(const void* logits, int dtype, long long tokens, int E, int top_k,
                                 int scoring, int renormalize, const float* bias, int* topk_ids,
                                 float* topk_w, int bs, int* sorted_ids, long long sorted_cap,
                                 int* expert_ids, long long expert_cap, int* ntpp,
                                 cudaStream_t stream) {
  const size_t smem = sizeof(int) * ((size_t)kWarps * E + 2 * E + 1 + kWarps);
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const int max_smem = (int)(sizeof(int) * ((size_t)kWarps * kMaxExperts + 2 * kMaxExperts + 1 + kWarps));
    cudaError_t err = cudaFuncSetAttribute(route_align_kernel<PER>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    if (err != cudaSuccess) return err;
    configured[dev] = true;
  }
  return launch_pdl(route_align_kernel<PER>, dim3(1), dim3(kThreads), smem, stream, logits, dtype,
                    tokens, E, top_k, scoring, renormalize, bias, topk_ids, topk_w, bs, sorted_ids,
                    sorted_cap, expert_ids, expert_cap, ntpp);
}

}  // namespace

cudaError_t launch_route_align(const void* logits, int dtype, long long tokens, int E, int top_k,
                               int scoring, int renormalize, const float* bias, int* topk_ids,
                               float* topk_w, int bs, int* sorted_ids, long long sorted_cap,
                               int* expert_ids, long long expert_cap, int* ntpp,
                               cudaStream_t stream) {
  const int per = (E + 31) / 32;
#define B200_ROUTE_ALIGN(P)                                                                    \
  return launch_route_align_t<P>(logits, dtype, tokens, E, top_k, scoring, renormalize, bias,  \
                                 topk_ids, topk_w, bs, sorted_ids, sorted_cap, expert_ids,     \
                                 expert_cap, ntpp, stream)
  if (per <= 1) B200_ROUTE_ALIGN(1);
  if (per <= 4) B200_ROUTE_ALIGN(4);
  if (per <= 8) B200_ROUTE_ALIGN(8);
  if (per <= 16) B200_ROUTE_ALIGN(16);
  B200_ROUTE_ALIGN(32);
#undef B200_ROUTE_ALIGN
}

cudaError_t launch_moe_align(const int* topk_ids, long long numel, int num_experts, int block_size,
                             int* sorted_ids, long long sorted_cap, int* expert_ids,
                             long long expert_cap, int* ntpp, cudaStream_t stream) {
  const size_t smem = sizeof(int) * ((size_t)kWarps * num_experts + 2 * num_experts + 1 + kWarps);
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const int max_smem = (int)(sizeof(int) * ((size_t)kWarps * kMaxExperts + 2 * kMaxExperts + 1 + kWarps));
    cudaError_t err = cudaFuncSetAttribute(moe_align_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    if (err != cudaSuccess) return err;
    configured[dev] = true;
  }
  return launch_pdl(moe_align_kernel, dim3(1), dim3(kThreads), smem, stream, topk_ids, numel,
                    num_experts, block_size, sorted_ids, sorted_cap, expert_ids, expert_cap, ntpp);
}

cudaError_t launch_moe_prep(const int* topk_ids, const float* topk_w, long long tokens, int top_k,
                            int num_experts, int shared, float shared_w, int* ids_out,
                            float* w_out, int block_size, int* sorted_ids, long long sorted_cap,
                            int* expert_ids, long long expert_cap, int* ntpp, const void* conv_in,
                            void* conv_out, long long conv_elems, cudaStream_t stream) {
  const size_t smem = sizeof(int) * ((size_t)kWarps * num_experts + 2 * num_experts + 1 + kWarps);
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const int max_smem = (int)(sizeof(int) * ((size_t)kWarps * kMaxExperts + 2 * kMaxExperts + 1 + kWarps));
    cudaError_t err = cudaFuncSetAttribute(moe_prep_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    if (err != cudaSuccess) return err;
    configured[dev] = true;
  }
  const long long n8 = conv_in != nullptr ? conv_elems / 8 : 0;
  long long conv_blocks = (n8 + kThreads - 1) / kThreads;
  const long long cap = device_sm_count();
  if (conv_blocks > cap) conv_blocks = cap;
  return launch_pdl(moe_prep_kernel, dim3((unsigned)(1 + conv_blocks)), dim3(kThreads), smem,
                    stream, topk_ids, topk_w, tokens, top_k, num_experts, shared, shared_w, ids_out,
                    w_out, block_size, sorted_ids, sorted_cap, expert_ids, expert_cap, ntpp,
                    static_cast<const uint4*>(conv_in), static_cast<uint4*>(conv_out), n8);
}

}  // namespace b200
