// Expert-parallel token exchange over peer memory (NVLink / NVSwitch P2P).
//
// Replaces the all-to-all dispatch / combine around the expert compute of an
// expert-parallel MoE layer. The reference has no all-to-all: its expert
// parallelism is upstream SGLang's dispatcher, which maps global expert ids to
// local ones and marks foreign routes -1
// (sglang_restomod/quant/sm70_fp8_moe/method.py:8-12, 253-283), and the expert
// method's combine (method.py:305-309). Here every rank owns a contiguous
// range of experts and one forward is five launches per rank, none of which
// involves the host:
//
//   dispatch (source)  every token's activation row is converted to f16 and
//                      stored once into each owner that holds one of its
//                      experts (P2P stores), with the token's top_k route
//                      slots (local expert or -1, router weight); the grid's
//                      last CTA publishes the per-owner row counts and raises
//                      the owner's dispatch flag;
//   receive  (owner)   waits for every source's flag, marks slots past each
//                      source's count empty and records where each row's
//                      return goes (the source's combine buffer);
//   expert GEMMs       (capi.cu) align + gate/up + down over the received
//                      rows as tokens, the down GEMM writing weighted route
//                      rows locally;
//   pre-sum  (owner)   adds each row's routes and stores the one summed row
//                      into the source's combine buffer (P2P stores), then
//                      raises each source's combine flag (signal);
//   combine  (source)  waits for every owner's flag, sums the (at most one per
//                      owner) returned rows of each token (+ shared expert,
//                      x routed_scaling_factor) and advances the step counter.
//
// A token whose top_k experts sit on d distinct owners crosses NVLink d
// times each way instead of top_k times (top-8 over 8 ranks: ~5.3 on
// average for uniform routing).
// Flags carry the step number (the region's local counter + 1), so nothing is
// reset between steps; every rank runs the same steps in the same order.
// Every wait is bounded (kWaitLimitNs) and reports kDevPeerTimeout in the
// region's status word instead of hanging. No TMA and no multicast: peer
// memory is touched only by plain loads and stores.
#include "common.cuh"
#include "internal.h"

namespace b200 {
namespace {

constexpr int kEpThreads = 256;

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int* hdr_of(uint8_t* region) { return reinterpret_cast<int*>(region); }

// Current step number + 1: the value this step's flags carry.
__device__ __forceinline__ int next_epoch(uint8_t* region) {
  return *reinterpret_cast<volatile int*>(hdr_of(region) + kEpHdrEpoch) + 1;
}

// Thread `who` < world waits until flags[who] reaches `want` (wrap-safe
// compare). Returns false after kWaitLimitNs, having set kDevPeerTimeout.
__device__ bool wait_flag(const int* flag, int want, int* status) {
  if (ld_acquire_sys(flag) - want >= 0) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_sys(flag) - want >= 0) return true;
    if ((i & 63u) == 0u && global_timer_ns() - t0 > kWaitLimitNs) {
      atomicOr(status, kDevPeerTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 raw) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[j]);
    __half2 h = __floats2half2_rn(__low2float(b), __high2float(b));
    o[j] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void st_u128(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

struct DispatchParams {
  const void* x;  // [tokens, hidden] bf16 / f16
  int x_f16;
  long long tokens, hidden;
  const int* ids;  // [tokens * top_k] global expert ids
  const float* w;  // [tokens * top_k]
  int top_k, num_experts, experts_per_rank, rank, world;
  int shared_expert;  // id num_experts = the shared expert: stays here as local expert experts_per_rank
  const unsigned long long* peers;  // [world] region bases in this process
  uint8_t* region;                  // this rank's region
  EpLayout L;
  int chunk;  // tokens per CTA
};

// Owner rank and local expert of global expert e (-1: not sent). With a
// fused shared expert, id num_experts is the shared expert, computed by the
// source rank itself as its local expert experts_per_rank.
__device__ __forceinline__ int route_owner(const DispatchParams& p, int e, int& local) {
  if (e >= 0 && e < p.num_experts) {
    const int o = e / p.experts_per_rank;
    local = e - o * p.experts_per_rank;
    return o;
  }
  if (p.shared_expert && e == p.num_experts) {
    local = p.experts_per_rank;
    return p.rank;
  }
  return -1;
}

// Owners token t's routes go to, as a bitmask.
__device__ __forceinline__ unsigned long long token_owners(const DispatchParams& p, long long t) {
  unsigned long long m = 0;
  for (int k = 0; k < p.top_k; ++k) {
    int local;
    const int o = route_owner(p, __ldg(p.ids + t * p.top_k + k), local);
    if (o >= 0) m |= 1ull << o;
  }
  return m;
}

// One CTA per chunk of tokens. Each (token, owner) pair becomes one row in
// the owner's segment for this source, at a position that follows token order
// (stable), so a receiver's rows are in the source's token order.
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(const DispatchParams p) {
  extern __shared__ int pos[];  // [chunk][world]
  __shared__ int base[kEpMaxWorld];
  __shared__ int mine[kEpMaxWorld];
  __shared__ int last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long c0 = (long long)blockIdx.x * p.chunk;
  const long long c1 = c0 + p.chunk < p.tokens ? c0 + p.chunk : p.tokens;
  const int epoch = next_epoch(p.region);
  int* hdr = hdr_of(p.region);
  unsigned long long* masks = reinterpret_cast<unsigned long long*>(p.region + p.L.off_mask);
  if (tid < kEpMaxWorld) {
    base[tid] = 0;
    mine[tid] = 0;
  }
  __syncthreads();
  // Rows of earlier chunks per owner.
  for (long long t = tid; t < c0; t += kEpThreads) {
    unsigned long long m = token_owners(p, t);
    while (m) {
      atomicAdd(&base[__ffsll((long long)m) - 1], 1);
      m &= m - 1;
    }
  }
  __syncthreads();
  if (warp == 0) {
    for (long long g = c0; g < c1; g += 32) {
      const long long t = g + lane;
      const unsigned long long m = t < c1 ? token_owners(p, t) : 0ull;
      if (t < c1) masks[t] = m;
      for (int d = 0; d < p.world; ++d) {
        const bool has = (m >> d) & 1ull;
        const unsigned b = __ballot_sync(0xffffffffu, has);
        if (t < c1) pos[(t - c0) * p.world + d] = has ? base[d] + __popc(b & ((1u << lane) - 1u)) : -1;
        __syncwarp();
        if (lane == 0) {
          base[d] += __popc(b);
          mine[d] += __popc(b);
        }
        __syncwarp();
      }
    }
  }
  __syncthreads();
  // Rows: one warp per (token, owner) pair, 16 bytes per lane per access;
  // lanes k < top_k write the row's route slots.
  const long long h8 = p.hidden / 8;
  const long long pairs = (c1 - c0) * p.world;
  for (long long q = warp; q < pairs; q += kEpThreads / 32) {
    const long long t = c0 + q / p.world;
    const int d = (int)(q % p.world);
    const int ps = pos[q];
    if (ps < 0) continue;
    uint8_t* dst = reinterpret_cast<uint8_t*>(p.peers[d]);
    const long long row = (long long)p.rank * p.L.cap + ps;
    if (lane < p.top_k) {
      const long long r = t * p.top_k + lane;
      int local = -1;
      const int o = route_owner(p, __ldg(p.ids + r), local);
      reinterpret_cast<int*>(dst + p.L.off_ids)[row * p.top_k + lane] = o == d ? local : -1;
      reinterpret_cast<float*>(dst + p.L.off_w)[row * p.top_k + lane] = __ldg(p.w + r);
    }
    if (lane == 0) reinterpret_cast<int*>(dst + p.L.off_orig)[row] = (int)t;
    const uint4* src = reinterpret_cast<const uint4*>(p.x) + t * h8;
    uint8_t* drow = dst + p.L.off_recv + row * p.hidden * 2;
    for (long long v = lane; v < h8; v += 32) {
      uint4 val = __ldg(src + v);
      if (!p.x_f16) val = bf16x8_to_f16x8(val);
      st_u128(drow + v * 16, val);
    }
  }
  // Publish: this CTA's per-owner row counts, then (last CTA) the totals + flags.
  if (tid < p.world && mine[tid] != 0)
    atomicAdd(reinterpret_cast<int*>(p.region + p.L.off_cnt_local) + tid, mine[tid]);
  __threadfence_system();
  __syncthreads();
  if (tid == 0) last = atomicAdd(hdr + kEpHdrDispatchDone, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (tid < p.world) {
    const int n = atomicExch(reinterpret_cast<int*>(p.region + p.L.off_cnt_local) + tid, 0);
    uint8_t* dst = reinterpret_cast<uint8_t*>(p.peers[tid]);
    *reinterpret_cast<volatile int*>(dst + p.L.off_count + 4 * p.rank) = n;
    __threadfence_system();
    st_release_sys(reinterpret_cast<int*>(dst + p.L.off_dflag) + p.rank, epoch);
  }
  if (tid == 0) hdr[kEpHdrDispatchDone] = 0;
}

// Owner: wait for every source, then per received row keep its route slots
// (local expert, weight) or mark them empty, and point the row's return at the
// source's combine buffer (token-major, this owner's column). Every CTA takes
// the waits itself.
__global__ void __launch_bounds__(kEpThreads) ep_receive_kernel(
    uint8_t* region, const unsigned long long* peers, int rank, int world, EpLayout L,
    int experts_local) {
  __shared__ int cnt[kEpMaxWorld];
  const int tid = threadIdx.x;
  int* hdr = hdr_of(region);
  const int epoch = next_epoch(region);
  if (tid < world) {
    const int* flag = reinterpret_cast<const int*>(region + L.off_dflag) + tid;
    int n = 0;
    if (wait_flag(flag, epoch, hdr + kEpHdrStatus)) {
      n = __ldcg(reinterpret_cast<const int*>(region + L.off_count) + tid);
      n = n < 0 ? 0 : (n > L.cap ? (int)L.cap : n);
    }
    cnt[tid] = n;
  }
  __syncthreads();
  __threadfence();
  int* ids = reinterpret_cast<int*>(region + L.off_ids);
  const int* orig = reinterpret_cast<const int*>(region + L.off_orig);
  unsigned long long* rows = reinterpret_cast<unsigned long long*>(region + L.off_rows);
  const long long total = (long long)world * L.cap;
  for (long long row = blockIdx.x * (long long)kEpThreads + tid; row < total;
       row += (long long)gridDim.x * kEpThreads) {
    const int s = (int)(row / L.cap);
    const long long j = row - (long long)s * L.cap;
    bool live = false;
    if (j < cnt[s]) {
      const int t = __ldcg(orig + row);
      if (t >= 0 && t < L.cap) {
        live = true;
        rows[row] = peers[s] + (unsigned long long)L.off_comb +
                    ((unsigned long long)t * world + rank) * (unsigned long long)L.hidden * 2ull;
      }
    }
    if (!live) rows[row] = 0ull;
    for (int k = 0; k < L.top_k; ++k) {
      const long long slot = row * L.top_k + k;
      int id = live ? __ldcg(ids + slot) : -1;
      if (id < 0 || id >= experts_local) id = -1;
      ids[slot] = id;
    }
  }
}

// Owner, after its down GEMM (stream order): one thread per 16 bytes of a
// received row sums the row's weighted route outputs (fp32) and stores the f16
// sum at the row's destination - the source's combine buffer, over NVLink.
// Element-parallel like the combine: a warp per row left most SMs idle.
__global__ void __launch_bounds__(kEpThreads) ep_presum_kernel(const uint8_t* region,
                                                               const uint8_t* routed, int world,
                                                               EpLayout L) {
  const int* ids = reinterpret_cast<const int*>(region + L.off_ids);
  const unsigned long long* rows = reinterpret_cast<const unsigned long long*>(region + L.off_rows);
  const long long h8 = L.hidden / 8;
  const long long total = (long long)world * L.cap * h8;
  for (long long id = blockIdx.x * (long long)kEpThreads + threadIdx.x; id < total;
       id += (long long)gridDim.x * kEpThreads) {
    const long long row = id / h8;
    const long long v = id - row * h8;
    const unsigned long long dst = __ldg(rows + row);
    if (dst == 0ull) continue;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < L.top_k; ++k) {
      if (__ldg(ids + row * L.top_k + k) < 0) continue;
      const uint4 raw =
          __ldcg(reinterpret_cast<const uint4*>(routed + (row * L.top_k + k) * L.hidden * 2) + v);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
      o[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    st_u128(reinterpret_cast<uint8_t*>(dst) + v * 16, make_uint4(o[0], o[1], o[2], o[3]));
  }
}

// Owner, after its pre-sum has completed (plain stream order): raise each
// source's combine flag.
__global__ void ep_signal_kernel(uint8_t* region, const unsigned long long* peers, int rank,
                                 int world, EpLayout L) {
  const int tid = threadIdx.x;
  const int epoch = next_epoch(region);
  __threadfence_system();
  if (tid < world) {
    uint8_t* dst = reinterpret_cast<uint8_t*>(peers[tid]);
    st_release_sys(reinterpret_cast<int*>(dst + L.off_cflag) + rank, epoch);
  }
}

struct CombineParams {
  uint8_t* region;
  EpLayout L;
  int world;
  long long tokens;
  float scale;
  const void* shared_out;
  int shared_f16;
  void* out;
  int out_f16;
};

// Source: wait for every owner, then out[t] = scale * sum over the owners
// token t went to of their returned row (+ shared[t]); the last CTA advances
// the step counter.
__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(const CombineParams p) {
  __shared__ int last;
  const int tid = threadIdx.x;
  int* hdr = hdr_of(p.region);
  const int epoch = next_epoch(p.region);
  if (tid < p.world) {
    const int* flag = reinterpret_cast<const int*>(p.region + p.L.off_cflag) + tid;
    wait_flag(flag, epoch, hdr + kEpHdrStatus);
  }
  __syncthreads();
  __threadfence();
  const uint8_t* rows = p.region + p.L.off_comb;
  const unsigned long long* masks =
      reinterpret_cast<const unsigned long long*>(p.region + p.L.off_mask);
  const long long hidden = p.L.hidden;
  const long long h8 = hidden / 8;
  const long long total = p.tokens * h8;
  for (long long id = blockIdx.x * (long long)kEpThreads + tid; id < total;
       id += (long long)gridDim.x * kEpThreads) {
    const long long t = id / h8;
    const long long c = (id - t * h8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    unsigned long long m = masks[t];
    while (m) {
      const int o = __ffsll((long long)m) - 1;
      m &= m - 1;
      const uint4 raw =
          __ldcg(reinterpret_cast<const uint4*>(rows + ((t * p.world + o) * hidden + c) * 2));
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= p.scale;
    if (p.shared_out != nullptr) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(
          reinterpret_cast<const uint8_t*>(p.shared_out) + (t * hidden + c) * 2));
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f;
        if (p.shared_f16)
          f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        else
          f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (p.out_f16) {
        __half2 h = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
        o[i] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        o[i] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.out) + (t * hidden + c) * 2) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  if (tid == 0) last = atomicAdd(hdr + kEpHdrCombineDone, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (last && tid == 0) {
    hdr[kEpHdrCombineDone] = 0;
    __threadfence();
    atomicExch(hdr + kEpHdrEpoch, epoch);
  }
}

int ep_grid(long long work) {
  long long blocks = (work + kEpThreads - 1) / kEpThreads;
  const long long cap = (long long)device_sm_count() * 4;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

}  // namespace

// Tokens per dispatch CTA: spread over up to 4 CTAs per SM (one warp per
// (token, owner) row, eight rows in flight per CTA).
int ep_dispatch_chunk(long long tokens) {
  const long long ctas = 4ll * device_sm_count();
  long long chunk = (tokens + ctas - 1) / ctas;
  return chunk < 1 ? 1 : (int)chunk;
}

cudaError_t launch_ep_dispatch(const void* x, int x_f16, long long tokens, long long hidden,
                               const int* ids, const float* w, int top_k, int num_experts,
                               int shared_expert, int experts_per_rank, int rank, int world,
                               const unsigned long long* peers, void* region, const EpLayout& L,
                               cudaStream_t stream) {
  // With no tokens one CTA still publishes this step's (zero) counts and flags.
  DispatchParams p;
  p.x = x;
  p.x_f16 = x_f16;
  p.tokens = tokens;
  p.hidden = hidden;
  p.ids = ids;
  p.w = w;
  p.top_k = top_k;
  p.num_experts = num_experts;
  p.shared_expert = shared_expert;
  p.experts_per_rank = experts_per_rank;
  p.rank = rank;
  p.world = world;
  p.peers = peers;
  p.region = static_cast<uint8_t*>(region);
  p.L = L;
  p.chunk = ep_dispatch_chunk(tokens);
  const int grid = tokens > 0 ? (int)((tokens + p.chunk - 1) / p.chunk) : 1;
  ep_dispatch_kernel<<<grid, kEpThreads, (size_t)p.chunk * world * 4, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_ep_receive(void* region, const unsigned long long* peers, int rank, int world,
                              const EpLayout& L, int experts_local, cudaStream_t stream) {
  ep_receive_kernel<<<ep_grid((long long)world * L.cap), kEpThreads, 0, stream>>>(
      static_cast<uint8_t*>(region), peers, rank, world, L, experts_local);
  return cudaGetLastError();
}

cudaError_t launch_ep_presum(const void* region, const void* routed, int world, const EpLayout& L,
                             cudaStream_t stream) {
  ep_presum_kernel<<<ep_grid((long long)world * L.cap * (L.hidden / 8)), kEpThreads, 0, stream>>>(
      static_cast<const uint8_t*>(region), static_cast<const uint8_t*>(routed), world, L);
  return cudaGetLastError();
}

cudaError_t launch_ep_signal(void* region, const unsigned long long* peers, int rank, int world,
                             const EpLayout& L, cudaStream_t stream) {
  ep_signal_kernel<<<1, 64, 0, stream>>>(static_cast<uint8_t*>(region), peers, rank, world, L);
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(void* region, const EpLayout& L, int world, long long tokens,
                              float scale, const void* shared_out, int shared_f16, void* out,
                              int out_f16, cudaStream_t stream) {
  CombineParams p;
  p.region = static_cast<uint8_t*>(region);
  p.L = L;
  p.world = world;
  p.tokens = tokens;
  p.scale = scale;
  p.shared_out = shared_out;
  p.shared_f16 = shared_f16;
  p.out = out;
  p.out_f16 = out_f16;
  ep_combine_kernel<<<ep_grid(tokens * (L.hidden / 8)), kEpThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace b200
