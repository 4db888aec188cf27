// Bandwidth-bound helpers around the expert GEMMs.
//
//   * bf16 -> f16 activation conversion (the stream GEMM's tensor-core
//     operand is f16, as the reference's activations are; sm70 has no bf16).
//   * moe_sum_reduce: out[t, :] = scale * sum_k in[t, k, :] in fp32, stored in
//     the input dtype. Same contract as the reference's Triton replacement
//     (sglang_restomod/quant/sm70_fp4_moe/sum_reduce.py:84-123).
//   * moe_combine: the top-k combine of SM70Fp8MoEMethod.apply
//     (sglang_restomod/quant/sm70_fp8_moe/method.py:305-309) for rows that the
//     down GEMM already multiplied by their router weight: routes whose
//     expert id is outside [0, E) (expert-parallel drops, id -1) contribute
//     nothing, the sum is fp32, then routed_scaling_factor, plus an optional
//     shared-expert row.
// All three move 16 bytes per thread per access.
#include "common.cuh"
#include "internal.h"

namespace b200 {
namespace {

__device__ __forceinline__ void load8(const void* base, long long idx, int f16, float (&v)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(
      reinterpret_cast<const uint8_t*>(base) + idx * 2);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (f16) {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      v[2 * i] = __low2float(h);
      v[2 * i + 1] = __high2float(h);
    } else {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      v[2 * i] = __low2float(h);
      v[2 * i + 1] = __high2float(h);
    }
  }
}

__device__ __forceinline__ void store8(void* base, long long idx, int f16, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (f16) {
      __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(base) + idx * 2) =
      make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void bf16_to_f16_kernel(const uint4* __restrict__ in, uint4* __restrict__ out,
                                   long long n8) {
  griddep_wait();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = bf16x8_to_f16x8(in[i]);
  griddep_launch_dependents();
}

// One thread per 8 hidden elements of one token.
__global__ void sum_reduce_kernel(const void* __restrict__ in, void* __restrict__ out,
                                  long long tokens, int top_k, long long hidden, int f16,
                                  float scale, const int* __restrict__ topk_ids, int num_experts,
                                  const void* __restrict__ shared_out, int shared_f16,
                                  int out_f16) {
  griddep_wait();
  const long long h8 = hidden / 8;
  const long long total = tokens * h8;
  for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
       id += (long long)gridDim.x * blockDim.x) {
    const long long t = id / h8;
    const long long c = (id - t * h8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // Four routes' rows in flight per step; a dropped route's row is never
    // read (it was not written).
    for (int k0 = 0; k0 < top_k; k0 += 4) {
      uint4 raw[4];
      bool use[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = k0 + j;
        use[j] = k < top_k;
        if (use[j] && topk_ids != nullptr) {
          const int e = __ldg(topk_ids + t * top_k + k);
          use[j] = e >= 0 && e < num_experts;
        }
        raw[j] = use[j] ? *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(in) +
                                                          ((t * top_k + k) * hidden + c) * 2)
                        : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 f;
          if (f16)
            f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
          else
            f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
          acc[2 * i] += f.x;
          acc[2 * i + 1] += f.y;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= scale;
    if (shared_out != nullptr) {
      float v[8];
      load8(shared_out, t * hidden + c, shared_f16, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += v[i];
    }
    store8(out, t * hidden + c, out_f16, acc);
  }
  griddep_launch_dependents();
}

// One warp per route slot, 16 bytes per lane per access. Reads the slot
// count written by moe_align on the device, so it is graph-capturable.
__global__ void __launch_bounds__(256) permute_rows_kernel(
    const uint8_t* __restrict__ x, int x_f16, long long ldx, long long x_rows, long long k,
    const int* __restrict__ sorted_ids, const int* __restrict__ ntpp, long long cap, int top_k,
    long long num_routes, uint8_t* __restrict__ out) {
  griddep_wait();
  long long n = ntpp[0];
  if (n > cap) n = cap;
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long k8 = k / 8;
  for (long long s = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); s < n;
       s += warps) {
    const int id = __ldg(sorted_ids + s);
    if (id < 0 || id >= num_routes) continue;
    const long long row = id / top_k;
    if (row >= x_rows) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + row * ldx * 2);
    uint4* dst = reinterpret_cast<uint4*>(out + s * k * 2);
    for (long long v = lane; v < k8; v += 32) {
      uint4 raw = __ldg(src + v);
      if (!x_f16) {
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[j]);
          __half2 h = __floats2half2_rn(__low2float(b), __high2float(b));
          o[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        raw = make_uint4(o[0], o[1], o[2], o[3]);
      }
      dst[v] = raw;
    }
  }
  griddep_launch_dependents();
}

// ids_out[t, :] = (topk_ids[t, :], shared_id), w_out[t, :] = (topk_weights[t, :],
// shared_weight): every token gains one route to the shared expert.
__global__ void __launch_bounds__(256) append_shared_route_kernel(
    const int* __restrict__ ids, const float* __restrict__ w, long long tokens, int top_k,
    int shared_id, float shared_weight, int* __restrict__ ids_out, float* __restrict__ w_out) {
  griddep_wait();
  const long long total = tokens * (top_k + 1);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / (top_k + 1);
    const int j = (int)(i - t * (top_k + 1));
    ids_out[i] = j < top_k ? __ldg(ids + t * top_k + j) : shared_id;
    w_out[i] = j < top_k ? __ldg(w + t * top_k + j) : shared_weight;
  }
  griddep_launch_dependents();
}

int grid_for(long long work, int threads) {
  long long blocks = (work + threads - 1) / threads;
  const long long cap = (long long)device_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

}  // namespace

cudaError_t launch_bf16_to_f16(const void* in, void* out, long long n, cudaStream_t stream) {
  const long long n8 = n / 8;
  if (n8 == 0) return cudaSuccess;
  return launch_pdl(bf16_to_f16_kernel, dim3(grid_for(n8, 256)), dim3(256), 0, stream,
                    reinterpret_cast<const uint4*>(in), reinterpret_cast<uint4*>(out), n8);
}

cudaError_t launch_permute_rows(const void* x, int x_f16, long long ldx, long long x_rows,
                                long long k, const int* sorted_ids, const int* ntpp, long long cap,
                                int top_k, long long num_routes, void* out, cudaStream_t stream) {
  if (cap <= 0) return cudaSuccess;
  long long blocks = (cap + 7) / 8;  // 8 warps of 256 threads, one slot each
  const long long limit = (long long)device_sm_count() * 8;
  if (blocks > limit) blocks = limit;
  return launch_pdl(permute_rows_kernel, dim3((unsigned)blocks), dim3(256), 0, stream,
                    static_cast<const uint8_t*>(x), x_f16, ldx, x_rows, k, sorted_ids, ntpp, cap,
                    top_k, num_routes, static_cast<uint8_t*>(out));
}

cudaError_t launch_append_shared_route(const int* ids, const float* w, long long tokens,
                                       int top_k, int shared_id, float shared_weight,
                                       int* ids_out, float* w_out, cudaStream_t stream) {
  const long long total = tokens * (top_k + 1);
  if (total == 0) return cudaSuccess;
  return launch_pdl(append_shared_route_kernel, dim3(grid_for(total, 256)), dim3(256), 0, stream,
                    ids, w, tokens, top_k, shared_id, shared_weight, ids_out, w_out);
}

cudaError_t launch_moe_sum_reduce(const void* in, void* out, long long tokens, int top_k,
                                  long long hidden, int f16, float scale, cudaStream_t stream) {
  const long long work = tokens * (hidden / 8);
  if (work == 0) return cudaSuccess;
  return launch_pdl(sum_reduce_kernel, dim3(grid_for(work, 256)), dim3(256), 0, stream, in, out,
                    tokens, top_k, hidden, f16, scale, static_cast<const int*>(nullptr), 0,
                    static_cast<const void*>(nullptr), 0, f16);
}

cudaError_t launch_moe_combine(const void* routed, int routed_f16, const int* topk_ids,
                               int num_experts, long long tokens, int top_k, long long hidden,
                               float scale, const void* shared_out, int shared_f16, void* out,
                               int out_f16, cudaStream_t stream) {
  const long long work = tokens * (hidden / 8);
  if (work == 0) return cudaSuccess;
  return launch_pdl(sum_reduce_kernel, dim3(grid_for(work, 256)), dim3(256), 0, stream, routed,
                    out, tokens, top_k, hidden, routed_f16, scale, topk_ids, num_experts,
                    shared_out, shared_f16, out_f16);
}

}  // namespace b200
