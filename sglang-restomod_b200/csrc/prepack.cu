// Load-time re-layout of checkpoint weights into the stream GEMM's units.
//
// Counterpart of the reference's load-time preparation:
//   * block-FP8 experts: prepare_experts / fp8_prepare(..., interleave_gated_silu)
//     (sglang_restomod/quant/sm70_fp8_moe/__init__.py:161-205, README.md:23-58);
//   * NVFP4 experts: prepare_moe_nvfp4 and qpn2.pack_expert
//     (sglang_restomod/quant/sm70_fp4_moe/method.py:290-382, qpn2.py:65-110).
// The layout itself is this library's own (stream_gemm.cu reads it).
//
// A unit covers 128 bank rows x 128 K. Bank rows map to logical weight rows:
//   plain : unit row block rb, warp w, lane row g (0..7):
//           top = rb*128 + 16w + g, bottom = top + 8
//   gated : gate/up interleaved so one lane holds gate j and up j:
//           top = rb*64 + 8w + g (gate j), bottom = N/2 + top (up j)
// Lane (g, c) of warp w covers K [kb*128 + 32c, +32) of its two rows.
//
// FP8 unit (16 KiB): [w:8][q:4][lane:32][16 B]; the 16 B are
//   top[k0 .. k0+8) ++ bottom[k0 .. k0+8) with k0 = kb*128 + 32c + 8q.
// NVFP4 unit (9 KiB): codes [w:8][lane:32][32 B] = top 16 B ++ bottom 16 B
//   (ModelOpt packing: byte b holds K 2b in the low nibble, 2b+1 high), then
//   scales [w:8][lane:32][4 B] = top g0, top g1, bottom g0, bottom g1 for the
//   two 16-K groups of the lane's K range.
#include "common.cuh"
#include "internal.h"

namespace b200 {
namespace {

__device__ __forceinline__ void bank_rows(int gated, int N, int rb, int w, int g, int& top,
                                          int& bot) {
  if (gated) {
    top = rb * 64 + w * 8 + g;
    bot = N / 2 + top;
  } else {
    top = rb * 128 + w * 16 + g;
    bot = top + 8;
  }
}

__global__ void prepack_fp8_kernel(const uint8_t* __restrict__ w, long long E, int N, int K,
                                   int gated, uint8_t* __restrict__ out) {
  const long long chunks = E * (long long)N * K / 16;
  const int nrb = N / 128, kch = K / 128;
  for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < chunks;
       id += (long long)gridDim.x * blockDim.x) {
    // id = ((((e*nrb + rb)*kch + kb)*8 + warp)*4 + q)*32 + lane
    long long t = id;
    const int lane = (int)(t % 32); t /= 32;
    const int q = (int)(t % 4); t /= 4;
    const int wp = (int)(t % 8); t /= 8;
    const int kb = (int)(t % kch); t /= kch;
    const int rb = (int)(t % nrb); t /= nrb;
    const long long e = t;
    int top, bot;
    bank_rows(gated, N, rb, wp, lane >> 2, top, bot);
    const long long k0 = (long long)kb * 128 + 32 * (lane & 3) + 8 * q;
    const uint8_t* base = w + e * (long long)N * K;
    const uint2 a = *reinterpret_cast<const uint2*>(base + (long long)top * K + k0);
    const uint2 b = *reinterpret_cast<const uint2*>(base + (long long)bot * K + k0);
    *reinterpret_cast<uint4*>(out + id * 16) = make_uint4(a.x, a.y, b.x, b.y);
  }
}

__global__ void prepack_nvfp4_kernel(const uint8_t* __restrict__ w,
                                     const uint8_t* __restrict__ scales, long long E, int N,
                                     int K, int gated, uint8_t* __restrict__ out) {
  const int nrb = N / 128, kch = K / 128;
  const long long lanes = E * nrb * (long long)kch * 8 * 32;
  for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < lanes;
       id += (long long)gridDim.x * blockDim.x) {
    long long t = id;
    const int lane = (int)(t % 32); t /= 32;
    const int wp = (int)(t % 8); t /= 8;
    const int kb = (int)(t % kch); t /= kch;
    const int rb = (int)(t % nrb); t /= nrb;
    const long long e = t;
    int top, bot;
    bank_rows(gated, N, rb, wp, lane >> 2, top, bot);
    const int c = lane & 3;
    const long long kbyte = (long long)kb * 64 + 16 * c;  // packed byte offset in the row
    const long long kgrp = (long long)kb * 8 + 2 * c;     // 16-K group index in the row
    const long long row_bytes = K / 2, row_groups = K / 16;
    const uint8_t* wb = w + e * (long long)N * row_bytes;
    const uint8_t* sb = scales + e * (long long)N * row_groups;
    const uint4 ct = *reinterpret_cast<const uint4*>(wb + (long long)top * row_bytes + kbyte);
    const uint4 cb = *reinterpret_cast<const uint4*>(wb + (long long)bot * row_bytes + kbyte);
    const uint32_t s = (uint32_t)sb[(long long)top * row_groups + kgrp] |
                       ((uint32_t)sb[(long long)top * row_groups + kgrp + 1] << 8) |
                       ((uint32_t)sb[(long long)bot * row_groups + kgrp] << 16) |
                       ((uint32_t)sb[(long long)bot * row_groups + kgrp + 1] << 24);
    const long long unit = (e * nrb + rb) * (long long)kch + kb;
    uint8_t* u = out + unit * (long long)kFp4UnitBytes;
    uint4* code_dst = reinterpret_cast<uint4*>(u + wp * 1024 + lane * 32);
    code_dst[0] = ct;
    code_dst[1] = cb;
    *reinterpret_cast<uint32_t*>(u + 8192 + wp * 128 + lane * 4) = s;
  }
}

int grid_for(long long work, int threads) {
  long long blocks = (work + threads - 1) / threads;
  const long long cap = (long long)device_sm_count() * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

}  // namespace

cudaError_t launch_prepack_fp8(const uint8_t* w, long long E, int N, int K, int gated,
                               uint8_t* out, cudaStream_t stream) {
  const long long chunks = E * (long long)N * K / 16;
  prepack_fp8_kernel<<<grid_for(chunks, 256), 256, 0, stream>>>(w, E, N, K, gated, out);
  return cudaGetLastError();
}

cudaError_t launch_prepack_nvfp4(const uint8_t* w, const uint8_t* scales, long long E, int N,
                                 int K, int gated, uint8_t* out, cudaStream_t stream) {
  const long long lanes = E * (long long)(N / 128) * (K / 128) * 8 * 32;
  prepack_nvfp4_kernel<<<grid_for(lanes, 256), 256, 0, stream>>>(w, scales, E, N, K, gated, out);
  return cudaGetLastError();
}

}  // namespace b200
