// W8A8 block-scaled FP8 GEMM for the prefill regime (opt-in): FP8 weights
// times FP8 activations on the tcgen05 tensor cores (kind::f8f6f4, twice the
// f16 rate), fp32 accumulation.
//
// The reference has no such path: its FP8 linears and experts are W8A16
// (quant/sm70_fp8_dense/_method.py:713-863, the TurboMind block-FP8 GEMMs).
// This is upstream SGLang's block-FP8 W8A8 arithmetic instead: activations
// quantized per (row, 128-K group) to e4m3 with one fp32 scale each
// (scale = max(amax / 448, 1e-8), the block-FP8 rule of
// quant/sm70_fp8_lm_head/__init__.py:33-41 applied to a 1x128 group), the
// checkpoint's e4m3 weights with their fp32 scale per 128x128 block, and
//   y[t, n] = sum over 128-K blocks kb of  sa[t, kb] * sw[n/128, kb] *
//             sum_{k in kb} qa[t, k] * qw[n, k].
// Quantizing the activations changes the results against the W8A16 path,
// which is why it is a separate entry point.
//
// Shape: D[128 weight rows, N <= 128 tokens] ("swap AB"), one 128-K block
// per pipeline stage. Weights (row-major, the checkpoint layout) and the
// quantized activations both arrive by 2-D TMA with 128-byte swizzle, the
// K-major layout the MMA's shared-memory descriptors read; the stage's 128
// activation scales come with them (a 512-byte bulk copy). The four
// K=32 MMAs of a block write a fresh fp32 partial into one of four tensor-
// memory buffers (all 512 columns); the epilogue warps load it, release the
// buffer at once, then multiply it by sa * sw and add it to their register
// accumulators (packed f32x2 math), so the MMAs run up to three blocks ahead
// of the promotion.
//
// Warps: 0-7 epilogue (warp w reads tensor-memory lanes 32 * (w % 4) ..,
// columns 64 * (w / 4) ..), 8 TMA producer, 9 MMA issuer (one elected lane)
// and tensor-memory owner, 10 item metadata (each output column's row and
// router weight, staged in shared memory ahead of the item's stores). Every
// wait is bounded; a timeout sets the status bit and every role stops.
//
// A gated gate/up bank (rows [gate | up], the checkpoint layout) is tiled so
// that one tile holds 64 gate rows and the 64 matching up rows: TMEM lanes
// 32q .. 32q+15 take gate rows 64t + 16q + 0..15, lanes 32q+16 .. 32q+31 the
// up rows of the same outputs, so silu(gate) * up is a shuffle within a warp.
#include <cstring>

#include "../../include/b200moe.h"
#include "common.cuh"
#include "internal.h"
#include "tcgen05.cuh"

namespace b200 {
namespace {

using namespace tcg;
using namespace tcg_host;

constexpr int kW8N = 128;  // MMA N (tokens / route slots) per item
constexpr int kW8Warps = 11;
constexpr int kW8Threads = kW8Warps * 32;
constexpr int kWarpEpiCount = 8;
constexpr int kWarpProd = 8, kWarpMma8 = 9, kWarpMeta8 = 10;
constexpr int kW8PBufs = 4;  // tensor-memory partial buffers
constexpr int kW8Stages = 6;
constexpr uint32_t kW8ATile = 128 * 128;  // 128 weight rows x 128 K e4m3
constexpr uint32_t kW8BTile = 128 * 128;  // 128 tokens x 128 K e4m3
constexpr uint32_t kW8SaBytes = kW8N * 4;
constexpr uint32_t kW8StageBytes = kW8ATile + kW8BTile + 1024;  // + scales, 1024-aligned
constexpr uint32_t kW8OffCtl = kW8Stages * kW8StageBytes;
constexpr uint32_t kW8OffMeta = kW8OffCtl + 1024;     // [2][kW8N] out rows, [2][kW8N] weights
constexpr size_t kW8Smem = kW8OffMeta + 4 * kW8N * 4 + 1024;  // + alignment slack
constexpr uint32_t kW8TmemCols = kW8PBufs * kW8N;           // 512: four partial buffers
constexpr uint32_t kW8StageTx = kW8ATile + kW8BTile + kW8SaBytes;
static_assert(kW8Smem <= 232448, "shared memory");
static_assert(kW8StageBytes % 1024 == 0, "stages stay 1024-byte aligned");

struct W8Params {
  const float* wscale;   // [E][N/128][K/128]
  const float* xscale;   // [K/128][xs_ld]: activation scales, rows (or slots) contiguous
  long long xs_ld;
  long long rows;        // activation rows: dense M, or route slots in moe mode
  const int* sorted_ids; // nullptr: dense
  const int* ntpp;
  int num_routes;
  const float* topk_w;
  int mul_w;
  int E, N, K;
  int gated;             // fused silu(gate) * up: output width N / 2
  void* out;
  long long ldo;
  int out_f16;
  int* status;
};

struct W8Ctl {
  uint64_t full[kW8Stages];   // A + B + scales landed (transaction bytes)
  uint64_t empty[kW8Stages];  // MMA commit + the 8 epilogue warps (scales read)
  uint64_t pfull[kW8PBufs];   // partial buffer written (MMA commit)
  uint64_t pempty[kW8PBufs];  // partial buffer read (8 epilogue warps)
  uint64_t mfull[2];          // item metadata staged (metadata warp)
  uint64_t mempty[2];         // item metadata used (8 epilogue warps)
  uint64_t done;
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(W8Ctl) <= 1024, "control block");

__device__ __forceinline__ uint32_t instr_desc_e4m3(int n) {
  // f32 accumulate, A and B e4m3 (format 0), both K-major, M = 128, N = n.
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]^T, e4m3 x e4m3 -> f32.
__device__ __forceinline__ void mma_ss_f8(uint32_t tmem_d, uint64_t da, uint64_t db,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      "  .reg .pred p;\n"
      "  setp.ne.b32 p, %4, 0;\n"
      "  tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ bool w8_wait(uint64_t* bar, uint32_t parity, W8Ctl* ctl, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u) {
      if (*reinterpret_cast<volatile int*>(&ctl->abort)) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        if (status) atomicOr(status, kDevWaitTimeout);
        *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool w8_warp_wait(uint64_t* bar, uint32_t parity, W8Ctl* ctl,
                                             int* status) {
  return __all_sync(0xffffffffu, w8_wait(bar, parity, ctl, status));
}

// One item: a 128-row weight tile of expert e against up to 128 activation
// rows (route slots) starting at slot0.
struct W8Item {
  int e, tile, rows;
  long long slot0;
};

__device__ __forceinline__ W8Item w8_item(const W8Params& p, const int2* plan, long long g,
                                          int ntiles, long long mchunks) {
  W8Item it;
  if (p.sorted_ids == nullptr) {
    // tile-major: consecutive items share a weight tile (L2 reuse)
    it.tile = (int)(g / mchunks);
    const long long c = g - (long long)it.tile * mchunks;
    it.e = 0;
    it.slot0 = c * kW8N;
    const long long left = p.rows - it.slot0;
    it.rows = left < kW8N ? (int)left : kW8N;
  } else {
    const long long pi = g / ntiles;
    it.tile = (int)(g - pi * ntiles);
    const int2 pe = __ldg(plan + pi);
    it.e = pe.y >> 9;
    it.slot0 = pe.x;
    it.rows = pe.y & 511;
  }
  return it;
}

__device__ __forceinline__ void fma_f32x2(uint64_t& acc, uint64_t v, uint64_t s, uint64_t w) {
  uint64_t t;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(v), "l"(s));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(t), "l"(w));
}

__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return make_float2(a, b);
}

__global__ void __launch_bounds__(kW8Threads, 1)
    w8a8_gemm_kernel(const W8Params p, const int2* __restrict__ plan,
                     const int* __restrict__ plan_count,
                     const __grid_constant__ CUtensorMap tmap_w,
                     const __grid_constant__ CUtensorMap tmap_x) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  W8Ctl* ctl = reinterpret_cast<W8Ctl*>(smem + kW8OffCtl);
  int* meta_row = reinterpret_cast<int*>(smem + kW8OffMeta);                  // [2][kW8N]
  float* meta_w = reinterpret_cast<float*>(smem + kW8OffMeta + 2 * kW8N * 4);  // [2][kW8N]
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int kch = p.K / 128;
  const int ntiles = p.N / 128;
  const bool dense = p.sorted_ids == nullptr;

  if (tid == 0) {
    for (int s = 0; s < kW8Stages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1 + kWarpEpiCount);
    }
    for (int b = 0; b < kW8PBufs; ++b) {
      mbar_init(&ctl->pfull[b], 1);
      mbar_init(&ctl->pempty[b], kWarpEpiCount);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->mfull[b], 1);
      mbar_init(&ctl->mempty[b], kWarpEpiCount);
    }
    mbar_init(&ctl->done, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMma8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&ctl->tmem)),
                 "r"(kW8TmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(&ctl->tmem);

  griddep_wait();
  if (tid == 0) griddep_launch_dependents();

  const long long mchunks = dense ? (p.rows + kW8N - 1) / kW8N : 1;
  const long long items = dense ? mchunks * ntiles : (long long)__ldg(plan_count) * ntiles;
  const long long my_items =
      items > (long long)blockIdx.x ? (items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const long long g0 = blockIdx.x, gs = gridDim.x;

  if (warp == kWarpProd) {
    // ------------------------------------------------------------ TMA
    long long t = 0;
    bool ok = true;
    const uint64_t pol = l2_policy_evict_last();
    for (long long j = 0; j < my_items && ok; ++j) {
      const W8Item it = w8_item(p, plan, g0 + j * gs, ntiles, mchunks);
      // 16-row boxes of the weight tile: box i lands at tile row 16 i.
      int ya[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const long long base = (long long)it.e * p.N;
        if (p.gated) {
          const int q = i >> 1, up = i & 1;
          ya[i] = (int)(base + (up ? p.N / 2 : 0) + 64 * it.tile + 16 * q);
        } else {
          ya[i] = (int)(base + 128 * it.tile + 16 * i);
        }
      }
      for (int kb = 0; kb < kch; ++kb, ++t) {
        const int s = (int)(t % kW8Stages);
        int good = 1;
        if (lane == 0) {
          good = w8_wait(&ctl->empty[s], (uint32_t)(((t / kW8Stages) & 1) ^ 1), ctl, p.status);
          if (good) {
            uint8_t* st = smem + s * kW8StageBytes;
            mbar_arrive_expect_tx(&ctl->full[s], kW8StageTx);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              tma_load_2d(st + i * 2048, &tmap_w, kb * 128, ya[i], &ctl->full[s]);
            tma_load_2d(st + kW8ATile, &tmap_x, kb * 128, (int)it.slot0, &ctl->full[s]);
            bulk_g2s(st + kW8ATile + kW8BTile, p.xscale + (long long)kb * p.xs_ld + it.slot0,
                     kW8SaBytes, &ctl->full[s], pol);
          }
        }
        if (!__shfl_sync(0xffffffffu, good, 0)) {
          ok = false;
          break;
        }
      }
    }
    // after an abort, copies in flight land before the CTA exits
    if (lane == 0 && !ok) {
      for (long long v = t > kW8Stages ? t - kW8Stages : 0; v < t; ++v)
        mbar_wait(&ctl->full[v % kW8Stages], (uint32_t)((v / kW8Stages) & 1), nullptr);
    }
  } else if (warp == kWarpMma8) {
    // ------------------------------------------------------------ MMA
    const uint32_t dhi = (uint32_t)(smem_desc_sw128(0) >> 32);
    const uint32_t lo0 = (uint32_t)smem_desc_sw128(smem_u32(smem));
    long long t = 0;
    bool ok = true;
    for (long long j = 0; j < my_items && ok; ++j) {
      const W8Item it = w8_item(p, plan, g0 + j * gs, ntiles, mchunks);
      int n = (it.rows + 15) & ~15;
      n = n < 16 ? 16 : (n > kW8N ? kW8N : n);
      const uint32_t idesc = instr_desc_e4m3(n);
      for (int kb = 0; kb < kch; ++kb, ++t) {
        const int s = (int)(t % kW8Stages);
        const int pb = (int)(t % kW8PBufs);
        ok = w8_warp_wait(&ctl->full[s], (uint32_t)((t / kW8Stages) & 1), ctl, p.status) &&
             w8_warp_wait(&ctl->pempty[pb], (uint32_t)(((t / kW8PBufs) & 1) ^ 1), ctl,
                          p.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t alo = lo0 + (uint32_t)(s * kW8StageBytes >> 4);
        const uint32_t blo = alo + (kW8ATile >> 4);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ss_f8(tmem + (uint32_t)pb * kW8N, ((uint64_t)dhi << 32) | (alo + 2u * kk),
                      ((uint64_t)dhi << 32) | (blo + 2u * kk), idesc, kk > 0 ? 1u : 0u);
          mma_commit(&ctl->empty[s]);
          mma_commit(&ctl->pfull[pb]);
        }
        __syncwarp();
      }
    }
    // every issued MMA completes before tensor memory is released
    if (elect_one()) {
      mma_commit(&ctl->done);
      mbar_wait(&ctl->done, 0u, nullptr);
    }
    __syncwarp();
  } else if (warp == kWarpMeta8) {
    // ---------------------------------------------------- item metadata
    // Output row (-1: nothing to store) and router weight of each column of
    // the item, at most one item ahead of the stores.
    bool ok = true;
    for (long long j = 0; j < my_items && ok; ++j) {
      const W8Item it = w8_item(p, plan, g0 + j * gs, ntiles, mchunks);
      const int mb = (int)(j & 1);
      ok = w8_warp_wait(&ctl->mempty[mb], (uint32_t)(((j >> 1) & 1) ^ 1), ctl, p.status);
      if (!ok) break;
#pragma unroll
      for (int i = 0; i < kW8N / 32; ++i) {
        const int col = 32 * i + lane;
        int orow = -1;
        float wt = 1.f;
        if (col < it.rows) {
          const long long slot = it.slot0 + col;
          if (dense) {
            orow = (int)slot;
          } else {
            const int id = __ldg(p.sorted_ids + slot);
            if (id >= 0 && id < p.num_routes) {
              orow = id;
              if (p.mul_w) wt = __ldg(p.topk_w + id);
            }
          }
        }
        meta_row[mb * kW8N + col] = orow;
        meta_w[mb * kW8N + col] = wt;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->mfull[mb]);
    }
  } else if (warp < kWarpEpiCount) {
    // ------------------------------------------- promotion and epilogue
    const int q = warp & 3;          // tensor-memory lanes 32q .. 32q + 31
    const int h = warp >> 2;         // columns 64h .. 64h + 63
    const int m = 32 * q + lane;     // row of the weight tile
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(64 * h);
    const bool up_lane = p.gated && lane >= 16;
    long long t = 0;
    bool ok = true;
    for (long long j = 0; j < my_items && ok; ++j) {
      const W8Item it = w8_item(p, plan, g0 + j * gs, ntiles, mchunks);
      // this lane's weight scale row (128-row block of the bank)
      long long srow;
      if (p.gated)
        srow = (long long)it.e * ntiles + (up_lane ? p.N / 256 : 0) + it.tile / 2;
      else
        srow = (long long)it.e * ntiles + it.tile;
      const float* swp = p.wscale + srow * kch;
      uint64_t acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = 0ull;
      float sw_next = __ldg(swp);
      for (int kb = 0; kb < kch; ++kb, ++t) {
        const int s = (int)(t % kW8Stages);
        const int pb = (int)(t % kW8PBufs);
        const float sw = sw_next;
        if (kb + 1 < kch) sw_next = __ldg(swp + kb + 1);
        ok = w8_warp_wait(&ctl->pfull[pb], (uint32_t)((t / kW8PBufs) & 1), ctl, p.status) &&
             w8_warp_wait(&ctl->full[s], (uint32_t)((t / kW8Stages) & 1), ctl, p.status);
        if (!ok) break;
        tc_fence_after();
        uint32_t v0[32], v1[32];
        tmem_ld32_nowait(lane_base + (uint32_t)pb * kW8N, v0);
        tmem_ld32_nowait(lane_base + (uint32_t)pb * kW8N + 32u, v1);
        tmem_ld_wait();
        // the partial is in registers: hand its buffer back to the MMAs
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->pempty[pb]);
        const float* sa = reinterpret_cast<const float*>(smem + s * kW8StageBytes + kW8ATile +
                                                         kW8BTile) + 64 * h;
        const uint64_t sw2 = pack2(sw, sw);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float4 s4 = *reinterpret_cast<const float4*>(sa + 4 * c);
          const uint32_t* v = c < 8 ? v0 : v1;
          const int o = (c & 7) * 4;
          fma_f32x2(acc[2 * c], pack2(__uint_as_float(v[o]), __uint_as_float(v[o + 1])),
                    pack2(s4.x, s4.y), sw2);
          fma_f32x2(acc[2 * c + 1], pack2(__uint_as_float(v[o + 2]), __uint_as_float(v[o + 3])),
                    pack2(s4.z, s4.w), sw2);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->empty[s]);
      }
      if (!ok) break;
      // ---- store: column c = token / slot 64h + c of the item
      const int mb = (int)(j & 1);
      ok = w8_warp_wait(&ctl->mfull[mb], (uint32_t)((j >> 1) & 1), ctl, p.status);
      if (!ok) break;
      const int* mrow = meta_row + mb * kW8N + 64 * h;
      const float* mw = meta_w + mb * kW8N + 64 * h;
      long long ocol;
      bool stores = true;
      if (p.gated) {
        ocol = 64ll * it.tile + 16 * q + (lane & 15);
        stores = !up_lane;
      } else {
        ocol = 128ll * it.tile + m;
      }
#pragma unroll
      for (int c2 = 0; c2 < 32; ++c2) {
        const float2 a2 = unpack2(acc[c2]);
        const int2 r2 = *reinterpret_cast<const int2*>(mrow + 2 * c2);
        const float2 w2 = *reinterpret_cast<const float2*>(mw + 2 * c2);
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          float val = w ? a2.y : a2.x;
          if (p.gated) {
            const float up = __shfl_down_sync(0xffffffffu, val, 16);
            val = silu_f32(val) * up;
          }
          const int orow = w ? r2.y : r2.x;  // uniform across the warp
          if (orow < 0 || !stores) continue;
          const float y = val * (w ? w2.y : w2.x);
          if (p.out_f16)
            reinterpret_cast<__half*>(p.out)[(long long)orow * p.ldo + ocol] = __float2half_rn(y);
          else
            reinterpret_cast<__nv_bfloat16*>(p.out)[(long long)orow * p.ldo + ocol] =
                __float2bfloat16_rn(y);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->mempty[mb]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma8) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kW8TmemCols)
                 : "memory");
  }
}

// ------------------------------------------------ activation quantization
// One half-warp per (output row, 128-K group), 8 elements (16 bytes) per
// lane: amax over the group, scale = max(amax / 448, 1e-8), e4m3 =
// rn_satfinite(x / scale). With a gather (sorted_ids) output row s takes
// activation row sorted_ids[s] / top_k, and rows whose id is padding are
// written as zeros. Scale rows [out_rows, ld) are zeroed too.
__global__ void __launch_bounds__(256) fp8_act_quant_kernel(
    const void* __restrict__ x, int x_f16, long long x_rows, int K, const int* __restrict__ ids,
    int top_k, long long num_routes, long long out_rows, uint8_t* __restrict__ q,
    float* __restrict__ scales, long long ld, int* status) {
  griddep_wait();
  const int kch = K / 128;
  const int hl = threadIdx.x & 15;  // lane within the half-warp
  const int half = (threadIdx.x >> 4) & 1;
  // Warp-uniform loop over pairs of groups (the shuffles below need every
  // lane of the warp): half-warp `half` takes group 2 * pair + half.
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long groups = ld * kch;
  for (long long pair = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
       2 * pair < groups; pair += warps) {
    const long long gid = 2 * pair + half;
    const bool in = gid < groups;
    const long long r = in ? gid / kch : 0;
    const int kb = in ? (int)(gid - r * kch) : 0;
    const bool row = in && r < out_rows;
    if (in && !row && hl == 0) scales[(long long)kb * ld + r] = 0.f;
    long long src = row ? r : -1;
    if (row && ids != nullptr) {
      const int id = __ldg(ids + r);
      src = (id >= 0 && id < num_routes) ? id / top_k : -1;
      if (src >= x_rows) {
        if (hl == 0 && status) atomicOr(status, kDevBadRoute);
        src = -1;
      }
    }
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    if (src >= 0) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(
          reinterpret_cast<const uint16_t*>(x) + src * K + kb * 128 + hl * 8));
      const uint32_t wds[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (x_f16) {
          const __half2 hh = *reinterpret_cast<const __half2*>(&wds[i]);
          v[2 * i] = __low2float(hh);
          v[2 * i + 1] = __high2float(hh);
        } else {
          const __nv_bfloat162 bb = *reinterpret_cast<const __nv_bfloat162*>(&wds[i]);
          v[2 * i] = __low2float(bb);
          v[2 * i + 1] = __high2float(bb);
        }
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    // the half-warp's 16 lanes hold the group (xor offsets below 16 stay in it)
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = fmaxf(amax / 448.f, 1e-8f);
    uint32_t packed[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint16_t lo, hi;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;"
          : "=h"(lo)
          : "f"(v[4 * i + 1] / scale), "f"(v[4 * i] / scale));
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;"
          : "=h"(hi)
          : "f"(v[4 * i + 3] / scale), "f"(v[4 * i + 2] / scale));
      packed[i] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    if (row) {
      *reinterpret_cast<uint2*>(q + r * K + kb * 128 + hl * 8) = make_uint2(packed[0], packed[1]);
      if (hl == 0) scales[(long long)kb * ld + r] = scale;
    }
  }
  griddep_launch_dependents();
}

}  // namespace

cudaError_t launch_fp8_act_quant(const void* x, int x_f16, long long x_rows, int K,
                                 const int* ids, int top_k, long long num_routes,
                                 long long out_rows, uint8_t* q, float* scales, long long ld,
                                 int* status, cudaStream_t stream) {
  const long long groups = ld * (K / 128);
  long long blocks = (groups + 15) / 16;  // 16 half-warps per block
  const long long cap = (long long)device_sm_count() * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return launch_pdl(fp8_act_quant_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, x, x_f16,
                    x_rows, K, ids, top_k, num_routes, out_rows, q, scales, ld, status);
}

cudaError_t launch_w8a8_gemm(const W8Launch& L, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(w8a8_gemm_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kW8Smem);
    if (err != cudaSuccess) return err;
    configured[dev] = true;
  }
  const unsigned long long wrows = (unsigned long long)L.E * (unsigned long long)L.N;
  if (wrows >= (1ull << 31) || L.rows <= 0 || L.rows >= (1ll << 31)) return cudaErrorInvalidValue;
  CUtensorMap tmap_w, tmap_x;
  if (!make_map(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.w, (unsigned long long)L.K, wrows,
                (unsigned long long)L.K, 128, 16, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
    return cudaErrorInvalidValue;
  if (!make_map(&tmap_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.xq, (unsigned long long)L.K,
                (unsigned long long)L.rows, (unsigned long long)L.K, 128, 128,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
    return cudaErrorInvalidValue;
  W8Params p{};
  p.wscale = L.wscale;
  p.xscale = L.xscale;
  p.xs_ld = L.xs_ld;
  p.rows = L.rows;
  p.sorted_ids = L.sorted_ids;
  p.ntpp = L.ntpp;
  p.num_routes = L.num_routes;
  p.topk_w = L.topk_w;
  p.mul_w = L.mul_w;
  p.E = L.E;
  p.N = L.N;
  p.K = L.K;
  p.gated = L.gated;
  p.out = L.out;
  p.ldo = L.ldo;
  p.out_f16 = L.out_f16;
  p.status = L.status;
  const int* count = reinterpret_cast<const int*>(L.plan_buf);
  const int2* plan = L.plan_buf == nullptr
                         ? nullptr
                         : reinterpret_cast<const int2*>(reinterpret_cast<const uint8_t*>(L.plan_buf) + 256);
  long long items;
  if (L.sorted_ids == nullptr)
    items = (L.rows + kW8N - 1) / kW8N * (L.N / 128);
  else
    items = (long long)L.plan_cap * (L.N / 128);
  long long grid = device_sm_count();
  if (grid > items) grid = items;
  if (grid < 1) grid = 1;
  return launch_pdl(w8a8_gemm_kernel, dim3((unsigned)grid), dim3(kW8Threads), kW8Smem, stream, p,
                    plan, count, tmap_w, tmap_x);
}

int w8a8_item_slots() { return kW8N; }

}  // namespace b200
