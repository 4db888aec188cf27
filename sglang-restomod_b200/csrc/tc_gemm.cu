// Tensor-core (tcgen05) grouped GEMM for the prefill regime: many routed
// tokens per expert, block-FP8 weights.
//
// Replaces, for large per-expert row counts, the reference's TurboMind block-
// FP8 expert GEMM (sglang_restomod/quant/sm70_fp8_moe/method.py:303-304,
// contract quant/sm70_fp8_moe/README.md:23-58) and its dense prefill dispatch
// (quant/sm70_fp8_dense/_method.py:713-784).
//
// Shape: D[128 weight rows, N tokens] = W_e[128 rows, K] . X[N tokens, K]^T
// ("swap AB": the weight row block is the MMA's M = 128; the expert's token
// group is N = 64..256, a multiple of 16, so short groups waste little).
//
// Per CTA (persistent, one per SM) and per 128-K step, two shared-memory
// stages alternate:
//   * all 256 threads dequantize the step's 16 KiB FP8 unit (the streamed
//     layout of prepack.cu, read straight from global, one step ahead in
//     registers) to f16(e4m3 * block scale) and store it as the A operand in
//     the K-major 128-byte swizzled layout;
//   * they copy the group's activation rows (f16, gathered through
//     sorted_token_ids) into the B operand with 16-byte cp.async, same layout;
//   * after a proxy fence and a CTA barrier, one thread issues eight
//     tcgen05.mma (M=128, N=BN, K=16, fp32 accumulate in tensor memory) and
//     commits them to the stage's mbarrier; the next step's loads overlap.
// The epilogue reads the accumulator with tcgen05.ld (warp w owns TMEM lanes
// 32*(w%4).., half of the columns) and applies SiLU*up (gate/up rows are
// 8 lanes apart in a gated bank), the router weight, and the store.
// Waits on MMA completion are bounded; a timeout records an error bit and the
// CTA still frees its tensor memory before returning.
#include "common.cuh"
#include "internal.h"

namespace b200 {
namespace {

constexpr int kTcThreads = 256;
constexpr uint32_t kABytes = 128 * 128 * 2;  // bf16 [128 rows][128 K], two 64-K atoms

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  // K-major, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart (SBO),
  // LBO field 1 (unused by swizzled K-major), version 1, layout type 2.
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

template <bool F16>
__host__ __device__ constexpr uint32_t instr_desc(int n) {
  // f32 accumulate, A/B = bf16 (1) or f16 (0), both K-major, M = 128.
  return (1u << 4) | ((F16 ? 0u : 1u) << 7) | ((F16 ? 0u : 1u) << 10) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n"
      "  .reg .pred p;\n"
      "  setp.ne.b32 p, %4, 0;\n"
      "  tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of 16-byte chunk (row, c16) of a [rows][64 x 16-bit] K-major
// 128B-swizzled atom.
__device__ __forceinline__ uint32_t sw128_off(int row, int c16) {
  return (uint32_t)row * 128u + (uint32_t)((c16 ^ (row & 7)) << 4);
}

template <bool F16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (F16) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// 8 E4M3 bytes (one 64-bit half of a 16-byte chunk) -> 8 16-bit values * s.
template <bool F16>
__device__ __forceinline__ uint4 dequant8(uint32_t lo, uint32_t hi, float s) {
  const uint32_t w[2] = {lo, hi};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t a = e4m3x2_to_f16x2((uint16_t)(w[i] & 0xffffu));
    const uint32_t b = e4m3x2_to_f16x2((uint16_t)(w[i] >> 16));
    const __half2 ha = *reinterpret_cast<const __half2*>(&a);
    const __half2 hb = *reinterpret_cast<const __half2*>(&b);
    o[2 * i] = pack2<F16>(__low2float(ha) * s, __high2float(ha) * s);
    o[2 * i + 1] = pack2<F16>(__low2float(hb) * s, __high2float(hb) * s);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int BN, bool F16>
struct TcLayout {
  static constexpr uint32_t kB = BN * 256u;  // [BN rows][128 K] 16-bit, two atoms
  static constexpr uint32_t kStage = kABytes + kB;
  static constexpr size_t kSmem = 2 * (size_t)kStage + 1024 /*align*/ + 64;
  static constexpr int kRowsPerThread = BN * 16 / kTcThreads;  // B chunks per thread per step
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;          // power of two >= 32
};

template <int BN, bool F16>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const StreamParams p) {
  using L = TcLayout<BN, F16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(smem + 2 * L::kStage);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(mma_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(mma_bar + 3);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nrb = p.N / 128;
  const int kch = p.K / 128;
  const bool dense = p.sorted_ids == nullptr;

  if (tid == 0) {
    mbar_init(&mma_bar[0], 1);
    mbar_init(&mma_bar[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32((const void*)tmem_slot)),
                 "r"(L::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  griddep_wait();
  if (tid == 0) griddep_launch_dependents();

  long long groups;
  if (dense) {
    groups = (long long)(p.dense_m + BN - 1) / BN;
  } else {
    groups = (long long)(p.ntpp[0] / p.block_m);
    if (groups < 0) groups = 0;
    if (groups > p.max_groups) groups = p.max_groups;
  }
  const long long items = groups * nrb;
  constexpr uint32_t kIdesc = instr_desc<F16>(BN);
  uint32_t phase[2] = {0u, 0u};
  int issued[2] = {0, 0};  // MMA batches committed to each stage barrier, not yet waited

  for (long long item = blockIdx.x; item < items; item += gridDim.x) {
    const long long gi = item / nrb;
    const int rb = (int)(item - gi * nrb);
    const int e = dense ? 0 : p.expert_ids[gi];
    if (e < 0 || e >= p.E) continue;

    // Activation rows this thread copies: chunk c = tid + 256*i of the
    // [BN rows][16 chunks] step tile -> row c/16, chunk c%16.
    const uint16_t* xrow[L::kRowsPerThread];
#pragma unroll
    for (int i = 0; i < L::kRowsPerThread; ++i) {
      const int n = (tid + kTcThreads * i) >> 4;
      const uint16_t* ptr = nullptr;
      if (dense) {
        const long long t = gi * BN + n;
        if (t < p.dense_m) ptr = reinterpret_cast<const uint16_t*>(p.x) + t * p.ldx;
      } else {
        const int r = p.sorted_ids[gi * p.block_m + n];
        if (r >= 0 && r < p.num_routes) {
          const long long row = r / p.top_k;
          if (row < p.x_rows) ptr = reinterpret_cast<const uint16_t*>(p.x) + row * p.ldx;
        }
      }
      xrow[i] = ptr;
    }

    // Weight scales of this row block (logical scale rows; gate/up banks
    // take the gate scale for the top rows and the up scale for the bottom).
    const int nsr = p.N / 128;
    const float* srow_top;
    const float* srow_bot;
    if (p.gated) {
      srow_top = p.wscale + ((long long)e * nsr + rb / 2) * kch;
      srow_bot = p.wscale + ((long long)e * nsr + p.N / 2 / 128 + rb / 2) * kch;
    } else {
      srow_top = p.wscale + ((long long)e * nsr + rb) * kch;
      srow_bot = srow_top;
    }
    const uint8_t* wunit = p.wq + ((long long)e * nrb + rb) * (long long)kch * kFp8UnitBytes;

    // Weight bytes for the next step, one step ahead in registers: chunk
    // j = tid + 256*i of the 16 KiB unit.
    uint4 wreg[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      wreg[i] = __ldg(reinterpret_cast<const uint4*>(wunit) + tid + kTcThreads * i);

    for (int kc = 0; kc < kch; ++kc) {
      const int s = kc & 1;
      uint8_t* stA = smem + s * L::kStage;
      uint8_t* stB = stA + kABytes;
      // Stage s was last read by the MMAs committed two steps ago.
      if (issued[s]) {
        bool ok = (*abort_flag == 0) && mbar_wait(&mma_bar[s], phase[s], p.status);
        phase[s] ^= 1u;
        issued[s] = 0;
        if (!ok) *abort_flag = 1;
      }
      tc_fence_after();
      // B: activation rows of this step.
#pragma unroll
      for (int i = 0; i < L::kRowsPerThread; ++i) {
        if (xrow[i] != nullptr) {
          const int c = tid + kTcThreads * i;
          const int n = c >> 4, j = c & 15;
          cp_async_16(stB + (j >> 3) * (BN * 128) + sw128_off(n, j & 7),
                      xrow[i] + (long long)kc * 128 + j * 8);
        }
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
      // A: dequantize this step's unit from registers, then fetch the next.
      const float st = __ldg(srow_top + kc);
      const float sb = __ldg(srow_bot + kc);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int jch = tid + kTcThreads * i;   // 16-byte chunk of the streamed unit
        const int wp = jch >> 7, q = (jch >> 5) & 3, ln = jch & 31;
        const int r0 = 16 * wp + (ln >> 2), r1 = r0 + 8;
        const int k0 = 32 * (ln & 3) + 8 * q;  // K of the chunk's 8 values
        const int atom = k0 >> 6, c16 = (k0 & 63) >> 3;
        *reinterpret_cast<uint4*>(stA + atom * 16384 + sw128_off(r0, c16)) =
            dequant8<F16>(wreg[i].x, wreg[i].y, st);
        *reinterpret_cast<uint4*>(stA + atom * 16384 + sw128_off(r1, c16)) =
            dequant8<F16>(wreg[i].z, wreg[i].w, sb);
      }
      if (kc + 1 < kch) {
        const uint4* nxt = reinterpret_cast<const uint4*>(wunit + (long long)(kc + 1) * kFp8UnitBytes);
#pragma unroll
        for (int i = 0; i < 4; ++i) wreg[i] = __ldg(nxt + tid + kTcThreads * i);
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
      fence_proxy_async();
      tc_fence_before();
      __syncthreads();
      if (tid == 0 && *abort_flag == 0) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(stA), b0 = smem_u32(stB);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)(kk & 3) * 32u;
          const uint64_t da = smem_desc_sw128(a0 + (kk >> 2) * 16384u + off);
          const uint64_t db = smem_desc_sw128(b0 + (kk >> 2) * (uint32_t)(BN * 128) + off);
          mma_bf16(tmem, da, db, kIdesc, (kc > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&mma_bar[s]);
      }
      issued[s] = 1;
    }

    // Wait for this item's last MMAs, then read the accumulator.
    {
      const int s = (kch - 1) & 1;
      bool ok = (*abort_flag == 0) && mbar_wait(&mma_bar[s], phase[s], p.status);
      phase[s] ^= 1u;
      issued[s] = 0;
      if (!ok) *abort_flag = 1;
      // The other stage's batch (if any) completed before this one.
      const int o = s ^ 1;
      if (issued[o]) {
        ok = (*abort_flag == 0) && mbar_wait(&mma_bar[o], phase[o], p.status);
        phase[o] ^= 1u;
        issued[o] = 0;
        if (!ok) *abort_flag = 1;
      }
    }
    tc_fence_after();
    if (*abort_flag == 0) {
      const int quarter = warp & 3;
      const int m = quarter * 32 + lane;  // accumulator lane = local weight row
      const int col0 = (warp >> 2) * (BN / 2);
      for (int cc = 0; cc < BN / 2; cc += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(col0 + cc), v);
        float up[16];
        if (p.gated) {
#pragma unroll
          for (int i = 0; i < 16; ++i) up[i] = __shfl_down_sync(0xffffffffu, v[i], 8);
        }
        const bool top = (m & 15) < 8;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int n = col0 + cc + i;
          long long orow;
          float w = 1.f;
          if (dense) {
            orow = gi * BN + n;
            if (orow >= p.dense_m) continue;
          } else {
            const int r = p.sorted_ids[gi * p.block_m + n];
            if (r < 0 || r >= p.num_routes) continue;
            orow = r;
            if (p.mul_w) w = p.topk_w[r];
          }
          long long col;
          float val;
          if (p.gated) {
            const long long j = (long long)rb * 64 + (m >> 4) * 8 + (m & 7);
            if (p.fuse_act) {
              if (!top) continue;
              col = j;
              val = silu_f32(v[i]) * up[i] * w;
            } else {
              col = top ? j : j + p.N / 2;
              val = v[i] * w;
            }
          } else {
            col = (long long)rb * 128 + m;
            val = v[i] * w;
          }
          if (p.out_f16)
            reinterpret_cast<__half*>(p.out)[orow * p.ldo + col] = __float2half_rn(val);
          else
            reinterpret_cast<__nv_bfloat16*>(p.out)[orow * p.ldo + col] = __float2bfloat16_rn(val);
        }
      }
    }
    // Every thread's accumulator reads finish before the next item's MMAs.
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(L::kTmemCols)
                 : "memory");
  }
}

template <int BN, bool F16>
cudaError_t launch_tc(const StreamParams& p, int grid, cudaStream_t stream) {
  using L = TcLayout<BN, F16>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(tc_gemm_kernel<BN, F16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)L::kSmem);
    if (err != cudaSuccess) return err;
    configured[dev] = true;
  }
  return launch_pdl(tc_gemm_kernel<BN, F16>, dim3(grid), dim3(kTcThreads), L::kSmem, stream, p);
}

}  // namespace

bool tc_gemm_supported(int block) { return block == 64 || block == 128 || block == 256; }

// Operands are f16: the weights dequantized as f16(e4m3 * scale), whose
// rounding (2^-11) keeps long-K sums as close to the exact dequantized
// product as the decode path; bf16 activations are converted by the caller.
cudaError_t launch_tc_gemm(int block, const StreamParams& p, int grid, cudaStream_t stream) {
  switch (block) {
    case 64: return launch_tc<64, true>(p, grid, stream);
    case 128: return launch_tc<128, true>(p, grid, stream);
    case 256: return launch_tc<256, true>(p, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace b200
