// Weight-streaming GEMM for the decode regime (few rows per weight tile).
//
// Replaces, for B200, the reference's decode kernels:
//   * FP8 block-scaled dense decode (sglang_restomod/quant/sm70_fp8_dense/csrc/
//     sm70_fp8_qpn8_decode.cu:60-149, gated variant :156-246);
//   * the TurboMind block-FP8 expert GEMM used by SM70Fp8MoEMethod.apply
//     (sglang_restomod/quant/sm70_fp8_moe/method.py:303-304, contract in
//     quant/sm70_fp8_moe/README.md:23-58);
//   * the NVFP4 MoE decode GEMVs routed by moe_align_block_size
//     (sglang_restomod/quant/sm70_fp4_moe/csrc/decode_gemv_qpn2.cu:63-200).
//
// Design (B200-first, not a port of any of the above):
//   * Weights are prepacked at load time into 128-row x 128-K "units" whose
//     bytes are ordered exactly as the consumer warps read them (prepack.cu).
//     A unit is one FP8 scale block: 16 KiB of E4M3, or 8 KiB of E2M1 codes
//     plus 1 KiB of E4M3 group scales.
//   * A persistent grid splits the flattened (row-group, row-block, K-stage)
//     space evenly across CTAs (stream-K), or, when there are no more
//     (row-group, row-block) pairs than CTAs and they are short, gives each
//     CTA one whole pair; a stage is 1, 2 or 4 consecutive K-units of one
//     pair. Each CTA runs one producer warp and 8 consumer
//     warps over a shared-memory ring of up to 4 stages tracked by mbarriers.
//     For every stage the producer issues one cp.async.bulk (TMA) of its
//     weight units (contiguous in the prepacked bank; L2 evict-first), and
//     its 32 lanes copy the group's activation rows (128-K slices) with
//     16-byte cp.async into padded tiles (row stride 304 B, second half at
//     +160 B: bank-conflict-free for the consumers' 16-byte reads); one lane
//     copies the units' FP8 block scales (4-byte cp.async). All the copies
//     complete on the stage's mbarrier.
//   * A consumer warp owns 16 weight rows of the unit. It converts its bytes
//     with the hardware cvt.rn.f16x2.{e4m3x2,e2m1x2} instructions straight
//     into m16n8k16 A fragments and multiplies them against f16 activation
//     fragments read from the tile (fp32 accumulate). FP8 block scales are
//     applied once per unit to the accumulators; NVFP4 group scales
//     (fp16_rne(e4m3 * global), as the reference rounds them) multiply the
//     fragments.
//   * The K index inside a unit is permuted consistently on both operands so
//     that every lane reads 32 contiguous K of its rows and of its activation
//     row - the sum over K is order-free.
//   * A (row-group, row-block) pair that straddles CTAs is reduced through a
//     zeroed fp32 workspace slot with an arrival counter; the last arriving
//     CTA applies the epilogue and leaves slot and counter zeroed again.
//   * Launched with programmatic dependent launch: the prologue overlaps the
//     previous kernel, every thread waits on it before reading its outputs.
#include "common.cuh"
#include "internal.h"

namespace b200 {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
// Tuning knobs (compile-time). The defaults are the best of a same-box A/B:
// more stages, register preloading of 16-row activation tiles, and an L2
// prefetch ahead of the PDL wait each measured slower.
#ifndef B200_STREAM_MAX_STAGES
#define B200_STREAM_MAX_STAGES 4
#endif
// Stages of the one-CTA-per-SM launch used when a call has no more
// (group, row block) pairs than SMs and each is short (small decode
// batches): the whole pair streams through one CTA, so the bytes it keeps
// in flight are what its latency is divided by.
#ifndef B200_STREAM_SOLO_MAX_STAGES
#define B200_STREAM_SOLO_MAX_STAGES 6
#endif
#ifndef B200_STREAM_PRELOAD_NT
#define B200_STREAM_PRELOAD_NT 1
#endif
#ifndef B200_STREAM_DENSE_PREFETCH
#define B200_STREAM_DENSE_PREFETCH 0
#endif
// K-units per pipeline stage (1, 2 or 4; fewer when two such stages would
// not fit): consecutive K-units of a pair share one barrier wait, one unit
// walk and one accumulate. Measured against one unit per stage: FP8 two
// units 10 % faster (config4 decode); NVFP4 two units 10 %, four 17-20 %.
// Pairs of at most this many stages are not split across CTAs when there
// are no more pairs than CTAs (0: always split evenly, stream-K).
#ifndef B200_STREAM_WHOLE_PAIR_MAX_STAGES
#define B200_STREAM_WHOLE_PAIR_MAX_STAGES 8
#endif
// FP8 block scales of a stage copied into the stage by the producer (one
// 4-byte cp.async per scale) instead of loaded by every consumer warp.
#ifndef B200_STREAM_STAGE_SCALES
#define B200_STREAM_STAGE_SCALES 1
#endif
#ifndef B200_STREAM_SUB_FP8
#define B200_STREAM_SUB_FP8 2
#endif
#ifndef B200_STREAM_SUB_NVFP4
#define B200_STREAM_SUB_NVFP4 4
#endif

constexpr int kSmemPerSm = 233472;  // 228 KiB of shared memory per SM
constexpr int kSmemReserved = 1024; // per CTA, kept by the system
constexpr int kRowStride = 304;  // bytes per activation row in the tile
constexpr int kHalf1 = 160;      // offset of the row's second 128 bytes

template <int NT>
struct CtasPerSm {
  static constexpr int value = NT >= 8 ? 1 : 2;
};

template <int Q>
struct UnitBytes;
template <>
struct UnitBytes<kQuantFp8Block> {
  static constexpr uint32_t value = kFp8UnitBytes;
};
template <>
struct UnitBytes<kQuantNvfp4> {
  static constexpr uint32_t value = kFp4UnitBytes;
};

template <int Q>
struct SubUnits {
  static constexpr int value = Q == kQuantFp8Block ? B200_STREAM_SUB_FP8 : B200_STREAM_SUB_NVFP4;
  static_assert(value == 1 || value == 2 || value == 4, "1, 2 or 4 units per stage");
};

// FP8 stages end with their units' block scales: (top, bottom) per unit.
template <int Q>
struct StageScaleBytes {
  static constexpr uint32_t value = Q == kQuantFp8Block && B200_STREAM_STAGE_SCALES ? 8 : 0;
};

constexpr uint32_t stage_bytes(int sub, uint32_t w, uint32_t x, uint32_t sc) {
  return (sub * (w + x + sc) + 127) / 128 * 128;
}

// Stage = kSub consecutive weight units of one pair (contiguous, one bulk
// copy) followed by their kSub activation tiles (and, FP8, their block
// scales); as many stages as fit when
// CPS CTAs share an SM, capped at B200_STREAM_MAX_STAGES (CPS = 1, the
// launch for a few short pairs, at B200_STREAM_SOLO_MAX_STAGES).
template <int Q, int NT, int CPS = CtasPerSm<NT>::value>
struct Layout {
  static constexpr uint32_t kW = UnitBytes<Q>::value;
  static constexpr uint32_t kX = 8 * NT * kRowStride;
  static constexpr uint32_t kSc = StageScaleBytes<Q>::value;
  static constexpr int kBudget = kSmemPerSm / CPS - kSmemReserved - 128;
  static constexpr int kReq = SubUnits<Q>::value;
  static constexpr int kSub =
      kReq >= 4 && 2 * stage_bytes(4, kW, kX, kSc) <= (uint32_t)kBudget   ? 4
      : kReq >= 2 && 2 * stage_bytes(2, kW, kX, kSc) <= (uint32_t)kBudget ? 2
                                                                           : 1;
  static constexpr uint32_t kXOff = kSub * kW;             // first activation tile
  static constexpr uint32_t kScOff = kSub * (kW + kX);     // block scales
  static constexpr uint32_t kStage = stage_bytes(kSub, kW, kX, kSc);
  static constexpr int kFit = kBudget / (int)kStage;
  static constexpr int kCap = CPS == 1 ? B200_STREAM_SOLO_MAX_STAGES : B200_STREAM_MAX_STAGES;
  static constexpr int kS = kFit > kCap ? kCap : kFit;
  static constexpr size_t kSmem = (size_t)kS * kStage + 2 * kS * sizeof(uint64_t) + 16;
  static_assert(kS >= 2, "stage does not fit");
  static_assert(kXOff % 16 == 0 && kX % 16 == 0 && kScOff % 8 == 0, "cp.async destinations");
};

__device__ __forceinline__ int chunk_pos(int j) { return j * 16 + (j >= 8 ? kHalf1 - 128 : 0); }

__device__ __forceinline__ long long cta_containing(long long u, long long U, long long G) {
  // Largest c with floor(c*U/G) <= u.
  long long c = ((u + 1) * G + U - 1) / U - 1;
  return c < G ? c : G - 1;
}

__device__ __forceinline__ uint32_t f16x2_splat(float v) {
  __half h = __float2half_rn(v);
  __half2 h2 = __halves2half2(h, h);
  return *reinterpret_cast<uint32_t*>(&h2);
}

// Activation row of slot `slot` of group `gi`, or nullptr for a padding slot.
template <int NT>
__device__ __forceinline__ const __half* slot_row(const StreamParams& p, long long gi, int slot,
                                                  bool dense) {
  if (dense) {
    const long long t = gi * (8 * NT) + slot;
    return t < p.dense_m ? p.x + t * p.ldx : nullptr;
  }
  const int r = p.sorted_ids[gi * p.block_m + slot];
  if (r < 0 || r >= p.num_routes) return nullptr;
  const long long row = r / p.top_k;
  if (row >= p.x_rows) return nullptr;
  return p.x + row * p.ldx;
}

template <int NT>
__device__ __forceinline__ void store_pair(const StreamParams& p, long long gi, int rb, int warp,
                                           int lane, const float (&acc)[NT][4]) {
  const int g8 = lane >> 2, cq = lane & 3;
  const int row_top = warp * 16 + g8;  // local row inside the 128-row block
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e2 = 0; e2 < 2; ++e2) {
      const int tok = nt * 8 + 2 * cq + e2;
      long long orow;
      float w = 1.0f;
      if (p.sorted_ids == nullptr) {
        orow = gi * (8 * NT) + tok;
        if (orow >= p.dense_m) continue;
      } else {
        const int r = p.sorted_ids[gi * p.block_m + tok];
        if (r < 0 || r >= p.num_routes) continue;
        orow = r;
        if (p.mul_w) w = p.topk_w[r];
      }
      const float vt = acc[nt][e2];
      const float vb = acc[nt][2 + e2];
      long long c0, c1 = -1;
      float v0, v1 = 0.f;
      if (p.gated) {
        c0 = (long long)rb * 64 + warp * 8 + g8;
        if (p.fuse_act) {
          v0 = silu_f32(vt) * vb * w;
        } else {
          v0 = vt * w;
          c1 = c0 + p.N / 2;
          v1 = vb * w;
        }
      } else {
        c0 = (long long)rb * 128 + row_top;
        c1 = c0 + 8;
        v0 = vt * w;
        v1 = vb * w;
      }
      // Both output dtypes are 2 bytes; an expert-parallel owner's row may
      // live on another GPU (out_rows).
      void* orow_p = p.out_rows != nullptr
                         ? reinterpret_cast<void*>(p.out_rows[orow])
                         : reinterpret_cast<void*>(reinterpret_cast<uint16_t*>(p.out) + orow * p.ldo);
      if (p.out_f16) {
        __half* o = reinterpret_cast<__half*>(orow_p);
        o[c0] = __float2half_rn(v0);
        if (c1 >= 0) o[c1] = __float2half_rn(v1);
      } else {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(orow_p);
        o[c0] = __float2bfloat16_rn(v0);
        if (c1 >= 0) o[c1] = __float2bfloat16_rn(v1);
      }
    }
  }
}

template <int Q, int NT, int CPS>
__global__ void __launch_bounds__(kThreads, CPS)
    stream_gemm_kernel(const StreamParams p) {
  using L = Layout<Q, NT, CPS>;
  constexpr uint32_t UB = L::kW;
  constexpr int kRows = 8 * NT;
  constexpr int kSub = L::kSub;
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kStages = L::kS;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * L::kStage);
  uint64_t* empty = full + kStages;
  volatile int* flag = reinterpret_cast<volatile int*>(empty + kStages);
  volatile int* abort_flag = flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nrb = p.N / kUnitRows;
  const int kch = p.K / kUnitK;            // K-units per (group, row block) pair
  const int kcs = (kch + kSub - 1) / kSub;  // stages per pair; the last may hold fewer units
  const bool dense = p.sorted_ids == nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1 + 32);  // TMA expect_tx arrive + one cp.async arrive per lane
      mbar_init(&empty[s], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // Routing, activations and the workspace come from earlier kernels: every
  // thread waits for them before its first global read of such data. Only the
  // dense producer runs ahead, prefetching static weights into L2.
  const bool early_producer = B200_STREAM_DENSE_PREFETCH && dense && warp == kConsumerWarps;
  if (!early_producer) griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();

  // The producer reads the expert of group blockIdx.x / nrb together with the
  // group count: when each CTA takes one whole pair (small batches) that is
  // its first pair's expert, and its first weight copy then waits for one
  // load instead of two in a row. (In bounds: expert_ids holds max_groups
  // entries; the value is used only for a group below the aligned count.)
  const long long gi_first = (long long)blockIdx.x / nrb;
  int e_first = -1;
  if (!dense && warp == kConsumerWarps && gi_first < p.max_groups) e_first = p.expert_ids[gi_first];

  long long groups;
  if (dense) {
    groups = (long long)(p.dense_m + kRows - 1) / kRows;
  } else {
    groups = (long long)(p.ntpp[0] / p.block_m);
    if (groups < 0) groups = 0;
    if (groups > p.max_groups) groups = p.max_groups;
  }
  const long long pairs = groups * nrb;
  const long long U = pairs * (long long)kcs;
  const long long G = gridDim.x;
  long long u0, u1;
  if (pairs <= G && kcs <= B200_STREAM_WHOLE_PAIR_MAX_STAGES) {
    // Few, short pairs (small decode batches): one whole pair per CTA, so no
    // pair is split and none pays the workspace reduction; the pairs' first
    // stages alone keep enough bytes in flight.
    u0 = blockIdx.x < pairs ? (long long)blockIdx.x * kcs : U;
    u1 = blockIdx.x < pairs ? u0 + kcs : U;
  } else {
    u0 = (long long)blockIdx.x * U / G;
    u1 = ((long long)blockIdx.x + 1) * U / G;
  }
  if (u0 >= u1) {
    if (early_producer) griddep_wait();
    return;
  }

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (early_producer) {
      // Dense units of one CTA are contiguous in memory: pull the first ones
      // into L2 while the previous kernel finishes.
      if (lane == 0) {
        // first K-unit of stage u0, and the units of its first 2 * kStages stages
        const long long unit0 = (u0 / kcs) * kch + (u0 % kcs) * kSub;
        const long long units = (long long)p.dense_m > 0 ? (long long)nrb * kch : 0;
        long long pre = units - unit0;
        if (pre > 2LL * kStages * kSub) pre = 2LL * kStages * kSub;
        if (pre > 0)
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.wq + unit0 * (long long)UB),
                       "r"((uint32_t)(pre * UB))
                       : "memory");
      }
      griddep_wait();
    }
    // Activation rows go through per-lane 16-byte cp.async copies, which
    // signal the stage barrier when they land (one arrival per lane); many
    // small bulk copies would bottleneck the TMA engine. With kRows <= 32,
    // kLanesPerRow lanes share a tile row, each copying kChunks 16-byte
    // chunks of its 256 bytes; with 64 rows every lane owns two rows.
    constexpr int kRowsPerLane = kRows > 32 ? kRows / 32 : 1;
    constexpr int kLanesPerRow = kRows >= 32 ? 1 : 32 / kRows;
    constexpr int kChunks = 16 / kLanesPerRow;
    const int my_row0 = kRows >= 32 ? lane : lane / kLanesPerRow;
    const int my_chunk0 = kRows >= 32 ? 0 : (lane % kLanesPerRow) * kChunks;
    const uint64_t pol_w = l2_policy_evict_first();
    const __half* rows[kRowsPerLane];
    // (group, row block, stage of the pair) of u0; advanced by counters.
    long long pair = u0 / kcs;
    int kc = (int)(u0 - pair * kcs);
    long long gi = pair / nrb;
    int rb = (int)(pair - gi * nrb);
    bool new_pair = true;
    int e = 0;
    int i = 0;
    for (long long u = u0; u < u1; ++u) {
      if (u != u0) {
        if (++kc == kcs) {
          kc = 0;
          new_pair = true;
          if (++rb == nrb) {
            rb = 0;
            ++gi;
          }
        }
      }
      if (new_pair) e = dense ? 0 : (gi == gi_first ? e_first : p.expert_ids[gi]);
      if (e < 0 || e >= p.E) {
        new_pair = false;
        continue;
      }
      if (new_pair) {
        new_pair = false;
#pragma unroll
        for (int r = 0; r < kRowsPerLane; ++r)
          rows[r] = slot_row<NT>(p, gi, my_row0 + 32 * r, dense);
      }
      const int s = i % kStages;
      if (i >= kStages) {
        int ok = 1;
        if (lane == 0) ok = mbar_wait(&empty[s], ((i / kStages) - 1) & 1, p.status) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
      }
      uint8_t* stage = smem + (size_t)s * L::kStage;
      const int ku = kc * kSub;  // first K-unit of this stage
      const int nsub = kch - ku < kSub ? kch - ku : kSub;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], UB * (uint32_t)nsub);
        const uint8_t* src = p.wq + (((long long)e * nrb + rb) * kch + ku) * (long long)UB;
        bulk_g2s(stage, src, UB * (uint32_t)nsub, &full[s], pol_w);
      }
#pragma unroll
      for (int r = 0; r < kRowsPerLane; ++r) {
        if (rows[r] != nullptr) {
#pragma unroll
          for (int sub = 0; sub < kSub; ++sub) {
            if (sub < nsub) {
              const __half* src = rows[r] + (long long)(ku + sub) * kUnitK + my_chunk0 * 8;
              uint8_t* dst = stage + L::kXOff + sub * L::kX + (my_row0 + 32 * r) * kRowStride;
#pragma unroll
              for (int c = 0; c < kChunks; ++c)
                cp_async_16(dst + chunk_pos(my_chunk0 + c), src + c * 8);
            }
          }
        }
      }
      if constexpr (L::kSc != 0) {
        if (lane == 31) {
          const int nsr = p.N / kUnitRows;  // scale rows per expert
          const long long top = p.gated ? (long long)e * nsr + rb / 2 : (long long)e * nsr + rb;
          const long long bot = p.gated ? top + p.N / 2 / kUnitRows : top;
          for (int sub = 0; sub < nsub; ++sub) {
            cp_async_4(stage + L::kScOff + sub * 8, p.wscale + top * kch + ku + sub);
            cp_async_4(stage + L::kScOff + sub * 8 + 4, p.wscale + bot * kch + ku + sub);
          }
        }
      }
      cp_async_arrive_noinc(&full[s]);
      ++i;
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // Every consumer warp walks the same unit sequence and takes the same
  // branches at pair ends, so the named barriers below always line up. A
  // timed-out wait raises the CTA abort flag instead of returning.
  const int g8 = lane >> 2;
  const int cq = lane & 3;
  float acc[NT][4];
  bool valid[NT];
  // 8-row tiles with no valid row at all (the padding at the end of a
  // group): their MMAs are skipped (warp-uniform).
  bool tile_live[NT];
  long long pair = u0 / kcs;
  int kc = (int)(u0 - pair * kcs);
  long long gi = pair / nrb;
  int rb = (int)(pair - gi * nrb);
  bool new_pair = true;
  int e = 0;
  int i = 0;
  float gs = 1.f;  // NVFP4 global scale of expert e

  for (long long u = u0; u < u1; ++u) {
    if (u != u0) {
      if (++kc == kcs) {
        kc = 0;
        new_pair = true;
        ++pair;
        if (++rb == nrb) {
          rb = 0;
          ++gi;
        }
      }
    }
    if (new_pair) e = dense ? 0 : p.expert_ids[gi];
    if (e < 0 || e >= p.E) {
      if (new_pair && e >= p.E && rb == 0 && warp == 0 && lane == 0) atomicOr(p.status, kDevBadExpert);
      new_pair = false;
      continue;
    }

    if (new_pair) {
      new_pair = false;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[nt][r] = 0.f;
        valid[nt] = slot_row<NT>(p, gi, nt * 8 + g8, dense) != nullptr;
        tile_live[nt] = __any_sync(0xffffffffu, valid[nt]);
      }
      if constexpr (Q == kQuantNvfp4) gs = __ldg(p.gscale + e);
    }

    const int ku = kc * kSub;  // first K-unit of this stage
    const int nsub = kch - ku < kSub ? kch - ku : kSub;
    const int s = i % kStages;
    const uint32_t parity = (uint32_t)((i / kStages) & 1);
    ++i;
    bool ok = (*abort_flag == 0);
    if (ok && !mbar_wait(&full[s], parity, p.status)) {
      *abort_flag = 1;
      ok = false;
    }
    if (p.loads_only) {
      // pipeline floor: release the stage unread; no math, no stores
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&empty[s]);
      continue;
    }
    if (ok) {
      const uint8_t* stage = smem + (size_t)s * L::kStage;
      // NT == 1 keeps two accumulators (even / odd K-steps) so the MMA
      // chain is half as long; wider tiles already interleave NT chains.
      constexpr int kChains = NT == 1 ? 2 : 1;
      // Small tiles copy their activation fragments out and release the
      // stage once the last unit's are read; wider tiles read them during
      // the MMA loop.
      constexpr bool kPre = NT <= B200_STREAM_PRELOAD_NT;
      float t[NT * kChains][4];
#pragma unroll
      for (int c = 0; c < NT * kChains; ++c)
#pragma unroll
        for (int r = 0; r < 4; ++r) t[c][r] = 0.f;

#pragma unroll
      for (int sub = 0; sub < kSub; ++sub) {
        if (sub >= nsub) break;
        const uint8_t* wunit = stage + sub * UB;
        const uint8_t* xt = stage + L::kXOff + sub * L::kX + g8 * kRowStride;
        auto load_b = [&](int nt, int q) -> uint4 {
          if (!valid[nt]) return make_uint4(0u, 0u, 0u, 0u);
          return ld_shared_u128(xt + nt * 8 * kRowStride + chunk_pos(4 * cq + q));
        };
        const bool last = sub == nsub - 1;

        if constexpr (Q == kQuantFp8Block) {
          float s_top, s_bot;
          const int nsr = p.N / kUnitRows;  // scale rows per expert
          if constexpr (L::kSc != 0) {
            s_top = __uint_as_float(ld_shared_u32(stage + L::kScOff + sub * 8));
            s_bot = __uint_as_float(ld_shared_u32(stage + L::kScOff + sub * 8 + 4));
          } else if (p.gated) {
            const int half_rows = p.N / 2 / kUnitRows;
            s_top = __ldg(p.wscale + ((long long)e * nsr + rb / 2) * kch + ku + sub);
            s_bot = __ldg(p.wscale + ((long long)e * nsr + half_rows + rb / 2) * kch + ku + sub);
          } else {
            s_top = __ldg(p.wscale + ((long long)e * nsr + rb) * kch + ku + sub);
            s_bot = s_top;
          }
          if (sub > 0) {
#pragma unroll
            for (int c = 0; c < NT * kChains; ++c)
#pragma unroll
              for (int r = 0; r < 4; ++r) t[c][r] = 0.f;
          }
          uint4 wa[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            wa[q] = ld_shared_u128(wunit + warp * 2048 + q * 512 + lane * 16);
          uint4 bpre[kPre ? NT : 1][4];
          if constexpr (kPre) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int q = 0; q < 4; ++q) bpre[nt][q] = load_b(nt, q);
            if (last) {
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[s]);
            }
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 b[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if constexpr (kPre)
                b[nt] = bpre[nt][q];
              else
                b[nt] = load_b(nt, q);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t top = h ? wa[q].y : wa[q].x;
              const uint32_t bot = h ? wa[q].w : wa[q].z;
              uint32_t a[4];
              a[0] = e4m3x2_to_f16x2((uint16_t)(top & 0xffffu));
              a[1] = e4m3x2_to_f16x2((uint16_t)(bot & 0xffffu));
              a[2] = e4m3x2_to_f16x2((uint16_t)(top >> 16));
              a[3] = e4m3x2_to_f16x2((uint16_t)(bot >> 16));
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
                if (NT == 1 || tile_live[nt])
                  mma_16816(t[nt * kChains + (kChains == 2 ? h : 0)], a, h ? b[nt].z : b[nt].x,
                            h ? b[nt].w : b[nt].y);
            }
          }
          if constexpr (!kPre) {
            if (last) {
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[s]);
            }
          }
          if constexpr (kChains == 2) {
#pragma unroll
            for (int r = 0; r < 4; ++r) t[0][r] += t[1][r];
          }
          // block scales differ per unit: fold this unit's sums in now
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            acc[nt][0] = fmaf(s_top, t[nt][0], acc[nt][0]);
            acc[nt][1] = fmaf(s_top, t[nt][1], acc[nt][1]);
            acc[nt][2] = fmaf(s_bot, t[nt][2], acc[nt][2]);
            acc[nt][3] = fmaf(s_bot, t[nt][3], acc[nt][3]);
          }
        } else {
          const uint4 ct = ld_shared_u128(wunit + warp * 1024 + lane * 32);
          const uint4 cb = ld_shared_u128(wunit + warp * 1024 + lane * 32 + 16);
          const uint32_t sc = ld_shared_u32(wunit + 8192 + warp * 128 + lane * 4);
          uint4 bpre[kPre ? NT : 1][4];
          if constexpr (kPre) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int q = 0; q < 4; ++q) bpre[nt][q] = load_b(nt, q);
            if (last) {
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[s]);
            }
          }
          // Group scales: fp16_rne(float(e4m3) * global), the single rounding
          // the reference applies (quant/sm70_fp4_moe/csrc/decode_gemv_qpn2.cu:40-45).
          const uint32_t st2 = e4m3x2_to_f16x2((uint16_t)(sc & 0xffffu));
          const uint32_t sb2 = e4m3x2_to_f16x2((uint16_t)(sc >> 16));
          const __half2 st_h = *reinterpret_cast<const __half2*>(&st2);
          const __half2 sb_h = *reinterpret_cast<const __half2*>(&sb2);
          const uint32_t st[2] = {f16x2_splat(__low2float(st_h) * gs),
                                  f16x2_splat(__high2float(st_h) * gs)};
          const uint32_t sb[2] = {f16x2_splat(__low2float(sb_h) * gs),
                                  f16x2_splat(__high2float(sb_h) * gs)};
          const uint32_t ctw[4] = {ct.x, ct.y, ct.z, ct.w};
          const uint32_t cbw[4] = {cb.x, cb.y, cb.z, cb.w};
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            uint32_t wt[4], wb[4];
            e2m1x8_to_f16x2x4(ctw[m], wt);
            e2m1x8_to_f16x2x4(cbw[m], wb);
            const uint32_t sct = st[m >> 1];
            const uint32_t scb = sb[m >> 1];
            uint4 b[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if constexpr (kPre)
                b[nt] = bpre[nt][m];
              else
                b[nt] = load_b(nt, m);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t a[4];
              a[0] = hmul2_u32(wt[2 * h], sct);
              a[1] = hmul2_u32(wb[2 * h], scb);
              a[2] = hmul2_u32(wt[2 * h + 1], sct);
              a[3] = hmul2_u32(wb[2 * h + 1], scb);
              // k-step j = 2m + h uses activation chunk m, half h
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
                if (NT == 1 || tile_live[nt])
                  mma_16816(t[nt * kChains + (kChains == 2 ? h : 0)], a, h ? b[nt].z : b[nt].x,
                            h ? b[nt].w : b[nt].y);
            }
          }
          if constexpr (!kPre) {
            if (last) {
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[s]);
            }
          }
        }
      }
      if constexpr (Q == kQuantNvfp4) {
        // group scales are already in the fragments: one accumulate per stage
        if constexpr (kChains == 2) {
#pragma unroll
          for (int r = 0; r < 4; ++r) t[0][r] += t[1][r];
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[nt][r] += t[nt][r];
      }
    }

    const bool pair_end = (kc == kcs - 1) || (u == u1 - 1);
    if (!pair_end) continue;

    const long long pu0 = pair * kcs;
    const long long pu1 = pu0 + kcs;
    if (pu0 >= u0 && pu1 <= u1) {
      if (*abort_flag == 0) store_pair<NT>(p, gi, rb, warp, lane, acc);
      continue;
    }
    // Split pair: reduce through the workspace slot of the CTA where it starts.
    const long long slot = cta_containing(pu0, U, G);
    float* wsl = p.ws + slot * kWsSlotFloats;
    const int my_units = (int)((pu1 < u1 ? pu1 : u1) - (pu0 > u0 ? pu0 : u0));
    const int row_top = warp * 16 + g8;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        const int tok = nt * 8 + 2 * cq + e2;
        atomicAdd(wsl + row_top * 64 + tok, acc[nt][e2]);
        atomicAdd(wsl + (row_top + 8) * 64 + tok, acc[nt][2 + e2]);
      }
    }
    __threadfence();
    named_bar_sync(1, kConsumerWarps * 32);
    if (warp == 0 && lane == 0) {
      const int old = atomicAdd(p.ws_cnt + slot, my_units);
      *flag = (old + my_units == kcs) ? 1 : 0;
    }
    named_bar_sync(1, kConsumerWarps * 32);
    if (*flag != 0) {
      __threadfence();
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const int tok = nt * 8 + 2 * cq + e2;
          acc[nt][e2] = atomicExch(wsl + row_top * 64 + tok, 0.f);
          acc[nt][2 + e2] = atomicExch(wsl + (row_top + 8) * 64 + tok, 0.f);
        }
      }
      if (*abort_flag == 0) store_pair<NT>(p, gi, rb, warp, lane, acc);
      if (warp == 0 && lane == 0) atomicExch(p.ws_cnt + slot, 0);
    }
    named_bar_sync(1, kConsumerWarps * 32);
  }
}

template <int Q, int NT, int CPS = CtasPerSm<NT>::value>
cudaError_t launch_one(const StreamParams& p, int grid, cudaStream_t stream) {
  const size_t smem = Layout<Q, NT, CPS>::kSmem;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(stream_gemm_kernel<Q, NT, CPS>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    configured[dev] = true;
  }
  return launch_pdl(stream_gemm_kernel<Q, NT, CPS>, dim3(grid), dim3(kThreads), smem, stream, p);
}

}  // namespace

int stream_gemm_whole_pair_max_stages() { return B200_STREAM_WHOLE_PAIR_MAX_STAGES; }

// K-units per stage of the nt <= 2 layouts (the same at one or two CTAs per SM).
int stream_gemm_stage_units(int quant) {
  return quant == kQuantFp8Block ? Layout<kQuantFp8Block, 1>::kSub : Layout<kQuantNvfp4, 1>::kSub;
}

int stream_gemm_ctas_per_sm(int nt) { return nt >= 8 ? CtasPerSm<8>::value : CtasPerSm<1>::value; }

cudaError_t launch_stream_gemm(int quant, int nt, const StreamParams& p, int grid,
                               cudaStream_t stream, bool solo) {
  if (solo && nt <= 2) {
    // one CTA per SM, deeper ring (few short pairs, one per CTA)
    if (quant == kQuantFp8Block)
      return nt == 1 ? launch_one<kQuantFp8Block, 1, 1>(p, grid, stream)
                     : launch_one<kQuantFp8Block, 2, 1>(p, grid, stream);
    return nt == 1 ? launch_one<kQuantNvfp4, 1, 1>(p, grid, stream)
                   : launch_one<kQuantNvfp4, 2, 1>(p, grid, stream);
  }
  if (quant == kQuantFp8Block) {
    switch (nt) {
      case 1: return launch_one<kQuantFp8Block, 1>(p, grid, stream);
      case 2: return launch_one<kQuantFp8Block, 2>(p, grid, stream);
      case 4: return launch_one<kQuantFp8Block, 4>(p, grid, stream);
      case 8: return launch_one<kQuantFp8Block, 8>(p, grid, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (nt) {
    case 1: return launch_one<kQuantNvfp4, 1>(p, grid, stream);
    case 2: return launch_one<kQuantNvfp4, 2>(p, grid, stream);
    case 4: return launch_one<kQuantNvfp4, 4>(p, grid, stream);
    case 8: return launch_one<kQuantNvfp4, 8>(p, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace b200
