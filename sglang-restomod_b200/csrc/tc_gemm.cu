// Tensor-core (tcgen05) grouped GEMM for the prefill regime: many routed
// tokens per expert, block-FP8 weights.
//
// Replaces, for large per-expert row counts, the reference's TurboMind block-
// FP8 expert GEMM (sglang_restomod/quant/sm70_fp8_moe/method.py:303-304,
// contract quant/sm70_fp8_moe/README.md:23-58) and its dense prefill dispatch
// (quant/sm70_fp8_dense/_method.py:713-784).
//
// Shape: D[128 weight rows, N tokens] = W_e[128 rows, K] . X[N tokens, K]^T
// ("swap AB": the weight row block is the MMA's M = 128; the tokens are
// N <= 192). An item is one 128-row weight block of one expert against up to
// 192 of that expert's route slots: a small pre-kernel (tc_plan_kernel) merges
// runs of consecutive moe_align blocks of the same expert into items, so an
// expert's weights are dequantized once per 192 routes, and the item's N is
// trimmed to its last valid route (rounded up to 16).
//
// The A operand (dequantized weights) lives in tensor memory; shared memory
// carries the raw FP8 units and the activation tiles, both written by TMA.
// One persistent CTA per SM, 16 warps with fixed roles, coupled only through
// mbarrier rings (every wait bounded, no named barriers):
//   warp 0       weights: per 16 KiB FP8 unit (one 128x128 block of
//                prepack.cu's streamed layout) its two f16 scale multipliers
//                and a 2-D TMA copy (128-byte swizzle) into the raw ring;
//                the warp computes 32 units' multipliers at a time and lane 0
//                issues their copies;
//   warp 1       MMA: lane 0 alone runs the main loop - per stage its B tile
//                (`bfull`) and A columns (`full`), tested one stage ahead,
//                tcgen05.mma (M=128, N<=192, K=16, A from tensor memory, B
//                from shared memory, f16 x f16 -> f32), four per 64 K, and one
//                tcgen05.commit that releases the stage (its A columns and its
//                B tile) to the producers;
//   warps 2-3    activations: the item's rows as 2-D TMA tiles of a
//                slot-ordered copy (lane 0 of warp 2), or gathered through
//                sorted_token_ids with 16-byte cp.async (both warps), into
//                128-byte-swizzled [rows][64 K] sub-tiles; the copies land on
//                the stage's `bfull` barrier;
//   warps 4-7    dequant: lane = weight row; each reads its row's FP8 bytes
//                from the swizzled raw unit (conflict-free 8-byte reads),
//                f16(e4m3) * m with one hmul2 per two values, and writes them
//                into the stage's tensor-memory columns (tcgen05.st), then
//                arrive on the stage's `full` barrier; warps 12-15 are a
//                second dequant group in two of the three configurations
//                (TcCfg: alternate units on the narrow tiles, the other 64-K
//                half of every unit on long wide items);
//   warps 8-15   epilogue (8-11 where 12-15 dequantize): tcgen05.ld of a
//                double-buffered accumulator, 2^E, SiLU*up, router weight and
//                store, overlapping the next item's main loop; with two
//                groups warps 8-11 drain buffer 0 (even items), warps 12-15
//                buffer 1.
// The MMA thread's loop is the pipeline's critical path. Measured on B200 with
// a per-stage timeline of every role: the producers ran ~2,000 clocks ahead
// while a warp-wide loop with separate A and B barriers spent 650-800 clocks
// per 64-K stage on control (warp votes, two commits, 64-bit ring arithmetic)
// against ~100 for its four MMAs; a barrier poll whose result feeds a branch
// costs ~190 clocks; and an N = 192 MMA issues at about the tensor rate, so
// nothing the MMA thread does besides issuing MMAs is hidden. Hence one
// thread, one commit per stage, 32-bit ring counters, 128-K stages, and the
// next stage's barriers tested while this stage's MMAs issue. (A separate
// "scout" warp that polled the barriers and published a ready count, so that
// the MMA thread never polled, measured 10-25 % slower on the wide tiles: its
// extra hop lands on the dequant refill chain that bounds them.)
// Tensor memory: accumulators in columns [0, 2 NMAX), then the A stages.
//
// Block scales. A 128x128 block's scale s is split as s = m * 2^E with one
// power of two E per (expert, 128-row scale block) - the exponent of the
// largest scale of that row - and m = f16(s * 2^-E) in (0, 2). The weights are
// dequantized as f16(e4m3 * m) (f16 rounding; values below 2^-24 of the row's
// largest block scale flush) and the accumulator is multiplied by 2^E exactly.
#include <cuda.h>  // CUtensorMap and its encoding enums (types only)

#include <cstring>

#include "common.cuh"
#include "internal.h"
#include "tcgen05.cuh"

namespace b200 {
namespace {

using namespace tcg;
using namespace tcg_host;

// 16 warps: four per SM sub-partition, so each thread may hold 128 registers.
constexpr int kTcWarps = 16;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kWarpMeta = 0, kWarpMma = 1, kWarpLoad = 2, kWarpDeq = 4, kWarpEpi = 8;
constexpr int kLoadThreads = (kWarpDeq - kWarpLoad) * 32;
constexpr uint32_t kUnitBytes = kFp8UnitBytes;           // 16 KiB
constexpr int kInfoSlots = 8;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSubCols = 32;                        // 64 K f16 = 32 tensor-memory columns
constexpr int kNMaxWide = 192;   // route slots (MMA N) per item: the prefill tiles
constexpr int kNMaxNarrow = 64;  // items of few routes (expert-parallel owners, dense M <= 64)

// Tile configuration by the item width NMAX. A stage is kSub 64-K sub-tiles:
// its A columns in tensor memory (a ring of kAStages) and its B tile
// ([NMAX rows][64 K] f16 per sub-tile) in shared memory (a ring of kBStages
// >= kAStages). Stage t uses A slot t % kAStages and B slot t % kBStages, and
// the MMA thread's one commit per stage lands on empty[t % kBStages]: the B
// producer reuses its slot after stage t - kBStages, the dequant warps theirs
// after stage t - kAStages. Stages are 128 K (one weight unit): measured per
// stage on B200, the MMA thread spends ~400 clocks per stage on its barrier
// tests, commit and loop whatever the stage's size, against 96 clocks of
// tensor work per N = 192 MMA, so a 64-K stage (four MMAs) left the tensor
// pipe idle about half the time. The wide configuration's two 192-column
// accumulators leave tensor memory for two 128-K A stages (the dequant warps
// refill a slot in ~250 clocks, well inside the other stage's ~770 of MMAs);
// its B tiles come from L2 ~2,000 clocks after they are asked for, so three
// 48 KiB B stages are in flight, and five raw weight units. The narrow
// configuration's 64-column accumulators leave room for six A stages.
// Configurations: kTcWideShort (items of 192 slots, fewer than 32 weight
// units), kTcWideLong (192 slots, 32 units or more), kTcNarrow (64 slots).
constexpr int kTcWideShort = 0, kTcWideLong = 1, kTcNarrow = 2;
template <int CFG>
struct TcCfg {
  static constexpr int NMAX = CFG == kTcNarrow ? 64 : 192;
  static constexpr int kNMax = NMAX;
  static constexpr int kLoadPasses = NMAX / (kLoadThreads / 2);  // rows per gather thread
  static constexpr int kRawStages = NMAX > 64 ? 5 : 8;             // 16 KiB units in flight
  static constexpr int kSub = 2;                                   // 64-K sub-tiles per stage
  static constexpr int kAStages = NMAX > 64 ? 2 : 6;               // tensor memory
  static constexpr int kBStages = NMAX > 64 ? 3 : 6;               // shared memory
  // Dequant and epilogue warp groups (four warps each, one per tensor-memory
  // lane quarter) among warps 4-15. Measured on B200: with long items the
  // one epilogue group keeps up, and two dequant groups pay - on the wide
  // tiles each converts one 64-K half of every unit (halving the refill
  // latency of the two A slots: config4 T=4096 gate/up 3.30 -> 2.98 ms), on
  // the narrow ones group g takes the units u with u % 2 == g (one group's
  // ~450 clocks per 128-K stage per warp paced them); with short wide items
  // (K = 512-2048) the second epilogue group is needed (config2 T=8192
  // gate/up 556 us with it, 630 us without).
  static constexpr int kDqGroups = CFG == kTcWideShort ? 1 : 2;
  static constexpr int kEpiGroups = 3 - kDqGroups;
  static constexpr bool kDqHalves = CFG == kTcWideLong;
  static constexpr uint32_t kSubTile = NMAX * 128;                 // [NMAX rows][64 K] f16
  static constexpr uint32_t kBStage = kSub * kSubTile;
  static constexpr uint32_t kStageCols = kSub * kSubCols;
  static constexpr uint32_t kOffB = 0;
  static constexpr uint32_t kOffRaw = kOffB + kBStages * kBStage;
  static constexpr uint32_t kOffCtl = kOffRaw + kRawStages * kUnitBytes;
  static constexpr uint32_t kAccCols = NMAX;                       // per accumulator buffer
  static constexpr uint32_t kACol0 = 2 * kAccCols;                 // first A-stage column
  static constexpr size_t kTcSmem = kOffCtl + 1024 + 1024;  // control block + alignment slack
  static_assert(kBStages >= kAStages, "an A slot is reused after its stage's commit");
  static_assert(kACol0 + kAStages * kStageCols <= kTmemCols, "tensor memory");
  static_assert(kSubTile % 1024 == 0 && kOffRaw % 1024 == 0, "swizzled tiles stay 1024-byte aligned");
  static_assert(kTcSmem <= 232448, "shared memory");
  static_assert(NMAX % 64 == 0 && kLoadPasses * (kLoadThreads / 2) == NMAX, "item width");
  static_assert(2 % kSub == 0, "a weight unit is two 64-K halves");
  static_assert(kDqGroups == 1 || kSub == 2, "two dequant groups need 128-K stages");
};

template <int R, int A, int B>
struct CtlT {
  uint64_t full[A];    // A columns written: the 4 dequant warps
  uint64_t empty[B];   // stage t consumed (slot t % B): one MMA commit
  uint64_t bfull[B];   // B tile landed: gather threads or the TMA issuer (+ bytes)
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t raw_full[R];      // expect_tx + the unit's bytes
  uint64_t raw_empty[R];     // 4 dequant warps
  uint64_t done;
  uint2 raw_mult[R];         // f16x2 multipliers: top 8 rows of every 16, bottom 8
  uint2 wmult[32];           // the weight warp's multipliers for its next 32 units
  int info[kInfoSlots];      // (item << 9) | N of the item's MMAs, atomicMax-combined
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(CtlT<8, 6, 6>) <= 1024, "control block");

// Position in a ring of N slots: slot index and the parity of its phase.
template <int N>
struct RingPos {
  uint32_t idx = 0, phase = 0;
  __device__ __forceinline__ void advance() {
    if (++idx == (uint32_t)N) {
      idx = 0;
      phase ^= 1u;
    }
  }
};


__device__ __forceinline__ uint32_t instr_desc_f16(int n) {
  // f32 accumulate, A/B f16, both K-major, M = 128, N = n.
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}


// D[tmem] (+)= A[tmem] . B[smem descriptor]^T
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      "  .reg .pred p;\n"
      "  setp.ne.b32 p, %4, 0;\n"
      "  tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n"
      "}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}




// Lane i of the warp writes v[0..31] to lane (taddr.lane + i), columns
// taddr.col .. +31; returns once the stores have completed.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Byte offset of 16-byte chunk (row, c16) of a [rows][64 x 16-bit] K-major
// 128B-swizzled tile.
__device__ __forceinline__ uint32_t sw128_off(int row, int c16) {
  return (uint32_t)row * 128u + (uint32_t)((c16 ^ (row & 7)) << 4);
}


// Bounded wait that also gives up once another role of the CTA has aborted.
template <class Ctl>
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Ctl* ctl, int* status) {
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

// Bounded wait for two barriers at once: both polls go out before the branch
// on their results, so a thread whose two operands are ready pays one poll
// latency (~190 clocks on B200), not two.
template <class Ctl>
__device__ __forceinline__ bool wait_bar2(uint64_t* bar_a, uint32_t par_a, uint64_t* bar_b,
                                          uint32_t par_b, Ctl* ctl, int* status) {
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 0;; ++i) {
    const bool a = mbar_try_wait(bar_a, par_a);
    const bool b = mbar_try_wait(bar_b, par_b);
    if (a && b) return true;
    if ((i & 63u) == 63u) {
      if (*reinterpret_cast<volatile int*>(&ctl->abort)) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        if (status) atomicOr(status, kDevWaitTimeout);
        *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
        return false;
      }
    }
  }
}

// The same wait for a role off the critical path: a pause of about pause_ns
// between polls leaves the SM's barrier unit to the MMA thread, whose waits,
// fences and commits otherwise queue behind a dozen spinning warps.
#ifndef B200_TC_PAUSE_NS
#define B200_TC_PAUSE_NS 64
#endif
template <class Ctl>
__device__ __forceinline__ bool wait_bar_lazy(uint64_t* bar, uint32_t parity, Ctl* ctl, int* status,
                                              uint32_t pause_ns = B200_TC_PAUSE_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (;;) {
    __nanosleep(pause_ns);
    if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile int*>(&ctl->abort)) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      if (status) atomicOr(status, kDevWaitTimeout);
      *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
      return false;
    }
  }
}

// A lazy wait taken by every lane of the warp, with one shared outcome.
template <class Ctl>
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, Ctl* ctl, int* status,
                                          uint32_t pause_ns = B200_TC_PAUSE_NS) {
  return __all_sync(0xffffffffu, wait_bar_lazy(bar, parity, ctl, status, pause_ns));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Binary exponent of a scale row's largest |scale|, clamped so that both 2^E
// and 2^-E are normal floats.
__device__ __forceinline__ int max_exponent(float mx) {
  const int e = (int)((__float_as_uint(mx) >> 23) & 0xffu) - 127;
  return e < -126 ? -126 : (e > 126 ? 126 : e);
}
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

__device__ __forceinline__ uint32_t mult_f16x2(float s, int e) {
  const uint16_t b = __half_as_ushort(__float2half_rn(s * pow2f(-e)));
  return (uint32_t)b | ((uint32_t)b << 16);
}

__device__ __forceinline__ float ldg_or0(const float* p, int k, int kch) {
  return k < kch ? __ldg(p + k) : 0.f;
}

// One item of the CTA's walk, decoded identically by every role.
struct Item {
  int e;            // expert (0 for dense)
  int rb;           // 128-row weight block
  long long slot0;  // first route slot (moe) or first activation row (dense)
  int rows;         // route slots / rows covered (<= the item width)
  int kc0, nk;      // 128-K units kc0 .. kc0+nk-1 (all of K unless split)
};

// Dense items with K split: item g = ((chunk * nrb) + rb) * ksplit + part.
__device__ __forceinline__ void item_k_range(const StreamParams& p, long long g, int kch,
                                             int& kc0, int& nk) {
  if (p.sorted_ids != nullptr || p.ksplit <= 1) {
    kc0 = 0;
    nk = kch;
    return;
  }
  const int kpart = (kch + p.ksplit - 1) / p.ksplit;
  kc0 = (int)(g % p.ksplit) * kpart;
  nk = kch - kc0 < kpart ? kch - kc0 : kpart;
}

__device__ __forceinline__ int2 plan_entry(const StreamParams& p, const int2* plan, long long g,
                                           int nrb) {
  if (p.sorted_ids == nullptr) return make_int2(0, 0);
  return __ldg(plan + g / nrb);
}

template <int kNMax>
__device__ __forceinline__ Item make_item(const StreamParams& p, int2 pe, long long g, int nrb,
                                          int kch) {
  Item it;
  item_k_range(p, g, kch, it.kc0, it.nk);
  if (p.sorted_ids == nullptr) {
    const long long gb = p.ksplit > 1 ? g / p.ksplit : g;
    const long long sb = gb / nrb;
    it.rb = (int)(gb - sb * nrb);
    it.e = 0;
    it.slot0 = sb * kNMax;
    const long long left = (long long)p.dense_m - it.slot0;
    it.rows = left < kNMax ? (int)left : kNMax;
  } else {
    const long long sb = g / nrb;
    it.rb = (int)(g - sb * nrb);
    it.e = pe.y >> 9;
    it.slot0 = pe.x;
    it.rows = pe.y & 511;
  }
  return it;
}

// Scale rows of an item's weight block: the gate row for the top 8 rows of
// every 16 and the up row for the bottom 8 in a gated bank.
__device__ __forceinline__ void scale_rows(const StreamParams& p, const Item& it, int kch,
                                           const float*& top, const float*& bot) {
  const int nsr = p.N / 128;
  if (p.gated) {
    top = p.wscale + ((long long)it.e * nsr + it.rb / 2) * kch;
    bot = p.wscale + ((long long)it.e * nsr + p.N / 2 / 128 + it.rb / 2) * kch;
  } else {
    top = p.wscale + ((long long)it.e * nsr + it.rb) * kch;
    bot = top;
  }
}

// Route id of slot n of the item (-1 past the item), loaded without use.
__device__ __forceinline__ int slot_id(const StreamParams& p, const Item& it, int n) {
  if (n >= it.rows) return -1;
  if (p.sorted_ids == nullptr) return (int)(it.slot0 + n);
  return __ldg(p.sorted_ids + it.slot0 + n);
}

// Slot id -> activation row, or -1 for padding / an out-of-range route.
__device__ __forceinline__ long long id_row(const StreamParams& p, int id) {
  if (p.sorted_ids == nullptr) return id;
  if (id < 0 || id >= p.num_routes) return -1;
  const long long row = id / p.top_k;
  if (row >= p.x_rows) {
    if (p.status) atomicOr(p.status, kDevBadRoute);
    return -1;
  }
  return row;
}

__device__ __forceinline__ uint32_t f16x2_splat(float v) {
  const uint16_t b = __half_as_ushort(__float2half_rn(v));
  return (uint32_t)b | ((uint32_t)b << 16);
}

template <typename T, int M>
__device__ __forceinline__ T pick(const T (&v)[M], int g) {
  T r = v[0];
#pragma unroll
  for (int i = 1; i < M; ++i) r = g == i ? v[i] : r;
  return r;
}

// kFp4: NVFP4 units (9 KiB: codes, then per-16-K E4M3 scales; weights
// e2m1 * fp16_rne(e4m3 * global)), else block-FP8 units (16 KiB).
template <bool kFp4, int CFG>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const StreamParams p, const int2* __restrict__ plan,
                   const int* __restrict__ plan_count, const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x) {
  using C = TcCfg<CFG>;
  using Ctl = CtlT<C::kRawStages, C::kAStages, C::kBStages>;
  constexpr int kNMax = C::kNMax;
  constexpr int kAStages = C::kAStages;
  constexpr int kBStages = C::kBStages;
  constexpr int kSub = C::kSub;
  constexpr int kLoadPasses = C::kLoadPasses;
  constexpr int kRawStages = C::kRawStages;
  constexpr uint32_t kSubTile = C::kSubTile;
  constexpr uint32_t kBStage = C::kBStage;
  constexpr uint32_t kStageCols = C::kStageCols;
  constexpr uint32_t kOffB = C::kOffB;
  constexpr uint32_t kOffRaw = C::kOffRaw;
  constexpr uint32_t kOffCtl = C::kOffCtl;
  constexpr uint32_t kAccCols = C::kAccCols;
  constexpr uint32_t kACol0 = C::kACol0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + kOffCtl);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nrb = p.N / 128;
  const int kch = p.K / 128;
  const bool dense = p.sorted_ids == nullptr;

  if (tid == 0) {
    // bfull: every gather thread (cp.async arrivals) or the one thread that
    // issues the stage's TMA tiles.
    const uint32_t b_arrivals = p.xs != nullptr ? 1u : (uint32_t)kLoadThreads;
    for (int s = 0; s < kAStages; ++s) mbar_init(&ctl->full[s], C::kDqHalves ? 8 : 4);
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&ctl->empty[s], 1);
      mbar_init(&ctl->bfull[s], b_arrivals);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&ctl->acc_full[s], 1);
      mbar_init(&ctl->acc_empty[s], 4);
    }
    for (int s = 0; s < kRawStages; ++s) {
      mbar_init(&ctl->raw_full[s], 1);
      mbar_init(&ctl->raw_empty[s], C::kDqHalves ? 8 : 4);
    }
    mbar_init(&ctl->done, 1);
    for (int i = 0; i < kInfoSlots; ++i) ctl->info[i] = 0;
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMeta) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&ctl->tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(&ctl->tmem);

  griddep_wait();
  if (tid == 0) griddep_launch_dependents();

  long long items;
  if (dense) {
    items = (long long)((p.dense_m + kNMax - 1) / kNMax) * nrb * (p.ksplit > 1 ? p.ksplit : 1);
  } else {
    items = (long long)__ldg(plan_count) * nrb;
  }
  // This CTA's items: g = blockIdx.x + j * gridDim.x, j < my_items.
  const long long my_items =
      items > (long long)blockIdx.x ? (items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const long long g0 = blockIdx.x, gs = gridDim.x;

  if (warp == kWarpMeta) {
    // ------------------------------------------------------------- weights
    long long u = 0;         // units issued by this CTA (lane 0)
    RingPos<kRawStages> rp;  // the next raw slot (lane 0)
    bool ok = true;
    int2 pe_next = my_items > 0 ? plan_entry(p, plan, g0, nrb) : make_int2(0, 0);
    for (long long j = 0; j < my_items && ok; ++j) {
      const Item it = make_item<kNMax>(p, pe_next, g0 + j * gs, nrb, kch);
      if (j + 1 < my_items) pe_next = plan_entry(p, plan, g0 + (j + 1) * gs, nrb);
      const float* stop = nullptr;
      const float* sbot = nullptr;
      int et = 0, eb = 0;
      float ct = 0.f, cb = 0.f, nt = 0.f, nb = 0.f, gsc = 0.f;
      if constexpr (kFp4) {
        gsc = __ldg(p.gscale + it.e);
      } else {
        scale_rows(p, it, kch, stop, sbot);
        // Lane l holds the scales of units 32c + l (window c); the row maxima
        // give the item's exponents. Runs right after the previous item's
        // last unit was issued, while the raw ring is full.
        float mt = 0.f, mb = 0.f;
        for (int k = lane; k < kch; k += 32) {
          mt = fmaxf(mt, fabsf(__ldg(stop + k)));
          mb = fmaxf(mb, fabsf(__ldg(sbot + k)));
        }
        et = max_exponent(warp_max(mt));
        eb = max_exponent(warp_max(mb));
        // Scale windows from the item's first unit on.
        ct = ldg_or0(stop, it.kc0 + lane, kch);
        cb = ldg_or0(sbot, it.kc0 + lane, kch);
        nt = ldg_or0(stop, it.kc0 + 32 + lane, kch);
        nb = ldg_or0(sbot, it.kc0 + 32 + lane, kch);
      }
      // The unit's rows of 128 bytes in the weight tensor map.
      constexpr int kUnitRows = (kFp4 ? kFp4UnitBytes : kFp8UnitBytes) / 128;
      const int row0 = (int)(((long long)it.e * nrb + it.rb) * kch * kUnitRows);
      // Windows of 32 units: every lane computes its unit's multipliers, then
      // lane 0 alone waits for raw slots and issues the copies.
      for (int w0 = 0; w0 < it.nk && ok; w0 += 32) {
        if (!kFp4 && w0 > 0) {
          ct = nt;
          cb = nb;
          nt = ldg_or0(stop, it.kc0 + w0 + 32 + lane, kch);
          nb = ldg_or0(sbot, it.kc0 + w0 + 32 + lane, kch);
        }
        if constexpr (kFp4)
          ctl->wmult[lane] = make_uint2(__float_as_uint(gsc), 0u);
        else
          ctl->wmult[lane] = make_uint2(mult_f16x2(ct, et), mult_f16x2(cb, eb));
        __syncwarp();
        const int nw = it.nk - w0 < 32 ? it.nk - w0 : 32;
        int good = 1;
        if (lane == 0) {
          for (int i = 0; i < nw; ++i) {
            if (!wait_bar_lazy(&ctl->raw_empty[rp.idx], rp.phase ^ 1u, ctl, p.status)) {
              good = 0;
              break;
            }
            ctl->raw_mult[rp.idx] = ctl->wmult[i];
            mbar_arrive_expect_tx(&ctl->raw_full[rp.idx], (uint32_t)(kUnitRows * 128));
            tma_load_2d(smem + kOffRaw + rp.idx * kUnitBytes, &tmap_w, 0,
                        row0 + (it.kc0 + w0 + i) * kUnitRows, &ctl->raw_full[rp.idx]);
            rp.advance();
            ++u;
          }
        }
        // Also holds the other lanes until lane 0 has read the window.
        if (!__shfl_sync(0xffffffffu, good, 0)) ok = false;
      }
    }
    // Copies still in flight land before the CTA exits (only after an abort).
    if (lane == 0 && !ok) {
      for (long long v = u > kRawStages ? u - kRawStages : 0; v < u; ++v)
        mbar_wait(&ctl->raw_full[v % kRawStages], (uint32_t)((v / kRawStages) & 1), nullptr);
    }
  } else if (warp == kWarpMma) {
    // ----------------------------------------------------------------- MMA
    // Lane 0 alone runs the loop: per stage its two barriers (`bfull`: B
    // landed, `full`: A written), kSub x 4 MMAs and one commit that releases
    // the stage. A barrier poll whose result feeds a branch costs ~190 clocks
    // (measured on B200), so the next stage's barriers are tested (test_wait,
    // which never suspends) before this stage's MMAs are issued and the
    // results are read at the next stage; when they were not yet complete the
    // thread polls both together.
    // A stage's B descriptor differs from stage 0's only in the start-address
    // field: + the stage's and the sub-tile's offsets, + 2 (32 bytes) per K=16
    // MMA.
    if (lane == 0) {
      const uint32_t dhi = (uint32_t)(smem_desc_sw128(0) >> 32);
      const uint32_t b_lo0 = (uint32_t)smem_desc_sw128(smem_u32(smem + kOffB));
      RingPos<kAStages> sa;  // A slot / `full`
      RingPos<kBStages> sb;  // B slot / `bfull` / `empty`
      bool ok = true;
      bool ready = false;  // the current stage's barriers, tested ahead
      for (long long j = 0; j < my_items && ok; ++j) {
        const int buf = (int)(j & 1);
        ok = wait_bar(&ctl->acc_empty[buf], (uint32_t)(((j >> 1) & 1) ^ 1), ctl, p.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t dcol = tmem + (uint32_t)buf * kAccCols;
        uint32_t idesc = 0;
        int kc0, nk;
        item_k_range(p, g0 + j * gs, kch, kc0, nk);
        const int nst = nk * (2 / kSub);
        for (int ts = 0; ts < nst; ++ts) {
          if (!ready) {
            ok = wait_bar2(&ctl->bfull[sb.idx], sb.phase, &ctl->full[sa.idx], sa.phase, ctl,
                           p.status);
            if (!ok) break;
          }
          tc_fence_after();
          if (ts == 0) {
            const int v = *reinterpret_cast<volatile int*>(&ctl->info[j % kInfoSlots]);
            int n = (v >> 9) == (int)(j & 0x3fffff) ? (v & 511) : kNMax;
            n = n < 16 ? 16 : (n > kNMax ? kNMax : n);
            idesc = instr_desc_f16(n);
          }
          RingPos<kAStages> na_pos = sa;
          RingPos<kBStages> nb_pos = sb;
          na_pos.advance();
          nb_pos.advance();
          const bool nb = mbar_test_wait(&ctl->bfull[nb_pos.idx], nb_pos.phase);
          const bool na = mbar_test_wait(&ctl->full[na_pos.idx], na_pos.phase);
          if (!p.loads_only) {
            const uint32_t acol = tmem + kACol0 + sa.idx * kStageCols;
            const uint32_t blo = b_lo0 + sb.idx * (kBStage >> 4);
#pragma unroll
            for (int q = 0; q < kSub; ++q)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_ts(dcol, acol + q * kSubCols + 8u * kk,
                       ((uint64_t)dhi << 32) | (blo + q * (kSubTile >> 4) + 2u * kk), idesc,
                       (ts > 0 || q > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&ctl->empty[sb.idx]);
          sa = na_pos;
          sb = nb_pos;
          ready = nb && na;
        }
        if (ok) mma_commit(&ctl->acc_full[buf]);
      }
      // Every issued MMA has completed before tensor memory is released.
      mma_commit(&ctl->done);
      mbar_wait(&ctl->done, 0u, nullptr);
    }
    __syncwarp();
  } else if (warp < kWarpDeq && p.xs != nullptr) {
    // ------------------------------------- B (activations) by 2-D TMA tiles
    // The operand is already in slot order: a 64-K sub-tile is ceil(rows / 64)
    // boxes of 64 rows x 64 K, landing in the 128-byte-swizzled K-major layout
    // the MMA descriptor reads. Lane 0 of warp 2 issues; warp 3 has nothing to
    // do.
    if (warp == kWarpLoad) {
      long long t = 0;  // stages issued (lane 0)
      RingPos<kBStages> sp;
      bool ok = true;
      for (long long j = 0; j < my_items && ok; ++j) {
        const long long g = g0 + j * gs;
        const Item it = make_item<kNMax>(p, plan_entry(p, plan, g, nrb), g, nrb, kch);
        // The MMA's N: slots up to the item's last valid route.
        int nmax = 0;
  #pragma unroll
        for (int q = 0; q < kNMax / 32; ++q) {
          const int n = q * 32 + lane;
          if (id_row(p, slot_id(p, it, n)) >= 0) nmax = n + 1;
        }
        nmax = (int)__reduce_max_sync(0xffffffffu, (unsigned)nmax);
        int good = 1;
        if (lane == 0) {
          atomicMax(&ctl->info[j % kInfoSlots], (int)(((j & 0x3fffff) << 9) | ((nmax + 15) & ~15)));
          const int nbox = nmax > 64 ? (nmax + 63) / 64 : 1;
          int kc0, nk;
          item_k_range(p, g, kch, kc0, nk);
          const int nst = nk * (2 / kSub);
          for (int ts = 0; ts < nst; ++ts) {
            if (!wait_bar_lazy(&ctl->empty[sp.idx], sp.phase ^ 1u, ctl, p.status)) {
              good = 0;
              break;
            }
            uint8_t* B = smem + kOffB + sp.idx * kBStage;
            mbar_arrive_expect_tx(&ctl->bfull[sp.idx], (uint32_t)(nbox * kSub) * 8192u);
  #pragma unroll
            for (int q = 0; q < kSub; ++q) {
              const int kofs = kc0 * 128 + (ts * kSub + q) * 64;
              for (int b = 0; b < nbox; ++b)
                tma_load_2d(B + q * kSubTile + b * 8192, &tmap_x, kofs, (int)(it.slot0 + 64 * b),
                            &ctl->bfull[sp.idx]);
            }
            sp.advance();
            ++t;
          }
        }
        if (!__shfl_sync(0xffffffffu, good, 0)) ok = false;
      }
      // After an abort, tiles still in flight land before the CTA exits.
      if (lane == 0 && !ok) {
        for (long long v = t > kBStages ? t - kBStages : 0; v < t; ++v)
          mbar_wait(&ctl->bfull[v % kBStages], (uint32_t)((v / kBStages) & 1), nullptr);
      }
    }
  } else if (warp < kWarpDeq) {
    // ---------------------------------------------------- B (activations)
    const int ltid = tid - kWarpLoad * 32;  // 0..kLoadThreads-1
    const int rsub = ltid >> 1;             // row within a pass of kLoadThreads/2 rows
    const int cpar = ltid & 1;              // chunk parity
    RingPos<kBStages> sp;
    bool ok = true;
    // Item j's route ids (ids_a), item j+1's plan entry (pe_b): one item ahead.
    int2 pe_a = my_items > 0 ? plan_entry(p, plan, g0, nrb) : make_int2(0, 0);
    int ids_a[kLoadPasses];
    {
      const Item it0 = make_item<kNMax>(p, pe_a, g0, nrb, kch);
#pragma unroll
      for (int q = 0; q < kLoadPasses; ++q)
        ids_a[q] = my_items > 0 ? slot_id(p, it0, q * (kLoadThreads / 2) + rsub) : -1;
    }
    int2 pe_b = my_items > 1 ? plan_entry(p, plan, g0 + gs, nrb) : make_int2(0, 0);
    for (long long j = 0; j < my_items && ok; ++j) {
      const uint16_t* rowp[kLoadPasses];
      int nmax = 0;
#pragma unroll
      for (int q = 0; q < kLoadPasses; ++q) {
        const long long row = id_row(p, ids_a[q]);
        rowp[q] = row >= 0 ? reinterpret_cast<const uint16_t*>(p.x) + row * p.ldx : nullptr;
        if (row >= 0) nmax = q * (kLoadThreads / 2) + rsub + 1;
      }
      nmax = (int)__reduce_max_sync(0xffffffffu, (unsigned)nmax);
      if (lane == 0)
        atomicMax(&ctl->info[j % kInfoSlots], (int)(((j & 0x3fffff) << 9) | ((nmax + 15) & ~15)));
      // Prefetch the next item's route ids and the one after's plan entry.
      int2 pe_c = make_int2(0, 0);
      if (j + 1 < my_items) {
        const Item itn = make_item<kNMax>(p, pe_b, g0 + (j + 1) * gs, nrb, kch);
#pragma unroll
        for (int q = 0; q < kLoadPasses; ++q)
          ids_a[q] = slot_id(p, itn, q * (kLoadThreads / 2) + rsub);
        if (j + 2 < my_items) pe_c = plan_entry(p, plan, g0 + (j + 2) * gs, nrb);
      }
      int kc0, nk;
      item_k_range(p, g0 + j * gs, kch, kc0, nk);
      const int nst = nk * (2 / kSub);
      for (int ts = 0; ts < nst; ++ts) {
        ok = warp_wait(&ctl->empty[sp.idx], sp.phase ^ 1u, ctl, p.status);
        if (!ok) break;
        uint8_t* B = smem + kOffB + sp.idx * kBStage;
#pragma unroll
        for (int sq = 0; sq < kSub; ++sq) {
          const long long kofs = (long long)kc0 * 128 + (ts * kSub + sq) * 64;
#pragma unroll
          for (int q = 0; q < kLoadPasses; ++q) {
            if (rowp[q] != nullptr) {
              const int n = q * (kLoadThreads / 2) + rsub;
#pragma unroll
              for (int c2 = 0; c2 < 4; ++c2) {
                const int c = 2 * c2 + cpar;
                cp_async_16(B + sq * kSubTile + sw128_off(n, c), rowp[q] + kofs + c * 8);
              }
            }
          }
        }
        cp_async_arrive_noinc(&ctl->bfull[sp.idx]);
        sp.advance();
      }
      pe_b = pe_c;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp < kWarpEpi || warp >= kWarpEpi + 4 * C::kEpiGroups) {
    // ------------------------------------------------------------- dequant
    // Lane = weight row m of this warp's tensor-memory quarter. In the
    // streamed unit, row m's 8 K values K = 32*kg4 + 8q + 0..7 are bytes
    // hf*8 .. +7 of 16-byte chunk wp*128 + q*32 + 4*(m&7) + kg4 (wp = m/16,
    // hf = (m/8)&1), i.e. unit byte wp*2048 + q*512 + (m&7)*64 + kg4*16 + hf*8.
    // The TMA copy stores the unit as 128 rows of 128 bytes with 16-byte chunk
    // c of row r at chunk c ^ (r & 7). A 64-K stage h takes kg4 = 2h + kg.
    const int quarter = warp & 3;
    const int dg = warp < kWarpEpi ? 0 : 1;  // dequant group (its units or its halves)
    const int m = quarter * 32 + lane;
    const int hf = (m >> 3) & 1;
    const int r8 = m & 7;
    const int rbase = (m >> 4) * 16 + (r8 >> 1);  // 128-byte row of q = 0
    const uint32_t tlane = (uint32_t)(quarter * 32) << 16;
    RingPos<kRawStages> rr;  // raw unit
    RingPos<kAStages> st;    // A slot / `full` of the current stage
    RingPos<kBStages> ew;    // the commit that frees it: stage t - kAStages
    int taken = 0;           // stages taken (by either group)
    int ug = 0;              // units passed (by either group)
    bool ok = true;
    int nk_left = 0;  // units left in the current item
    // Half h of a unit is sub-tile h % kSub of the current stage: the stage's
    // A slot is taken at sub-tile 0 (once the MMAs of the stage kAStages
    // earlier have completed) and handed to the MMA thread after the last one.
    auto take_stage = [&]() -> bool {
      if (taken >= kAStages) {
        // On the critical path when the A ring is short: polled without pauses.
        if (!__all_sync(0xffffffffu, wait_bar(&ctl->empty[ew.idx], ew.phase, ctl, p.status)))
          return false;
        ew.advance();
      }
      ++taken;
      tc_fence_after();
      return true;
    };
    auto give_stage = [&]() -> bool {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->full[st.idx]);
      st.advance();
      return true;
    };
    for (long long j = 0; ok;) {
      if (nk_left == 0) {
        if (j >= my_items) break;
        int kc0;
        item_k_range(p, g0 + j * gs, kch, kc0, nk_left);
        ++j;
      }
      --nk_left;
      if constexpr (C::kDqGroups > 1 && !C::kDqHalves) {
        // The other group's unit (one stage): only the ring positions move.
        if (ug++ % C::kDqGroups != dg) {
          rr.advance();
          st.advance();
          if (taken >= kAStages) ew.advance();
          ++taken;
          continue;
        }
      }
      ok = warp_wait(&ctl->raw_full[rr.idx], rr.phase, ctl, p.status);
      if (!ok) break;
      const volatile uint32_t* mm = reinterpret_cast<volatile uint32_t*>(&ctl->raw_mult[rr.idx]);
      const uint32_t m2 = hf ? mm[1] : mm[0];  // FP8: this row's multiplier
      const float gsc = __uint_as_float(mm[0]);  // NVFP4: the expert's global scale
      const uint8_t* raw = smem + kOffRaw + rr.idx * kUnitBytes;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (C::kDqHalves && h != dg) continue;  // the other group's half
        const int sq = h % kSub;
        const bool first = C::kDqHalves || sq == 0;        // takes the stage
        const bool last = C::kDqHalves || sq == kSub - 1;  // hands it on
        if (p.loads_only) {
          // pipeline floor: hand the stage on without dequantizing into it
          if (first && !(ok = take_stage())) break;
          if (last && !(ok = give_stage())) break;
          continue;
        }
        uint32_t v[32];
        if constexpr (kFp4) {
          // NVFP4: row m's codes for K 32c .. +31 are bytes hf*16 .. +15 of
          // the 32-byte lane record (w = m/16, lane 4*(m&7) + c), i.e. 128-byte
          // row 8w + (m&7), chunk 2c + hf; its two group scales are bytes
          // 2hf, 2hf+1 of the record's 4 scale bytes, in row 64 + w at byte
          // 16*(m&7) + 4c. Half h takes c = 2h, 2h + 1.
          const int wr = m >> 4, g = m & 7;
          const int row = 8 * wr + g;
          uint4 code[2];
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int chunk = ((2 * (2 * h + cc) + hf) ^ g) & 7;
            code[cc] = *reinterpret_cast<const uint4*>(raw + row * 128 + chunk * 16);
          }
          const uint2 sc = *reinterpret_cast<const uint2*>(
              raw + (64 + wr) * 128 + ((g ^ wr) & 7) * 16 + 8 * h);
          if (first && !(ok = take_stage())) break;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            // Scale bytes of record c: top g0, top g1, bottom g0, bottom g1.
            const uint32_t sw = cc ? sc.y : sc.x;
            const uint32_t sp = e4m3x2_to_f16x2((uint16_t)(hf ? (sw >> 16) : (sw & 0xffffu)));
            const __half2 sh = *reinterpret_cast<const __half2*>(&sp);
            const uint32_t s0 = f16x2_splat(__low2float(sh) * gsc);
            const uint32_t s1 = f16x2_splat(__high2float(sh) * gsc);
            const uint32_t cw[4] = {code[cc].x, code[cc].y, code[cc].z, code[cc].w};
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
              uint32_t f[4];
              e2m1x8_to_f16x2x4(cw[wd], f);
#pragma unroll
              for (int i = 0; i < 4; ++i) v[16 * cc + 4 * wd + i] = hmul2_u32(f[i], wd < 2 ? s0 : s1);
            }
          }
        } else {
          uint2 r[8];  // [kg][q]
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int kg4 = 2 * h + (i >> 2), q = i & 3;
            const int row = rbase + 4 * q;
            const int chunk = (((r8 & 1) * 4 + kg4) ^ row) & 7;
            r[i] = *reinterpret_cast<const uint2*>(raw + row * 128 + chunk * 16 + hf * 8);
          }
          if (first && !(ok = take_stage())) break;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            uint32_t* o = v + 16 * (i >> 2) + 4 * (i & 3);
            o[0] = hmul2_u32(e4m3x2_to_f16x2((uint16_t)(r[i].x & 0xffffu)), m2);
            o[1] = hmul2_u32(e4m3x2_to_f16x2((uint16_t)(r[i].x >> 16)), m2);
            o[2] = hmul2_u32(e4m3x2_to_f16x2((uint16_t)(r[i].y & 0xffffu)), m2);
            o[3] = hmul2_u32(e4m3x2_to_f16x2((uint16_t)(r[i].y >> 16)), m2);
          }
        }
        tmem_st32(tmem + tlane + kACol0 + st.idx * kStageCols + (uint32_t)sq * kSubCols, v);
        if (last && !(ok = give_stage())) break;
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->raw_empty[rr.idx]);
      rr.advance();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Item j's accumulator is TMEM buffer j & 1. With two groups warps 8-11
    // take the even items and warps 12-15 the odd ones (each has two items'
    // main-loop time for one); with one group warps 8-11 take them all.
    const int quarter = warp & 3;  // tensor-memory lanes 32*quarter..+31
    const int eg = (warp - kWarpEpi) >> 2;
    const int m = quarter * 32 + lane;  // weight row within the block
    const bool top = (m & 15) < 8;
    const bool fused = p.gated && p.fuse_act;
    const bool lane_stores = !fused || top;
    const uint32_t tlanes = tmem + ((uint32_t)(quarter * 32) << 16);
    constexpr int kGroups = kNMax / 32;
    for (long long j = eg; j < my_items; j += C::kEpiGroups) {
      const int ab = (int)(j & 1);
      const uint32_t tbase = tlanes + (uint32_t)ab * kAccCols;
      const long long g = g0 + j * gs;
      const Item it = make_item<kNMax>(p, plan_entry(p, plan, g, nrb), g, nrb, kch);
      float fself = 1.f;  // this lane's row: 2^E (FP8), 1 (NVFP4)
      if constexpr (!kFp4) {
        const float* stop;
        const float* sbot;
        scale_rows(p, it, kch, stop, sbot);
        float mt = 0.f, mb = 0.f;
        for (int k = lane; k < kch; k += 32) {
          mt = fmaxf(mt, fabsf(__ldg(stop + k)));
          mb = fmaxf(mb, fabsf(__ldg(sbot + k)));
        }
        const int et = max_exponent(warp_max(mt));
        const int eb = max_exponent(warp_max(mb));
        fself = pow2f(top ? et : eb);
      }
      long long mycol;
      if (p.gated) {
        const long long jj = (long long)it.rb * 64 + (m >> 4) * 8 + (m & 7);
        mycol = top ? jj : jj + p.N / 2;
      } else {
        mycol = (long long)it.rb * 128 + m;
      }
      // Output row and router weight of column 32g + lane.
      int orow[kGroups];
      float wr[kGroups];
#pragma unroll
      for (int gg = 0; gg < kGroups; ++gg) {
        const int id = slot_id(p, it, gg * 32 + lane);
        orow[gg] = -1;
        wr[gg] = 1.f;
        if (dense) {
          orow[gg] = id;
        } else if (id >= 0 && id < p.num_routes && id / p.top_k < p.x_rows) {
          orow[gg] = p.out_by_slot ? (int)(it.slot0 + gg * 32 + lane) : id;
          if (p.mul_w) wr[gg] = __ldg(p.topk_w + id);
        }
      }
      if (!warp_wait(&ctl->acc_full[ab], (uint32_t)((j >> 1) & 1), ctl, p.status, 4 * B200_TC_PAUSE_NS))
        break;
      tc_fence_after();
      const int ngroups = p.loads_only ? 0 : (it.rows + 31) >> 5;
      for (int gg = 0; gg < ngroups; ++gg) {
        const int og = pick(orow, gg);
        const float wg = pick(wr, gg);
        const unsigned vmask = __ballot_sync(0xffffffffu, og >= 0);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (((vmask >> (16 * hh)) & 0xffffu) == 0u) continue;
          float v[16];
          tmem_ld16(tbase + (uint32_t)(gg * 32 + hh * 16), v);
          // Column metadata first (independent shuffles), then branch-free
          // math and predicated stores.
          int orw[16];
          float wv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            orw[i] = __shfl_sync(0xffffffffu, og, hh * 16 + i);
            wv[i] = __shfl_sync(0xffffffffu, wg, hh * 16 + i);
          }
          // Each lane scales its own row; a gated top lane then takes the
          // (scaled) up value of the row 8 lanes below.
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] *= fself;
          if (p.ksplit > 1) {
            // K split (dense): add this part's sums; the finishing kernel
            // applies the activation. Gate and up rows land in columns j and
            // N/2 + j of the [rows][N] fp32 buffer.
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (orw[i] >= 0) atomicAdd(p.ws + (long long)orw[i] * p.N + mycol, v[i]);
            continue;
          }
          if (fused) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float up = __shfl_down_sync(0xffffffffu, v[i], 8);
              v[i] = silu_f32(v[i]) * up;
            }
          }
          if (p.out_rows != nullptr) {
            // Expert-parallel owner: each route's row is in its source
            // rank's combine buffer (a peer address).
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (lane_stores && orw[i] >= 0) {
                uint16_t* o = reinterpret_cast<uint16_t*>(__ldg(p.out_rows + orw[i]));
                const float x = v[i] * wv[i];
                o[mycol] = p.out_f16 ? __half_as_ushort(__float2half_rn(x))
                                     : __bfloat16_as_ushort(__float2bfloat16_rn(x));
              }
          } else if (p.out_f16) {
            __half* o = reinterpret_cast<__half*>(p.out);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (lane_stores && orw[i] >= 0)
                o[(long long)orw[i] * p.ldo + mycol] = __float2half_rn(v[i] * wv[i]);
          } else {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (lane_stores && orw[i] >= 0)
                o[(long long)orw[i] * p.ldo + mycol] = __float2bfloat16_rn(v[i] * wv[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->acc_empty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMeta) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------------------ plan
// Block-wide inclusive max / exclusive sum (blockDim.x == 1024).
__device__ __forceinline__ int block_incl_max(int v, int* sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = max(v, x);
  }
  if (lane == 31) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    int x = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x = max(x, y);
    }
    sh[lane] = x;
  }
  __syncthreads();
  if (w > 0) v = max(v, sh[w - 1]);
  __syncthreads();
  return v;
}

__device__ __forceinline__ int block_excl_sum(int v, int* sh, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[w] = x;
  __syncthreads();
  if (w == 0) {
    int s = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    sh[lane] = s;
  }
  __syncthreads();
  total = sh[31];
  const int excl = x - v + (w > 0 ? sh[w - 1] : 0);
  __syncthreads();
  return excl;
}

// Items of the grouped GEMM. The route slots are cut into virtual blocks of
// `vblock` (the moe_align block, or half of it when the block exceeds the
// item width);
// every run of consecutive virtual blocks of the same (valid) expert is cut
// into items of at most nb_max of them.
// plan[i] = {first slot, expert << 9 | slots}; *count = number of items.
__global__ void __launch_bounds__(1024) tc_plan_kernel(const int* __restrict__ expert_ids,
                                                       const int* __restrict__ ntpp, int block_m,
                                                       int vblock, long long max_groups, int E,
                                                       int nb_max, int2* __restrict__ plan,
                                                       int* __restrict__ count, int cap) {
  __shared__ int sh[32];
  __shared__ int carry_sh;
  griddep_wait();
  long long groups = ntpp[0] / block_m;
  if (groups < 0) groups = 0;
  if (groups > max_groups) groups = max_groups;
  const int vpb = block_m / vblock;
  long long vgroups = groups * vpb;
  if (vgroups > cap) vgroups = cap;
  int carry = -1, total = 0;
  for (long long v0 = 0; v0 < vgroups; v0 += blockDim.x) {
    const int v = (int)(v0 + threadIdx.x);
    const bool in = v < vgroups;
    const int e = in ? expert_ids[v / vpb] : -1;
    const bool valid = in && e >= 0 && e < E;
    const int pe = (in && v > 0) ? expert_ids[(v - 1) / vpb] : -1;
    const bool run_start = valid && (v == 0 || pe != e);
    int rs = block_incl_max(run_start ? v : -1, sh);
    rs = max(rs, carry);
    const bool item = valid && ((v - rs) % nb_max) == 0;
    int nb = 0;
    if (item) {
      nb = 1;
      for (int k = 1; k < nb_max; ++k) {
        if (v + k >= vgroups || expert_ids[(v + k) / vpb] != e) break;
        ++nb;
      }
    }
    int tile_total = 0;
    const int idx = total + block_excl_sum(item ? 1 : 0, sh, tile_total);
    if (item && idx < cap) plan[idx] = make_int2(v * vblock, (e << 9) | (nb * vblock));
    total += tile_total;
    // The last thread's run start carries into the next tile.
    if (threadIdx.x == blockDim.x - 1) carry_sh = rs;
    __syncthreads();
    carry = carry_sh;
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = total < cap ? total : cap;
  griddep_launch_dependents();
}

__global__ void __launch_bounds__(256) tc_split_finish_kernel(const StreamParams p) {
  griddep_wait();
  const int cols = p.fuse_act ? p.N / 2 : p.N;
  const long long total = (long long)p.dense_m * cols;
  for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
       id += (long long)gridDim.x * blockDim.x) {
    const long long r = id / cols;
    const int c = (int)(id - r * cols);
    float* row = p.ws + r * p.N;
    float v = row[c];
    row[c] = 0.f;
    if (p.fuse_act) {
      const float up = row[p.N / 2 + c];
      row[p.N / 2 + c] = 0.f;
      v = silu_f32(v) * up;
    }
    if (p.out_f16)
      reinterpret_cast<__half*>(p.out)[r * p.ldo + c] = __float2half_rn(v);
    else
      reinterpret_cast<__nv_bfloat16*>(p.out)[r * p.ldo + c] = __float2bfloat16_rn(v);
  }
  griddep_launch_dependents();
}

}  // namespace

int64_t tc_plan_bytes(int cap) { return 256 + (int64_t)cap * (int64_t)sizeof(int2); }

bool tc_gemm_supported(int block) {
  return block == 16 || block == 32 || block == 64 || block == 128 || block == 256;
}

int tc_plan_slots_per_group(int block) { return block > kNMaxWide ? 2 : 1; }

int tc_narrow_slots() { return kNMaxNarrow; }

cudaError_t launch_tc_plan_slots(const StreamParams& p, void* plan_buf, int cap, int max_slots,
                                cudaStream_t stream) {
  int* count = reinterpret_cast<int*>(plan_buf);
  int2* plan = reinterpret_cast<int2*>(reinterpret_cast<uint8_t*>(plan_buf) + 256);
  const int vblock = p.block_m > max_slots ? p.block_m / 2 : p.block_m;
  if (vblock > max_slots || vblock <= 0) return cudaErrorInvalidValue;
  return launch_pdl(tc_plan_kernel, dim3(1), dim3(1024), 0, stream, p.expert_ids, p.ntpp,
                    p.block_m, vblock, p.max_groups, p.E, max_slots / vblock, plan, count, cap);
}

cudaError_t launch_tc_plan(const StreamParams& p, void* plan_buf, int cap, cudaStream_t stream) {
  return launch_tc_plan_slots(p, plan_buf, cap, kNMaxWide, stream);
}

cudaError_t launch_tc_split_finish(const StreamParams& p, cudaStream_t stream) {
  const long long work = (long long)p.dense_m * (p.fuse_act ? p.N / 2 : p.N);
  long long blocks = (work + 255) / 256;
  const long long cap = (long long)device_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return launch_pdl(tc_split_finish_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, p);
}


// Operands are f16: FP8 weights dequantized as f16(e4m3 * m) with the
// scale's power of two applied to the fp32 accumulator, NVFP4 weights as
// e2m1 * fp16_rne(e4m3 * global); bf16 activations are converted by the
// caller. `plan_buf` holds launch_tc_plan's output (moe mode).
namespace {

template <bool kFp4, int CFG>
cudaError_t launch_tc_config(const StreamParams& p, const int2* plan, const int* count, int grid,
                             const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                             cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  constexpr size_t smem = TcCfg<CFG>::kTcSmem;
  if (!configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(tc_gemm_kernel<kFp4, CFG>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    configured[dev] = true;
  }
  return launch_pdl(tc_gemm_kernel<kFp4, CFG>, dim3(grid), dim3(kTcThreads), smem, stream, p,
                    plan, count, tmap_w, tmap_x);
}

}  // namespace

cudaError_t launch_tc_gemm(int quant, const StreamParams& p, const void* plan_buf, int grid,
                           cudaStream_t stream, bool narrow) {
  const bool fp4 = quant == kQuantNvfp4;
  // Weights: every unit is rows of 128 bytes (FP8 128 rows, NVFP4 72), one
  // box per unit.
  const unsigned unit_rows = (fp4 ? kFp4UnitBytes : kFp8UnitBytes) / 128;
  const long long experts = p.sorted_ids == nullptr ? 1 : p.E;
  const unsigned long long wrows =
      (unsigned long long)experts * (p.N / 128) * (p.K / 128) * unit_rows;
  if (wrows >= (1ull << 31)) return cudaErrorInvalidValue;
  CUtensorMap tmap_w;
  if (!make_map(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.wq, 128, wrows, 128, 128, unit_rows,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
    return cudaErrorInvalidValue;
  // Slot-ordered activations: boxes of 64 K (128 bytes) x 64 rows; rows past
  // xs_rows read as zero.
  CUtensorMap tmap_x;
  memset(&tmap_x, 0, sizeof(tmap_x));
  if (p.xs != nullptr) {
    if (p.xs_rows <= 0 || p.xs_rows >= (1ll << 31) || p.ldx % 8 != 0 || p.ldx < p.K ||
        (reinterpret_cast<uintptr_t>(p.xs) & 15u) != 0)
      return cudaErrorInvalidValue;
    if (!make_map(&tmap_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.xs, (unsigned long long)p.K,
                  (unsigned long long)p.xs_rows, (unsigned long long)p.ldx * 2, 64, 64,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
      return cudaErrorInvalidValue;
  }
  const int* count = reinterpret_cast<const int*>(plan_buf);
  const int2* plan = reinterpret_cast<const int2*>(reinterpret_cast<const uint8_t*>(plan_buf) + 256);
  // Weight units per item (per K part when K is split).
  const int kch = p.K / 128;
  const int item_units =
      p.sorted_ids == nullptr && p.ksplit > 1 ? (kch + p.ksplit - 1) / p.ksplit : kch;
  const int cfg = narrow ? kTcNarrow : (item_units >= 32 ? kTcWideLong : kTcWideShort);
  if (fp4) {
    if (cfg == kTcNarrow)
      return launch_tc_config<true, kTcNarrow>(p, plan, count, grid, tmap_w, tmap_x, stream);
    if (cfg == kTcWideLong)
      return launch_tc_config<true, kTcWideLong>(p, plan, count, grid, tmap_w, tmap_x, stream);
    return launch_tc_config<true, kTcWideShort>(p, plan, count, grid, tmap_w, tmap_x, stream);
  }
  if (cfg == kTcNarrow)
    return launch_tc_config<false, kTcNarrow>(p, plan, count, grid, tmap_w, tmap_x, stream);
  if (cfg == kTcWideLong)
    return launch_tc_config<false, kTcWideLong>(p, plan, count, grid, tmap_w, tmap_x, stream);
  return launch_tc_config<false, kTcWideShort>(p, plan, count, grid, tmap_w, tmap_x, stream);
}

}  // namespace b200
