// Internal launch interface shared by the .cu files of libb200moe. Nothing in
// here crosses the C ABI; include/b200moe.h is the public surface.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace b200 {

// Weight-streaming GEMM: Y[rows, N] = X[rows, K] * dequant(W[N, K])^T, with
// rows either a dense batch or route slots grouped by expert (the
// moe_align_block_size output).
enum StreamQuant : int { kQuantFp8Block = 0, kQuantNvfp4 = 1 };

struct StreamParams {
  const uint8_t* wq;     // prepacked weight units (see prepack.cu)
  const float* wscale;   // FP8: [E][N/128][K/128] fp32 block scales (logical rows)
  const float* gscale;   // NVFP4: [E] fp32 global scale
  const __half* x;       // activations, f16, rows of ldx elements
  long long ldx;
  // tcgen05 GEMM only: activations already in slot order (row s = route slot
  // s of the moe_align output, or dense row s), f16 rows of ldx elements;
  // B tiles then come by 2-D TMA instead of the per-route gather.
  const __half* xs;
  long long xs_rows;
  int out_by_slot;       // tcgen05 moe mode: output row = route slot, not route id
  long long x_rows;      // number of activation rows (route rows are checked against it)
  const int* sorted_ids; // nullptr: dense mode
  const int* expert_ids;
  const int* ntpp;       // num_tokens_post_padded (device)
  int block_m;           // route slots per group (moe mode); == 8 * NT
  long long max_groups;  // moe mode: groups readable from sorted_ids / expert_ids
  int top_k;             // activation row = route / top_k
  int num_routes;        // route ids >= num_routes are padding
  const float* topk_w;   // one weight per route (mul_w)
  int dense_m;           // dense mode: number of rows
  int E, N, K;           // N = weight rows (2I for a gated gate/up bank)
  int gated;             // bank rows interleaved gate/up
  int fuse_act;          // gated: write silu(gate)*up [.., N/2]; else gate | up halves
  int mul_w;             // multiply each route's row by topk_w[route]
  void* out;
  long long ldo;
  // Optional: output row of route r at address out_rows[r] (expert-parallel
  // owners store straight into the source rank's buffer); nullptr: out + r*ldo.
  const unsigned long long* out_rows;
  int out_f16;           // 1: f16 output, 0: bf16
  int ksplit;            // tcgen05 dense mode: K ranges per item (1 = none); >1 sums into ws
  float* ws;             // split-pair partial sums, kWsSlotFloats per grid slot, zeroed
  int* ws_cnt;           // one arrival counter per grid slot, zeroed
  int* status;           // device error bits
  // Loads only (pipeline floor, for measurement): every copy and barrier
  // hand-off of the call runs, the conversions, MMAs and stores do not.
  int loads_only;
};

constexpr int kWsSlotFloats = 128 * 64;

// Stream GEMM tiling constants (also used by the host for sizing).
constexpr int kUnitRows = 128;
constexpr int kUnitK = 128;
constexpr uint32_t kFp8UnitBytes = kUnitRows * kUnitK;                       // 16 KiB
constexpr uint32_t kFp4UnitBytes = kUnitRows * kUnitK / 2 + kUnitRows * 8;   // 9 KiB

// solo: one CTA per SM with a deeper stage ring, for calls whose (group, row
// block) pairs each fit one CTA (grid <= SMs; nt <= 2, else ignored).
cudaError_t launch_stream_gemm(int quant, int nt, const StreamParams& p, int grid,
                               cudaStream_t stream, bool solo = false);
int stream_gemm_whole_pair_max_stages();
int stream_gemm_stage_units(int quant);
int stream_gemm_ctas_per_sm(int nt);

// tcgen05 grouped GEMM (FP8 or NVFP4 weights, f16 activations). Moe mode first runs
// launch_tc_plan (items = runs of same-expert groups, up to 256 route slots
// each) into a buffer of tc_plan_bytes(cap); groups beyond `cap` are not
// planned, so callers pick the stream GEMM when max_groups > cap.
bool tc_gemm_supported(int block);  // block_m in {16, 32, 64, 128, 256}
int tc_plan_slots_per_group(int block);  // plan entries a moe_align group may need
int64_t tc_plan_bytes(int cap);
cudaError_t launch_tc_plan(const StreamParams& p, void* plan_buf, int cap, cudaStream_t stream);
// narrow: items of at most tc_narrow_slots() route slots / rows with a deeper
// weight ring (few routes per expert, dense M <= 64); the moe plan must then
// come from launch_tc_plan_slots(.., tc_narrow_slots(), ..).
cudaError_t launch_tc_gemm(int quant, const StreamParams& p, const void* plan_buf, int grid,
                           cudaStream_t stream, bool narrow = false);
int tc_narrow_slots();
// The same plan with items of at most max_slots route slots (blocks larger
// than max_slots are cut in half first).
cudaError_t launch_tc_plan_slots(const StreamParams& p, void* plan_buf, int cap, int max_slots,
                                 cudaStream_t stream);
// After a dense tcgen05 GEMM with ksplit > 1: fp32 sums in p.ws -> output
// (SiLU*up for a fused gated bank), and the sums back to zero.
cudaError_t launch_tc_split_finish(const StreamParams& p, cudaStream_t stream);

// moe_align_block_size: stable expert-major counting sort with per-expert
// padding to block_size.
cudaError_t launch_moe_align(const int* topk_ids, long long numel, int num_experts, int block_size,
                             int* sorted_ids, long long sorted_cap, int* expert_ids,
                             long long expert_cap, int* ntpp, cudaStream_t stream);
int moe_align_max_experts();
// Router top-k and single-CTA align in one launch (decode-size batches):
// writes topk_ids / topk_w and the moe_align outputs.
cudaError_t launch_route_align(const void* logits, int dtype, long long tokens, int E, int top_k,
                               int scoring, int renormalize, const float* bias, int* topk_ids,
                               float* topk_w, int bs, int* sorted_ids, long long sorted_cap,
                               int* expert_ids, long long expert_cap, int* ntpp,
                               cudaStream_t stream);
// Multi-CTA variant (same output) for large route counts; `scratch` holds
// moe_align_scratch_ints(numel, E) ints.
long long moe_align_scratch_ints(long long numel, int num_experts);
cudaError_t launch_moe_align_multi(const int* topk_ids, long long numel, int num_experts,
                                   int block_size, int* sorted_ids, long long sorted_cap,
                                   int* expert_ids, long long expert_cap, int* ntpp, int* scratch,
                                   cudaStream_t stream);

// Router top-k (softmax or sigmoid scoring, optional selection bias and
// renormalisation); logits dtype 0 bf16, 1 f16, 2 f32.
int router_max_experts();
// groups > 0: only the topk_group best of `groups` contiguous expert groups
// are selectable (upstream SGLang's grouped top-k).
cudaError_t launch_topk_route(const void* logits, int dtype, long long tokens, int num_experts,
                              int top_k, int scoring, int renormalize, const float* bias,
                              int* topk_ids, float* topk_w, cudaStream_t stream, int groups = 0,
                              int topk_group = 0);

// Elementwise / reduction kernels.
cudaError_t launch_append_shared_route(const int* ids, const float* w, long long tokens,
                                       int top_k, int shared_id, float shared_weight,
                                       int* ids_out, float* w_out, cudaStream_t stream);
cudaError_t launch_bf16_to_f16(const void* in, void* out, long long n, cudaStream_t stream);
// Shared-route append (optional), moe_align and the bf16 -> f16 activation
// conversion (optional: conv_in == nullptr skips it) in one launch; the
// single-CTA align, so for route counts the single-CTA path takes.
cudaError_t launch_moe_prep(const int* topk_ids, const float* topk_w, long long tokens, int top_k,
                            int num_experts, int shared, float shared_w, int* ids_out,
                            float* w_out, int block_size, int* sorted_ids, long long sorted_cap,
                            int* expert_ids, long long expert_cap, int* ntpp, const void* conv_in,
                            void* conv_out, long long conv_elems, cudaStream_t stream);
// out[s, :k] (f16) = x[sorted_ids[s] / top_k, :k] for the valid route slots
// s < min(*ntpp, cap); padding slots are left as they are.
cudaError_t launch_permute_rows(const void* x, int x_f16, long long ldx, long long x_rows,
                                long long k, const int* sorted_ids, const int* ntpp, long long cap,
                                int top_k, long long num_routes, void* out, cudaStream_t stream);
cudaError_t launch_moe_sum_reduce(const void* in, void* out, long long tokens, int top_k,
                                  long long hidden, int f16, float scale, cudaStream_t stream);
cudaError_t launch_moe_combine(const void* routed, int routed_f16, const int* topk_ids,
                               int num_experts, long long tokens, int top_k, long long hidden,
                               float scale, const void* shared_out, int shared_f16, void* out,
                               int out_f16, cudaStream_t stream);

// Load-time re-layouts.
cudaError_t launch_prepack_fp8(const uint8_t* w, long long E, int N, int K, int gated,
                               uint8_t* out, cudaStream_t stream);
cudaError_t launch_prepack_nvfp4(const uint8_t* w, const uint8_t* scales, long long E, int N,
                                 int K, int gated, uint8_t* out, cudaStream_t stream);

int device_sm_count();

// Expert-parallel exchange region: one per rank, identical layout on every
// rank, mapped into every peer (CUDA IPC). Offsets in bytes, each 256-aligned.
constexpr int kEpMaxWorld = 64;
enum EpHdr : int { kEpHdrStatus = 0, kEpHdrEpoch = 1, kEpHdrDispatchDone = 2, kEpHdrCombineDone = 3 };
// A source sends each token's activation row once per owner that holds one
// of its experts (a "row"), with the token's top_k route slots (local expert
// id, -1 for the routes elsewhere, and router weight); the owner returns one
// row per received row, the weighted sum of its experts' outputs.
struct EpLayout {
  long long cap;     // rows one source may send to one owner (max tokens)
  int top_k;
  long long hidden;
  long long off_dflag, off_cflag, off_count, off_cnt_local;  // [kEpMaxWorld] ints each
  long long off_ids, off_w;  // [world * cap * top_k]: local expert id (-1 none), router weight
  long long off_orig;        // [world * cap]: source token of each received row
  long long off_rows;        // [world * cap] u64: destination of each row's summed return (0 = none)
  long long off_recv;        // [world * cap][hidden] f16: received activation rows
  long long off_comb;        // [cap * world][hidden] f16: returned rows, token t of owner o at t*world+o
  long long off_mask;        // [cap] u64: owners each token of the last dispatch went to (source)
  long long total;
};
inline EpLayout ep_layout(int world, long long max_tokens, int top_k, long long hidden) {
  auto up = [](long long v) { return (v + 255) / 256 * 256; };
  EpLayout L;
  L.cap = max_tokens;
  L.top_k = top_k;
  L.hidden = hidden;
  long long o = 256;  // header: status, step counter, two done counters
  L.off_dflag = o; o += up(4 * kEpMaxWorld);
  L.off_cflag = o; o += up(4 * kEpMaxWorld);
  L.off_count = o; o += up(4 * kEpMaxWorld);
  L.off_cnt_local = o; o += up(4 * kEpMaxWorld);
  const long long rows = (long long)world * max_tokens;
  L.off_ids = o; o += up(4 * rows * top_k);
  L.off_w = o; o += up(4 * rows * top_k);
  L.off_orig = o; o += up(4 * rows);
  L.off_rows = o; o += up(8 * rows);
  L.off_recv = o; o += up(2 * rows * hidden);
  L.off_comb = o; o += up(2 * rows * hidden);
  L.off_mask = o; o += up(8 * max_tokens);
  L.total = o;
  return L;
}
int ep_dispatch_chunk(long long tokens);
cudaError_t launch_ep_dispatch(const void* x, int x_f16, long long tokens, long long hidden,
                               const int* ids, const float* w, int top_k, int num_experts,
                               int shared_expert, int experts_per_rank, int rank, int world,
                               const unsigned long long* peers, void* region, const EpLayout& L,
                               cudaStream_t stream);
cudaError_t launch_ep_receive(void* region, const unsigned long long* peers, int rank, int world,
                              const EpLayout& L, int experts_local, cudaStream_t stream);
// Owner, after its down GEMM: row r's return = sum over its valid route slots
// of routed[r * top_k + k] (f16 [world * cap * top_k][hidden]), stored at the
// row's destination (a peer address).
cudaError_t launch_ep_presum(const void* region, const void* routed, int world, const EpLayout& L,
                             cudaStream_t stream);
cudaError_t launch_ep_signal(void* region, const unsigned long long* peers, int rank, int world,
                             const EpLayout& L, cudaStream_t stream);
cudaError_t launch_ep_combine(void* region, const EpLayout& L, int world, long long tokens,
                              float scale, const void* shared_out, int shared_f16, void* out,
                              int out_f16, cudaStream_t stream);

// W8A8 block-FP8 GEMM (w8a8.cu): e4m3 weights [E][N][K] row-major with fp32
// scales per 128x128 block, times e4m3 activations [rows][K] with fp32 scales
// per (row, 128-K group) stored [K/128][xs_ld]. Dense (sorted_ids == nullptr):
// output row = activation row. Moe: activation rows are route slots in
// moe_align order, items from launch_tc_plan_slots(.., w8a8_item_slots()),
// output row = route id (times topk_w[route] when mul_w). gated: the bank is
// [gate | up] and the output is silu(gate) * up, N / 2 wide.
struct W8Launch {
  const uint8_t* w;
  const float* wscale;
  const uint8_t* xq;
  const float* xscale;
  long long xs_ld;
  long long rows;
  const int* sorted_ids;
  const int* ntpp;
  int num_routes;
  const float* topk_w;
  int mul_w;
  int E, N, K, gated;
  void* out;
  long long ldo;
  int out_f16;
  int* status;
  const void* plan_buf;  // moe mode: the plan (count + entries)
  int plan_cap;          // moe mode: plan entries the buffer holds
};
cudaError_t launch_w8a8_gemm(const W8Launch& L, cudaStream_t stream);
int w8a8_item_slots();
// Per (row, 128-K group) e4m3 quantization: q [out_rows][K], scales
// [K/128][ld] (rows out_rows .. ld-1 zeroed). ids != nullptr: row s quantizes
// activation row ids[s] / top_k (zeros for padding ids >= num_routes).
cudaError_t launch_fp8_act_quant(const void* x, int x_f16, long long x_rows, int K,
                                 const int* ids, int top_k, long long num_routes,
                                 long long out_rows, uint8_t* q, float* scales, long long ld,
                                 int* status, cudaStream_t stream);

// Records `message` as this thread's b200_last_error() and returns `code`.
int set_last_error(int code, const char* message);

// GEMM workspace layout (capi.cu): the status word and the arrival counters
// sit at the front, in ws_head_bytes(); the fixed part (head, tcgen05 plan,
// split partial sums) is ws_fixed_bytes() on the current device.
int64_t ws_head_bytes();
int64_t ws_fixed_bytes();

}  // namespace b200
