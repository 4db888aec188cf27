// b200_linear_noalloc: the dense linear for callers that cannot allocate.
//
// b200_linear needs a workspace (split-K partial sums, arrival counters, a
// status word, and room to convert bf16 activations to f16). Most callers
// hand it a buffer they allocated once. Some cannot: an engine that reserved
// all device memory for its own pool before loading plugins (a foreign
// cudaMalloc fails or breaks its accounting), or a binding with no handle on
// the device allocator. For them this entry point keeps the workspace in a
// fixed array compiled into the library: 16 MiB per device that loads the
// library, held until the process exits. It calls no cudaMalloc, cudaFree or
// allocating library routine.
//
// The array is shared by every call on a device and keeps whatever the last
// call left in it. The kernels return every arrival counter and partial sum
// they touch to zero when they finish, and a static device array starts
// zero-filled, so a call needs no clearing beyond:
//   * the first call on a device clears the whole fixed part (status word,
//     counters, tcgen05 plan, partial sums) once;
//   * every call clears the arrival counters (4 KiB), so a call that gave up
//     part-way (a timed-out pipeline wait) cannot skew the next call's
//     reductions;
//   * b200_linear_noalloc_status(.., reset != 0) that finds error bits set
//     clears the whole fixed part again (the partial sums of an aborted call).
// The status word is sticky: calls never clear it, so an error any earlier
// call recorded stays visible until the caller reads it with reset.
// Two calls that overlap on the GPU (different streams, no ordering between
// them) race on the array and produce wrong results; order them.
//
// In host code the array's name does not denote device memory. The first
// call on each device looks up the array's device address with
// cudaGetSymbolAddress while that device is current, and keeps it for the
// life of the process; make that first call before capturing the calls into
// a CUDA graph. cudaDeviceReset after the first call on a device is not
// supported (the kept address would be stale).
#include <cstdio>
#include <mutex>

#include "../../include/b200moe.h"
#include "internal.h"

namespace {

constexpr int64_t kScratchBytes = 16ll << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_linear_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_dev[kMaxDevices] = {};
bool g_cleared[kMaxDevices] = {};

int cuda_fail(const char* what, cudaError_t err) {
  char msg[256];
  snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(err));
  return b200::set_last_error(B200_ERR_CUDA, msg);
}

// Device address of g_linear_scratch on the current device (looked up once)
// and the device ordinal.
int scratch_for_current_device(void** out, int* dev_out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return b200::set_last_error(B200_ERR_CUDA, "b200_linear_noalloc: no usable current device");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_dev[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_linear_scratch);
    if (err != cudaSuccess || ptr == nullptr)
      return cuda_fail("b200_linear_noalloc: cudaGetSymbolAddress failed", err);
    g_scratch_dev[dev] = ptr;
  }
  *out = g_scratch_dev[dev];
  *dev_out = dev;
  return B200_OK;
}

}  // namespace

extern "C" int64_t b200_linear_noalloc_scratch_bytes(void) { return kScratchBytes; }

extern "C" int b200_linear_noalloc(int32_t quant, const void* x, int32_t x_dtype, int64_t m,
                                   int64_t k, const uint8_t* w_packed, const float* w_scales,
                                   const float* global_scale, int64_t n, int32_t gated_mode,
                                   void* y, int32_t y_dtype, void* stream) {
  if (m < 0 || k <= 0 || m >= (1ll << 31) || k >= (1ll << 31))
    return b200::set_last_error(B200_ERR_INVALID, "b200_linear_noalloc: bad M or K");
  const int64_t convert = x_dtype == B200_DTYPE_BF16 ? m * k : 0;
  const int64_t need = b200_gemm_workspace_bytes(convert);
  if (need < 0 || need > kScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "b200_linear_noalloc: this call needs %lld bytes of scratch, the static array holds "
             "%lld (bf16 activations: M*K=%lld too large; pass f16 or use b200_linear)",
             (long long)need, (long long)kScratchBytes, (long long)convert);
    return b200::set_last_error(B200_ERR_INVALID, msg);
  }
  if (m == 0) return B200_OK;
  void* scratch = nullptr;
  int dev = 0;
  int rc = scratch_for_current_device(&scratch, &dev);
  if (rc != B200_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  bool first = false;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    first = !g_cleared[dev];
    g_cleared[dev] = true;
  }
  cudaError_t err;
  if (first) {
    err = cudaMemsetAsync(base, 0, (size_t)b200::ws_fixed_bytes(), st);
  } else {
    // counters only: they follow the 256-byte status block
    const int64_t status_bytes = 256;
    err = cudaMemsetAsync(base + status_bytes, 0, (size_t)(b200::ws_head_bytes() - status_bytes),
                          st);
  }
  if (err != cudaSuccess) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (first) g_cleared[dev] = false;
    return cuda_fail("b200_linear_noalloc: clearing the scratch failed", err);
  }
  return b200_linear(quant, x, x_dtype, m, k, w_packed, w_scales, global_scale, n, gated_mode, y,
                     y_dtype, scratch, kScratchBytes, stream);
}

extern "C" int b200_linear_noalloc_status(int32_t* bits, int32_t reset, void* stream) {
  if (bits == nullptr) return b200::set_last_error(B200_ERR_INVALID, "null argument");
  void* scratch = nullptr;
  int dev = 0;
  int rc = scratch_for_current_device(&scratch, &dev);
  if (rc != B200_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int32_t host = 0;
  cudaError_t err = cudaMemcpyAsync(&host, scratch, sizeof(host), cudaMemcpyDeviceToHost, st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  if (err != cudaSuccess) return cuda_fail("b200_linear_noalloc_status: status read", err);
  *bits = host;
  if (reset && host != 0) {
    // An errored call may have left partial sums behind: clear the fixed part.
    err = cudaMemsetAsync(scratch, 0, (size_t)b200::ws_fixed_bytes(), st);
    if (err != cudaSuccess) return cuda_fail("b200_linear_noalloc_status: reset", err);
  }
  return B200_OK;
}
