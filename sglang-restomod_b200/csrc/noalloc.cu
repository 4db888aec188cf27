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
// call left in it, so each call first clears the part that must start at
// zero (status, counters, partial sums) with cudaMemsetAsync on the caller's
// stream. Two calls that overlap on the GPU (different streams, no ordering
// between them) race on the array and produce wrong results; order them.
//
// In host code the array's name does not denote device memory. The first
// call on each device looks up the array's device address with
// cudaGetSymbolAddress while that device is current; make that first call
// before capturing the calls into a CUDA graph.
#include <cstdio>
#include <mutex>

#include "../../include/b200moe.h"
#include "internal.h"

namespace {

constexpr int64_t kScratchBytes = 16ll << 20;

__device__ __align__(256) uint8_t g_linear_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_dev[64] = {};

// Device address of g_linear_scratch on the current device, looked up once.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess || dev < 0 || dev >= 64)
    return b200::set_last_error(B200_ERR_CUDA, "b200_linear_noalloc: no usable current device");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_dev[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_linear_scratch);
    if (err != cudaSuccess || ptr == nullptr) {
      char msg[256];
      snprintf(msg, sizeof(msg), "b200_linear_noalloc: cudaGetSymbolAddress failed: %s",
               cudaGetErrorString(err));
      return b200::set_last_error(B200_ERR_CUDA, msg);
    }
    g_scratch_dev[dev] = ptr;
  }
  *out = g_scratch_dev[dev];
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
  int rc = scratch_for_current_device(&scratch);
  if (rc != B200_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t zeroed = b200_gemm_workspace_bytes(0);  // status, counters, partials
  cudaError_t err = cudaMemsetAsync(scratch, 0, (size_t)zeroed, st);
  if (err != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "b200_linear_noalloc: clearing the scratch failed: %s",
             cudaGetErrorString(err));
    return b200::set_last_error(B200_ERR_CUDA, msg);
  }
  return b200_linear(quant, x, x_dtype, m, k, w_packed, w_scales, global_scale, n, gated_mode, y,
                     y_dtype, scratch, kScratchBytes, stream);
}
