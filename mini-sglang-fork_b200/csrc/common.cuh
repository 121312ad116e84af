// Shared host-side plumbing of the W8A8 library: status codes, the
// thread-local error message, CUDA checks and per-device facts.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/w8a8_tp.h"

namespace w8a8 {

// Device-side error bits, OR-ed into the per-device error word.
enum DeviceErrorBits : unsigned int {
  kErrGemmWait = 1u << 0,   // a GEMM mbarrier wait ran out of time
  kErrCommWait = 1u << 1,   // a cross-rank flag wait ran out of time
  kErrGemmDrain = 1u << 2,  // draining in-flight copies/MMAs after an abort timed out
};

// Records a formatted message for w8a8_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
void clear_error();

// Address (on the current device) of the device error word; nullptr and a
// recorded error if the symbol cannot be resolved.
unsigned int* device_error_word();

// Streaming multiprocessor count / compute capability of the current device
// (cached per device).
int current_device();
int sm_count();
int device_cc_major();

constexpr long long kDefaultGemmTimeoutNs = 4000000000LL;  // 4 s

}  // namespace w8a8

#define W8A8_CUDA_TRY(expr)                                                              \
  do {                                                                                   \
    cudaError_t e__ = (expr);                                                            \
    if (e__ != cudaSuccess)                                                              \
      return ::w8a8::fail(W8A8_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                 \
                          cudaGetErrorString(e__), __FILE__, __LINE__);                  \
  } while (0)

#define W8A8_REQUIRE(cond, code, ...)                                                    \
  do {                                                                                   \
    if (!(cond)) return ::w8a8::fail((code), __VA_ARGS__);                               \
  } while (0)

// 16-byte alignment test of a device pointer.
#define W8A8_ALIGNED16(p) ((reinterpret_cast<uintptr_t>(p) & 15u) == 0)

namespace w8a8 {

// Launch with programmatic stream serialisation (PDL): the kernel may begin
// its prologue while the previous kernel of the stream drains; it must call
// dev::griddep_wait() before touching that kernel's inputs or outputs.
template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace w8a8
