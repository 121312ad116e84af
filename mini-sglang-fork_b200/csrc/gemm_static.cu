// No-allocation entry point of the W8A8 GEMM: the same kernels and the same
// plan as w8a8_gemm, with the stream-K scratch (tile counters + int32 partial
// tiles) held in a fixed, file-scope device array instead of a caller-provided
// workspace.
//
// Callers that cannot allocate at call time:
//  * a serving engine that hands the HBM left after loading the weights to its
//    KV-cache page pool: a workspace allocated later can fail with
//    out-of-memory, or evict pages the scheduler already counted on;
//  * C / FFI callers (ctypes, cgo, JNI) without a caching allocator: a
//    cudaMalloc / cudaFree in the middle of a step synchronises the whole
//    device and stalls the host's overlap of scheduling with the GPU.
// This entry point calls no allocator (no cudaMalloc / cudaFree, no library
// that allocates): the scratch is part of the module image, resolved once.
//
// Limits:
//  * kStaticScratchBytes (20 MiB) per device: the 256 KiB counter region plus
//    two partial-tile slots per CTA.  On a 148-SM device that covers every
//    stream-K plan the planner makes (the largest, 128 x 128 tiles with a cut
//    remainder, needs 19.7 MB); a plan that needs more (possible on a device
//    with more SMs) is rejected with W8A8_ERR_WORKSPACE before any launch.
//  * Set-up: the first accepted non-empty call on a device (with that device
//    current) resolves the array's address with cudaGetSymbolAddress and clears
//    the counter region, synchronously.  Make that first call before any
//    stream capture.
//  * Every call that cuts tiles clears the counters it uses on its own stream
//    before the launch, so a call after one that gave up (device error word
//    set) starts from zero counters.
//  * One array per device: overlapping calls on one device (two streams, or
//    two host threads) share it and race.  Serialise them.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "gemm_api.h"
#include "gemm_plan.h"

namespace {

constexpr size_t kStaticScratchBytes = 20ull << 20;
static_assert(kStaticScratchBytes > w8a8::kCounterBytes, "scratch must hold the counter region");

__device__ __align__(256) unsigned char g_gemm_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Address of the current device's scratch; the first call per device resolves
// it and zeroes the counter region.
int static_scratch(void** out) {
  int dev = -1;
  W8A8_CUDA_TRY(cudaGetDevice(&dev));
  W8A8_REQUIRE(dev >= 0 && dev < kMaxDevices, W8A8_ERR_UNSUPPORTED,
               "gemm_static_scratch: device %d beyond the %d supported", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemm_static_scratch);
    W8A8_REQUIRE(e == cudaSuccess && p != nullptr, W8A8_ERR_CUDA,
                 "gemm_static_scratch: cudaGetSymbolAddress of the static scratch failed on device %d: %s", dev,
                 cudaGetErrorString(e));
    W8A8_REQUIRE((reinterpret_cast<uintptr_t>(p) & 255u) == 0, W8A8_ERR_ALIGNMENT,
                 "gemm_static_scratch: static scratch is not 256-byte aligned");
    W8A8_CUDA_TRY(cudaMemset(p, 0, w8a8::kCounterBytes));
    W8A8_CUDA_TRY(cudaDeviceSynchronize());
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return W8A8_OK;
}

}  // namespace

extern "C" {

int w8a8_gemm_static_scratch(const int8_t* A, const int8_t* B, const float* sa, const float* sb,
                             const void* bias, void* C, int32_t* c_i32, int64_t M, int64_t N, int64_t K,
                             void* stream) {
  W8A8_REQUIRE(M >= 0 && N >= 0 && K >= 0, W8A8_ERR_INVALID_ARG, "gemm_static_scratch: negative shape");
  if (M == 0) return W8A8_OK;  // empty batch, as w8a8_gemm
  W8A8_REQUIRE(N > 0 && K > 0, W8A8_ERR_INVALID_ARG, "gemm_static_scratch: empty N or K");
  // Every check that can reject the call runs before the set-up below, so a
  // rejected call touches no device state (and cannot disturb a capture).
  int rc = w8a8::validate_gemm_args(A, B, sa, sb, C, M, N, K);
  if (rc) return rc;
  W8A8_REQUIRE(w8a8::device_cc_major() == 10, W8A8_ERR_UNSUPPORTED,
               "gemm_static_scratch: the tcgen05 kernels need an sm_100 (B200) device; found compute capability %d.x",
               w8a8::device_cc_major());
  W8A8_REQUIRE(W8A8_ALIGNED16(c_i32), W8A8_ERR_ALIGNMENT, "gemm_static_scratch: c_i32 must be 16-byte aligned");
  const int nsm = w8a8::sm_count();
  W8A8_REQUIRE(nsm > 0, W8A8_ERR_CUDA, "gemm_static_scratch: no CUDA device");
  // The plan w8a8_gemm makes when its workspace is large enough.
  w8a8::GemmPlan p;
  W8A8_REQUIRE(w8a8::plan_gemm(M, N, K, 0, 0, static_cast<size_t>(-1), nsm, &p) == 0, W8A8_ERR_INVALID_ARG,
               "gemm_static_scratch: invalid shape");
  W8A8_REQUIRE(p.ws_bytes <= kStaticScratchBytes, W8A8_ERR_WORKSPACE,
               "gemm_static_scratch: the plan for %lld x %lld x %lld needs %zu bytes of scratch, above the static "
               "maximum of %zu bytes; call w8a8_gemm with a workspace",
               (long long)M, (long long)N, (long long)K, p.ws_bytes, kStaticScratchBytes);
  void* scratch = nullptr;
  rc = static_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p.cut_tiles)
    W8A8_CUDA_TRY(cudaMemsetAsync(scratch, 0, w8a8::plan_counter_words(p) * sizeof(uint32_t), s));
  return w8a8::run_gemm(A, B, sa, sb, bias, C, c_i32, M, N, K, 0, 0, scratch, kStaticScratchBytes, s,
                        w8a8::kDefaultGemmTimeoutNs, nullptr);
}

}  // extern "C"
