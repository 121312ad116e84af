// Measurement kernel: the int8 tensor-core ceiling of this device, used as
// the denominator of the GEMM's roofline fraction.
//
// An MMA-only loop: every CTA keeps one k block of both operands resident in
// shared memory (filled once with pseudo-random bytes, read through the same
// 128-byte swizzled K-major descriptors the GEMM uses) and issues `iters` x 4
// back-to-back tcgen05.mma kind::i8 into one TMEM accumulator, with no
// global-memory traffic at all.  The issuing thread
// then commits and waits (bounded) for the MMAs to drain.  ops per launch =
// 2 * M_mma * N_mma * 32 * 4 * iters per CTA (pair: per cluster).
//   pair = 0: one CTA per SM, M = 128, N = 256 (cta_group::1)
//   pair = 1: CTA pairs, M = 256, N = 256 (cta_group::2, the prefill kernel's
//             instruction shape)
#include "common.cuh"
#include "sm100.cuh"

namespace {

constexpr int kProbeThreads = 128;
constexpr int kProbeOperandBytes = 128 * 128;  // one 128-row x 128-byte k block per operand and CTA

struct ProbeSmem {
  uint8_t a[kProbeOperandBytes];
  uint8_t b[2 * kProbeOperandBytes];  // up to 256 rows of B for the 1-SM N = 256 shape
  uint64_t done;
  uint32_t tmem;
};

template <bool PAIR>
__global__ void __launch_bounds__(kProbeThreads, 1) mma_peak_kernel(long long iters, unsigned int* err,
                                                                    long long timeout_ns) {
  extern __shared__ __align__(1024) uint8_t raw[];
  ProbeSmem* s = reinterpret_cast<ProbeSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  // pseudo-random operand bytes (an all-zero operand would draw less power
  // than real data and flatter the ceiling)
  for (int i = threadIdx.x; i < (3 * kProbeOperandBytes) / 4; i += kProbeThreads) {
    uint32_t h = (static_cast<uint32_t>(i) + 0x9e3779b9u * (blockIdx.x + 1u)) * 0x85ebca6bu;
    h ^= h >> 13;
    h *= 0xc2b2ae35u;
    h ^= h >> 16;
    reinterpret_cast<uint32_t*>(s->a)[i] = h;
  }
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    w8a8::dev::mbar_init(w8a8::dev::smem_u32(&s->done), 1);
    w8a8::dev::fence_mbar_init();
  }
  if (warp == 0) {
    if constexpr (PAIR) {
      w8a8::dev::tmem_alloc2(w8a8::dev::smem_u32(&s->tmem), 256);
      w8a8::dev::tmem_relinquish2();
    } else {
      w8a8::dev::tmem_alloc(w8a8::dev::smem_u32(&s->tmem), 256);
      w8a8::dev::tmem_relinquish();
    }
  }
  // the generic-proxy operand stores must be visible to the tensor core's async proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  w8a8::dev::tc_fence_before();
  if constexpr (PAIR) {
    w8a8::dev::cluster_sync();
  } else {
    __syncthreads();
  }
  w8a8::dev::tc_fence_after();
  const uint32_t tmem = s->tmem;
  const bool issuer = threadIdx.x == 0 && (!PAIR || w8a8::dev::cluster_rank() == 0);
  if (issuer) {
    const uint64_t da = w8a8::dev::sdesc_k_sw128(w8a8::dev::smem_u32(s->a));
    const uint64_t db = w8a8::dev::sdesc_k_sw128(w8a8::dev::smem_u32(s->b));
    constexpr uint32_t idesc = PAIR ? w8a8::dev::idesc_i8(256, 256) : w8a8::dev::idesc_i8(128, 256);
    for (long long it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t off = static_cast<uint64_t>((k * 32) >> 4);
        if constexpr (PAIR) {
          w8a8::dev::mma_i8_pair(tmem, da + off, db + off, idesc, (it > 0 || k > 0) ? 1u : 0u);
        } else {
          w8a8::dev::mma_i8(tmem, da + off, db + off, idesc, (it > 0 || k > 0) ? 1u : 0u);
        }
      }
    }
    if constexpr (PAIR) {
      w8a8::dev::tc_commit_pair(w8a8::dev::smem_u32(&s->done));
    } else {
      w8a8::dev::tc_commit(w8a8::dev::smem_u32(&s->done));
    }
    if (!w8a8::dev::mbar_wait_drain(w8a8::dev::smem_u32(&s->done), 0, timeout_ns)) {
      if (err) atomicOr(err, w8a8::kErrGemmDrain);
    }
  }
  w8a8::dev::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) w8a8::dev::cluster_sync();
  w8a8::dev::tc_fence_after();
  if (warp == 0) {
    if constexpr (PAIR) {
      w8a8::dev::tmem_dealloc2(tmem, 256);
    } else {
      w8a8::dev::tmem_dealloc(tmem, 256);
    }
  }
}

template <bool PAIR>
int launch_probe(long long iters, unsigned int* err, cudaStream_t stream, int nsm) {
  auto kern = mma_peak_kernel<PAIR>;
  const size_t smem = sizeof(ProbeSmem) + 1024;
  W8A8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(PAIR ? (nsm / 2) * 2 : nsm));
  cfg.blockDim = dim3(kProbeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  W8A8_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, iters, err, w8a8::kDefaultGemmTimeoutNs));
  return W8A8_OK;
}

}  // namespace

extern "C" {

int w8a8_mma_peak_probe(int pair, int64_t iters, int64_t* ops_out, void* stream) {
  W8A8_REQUIRE(pair == 0 || pair == 1, W8A8_ERR_INVALID_ARG, "mma_peak_probe: pair must be 0 or 1");
  W8A8_REQUIRE(iters > 0 && iters <= (1LL << 24), W8A8_ERR_INVALID_ARG,
               "mma_peak_probe: iters %lld not in (0, 2^24]", (long long)iters);
  W8A8_REQUIRE(ops_out != nullptr, W8A8_ERR_INVALID_ARG, "mma_peak_probe: ops_out is null");
  W8A8_REQUIRE(w8a8::device_cc_major() == 10, W8A8_ERR_UNSUPPORTED,
               "mma_peak_probe: needs an sm_100 (B200) device; found compute capability %d.x",
               w8a8::device_cc_major());
  const int nsm = w8a8::sm_count();
  W8A8_REQUIRE(nsm >= 2, W8A8_ERR_CUDA, "mma_peak_probe: no CUDA device");
  unsigned int* err = w8a8::device_error_word();
  if (!err) return W8A8_ERR_CUDA;
  // per CTA (1-SM) or per pair: 4 MMAs of M x 256 x 32 per iteration
  const long long units = pair ? nsm / 2 : nsm;
  const long long m = pair ? 256 : 128;
  *ops_out = static_cast<int64_t>(units * iters * 4LL * 2LL * m * 256LL * 32LL);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return pair ? launch_probe<true>(iters, err, st, nsm) : launch_probe<false>(iters, err, st, nsm);
}

}  // extern "C"
