// Host side of kernel 2: tile-configuration planning, TMA descriptor
// encoding and launch of the tcgen05 W8A8 GEMM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "gemm2_sm100.cuh"
#include "gemm_api.h"
#include "gemm_plan.h"

namespace w8a8 {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

}  // namespace

// Tensor map over a row-major int8 matrix [rows, K] read as boxes of
// box_rows x 128 bytes with the 128-byte swizzle; out-of-range rows/columns
// read as zero.
int encode_operand(CUtensorMap* tm, const void* base, int64_t rows, int64_t K, int box_rows) {
  auto enc = tensor_map_encoder();
  W8A8_REQUIRE(enc != nullptr, W8A8_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
  cuuint32_t box[2] = {128u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  W8A8_REQUIRE(r == CUDA_SUCCESS, W8A8_ERR_CUDA,
               "cuTensorMapEncodeTiled failed (%d) for rows=%lld K=%lld box_rows=%d", (int)r,
               (long long)rows, (long long)K, box_rows);
  return W8A8_OK;
}

namespace {

template <int BN, int STAGES, bool SWAP, bool FUSED>
int launch_variant(const GemmPlan& p, const CUtensorMap& tw, const CUtensorMap& tn, const GemmArgs& args,
                   const CommView& cv, cudaStream_t stream) {
  using T = GemmTraits<BN, STAGES, SWAP>;
  constexpr int kSmem = T::smem_bytes(FUSED);
  auto kern = w8a8_gemm_kernel<BN, STAGES, SWAP, FUSED>;
  static std::mutex mu;
  static bool configured[64] = {false};
  const int dev = current_device();
  W8A8_REQUIRE(dev >= 0 && dev < 64, W8A8_ERR_CUDA, "no current device");
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!configured[dev]) {
      W8A8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
      configured[dev] = true;
    }
  }
  W8A8_CUDA_TRY(launch_pdl(kern, dim3(p.grid), dim3(gemm_block_threads<FUSED>()), kSmem, stream, tw, tn,
                           args, cv));
  return W8A8_OK;
}

}  // namespace

int validate_gemm_args(const int8_t* A, const int8_t* B, const float* sa, const float* sb, const void* C,
                       int64_t M, int64_t N, int64_t K) {
  W8A8_REQUIRE(M >= 0 && N >= 0 && K >= 0, W8A8_ERR_INVALID_ARG, "gemm: negative shape");
  W8A8_REQUIRE(A && B && sa && sb && C, W8A8_ERR_INVALID_ARG, "gemm: null pointer (A, B, sa, sb, C required)");
  W8A8_REQUIRE(K > 0 && K % 16 == 0, W8A8_ERR_INVALID_ARG, "gemm: K=%lld must be a positive multiple of 16",
               (long long)K);
  W8A8_REQUIRE(N > 0 && N % 16 == 0, W8A8_ERR_INVALID_ARG, "gemm: N=%lld must be a positive multiple of 16",
               (long long)N);
  W8A8_REQUIRE(M <= (1LL << 30) && N <= (1LL << 30) && K <= (1LL << 30), W8A8_ERR_UNSUPPORTED,
               "gemm: shape too large");
  W8A8_REQUIRE(W8A8_ALIGNED16(A) && W8A8_ALIGNED16(B) && W8A8_ALIGNED16(C), W8A8_ERR_ALIGNMENT,
               "gemm: A, B and C must be 16-byte aligned");
  return W8A8_OK;
}

template <int STAGES, bool FUSED>
int launch_pair_variant(const GemmPlan& p, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args,
                        const CommView& cv, cudaStream_t stream) {
  using T = Gemm2Traits<STAGES>;
  constexpr int kSmem = T::smem_bytes(FUSED);
  static_assert(kSmem <= 227 * 1024, "shared memory");
  auto kern = w8a8_gemm2_kernel<STAGES, FUSED>;
  static std::mutex mu;
  static bool configured[64] = {false};
  const int dev = current_device();
  W8A8_REQUIRE(dev >= 0 && dev < 64, W8A8_ERR_CUDA, "no current device");
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!configured[dev]) {
      W8A8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
      configured[dev] = true;
    }
  }
  W8A8_CUDA_TRY(launch_pdl(kern, dim3(p.grid), dim3(gemm2_block_threads<FUSED>()), kSmem, stream, ta, tb,
                           args, cv));
  return W8A8_OK;
}

template <bool FUSED>
int dispatch_variant(const GemmPlan& p, const CUtensorMap& tw, const CUtensorMap& tn, const GemmArgs& args,
                     const CommView& cv, cudaStream_t stream) {
  switch (p.variant) {
    case 1: return launch_variant<256, 4, false, FUSED>(p, tw, tn, args, cv, stream);
    case 2: return launch_variant<128, 6, false, FUSED>(p, tw, tn, args, cv, stream);
    // (a 5-stage decode ring, small enough for the next decode GEMM's CTA to
    // become resident beside this one, measured slower per decode step)
    case 3: return launch_variant<16, 10, true, FUSED>(p, tw, tn, args, cv, stream);
    case 4: return launch_variant<32, 9, true, FUSED>(p, tw, tn, args, cv, stream);
    case 5: return launch_variant<64, 8, true, FUSED>(p, tw, tn, args, cv, stream);
    case 6: return launch_variant<128, 6, true, FUSED>(p, tw, tn, args, cv, stream);
    case 7: return launch_pair_variant<6, FUSED>(p, tw, tn, args, cv, stream);
    default: return fail(W8A8_ERR_INVALID_ARG, "gemm: unknown variant %d", p.variant);
  }
}

int run_gemm(const int8_t* A, const int8_t* B, const float* sa, const float* sb, const void* bias, void* C,
             int32_t* c_i32, int64_t M, int64_t N, int64_t K, int variant, int ctas, void* workspace,
             size_t workspace_bytes, cudaStream_t stream, long long timeout_ns, const CommView* comm,
             uint32_t* silu_amax) {
  W8A8_REQUIRE(M >= 0 && N >= 0 && K >= 0, W8A8_ERR_INVALID_ARG, "gemm: negative shape");
  if (M == 0) return W8A8_OK;  // empty batch: nothing to compute (its tensors may be null)
  int rc = validate_gemm_args(A, B, sa, sb, C, M, N, K);
  if (rc) return rc;
  W8A8_REQUIRE(device_cc_major() == 10, W8A8_ERR_UNSUPPORTED,
               "gemm: the tcgen05 kernels need an sm_100 (B200) device; found compute capability %d.x",
               device_cc_major());
  W8A8_REQUIRE(W8A8_ALIGNED16(c_i32), W8A8_ERR_ALIGNMENT, "gemm: c_i32 must be 16-byte aligned");
  GemmPlan p;
  rc = plan_gemm(M, N, K, variant, ctas, workspace_bytes, sm_count(), &p);
  W8A8_REQUIRE(rc == 0, W8A8_ERR_INVALID_ARG, "gemm: %s", plan_error(rc));
  if (silu_amax) {
    W8A8_REQUIRE(comm == nullptr && c_i32 == nullptr, W8A8_ERR_INVALID_ARG,
                 "gemm_silu: no int32 output and no fused reduce with the SiLU epilogue");
    W8A8_REQUIRE(N % 256 == 0, W8A8_ERR_UNSUPPORTED, "gemm_silu: 2I = %lld must be a multiple of 256",
                 (long long)N);
    W8A8_REQUIRE(W8A8_ALIGNED16(silu_amax), W8A8_ERR_ALIGNMENT, "gemm_silu: amax must be 16-byte aligned");
    // the SiLU epilogue lives in the 2-SM pair kernel: take its plan whenever
    // the pairs have whole 256-row blocks to work on
    if (p.variant != 7 && M > 128) {
      GemmPlan q;
      if (plan_gemm(M, N, K, 7, ctas, workspace_bytes, sm_count(), &q) == 0) p = q;
    }
    W8A8_REQUIRE(p.variant == 7, W8A8_ERR_UNSUPPORTED,
                 "gemm_silu: M=%lld is below the 2-SM pair plan's range (needs M > 128)", (long long)M);
  }
  if (comm) {
    W8A8_REQUIRE(p.num_tiles <= kMaxSlots, W8A8_ERR_UNSUPPORTED,
                 "gemm_allreduce: %d output tiles exceed the %d flag slots", p.num_tiles, kMaxSlots);
    W8A8_REQUIRE(static_cast<unsigned long long>(M) * N * 2 <= comm->slot_bytes, W8A8_ERR_INVALID_ARG,
                 "gemm_allreduce: output of %lld x %lld bf16 exceeds the communicator's max_bytes %llu",
                 (long long)M, (long long)N, comm->slot_bytes);
    W8A8_REQUIRE(c_i32 == nullptr, W8A8_ERR_INVALID_ARG, "gemm_allreduce: no int32 output in fused mode");
    // a CTA hands over at most its share of whole tiles plus two stream-K
    // fix-ups; the hand-over ring must hold them all without reuse
    W8A8_REQUIRE((p.num_tiles + p.grid - 1) / p.grid + 2 <= kSignalRing, W8A8_ERR_UNSUPPORTED,
                 "gemm_allreduce: %d tiles over %d CTAs exceed the %d-tile hand-over ring", p.num_tiles, p.grid,
                 kSignalRing);
    // receive slots hold whole (padded) tiles
    W8A8_REQUIRE(static_cast<unsigned long long>(p.num_tiles) * 128 * p.bn * 2 <= comm->slot_bytes,
                 W8A8_ERR_INVALID_ARG,
                 "gemm_allreduce: %d padded %dx%d output tiles exceed the communicator's max_bytes %llu", p.num_tiles,
                 p.swap ? p.bn : 128, p.swap ? 128 : p.bn, comm->slot_bytes);
  }
  if (p.variant == 7 && (comm != nullptr || silu_amax != nullptr) && p.pair_split) {
    // the K split of the last wave is a plain-epilogue schedule: the fused
    // reduce and the SiLU epilogue deal whole blocks
    p.pair_split = 0;
    p.cut_tiles = false;
    p.ws_counter_bytes = 0;
    p.ws_bytes = 0;
  }
  if (p.cut_tiles) {
    W8A8_REQUIRE(workspace != nullptr && workspace_bytes >= p.ws_bytes, W8A8_ERR_WORKSPACE,
                 "gemm: stream-K needs a workspace of %zu bytes with zeroed counters", p.ws_bytes);
    W8A8_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, W8A8_ERR_ALIGNMENT,
                 "gemm: workspace must be 256-byte aligned");
  }
  unsigned int* err = device_error_word();
  if (!err) return W8A8_ERR_CUDA;

  const int8_t* wide = p.swap ? B : A;
  const int8_t* narrow = p.swap ? A : B;
  const int64_t rows_w = p.swap ? N : M;
  const int64_t rows_n = p.swap ? M : N;
  CUtensorMap tw, tn;
  rc = encode_operand(&tw, wide, rows_w, K, 128);
  if (rc) return rc;
  rc = encode_operand(&tn, narrow, rows_n, K, p.variant == 7 ? 128 : p.bn);
  if (rc) return rc;

  GemmArgs args;
  std::memset(&args, 0, sizeof(args));
  args.sa = sa;
  args.sb = sb;
  args.bias = static_cast<const __nv_bfloat16*>(bias);
  args.C = static_cast<__nv_bfloat16*>(C);
  args.c_i32 = c_i32;
  args.counters = p.cut_tiles ? static_cast<uint32_t*>(workspace) : nullptr;
  args.ws = p.cut_tiles ? reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + p.ws_counter_bytes)
                         : nullptr;
  args.err = err;
  args.timeout_ns = timeout_ns;
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.K = static_cast<int>(K);
  args.ldc = static_cast<int>(N);
  args.tiles_w = p.tiles_w;
  args.tiles_n = p.tiles_n;
  args.num_tiles = p.num_tiles;
  args.dp_tiles = p.dp_tiles;
  args.sk_ctas = p.sk_ctas;
  args.gran = p.gran;
  args.kblocks = p.kblocks;
  args.units = p.units;
  args.wide_fast = p.wide_fast;
  args.vec_scales = ((reinterpret_cast<uintptr_t>(sb) & 15u) == 0 && (reinterpret_cast<uintptr_t>(bias) & 15u) == 0) ? 1 : 0;
  // the K split of the pair kernel's last wave: plain, non-SiLU epilogue only
  args.pair_split = p.pair_split;
  if (silu_amax) {
    args.silu_i = static_cast<int>(N / 2);
    args.amax = silu_amax;
    args.ldc = static_cast<int>(N / 2);
  }

  if (comm) {
    CommView cv = *comm;
    if (p.swap) cv.two_shot = cv.nvls = 0;  // weight-stationary tiles push every partial to every rank
    return dispatch_variant<true>(p, tw, tn, args, cv, stream);
  }
  CommView none;
  std::memset(&none, 0, sizeof(none));
  return dispatch_variant<false>(p, tw, tn, args, none, stream);
}

}  // namespace w8a8

extern "C" {

size_t w8a8_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  w8a8::GemmPlan p;
  int nsm = w8a8::sm_count();
  if (nsm <= 0) nsm = 148;
  if (w8a8::plan_gemm(M, N, K, 0, 0, static_cast<size_t>(-1), nsm, &p) != 0) return 0;
  return p.ws_bytes;
}

int w8a8_gemm_plan(int64_t M, int64_t N, int64_t K, int variant, int ctas, size_t workspace_bytes,
                   int num_sms, int64_t* out) {
  W8A8_REQUIRE(out != nullptr, W8A8_ERR_INVALID_ARG, "gemm_plan: out is null");
  w8a8::GemmPlan p;
  const int rc = w8a8::plan_gemm(M, N, K, variant, ctas, workspace_bytes, num_sms, &p);
  W8A8_REQUIRE(rc == 0, W8A8_ERR_INVALID_ARG, "gemm_plan: %s",
               w8a8::plan_error(rc));
  out[0] = p.variant;
  out[1] = p.bn;
  out[2] = p.swap ? 1 : 0;
  out[3] = p.num_tiles;
  out[4] = p.grid;
  out[5] = p.kblocks;
  out[6] = p.gran;
  out[7] = static_cast<int64_t>(p.ws_bytes);
  return W8A8_OK;
}

int w8a8_gemm(const int8_t* A, const int8_t* B, const float* sa, const float* sb, const void* bias, void* C,
              int32_t* c_i32, int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
              void* stream) {
  return w8a8::run_gemm(A, B, sa, sb, bias, C, c_i32, M, N, K, 0, 0, workspace, workspace_bytes,
                        static_cast<cudaStream_t>(stream), w8a8::kDefaultGemmTimeoutNs, nullptr);
}

int w8a8_gemm_silu(const int8_t* A, const int8_t* B, const float* sa, const float* sb, const void* bias, void* Y,
                   uint32_t* amax, int64_t M, int64_t N2, int64_t K, void* workspace, size_t workspace_bytes,
                   void* stream) {
  W8A8_REQUIRE(amax != nullptr || M == 0, W8A8_ERR_INVALID_ARG, "gemm_silu: amax is null");
  if (M == 0) return W8A8_OK;
  return w8a8::run_gemm(A, B, sa, sb, bias, Y, nullptr, M, N2, K, 0, 0, workspace, workspace_bytes,
                        static_cast<cudaStream_t>(stream), w8a8::kDefaultGemmTimeoutNs, nullptr, amax);
}

int w8a8_gemm_config(const int8_t* A, const int8_t* B, const float* sa, const float* sb, const void* bias,
                     void* C, int32_t* c_i32, int64_t M, int64_t N, int64_t K, int variant, int ctas,
                     void* workspace, size_t workspace_bytes, void* stream) {
  W8A8_REQUIRE(variant >= 0 && variant <= w8a8::kMaxVariant, W8A8_ERR_INVALID_ARG,
               "gemm_config: variant %d out of range",
               variant);
  W8A8_REQUIRE(ctas >= 0, W8A8_ERR_INVALID_ARG, "gemm_config: negative ctas");
  return w8a8::run_gemm(A, B, sa, sb, bias, C, c_i32, M, N, K, variant, ctas, workspace, workspace_bytes,
                        static_cast<cudaStream_t>(stream), w8a8::kDefaultGemmTimeoutNs, nullptr);
}

}  // extern "C"
