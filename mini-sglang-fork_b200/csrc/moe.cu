// Mixture-of-experts W8A8 path: routing layout, grouped expert GEMMs and the
// top-k combine -- the B200 counterpart of fused_experts_impl
// (M/moe/fused.py:135-215) for int8 expert weights.
//
//   w8a8_moe_align          moe_align_block_size (M/moe/fused.py:32-83) with
//                           128-row blocks: expert-sorted slot order, block ->
//                           expert table, slot -> row map
//   w8a8_moe_quant_scatter  per-token quantiser whose int8 row and scale go to
//                           each of the token's top-k rows (quant.cu)
//   w8a8_moe_gemm           the grouped GEMM (moe_sm100.cuh): gate_up with the
//                           SiLU*mul epilogue, or down with the routing weight
//   w8a8_moe_quant_rows     row quantiser of y with the known absmax
//   w8a8_moe_sum            moe_sum_reduce (M/kernel/triton/fused_moe.py:5-48)
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "gemm_api.h"
#include "moe_sm100.cuh"

namespace w8a8 {

int64_t moe_max_blocks(int64_t num_slots, int64_t num_experts);
int launch_rows_amax(const __nv_bfloat16* y, int64_t ld, const uint32_t* amax, int8_t* q, float* scale, int64_t M,
                     int width, const int32_t* num_blocks, cudaStream_t s);

namespace {

constexpr int kAlignThreads = 1024;
constexpr int kMaxExperts = kAlignThreads;
constexpr int kMoeStages = 4;

// G CTAs, no communication between them: every CTA counts ALL slots per
// expert (shared-memory atomics; the ids are read from L2 after the first
// CTA), and separately the slots before its own range, so it knows each
// expert's first row (an exclusive scan of the per-expert block counts) and
// where its own slots of each expert start.  It then places the slots of its
// range [g * chunk, (g + 1) * chunk): every slot takes the next row of its
// expert.  The scattered row stores are spread over the G SMs; the counting
// is repeated G times but runs in parallel.  Each thread loads kAlignIds ids
// at once (coalesced across the CTA) before touching the counters.
// The order of the slots inside an expert follows the atomics (not the slot
// order); nothing downstream depends on it: every row of the grouped GEMM is
// computed on its own, and the combine sums a token's choices in choice order
// through the slot -> row map.  Slots whose expert id is outside [0, E) are
// dropped (inv_pos = -1) and contribute nothing.  Padding rows get the slot
// id num_slots and scale 0, written row-contiguously (rows shared out over
// the CTAs); CTA 0 writes the block -> expert table and the block count.
constexpr int kAlignIds = 16;
constexpr int kAlignSharedBlocks = 4096;  // block -> expert table held in shared memory
__global__ void __launch_bounds__(kAlignThreads) moe_align_kernel(const int32_t* __restrict__ ids, int num_slots,
                                                                  int E, int chunk, int32_t* __restrict__ sorted_ids,
                                                                  int32_t* __restrict__ block_expert,
                                                                  int32_t* __restrict__ num_blocks,
                                                                  int32_t* __restrict__ inv_pos,
                                                                  float* __restrict__ sa_sorted) {
  __shared__ int cnt[kMaxExperts];
  __shared__ int before[kMaxExperts];
  __shared__ int first_row[kMaxExperts];
  __shared__ int next_row[kMaxExperts];
  __shared__ int warp_sum[kAlignThreads / 32];
  __shared__ uint16_t blk_e[kAlignSharedBlocks];
  dev::griddep_launch();
  dev::griddep_wait();  // the expert ids are the router's output
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int my_begin = blockIdx.x * chunk;
  const int my_end = min(num_slots, my_begin + chunk);
  constexpr int kStep = kAlignThreads * kAlignIds;
  cnt[t] = 0;
  before[t] = 0;
  __syncthreads();
  for (int base = 0; base < num_slots; base += kStep) {
    int e[kAlignIds];
#pragma unroll
    for (int j = 0; j < kAlignIds; ++j) {
      const int s = base + j * kAlignThreads + t;
      e[j] = s < num_slots ? __ldg(ids + s) : -1;
    }
#pragma unroll
    for (int j = 0; j < kAlignIds; ++j) {
      if (e[j] >= 0 && e[j] < E) {
        atomicAdd(&cnt[e[j]], 1);
        if (base + j * kAlignThreads + t < my_begin) atomicAdd(&before[e[j]], 1);
      }
    }
  }
  __syncthreads();
  const int c = t < E ? cnt[t] : 0;
  const int nbk = (c + 127) >> 7;
  int incl = nbk;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_sum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = warp_sum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    warp_sum[lane] = v;
  }
  __syncthreads();
  const int first_block = incl - nbk + (warp > 0 ? warp_sum[warp - 1] : 0);
  const int total = warp_sum[kAlignThreads / 32 - 1];
  if (t < E) {
    first_row[t] = first_block * 128;
    next_row[t] = first_block * 128 + before[t];
    for (int k = 0; k < nbk; ++k) {
      if (blockIdx.x == 0) block_expert[first_block + k] = t;
      if (first_block + k < kAlignSharedBlocks) blk_e[first_block + k] = static_cast<uint16_t>(t);
    }
  }
  if (blockIdx.x == 0 && t == 0) *num_blocks = total;
  __syncthreads();
  if (total <= kAlignSharedBlocks) {
    // row r is padding when it lies past its expert's c_e slots
    for (int r = blockIdx.x * kAlignThreads + t; r < total * 128; r += gridDim.x * kAlignThreads) {
      const int e = blk_e[r >> 7];
      if (r - first_row[e] >= cnt[e]) {
        sorted_ids[r] = num_slots;
        sa_sorted[r] = 0.0f;
      }
    }
  } else if (blockIdx.x == 0 && t < E) {
    for (int r = first_block * 128 + c; r < (first_block + nbk) * 128; ++r) {
      sorted_ids[r] = num_slots;
      sa_sorted[r] = 0.0f;
    }
  }
  for (int base = my_begin; base < my_end; base += kStep) {
    int e[kAlignIds];
#pragma unroll
    for (int j = 0; j < kAlignIds; ++j) {
      const int s = base + j * kAlignThreads + t;
      e[j] = s < my_end ? __ldg(ids + s) : -1;
    }
#pragma unroll
    for (int j = 0; j < kAlignIds; ++j) {
      const int s = base + j * kAlignThreads + t;
      if (s >= my_end) continue;
      if (e[j] >= 0 && e[j] < E) {
        const int r = atomicAdd(&next_row[e[j]], 1);
        sorted_ids[r] = s;
        inv_pos[s] = r;
      } else {
        inv_pos[s] = -1;
      }
    }
  }
}

// out[t] = bf16(sum_j f32(C[row(t, j)])), j = 0..topk-1 in order, from an
// fp32 zero -- moe_sum_reduce_kernel's arithmetic.  One thread per 8 columns
// of a token; a dropped choice (row -1) adds nothing.  With topk <= KMAX the
// rows and then the values of all choices are loaded before the sum.
constexpr int kSumThreads = 256;
template <int KMAX>
__global__ void __launch_bounds__(kSumThreads) moe_sum_kernel(const __nv_bfloat16* __restrict__ c, int64_t ldc,
                                                              const int32_t* __restrict__ inv_pos, int64_t T,
                                                              int topk, int nvec, __nv_bfloat16* __restrict__ out,
                                                              int64_t ldo) {
  dev::griddep_launch();
  dev::griddep_wait();  // the rows are the down GEMM's output
  const int64_t total = T * nvec;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kSumThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kSumThreads) {
    const int64_t tok = i / nvec;
    const int v = static_cast<int>(i - tok * nvec);
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
    auto add = [&](const uint4& raw) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        acc[2 * k] = __fadd_rn(acc[2 * k], f.x);
        acc[2 * k + 1] = __fadd_rn(acc[2 * k + 1], f.y);
      }
    };
    if (KMAX > 0) {
      int r[KMAX > 0 ? KMAX : 1];
      uint4 raw[KMAX > 0 ? KMAX : 1];
#pragma unroll
      for (int j = 0; j < KMAX; ++j) r[j] = j < topk ? __ldg(inv_pos + tok * topk + j) : -1;
#pragma unroll
      for (int j = 0; j < KMAX; ++j)
        if (r[j] >= 0) raw[j] = __ldg(reinterpret_cast<const uint4*>(c + static_cast<int64_t>(r[j]) * ldc) + v);
#pragma unroll
      for (int j = 0; j < KMAX; ++j)
        if (r[j] >= 0) add(raw[j]);
    } else {
      for (int j = 0; j < topk; ++j) {
        const int r = __ldg(inv_pos + tok * topk + j);
        if (r >= 0) add(__ldg(reinterpret_cast<const uint4*>(c + static_cast<int64_t>(r) * ldc) + v));
      }
    }
    uint4 pk;
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
    reinterpret_cast<uint4*>(out + tok * ldo)[v] = pk;
  }
}

template <bool SILU>
int launch_moe_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const MoeGemmArgs& args, int grid,
                    cudaStream_t stream) {
  using T = MoeTraits<kMoeStages>;
  auto kern = w8a8_moe_gemm_kernel<kMoeStages, SILU>;
  static std::mutex mu;
  static bool configured[64] = {false};
  const int dev = current_device();
  W8A8_REQUIRE(dev >= 0 && dev < 64, W8A8_ERR_CUDA, "no current device");
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!configured[dev]) {
      W8A8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T::kSmemBytes));
      configured[dev] = true;
    }
  }
  W8A8_CUDA_TRY(launch_pdl(kern, dim3(grid), dim3(T::kThreads), T::kSmemBytes, stream, ta, tb, args));
  return W8A8_OK;
}

}  // namespace

// Upper bound of the 128-row blocks the routing can need: sum_e ceil(c_e/128)
// <= (num_slots + 127 E) / 128, and at most one block per slot.
int64_t moe_max_blocks(int64_t num_slots, int64_t num_experts) {
  const int64_t b = (num_slots + 127 * num_experts) / 128;
  return b < num_slots ? b : num_slots;
}

}  // namespace w8a8

extern "C" {

int64_t w8a8_moe_max_blocks(int64_t num_slots, int64_t num_experts) {
  if (num_slots <= 0 || num_experts <= 0) return 0;
  return w8a8::moe_max_blocks(num_slots, num_experts);
}

int w8a8_moe_align(const int32_t* topk_ids, int64_t num_slots, int num_experts, int32_t* sorted_ids,
                   int32_t* block_expert, int32_t* num_blocks, int32_t* inv_pos, float* sa_sorted, void* stream) {
  using namespace w8a8;
  W8A8_REQUIRE(num_slots >= 0, W8A8_ERR_INVALID_ARG, "moe_align: negative slot count");
  W8A8_REQUIRE(num_experts >= 1 && num_experts <= kMaxExperts, W8A8_ERR_UNSUPPORTED,
               "moe_align: %d experts (1..%d supported)", num_experts, kMaxExperts);
  W8A8_REQUIRE(num_slots <= (1LL << 30), W8A8_ERR_UNSUPPORTED, "moe_align: %lld slots too many",
               (long long)num_slots);
  W8A8_REQUIRE(num_blocks != nullptr, W8A8_ERR_INVALID_ARG, "moe_align: null num_blocks");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (num_slots == 0) {
    W8A8_CUDA_TRY(cudaMemsetAsync(num_blocks, 0, sizeof(int32_t), s));
    return W8A8_OK;
  }
  W8A8_REQUIRE(topk_ids && sorted_ids && block_expert && inv_pos && sa_sorted, W8A8_ERR_INVALID_ARG,
               "moe_align: null pointer");
  // one CTA per 2048 slots, at most 64 (every CTA counts all slots)
  int64_t grid = (num_slots + 2047) / 2048;
  if (grid > 64) grid = 64;
  const int chunk = static_cast<int>((num_slots + grid - 1) / grid);
  W8A8_CUDA_TRY(launch_pdl(moe_align_kernel, dim3(static_cast<unsigned>(grid)), dim3(kAlignThreads), 0, s, topk_ids,
                           static_cast<int>(num_slots), num_experts, chunk, sorted_ids, block_expert, num_blocks,
                           inv_pos, sa_sorted));
  return W8A8_OK;
}

int w8a8_moe_gemm(const int8_t* a_sorted, const int8_t* w, const float* sa_sorted, const float* sw,
                  const int32_t* block_expert, const int32_t* num_blocks, int64_t max_blocks,
                  const int32_t* sorted_ids, const float* route_w, int64_t num_slots, void* C, uint32_t* silu_amax,
                  int num_experts, int64_t N, int64_t K, void* stream) {
  using namespace w8a8;
  W8A8_REQUIRE(max_blocks >= 0 && num_slots >= 0 && N >= 0 && K >= 0, W8A8_ERR_INVALID_ARG,
               "moe_gemm: negative size");
  if (max_blocks == 0) return W8A8_OK;
  W8A8_REQUIRE(a_sorted && w && sa_sorted && sw && block_expert && num_blocks && C, W8A8_ERR_INVALID_ARG,
               "moe_gemm: null pointer");
  W8A8_REQUIRE(route_w == nullptr || sorted_ids != nullptr, W8A8_ERR_INVALID_ARG,
               "moe_gemm: routing weights need sorted_ids");
  W8A8_REQUIRE(silu_amax == nullptr || route_w == nullptr, W8A8_ERR_INVALID_ARG,
               "moe_gemm: no routing weight with the SiLU epilogue");
  W8A8_REQUIRE(num_experts >= 1 && num_experts <= kMaxExperts, W8A8_ERR_UNSUPPORTED, "moe_gemm: %d experts",
               num_experts);
  W8A8_REQUIRE(K > 0 && K % 16 == 0, W8A8_ERR_INVALID_ARG, "moe_gemm: K=%lld must be a positive multiple of 16",
               (long long)K);
  W8A8_REQUIRE(N > 0 && N % (silu_amax ? 32 : 16) == 0, W8A8_ERR_INVALID_ARG,
               "moe_gemm: N=%lld must be a positive multiple of %d", (long long)N, silu_amax ? 32 : 16);
  W8A8_REQUIRE(static_cast<int64_t>(num_experts) * N <= (1LL << 31) - 256 && K <= (1LL << 30) &&
                   max_blocks * 128 <= (1LL << 31) - 1 && num_slots <= (1LL << 30),
               W8A8_ERR_UNSUPPORTED, "moe_gemm: sizes too large");
  W8A8_REQUIRE(W8A8_ALIGNED16(a_sorted) && W8A8_ALIGNED16(w) && W8A8_ALIGNED16(C) && W8A8_ALIGNED16(sw),
               W8A8_ERR_ALIGNMENT, "moe_gemm: a_sorted, w, sw and C must be 16-byte aligned");
  W8A8_REQUIRE(device_cc_major() == 10, W8A8_ERR_UNSUPPORTED,
               "moe_gemm: the tcgen05 kernels need an sm_100 (B200) device; found compute capability %d.x",
               device_cc_major());
  unsigned int* err = device_error_word();
  if (!err) return W8A8_ERR_CUDA;
  const int64_t rows_a = max_blocks * 128;
  CUtensorMap ta, tb;
  int rc = encode_operand(&ta, a_sorted, rows_a, K, 128);
  if (rc) return rc;
  rc = encode_operand(&tb, w, static_cast<int64_t>(num_experts) * N, K, 128);
  if (rc) return rc;
  MoeGemmArgs args;
  std::memset(&args, 0, sizeof(args));
  args.sa = sa_sorted;
  args.sb = sw;
  args.C = static_cast<__nv_bfloat16*>(C);
  args.amax = silu_amax;
  args.block_expert = block_expert;
  args.num_blocks = num_blocks;
  args.sorted_ids = sorted_ids;
  args.route_w = route_w;
  args.err = err;
  args.timeout_ns = kDefaultGemmTimeoutNs;
  args.num_slots = static_cast<int>(num_slots);
  args.num_experts = num_experts;
  args.N = static_cast<int>(N);
  args.K = static_cast<int>(K);
  args.kblocks = static_cast<int>((K + 127) / 128);
  args.silu_i = silu_amax ? static_cast<int>(N / 2) : 0;
  args.ldc = silu_amax ? static_cast<int>(N / 2) : static_cast<int>(N);
  args.tiles_n = silu_amax ? static_cast<int>((N / 2 + 127) / 128) : static_cast<int>((N + 255) / 256);
  args.max_blocks = static_cast<int>(max_blocks);
  const int64_t tiles = max_blocks * args.tiles_n;
  const int nsm = sm_count();
  W8A8_REQUIRE(nsm > 0, W8A8_ERR_CUDA, "moe_gemm: no CUDA device");
  const int grid = static_cast<int>(tiles < nsm ? tiles : nsm);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return silu_amax ? launch_moe_gemm<true>(ta, tb, args, grid, s) : launch_moe_gemm<false>(ta, tb, args, grid, s);
}

int w8a8_moe_quant_rows(const void* y, int64_t ldy, const uint32_t* amax, int8_t* q, float* scale,
                        const int32_t* num_blocks, int64_t max_blocks, int64_t K, void* stream) {
  using namespace w8a8;
  W8A8_REQUIRE(max_blocks >= 0 && K >= 0, W8A8_ERR_INVALID_ARG, "moe_quant_rows: negative shape");
  if (max_blocks == 0) return W8A8_OK;
  W8A8_REQUIRE(y && amax && q && scale && num_blocks, W8A8_ERR_INVALID_ARG, "moe_quant_rows: null pointer");
  W8A8_REQUIRE(K > 0 && K % 8 == 0 && K <= 0x7fffffff, W8A8_ERR_INVALID_ARG,
               "moe_quant_rows: K=%lld must be a positive multiple of 8", (long long)K);
  W8A8_REQUIRE(ldy >= K && ldy % 8 == 0, W8A8_ERR_INVALID_ARG,
               "moe_quant_rows: row stride %lld must be >= K and a multiple of 8", (long long)ldy);
  W8A8_REQUIRE(W8A8_ALIGNED16(y) && W8A8_ALIGNED16(q), W8A8_ERR_ALIGNMENT,
               "moe_quant_rows: y and q must be 16-byte aligned");
  return launch_rows_amax(static_cast<const __nv_bfloat16*>(y), ldy, amax, q, scale, max_blocks * 128,
                          static_cast<int>(K), num_blocks, static_cast<cudaStream_t>(stream));
}

int w8a8_moe_sum(const void* c_sorted, int64_t ldc, const int32_t* inv_pos, int64_t T, int topk, int64_t H,
                 void* out, int64_t ldo, void* stream) {
  using namespace w8a8;
  W8A8_REQUIRE(T >= 0 && H >= 0 && topk >= 0, W8A8_ERR_INVALID_ARG, "moe_sum: negative shape");
  if (T == 0) return W8A8_OK;
  W8A8_REQUIRE(c_sorted && inv_pos && out, W8A8_ERR_INVALID_ARG, "moe_sum: null pointer");
  W8A8_REQUIRE(topk >= 1 && topk <= 64, W8A8_ERR_UNSUPPORTED, "moe_sum: top-k %d (1..64 supported)", topk);
  W8A8_REQUIRE(H > 0 && H % 8 == 0 && H <= (1LL << 30), W8A8_ERR_INVALID_ARG,
               "moe_sum: H=%lld must be a positive multiple of 8", (long long)H);
  W8A8_REQUIRE(ldc >= H && ldc % 8 == 0 && ldo >= H && ldo % 8 == 0, W8A8_ERR_INVALID_ARG,
               "moe_sum: row strides must be >= H and multiples of 8");
  W8A8_REQUIRE(W8A8_ALIGNED16(c_sorted) && W8A8_ALIGNED16(out), W8A8_ERR_ALIGNMENT,
               "moe_sum: c_sorted and out must be 16-byte aligned");
  const int nvec = static_cast<int>(H / 8);
  const int64_t total = T * nvec;
  const int nsm = sm_count();
  W8A8_REQUIRE(nsm > 0, W8A8_ERR_CUDA, "moe_sum: no CUDA device");
  int64_t grid = (total + kSumThreads - 1) / kSumThreads;
  const int64_t cap = static_cast<int64_t>(nsm) * 8;
  if (grid > cap) grid = cap;
  auto kern = topk <= 2 ? moe_sum_kernel<2> : topk <= 4 ? moe_sum_kernel<4> : topk <= 8 ? moe_sum_kernel<8>
                                                                                   : moe_sum_kernel<0>;
  W8A8_CUDA_TRY(launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(kSumThreads), 0,
                           static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(c_sorted), ldc,
                           inv_pos, T, topk, nvec, static_cast<__nv_bfloat16*>(out), ldo));
  return W8A8_OK;
}

}  // extern "C"
