// Grouped (mixture-of-experts) W8A8 GEMM for sm_100a: the expert GEMMs of
// fused_experts_impl (M/moe/fused.py:135-215), which the reference runs as the
// Triton fused_moe_kernel (M/kernel/triton/fused_moe.py:51-190) over token
// rows gathered by sorted_token_ids.
//
// Layout.  The routed rows (token t, choice j) -- "slots" s = t * topk + j --
// sit in expert order in HBM: expert e owns rows [start_e, start_e + 128 b_e)
// of the sorted operand, its c_e slots first and padding after, b_e =
// ceil(c_e / 128) row blocks (w8a8_moe_align builds the order, the block ->
// expert table and the slot -> row map).  A tile is one 128-row block x 256
// output columns of one expert: A rows by TMA from the sorted int8 operand,
// B rows by TMA from the stacked int8 weight [E * N, K] at row e * N, so each
// tile is a plain 128 x 256 x K tcgen05 GEMM (kind::i8, int32 in TMEM).  The
// number of blocks in use is read on the device (the launch covers the
// host-side bound), so the call needs no host sync and captures in a graph.
//
// Modes.
//  * SiLU (gate_up): the expert weight is [gate (I rows); up (I rows)].  A
//    tile covers 128 features: its B rows are gate rows tn*128.. and the
//    matching up rows I + tn*128.. (two TMA boxes of 128 rows), so the
//    accumulator holds gate features in columns 0-127 and their up features
//    in 128-255.  The epilogue writes y = bf16(silu(g) * u), g and u the bf16
//    values a plain epilogue would write, to C [P, I] and folds every row's
//    max |y| into amax (float bits) for the row quantiser.
//  * plain (down): C [P, N] = bf16(dequant(acc) * w), w the slot's routing
//    weight (1 without one) -- the MUL_ROUTED_WEIGHT step of fused_moe_kernel
//    on the fp32 value before the cast.
//
// Roles: warp 0 lane 0 issues the TMA loads (a ring of STAGES stages), warp 1
// lane 0 issues the MMAs into one of two TMEM accumulators, warps 2-9 run the
// epilogue (two warps per TMEM lane quarter, each taking half of the tile's
// columns).  Every wait is bounded: on expiry the CTA raises its abort flag
// and the device error word, drains what it issued, frees TMEM and exits.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdint>

#include "gemm_sm100.cuh"
#include "silu.cuh"

namespace w8a8 {

struct MoeGemmArgs {
  const float* sa;             // [P] scales of the sorted rows (0 on padding rows)
  const float* sb;             // [E * N] per-channel weight scales
  __nv_bfloat16* C;            // [P, ldc] output rows in sorted order
  uint32_t* amax;              // SiLU mode: [P] max |y| of each row (float bits; zeroed by the caller)
  const int32_t* block_expert; // [max_blocks] expert of each 128-row block
  const int32_t* num_blocks;   // device scalar: blocks in use
  const int32_t* sorted_ids;   // [P] slot of each sorted row (num_slots on padding rows)
  const float* route_w;        // plain mode: [num_slots] routing weight of each slot, or null
  unsigned int* err;           // device error word
  long long timeout_ns;
  int num_slots;
  int num_experts;
  int N, K, kblocks;           // N: output channels of one expert (2I in SiLU mode)
  int ldc;                     // N (plain) or I (SiLU)
  int tiles_n;                 // 256-column tiles (SiLU: 128-feature tiles)
  int silu_i;                  // SiLU mode: I; 0 in plain mode
  int max_blocks;
};

template <int STAGES>
struct MoeTraits {
  static constexpr int kBM = 128;
  static constexpr int kBN = 256;
  static constexpr int kBK = 128;  // bytes of K per stage (= int8 elements)
  static constexpr int kMmaK = 32;
  static constexpr int kTileABytes = kBM * kBK;
  static constexpr int kTileBBytes = kBN * kBK;
  static constexpr int kStageBytes = kTileABytes + kTileBBytes;
  static constexpr int kEpiWarps = 8;
  static constexpr int kEpiThreads = 32 * kEpiWarps;
  static constexpr int kThreads = 32 * (2 + kEpiWarps);
  static constexpr int kBarrierBytes = 256;
  static constexpr int kStagingBytes = kEpiWarps * 2048;  // a 32 x 32 bf16 transpose buffer per warp
  static constexpr int kScaleBytes = 2 * kBN * 4;          // double-buffered weight scales of a tile
  static constexpr int kSmemBytes = 1024 + STAGES * kStageBytes + kBarrierBytes + kStagingBytes + kScaleBytes;
  static constexpr int kTmemCols = 2 * kBN;
  static constexpr uint32_t kIdesc = dev::idesc_i8(kBM, kBN);
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

// A staged 32-row x 32-column chunk (rows row0.., columns n0..) to C with
// row-contiguous 16-byte stores; columns >= n_limit are skipped.
__device__ __forceinline__ void moe_store_staged(const MoeGemmArgs& a, const uint4* stg, int lane, int row0, int n0,
                                                 int n_limit) {
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = j * 8 + (lane >> 2), g = lane & 3;
    const int n = n0 + g * 8;
    if (n < n_limit)
      *reinterpret_cast<uint4*>(a.C + static_cast<size_t>(row0 + r) * a.ldc + n) = stg[stage_slot(r, g)];
  }
  __syncwarp();  // the next chunk may overwrite the staging buffer
}

// bf16 values of one 32-column chunk, (f32(acc) * sa) * sb rounded once (the
// dense epilogue's arithmetic without a bias), packed eight to a uint4; with
// ROUTE each value is multiplied by w before the cast.
template <bool ROUTE>
__device__ __forceinline__ void moe_dequant32(float sa, const float* sbs, float w, const uint32_t (&v)[32],
                                              uint4 (&out)[4]) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float4 s0 = reinterpret_cast<const float4*>(sbs)[g * 2];
    const float4 s1 = reinterpret_cast<const float4*>(sbs)[g * 2 + 1];
    const float sb[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&out[g]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float y0 = dequant1(static_cast<int32_t>(v[g * 8 + 2 * j]), sa, sb[2 * j]);
      float y1 = dequant1(static_cast<int32_t>(v[g * 8 + 2 * j + 1]), sa, sb[2 * j + 1]);
      if (ROUTE) {
        y0 = __fmul_rn(y0, w);
        y1 = __fmul_rn(y1, w);
      }
      h[j] = __floats2bfloat162_rn(y0, y1);
    }
  }
}

template <int STAGES, bool SILU>
__global__ void __launch_bounds__(MoeTraits<STAGES>::kThreads, 1)
    w8a8_moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                         const MoeGemmArgs args) {
  using T = MoeTraits<STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * T::kTileABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_b + STAGES * T::kTileBBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* staging = reinterpret_cast<uint8_t*>(bars) + T::kBarrierBytes;
  float* scale_stage = reinterpret_cast<float*>(staging + T::kStagingBytes);  // [2][256]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      dev::mbar_init(dev::smem_u32(full + s), 1);
      dev::mbar_init(dev::smem_u32(empty + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(dev::smem_u32(acc_full + s), 1);
      dev::mbar_init(dev::smem_u32(acc_empty + s), T::kEpiThreads);
    }
    dev::mbar_init(dev::smem_u32(drain), 1);
    *abort_flag = 0;
    dev::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    dev::prefetch_tmap(&tm_a);
    dev::prefetch_tmap(&tm_b);
  }
  if (warp == 1) {
    dev::tmem_alloc(dev::smem_u32(tmem_slot), T::kTmemCols);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const long long tmo = args.timeout_ns;
  dev::griddep_launch();
  // the block table, the sorted rows and their scales are the previous
  // kernels' output
  dev::griddep_wait();
  int nb = *args.num_blocks;
  nb = nb < 0 ? 0 : (nb > args.max_blocks ? args.max_blocks : nb);
  const int ntiles = nb * args.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        const int b = t / args.tiles_n;
        const int tn = t - b * args.tiles_n;
        const int e = __ldg(args.block_expert + b);
        const int row_a = b * T::kBM;
        const int row_b0 = SILU ? e * args.N + tn * 128 : e * args.N + tn * T::kBN;
        const int row_b1 = SILU ? e * args.N + args.silu_i + tn * 128 : row_b0 + 128;
        for (int kb = 0; kb < args.kblocks; ++kb) {
          if (!dev::mbar_wait(dev::smem_u32(empty + stage), phase ^ 1u, abort_flag, args.err, kErrGemmWait, tmo)) {
            ok = false;
            break;
          }
          const uint32_t fb = dev::smem_u32(full + stage);
          dev::mbar_expect_tx(fb, T::kStageBytes);
          dev::tma_load_2d(dev::smem_u32(s_a + stage * T::kTileABytes), &tm_a, fb, kb * T::kBK, row_a);
          uint8_t* sb_dst = s_b + stage * T::kTileBBytes;
          dev::tma_load_2d(dev::smem_u32(sb_dst), &tm_b, fb, kb * T::kBK, row_b0);
          dev::tma_load_2d(dev::smem_u32(sb_dst + 128 * T::kBK), &tm_b, fb, kb * T::kBK, row_b1);
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every issued load must land before the CTA may exit.
      for (int s = 0; s < STAGES; ++s) {
        if (issued_mask & (1u << s)) {
          if (!dev::mbar_wait_drain(dev::smem_u32(full + s), (issued_phase >> s) & 1u, tmo)) {
            if (args.err) atomicOr(args.err, kErrGemmDrain);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        if (!dev::mbar_wait(dev::smem_u32(acc_empty + acc), acc_phase ^ 1u, abort_flag, args.err, kErrGemmWait,
                            tmo)) {
          break;
        }
        dev::tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * T::kBN);
        for (int kb = 0; kb < args.kblocks; ++kb) {
          if (!dev::mbar_wait(dev::smem_u32(full + stage), phase, abort_flag, args.err, kErrGemmWait, tmo)) {
            ok = false;
            break;
          }
          dev::tc_fence_after();
          const uint64_t da = dev::sdesc_k_sw128(dev::smem_u32(s_a + stage * T::kTileABytes));
          const uint64_t db = dev::sdesc_k_sw128(dev::smem_u32(s_b + stage * T::kTileBBytes));
#pragma unroll
          for (int k = 0; k < T::kBK / T::kMmaK; ++k) {
            const uint64_t off = static_cast<uint64_t>((k * T::kMmaK) >> 4);
            dev::mma_i8(d_tmem, da + off, db + off, T::kIdesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          dev::tc_commit(dev::smem_u32(empty + stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        dev::tc_commit(dev::smem_u32(acc_full + acc));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // All MMAs this thread issued must finish before TMEM is freed.
      dev::tc_commit(dev::smem_u32(drain));
      if (!dev::mbar_wait_drain(dev::smem_u32(drain), 0, tmo)) {
        if (args.err) atomicOr(args.err, kErrGemmDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;     // 0..7
    const int quarter = warp & 3;  // TMEM lane quarter (warp id mod 4)
    const int hh = ew >> 2;        // which half of the tile's columns
    const int et = threadIdx.x - 64;
    uint4* stg = reinterpret_cast<uint4*>(staging + ew * 2048);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t nt = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++nt) {
      const int b = t / args.tiles_n;
      const int tn = t - b * args.tiles_n;
      const int e = __ldg(args.block_expert + b);
      // The tile's 256 weight scales into shared memory (buffer nt & 1)
      // before waiting; the barrier below publishes them, and no warp still
      // reads this buffer (it belonged to tile nt - 2).
      float* sbs = scale_stage + (nt & 1u) * T::kBN;
      {
        int ch;
        bool valid;  // an expert id outside [0, E) reads no scale (its B rows load as zeros)
        if (SILU) {
          const int f = tn * 128 + (et & 127);
          valid = f < args.silu_i;
          ch = e * args.N + (et < 128 ? 0 : args.silu_i) + f;
        } else {
          const int n = tn * T::kBN + et;
          valid = n < args.N;
          ch = e * args.N + n;
        }
        valid = valid && e >= 0 && e < args.num_experts;
        sbs[et] = valid ? __ldg(args.sb + ch) : 0.0f;
      }
      const int row0 = b * T::kBM + quarter * 32;
      const int row = row0 + lane;
      const float sa = __ldg(args.sa + row);
      float w = 1.0f;
      if (!SILU && args.route_w != nullptr) {
        const int slot = __ldg(args.sorted_ids + row);
        w = (slot >= 0 && slot < args.num_slots) ? __ldg(args.route_w + slot) : 0.0f;
      }
      const bool ok = dev::mbar_wait(dev::smem_u32(acc_full + acc), acc_phase, abort_flag, args.err, kErrGemmWait,
                                     tmo);
      if (dev::named_bar_or(1, T::kEpiThreads, !ok)) break;  // uniform exit of all epilogue threads
      dev::tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_base + static_cast<uint32_t>(acc * T::kBN);
      if constexpr (SILU) {
        // features [64 hh, 64 hh + 64) of the tile in two 32-feature chunks
        __nv_bfloat162 m2 = __float2bfloat162_rn(0.0f);
#pragma unroll 1
        for (int j = 0; j < 2; ++j) {
          const int fc = hh * 64 + j * 32;
          uint32_t vg[32], vu[32];
          dev::tmem_ld32(t_acc + fc, vg);
          dev::tmem_ld32(t_acc + 128 + fc, vu);
          dev::tmem_wait_ld(vg);
          dev::tmem_wait_ld(vu);
          if (j == 1) {
            dev::tc_fence_before();
            dev::mbar_arrive(dev::smem_u32(acc_empty + acc));
          }
          uint4 pg[4], pu[4];
          moe_dequant32<false>(sa, sbs + fc, 1.0f, vg, pg);
          moe_dequant32<false>(sa, sbs + 128 + fc, 1.0f, vu, pu);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 y = act::silu_mul_vec8(pg[i], pu[i]);
            m2 = act::vec8_absmax2(y, m2);
            stg[stage_slot(lane, i)] = y;
          }
          moe_store_staged(args, stg, lane, row0, tn * 128 + fc, args.silu_i);
        }
        const float mx = act::absmax_of(m2);
        if (mx > 0.0f) atomicMax(args.amax + row, __float_as_uint(mx));
      } else {
        // columns [128 hh, 128 hh + 128) of the tile in four 32-column chunks,
        // chunk c + 1 loading from TMEM while chunk c is converted
        uint32_t vn[32];
        dev::tmem_ld32(t_acc + hh * 128, vn);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          dev::tmem_wait_ld(vn);
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = vn[q];
          const int col = hh * 128 + c * 32;
          if (c < 3) {
            dev::tmem_ld32(t_acc + col + 32, vn);
          } else {
            dev::tc_fence_before();
            dev::mbar_arrive(dev::smem_u32(acc_empty + acc));
          }
          uint4 pk[4];
          if (args.route_w != nullptr) {
            moe_dequant32<true>(sa, sbs + col, w, v, pk);
          } else {
            moe_dequant32<false>(sa, sbs + col, 1.0f, v, pk);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) stg[stage_slot(lane, i)] = pk[i];
          moe_store_staged(args, stg, lane, row0, tn * T::kBN + col, args.N);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    dev::tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem_base, T::kTmemCols);
  }
}

}  // namespace w8a8
