// Kernel 2, pair variant: W8A8 GEMM with the 2-SM MMA (tcgen05 cta_group::2)
// for large (prefill) shapes, optionally fused with the row-parallel reduce.
//
// A cluster of two CTAs computes one 256 x 256 output block: CTA h of the
// pair stages rows [128h, 128h + 128) of the A block and rows
// [128h, 128h + 128) of the 256-row B (weight) block, 32 KB per 128-byte k
// block; the even CTA issues tcgen05.mma.cta_group::2 (M = 256, N = 256,
// K = 32), which reads both CTAs' shared memory and writes each CTA's own 128
// TMEM lanes x 256 columns.  Per SM that is 128 MACs per staged byte against
// 87 for the single-CTA 128 x 256 tile, which is what the single-CTA kernel is
// bound by at prefill sizes.
//
// Synchronisation across the pair (no cluster multicast anywhere):
//   * both producers load into their own shared memory and count the bytes
//     on the leader's `full` barrier (cp.async.bulk.tensor ... cta_group::2);
//     the leader arms it for both CTAs' bytes;
//   * the leader's MMA thread frees a stage in both CTAs and announces a
//     finished accumulator to both CTAs with one tcgen05.commit per CTA;
//   * both epilogues release the accumulator on the leader's `acc_empty`
//     barrier (the odd CTA with a remote arrive).
// The schedule is whole 256 x 256 blocks in grid-stride order over the pairs
// (the planner only picks this variant when that keeps every pair busy).  An
// odd number of 128-row tiles leaves the last pair's second half outside C:
// that CTA computes it (zero rows) and stores nothing.  Output tiles keep the
// 128 x 256 numbering of the single-CTA BN = 256 variant, so the fused reduce,
// its flags and receive-slot layout are shared with it.
#pragma once

#include "gemm_sm100.cuh"
#include "silu.cuh"

namespace w8a8 {

template <int STAGES>
struct Gemm2Traits {
  static constexpr int kBK = 128;
  static constexpr int kTileABytes = 128 * kBK;  // this CTA's 128 rows of A
  static constexpr int kTileBBytes = 128 * kBK;  // this CTA's 128 rows of B
  static constexpr int kStageBytes = kTileABytes + kTileBBytes;
  static constexpr int kBN = 256;
  static constexpr int kAccCols = 256;
  static constexpr int kTmemCols = 512;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kTileOutBytes = 128 * kBN * 2;
  // the staging buffers (2 KB per epilogue warp) serve both modes (the
  // epilogue's row-contiguous stores); the hand-over state only the fused one
  static constexpr int staging_bytes(bool fused) { return (fused ? 4 : 8) * 2048; }
  static constexpr int kScaleBytes = 2 * 2 * kBN * 4;  // double-buffered scales and bias of the tile (fp32)
  static constexpr int kSmemBytesPlain =
      1024 + STAGES * kStageBytes + kBarrierBytes + staging_bytes(false) + kScaleBytes;
  static constexpr int kSmemBytes =
      1024 + STAGES * kStageBytes + kBarrierBytes + staging_bytes(true) + kScaleBytes + kSignalBytes;
  static constexpr int smem_bytes(bool fused) { return fused ? kSmemBytes : kSmemBytesPlain; }
  static constexpr uint32_t kIdesc = dev::idesc_i8(256, 256);
  // (the launch checks the footprint of the mode it launches: a 7-stage ring
  // fits only without the fused-mode buffers)
  static_assert(kSmemBytesPlain <= 227 * 1024, "shared memory");
};

// Epilogue warps (warps 2, 3, ...): four in fused mode, one per TMEM lane
// quarter (warps 6-7 reduce there); eight in plain mode, two per lane quarter,
// each converting half of the block's 256 accumulator columns, which halves
// the per-block epilogue that sets the time of short-K GEMMs.
template <bool FUSED>
constexpr int gemm2_epi_warps() {
  return FUSED ? 4 : 8;
}
template <bool FUSED>
constexpr int gemm2_block_threads() {
  return FUSED ? gemm_block_threads<true>() : 32 * (2 + gemm2_epi_warps<false>());
}

// Pair p -> (pw, tn): 256-row block index and 256-column block index.
__device__ __forceinline__ void pair_coords(const GemmArgs& a, int pairs_w, int p, int& pw, int& tn) {
  if (a.wide_fast) {
    pw = p % pairs_w;
    tn = p / pairs_w;
  } else {
    tn = p % a.tiles_n;
    pw = p / a.tiles_n;
  }
}

// The work of one CTA pair (cluster c of G): whole blocks c, c + G, ... and,
// when the last wave is split along K (args.pair_split = s > 1), after them
// one fragment f = c of the last wave's rem = num_pairs % G blocks: block
// num_pairs - rem + f / s, k blocks [j kb / s, (j + 1) kb / s) with j = f % s.
// Every role of both CTAs walks the same sequence.
struct PairWalk {
  int p, num_pairs, G, full, split, frag;
  __device__ __forceinline__ PairWalk(const GemmArgs& a, int num_pairs_, int c, int G_)
      : p(c), num_pairs(num_pairs_), G(G_), full(num_pairs_), split(a.pair_split > 1 ? a.pair_split : 0),
        frag(-1) {
    if (split) {
      const int rem = num_pairs % G;
      full = num_pairs - rem;
      frag = c < rem * split ? c : -1;
    }
  }
  // block, k range, j (-1: whole block)
  __device__ __forceinline__ bool next(const GemmArgs& a, int& blk, int& kb0, int& kb1, int& j) {
    if (p < full) {
      blk = p;
      kb0 = 0;
      kb1 = a.kblocks;
      j = -1;
      p += G;
      return true;
    }
    if (frag < 0) return false;
    blk = full + frag / split;
    j = frag % split;
    kb0 = j * a.kblocks / split;
    kb1 = (j + 1) * a.kblocks / split;
    frag = -1;
    return true;
  }
};

// Index of output tile (tw, tn) in tile_coords' numbering.
__device__ __forceinline__ int tile_index(const GemmArgs& a, int tw, int tn) {
  return a.wide_fast ? tn * a.tiles_w + tw : tw * a.tiles_n + tn;
}

template <int STAGES, bool FUSED>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm2_block_threads<FUSED>(), 1)
    w8a8_gemm2_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                      const GemmArgs args, const CommView cv) {
  using T = Gemm2Traits<STAGES>;
  constexpr int kEpi = gemm2_epi_warps<FUSED>();
  constexpr int kEpiThreads = 32 * kEpi;
  constexpr int kChunksPerWarp = 8 * 4 / kEpi;  // 32-column chunks of the 256 per warp
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
  volatile uint32_t* epoch_slot = reinterpret_cast<volatile uint32_t*>(abort_flag + 2);
  uint8_t* staging = reinterpret_cast<uint8_t*>(bars) + T::kBarrierBytes;
  float* scale_stage = reinterpret_cast<float*>(staging + T::staging_bytes(FUSED));  // [2][256] sb, [2][256] bias
  FusedState* sigq = reinterpret_cast<FusedState*>(staging + T::staging_bytes(FUSED) + T::kScaleBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t half = dev::cluster_rank();  // 0 = leader
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;
  const int pairs_w = (args.tiles_w + 1) >> 1;
  const int num_pairs = pairs_w * args.tiles_n;

  if (threadIdx.x == 0) {
    if constexpr (FUSED) init_fused_state(sigq);  // plain launches carry no staging / hand-over region
    for (int s = 0; s < STAGES; ++s) {
      dev::mbar_init(dev::smem_u32(full + s), 1);
      dev::mbar_init(dev::smem_u32(empty + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(dev::smem_u32(acc_full + s), 1);
      dev::mbar_init(dev::smem_u32(acc_empty + s), 2 * kEpiThreads);  // the epilogue threads of both CTAs
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
    dev::tmem_alloc2(dev::smem_u32(tmem_slot), T::kTmemCols);
    dev::tmem_relinquish2();
  }
  dev::tc_fence_before();
  dev::cluster_sync();  // barriers of both CTAs initialised before any cross-CTA use
  dev::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const long long tmo = args.timeout_ns;
  dev::griddep_launch();
  uint32_t epoch = 0;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      dev::griddep_wait();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      PairWalk walk(args, num_pairs, cluster, nclusters);
      int p, kb0, kb1, jf;
      while (ok && walk.next(args, p, kb0, kb1, jf)) {
        int pw, tn;
        pair_coords(args, pairs_w, p, pw, tn);
        const int tw = 2 * pw + static_cast<int>(half);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!dev::mbar_wait(dev::smem_u32(empty + stage), phase ^ 1u, abort_flag, args.err, kErrGemmWait,
                              tmo)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = dev::mapa(dev::smem_u32(full + stage), 0);
          if (half == 0) dev::mbar_expect_tx(dev::smem_u32(full + stage), 2 * T::kStageBytes);
          dev::tma_load_2d_pair(dev::smem_u32(s_a + stage * T::kTileABytes), &tm_a, leader_full, kb * T::kBK,
                                tw * 128);
          // B rows of this CTA's half: the block's next 128 weight rows, or
          // (SiLU epilogue) the block's 128 gate rows / their 128 up rows
          const int b_row = args.silu_i ? tn * 128 + static_cast<int>(half) * args.silu_i
                                        : tn * 256 + static_cast<int>(half) * 128;
          dev::tma_load_2d_pair(dev::smem_u32(s_b + stage * T::kTileBBytes), &tm_b, leader_full, kb * T::kBK,
                                b_row);
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // The leader's full barriers count both CTAs' bytes: once they have
      // landed, no copy of either CTA is in flight (the pair then meets at the
      // closing cluster barrier).
      if (half == 0) {
        for (int s = 0; s < STAGES; ++s) {
          if (issued_mask & (1u << s)) {
            if (!dev::mbar_wait_drain(dev::smem_u32(full + s), (issued_phase >> s) & 1u, tmo)) {
              if (args.err) atomicOr(args.err, kErrGemmDrain);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && half == 0) {
      // --------------------------------------------- MMA issuer (leader only)
      dev::griddep_wait();
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      PairWalk walk(args, num_pairs, cluster, nclusters);
      int p, kb0, kb1, jf;
      while (ok && walk.next(args, p, kb0, kb1, jf)) {
        if (!dev::mbar_wait_cluster(dev::smem_u32(acc_empty + acc), acc_phase ^ 1u, abort_flag, args.err,
                                    kErrGemmWait, tmo)) {
          break;
        }
        dev::tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * T::kAccCols);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!dev::mbar_wait(dev::smem_u32(full + stage), phase, abort_flag, args.err, kErrGemmWait, tmo)) {
            ok = false;
            break;
          }
          dev::tc_fence_after();
          const uint64_t da = dev::sdesc_k_sw128(dev::smem_u32(s_a + stage * T::kTileABytes));
          const uint64_t db = dev::sdesc_k_sw128(dev::smem_u32(s_b + stage * T::kTileBBytes));
#pragma unroll
          for (int k = 0; k < T::kBK / 32; ++k) {
            const uint64_t off = static_cast<uint64_t>((k * 32) >> 4);
            dev::mma_i8_pair(d_tmem, da + off, db + off, T::kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          dev::tc_commit_pair(dev::smem_u32(empty + stage));
          dev::tc_commit_pair(dev::mapa(dev::smem_u32(empty + stage), 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        dev::tc_commit_pair(dev::smem_u32(acc_full + acc));
        dev::tc_commit_pair(dev::mapa(dev::smem_u32(acc_full + acc), 1));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      dev::tc_commit_pair(dev::smem_u32(drain));
      if (!dev::mbar_wait_drain(dev::smem_u32(drain), 0, tmo)) {
        if (args.err) atomicOr(args.err, kErrGemmDrain);
      }
    }
  } else if (warp < 2 + kEpi) {
    // ------------------------------------------------------------ epilogue
    dev::griddep_wait();
    if constexpr (FUSED) epoch = dev::ld_relaxed_gpu(dev::ctrl_ptr(cv.base[cv.rank])) + 1u;
    const size_t my_slot = kHeaderBytes + static_cast<size_t>(epoch & 1u) * cv.half_bytes +
                           static_cast<size_t>(cv.rank) * cv.slot_bytes;
    uint4* stg = reinterpret_cast<uint4*>(staging + (warp - 2) * 2048);
    int cur_m0 = 0, cur_hm = 1, cur_n0 = 0, cur_tile = 0;
    auto emit16 = [&](int, int n, const uint4& val) { stg[stage_slot(lane, (n & 31) >> 3)] = val; };
    auto push_chunk = [&](int c) {
      if constexpr (FUSED) {
        __syncwarp();
        const size_t blk = static_cast<size_t>(cur_tile) * T::kTileOutBytes + static_cast<size_t>(c) * 8192 +
                           static_cast<size_t>(warp & 3) * 2048;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = lane + 32 * j;
          const int r = (warp & 3) * 32 + (k >> 2);
          if (r >= cur_hm) continue;
          const uint4 val = stg[stage_slot(k >> 2, k & 3)];
          const size_t off = blk + static_cast<size_t>(k) * 16;
          if (cv.nvls) {
            *reinterpret_cast<uint4*>(dev::nv_partials(cv, cv.nv_local, epoch) + off) = val;
          } else if (cv.two_shot) {
            const int owner = min(row_owner(cur_m0 + r, cur_m0, cur_hm, cv.world), cv.world - 1);
            *reinterpret_cast<uint4*>(cv.base[owner] + my_slot + off) = val;
          } else {
            for (int d = 0; d < cv.world; ++d) *reinterpret_cast<uint4*>(cv.base[d] + my_slot + off) = val;
          }
        }
        if (cv.nvls) dev::fence_proxy_alias();  // before the tile's ready flag (read via multicast)
        __syncwarp();
      }
    };
    const int quarter = warp & 3;                        // TMEM lane quarter (warp id mod 4)
    const int c0 = ((warp - 2) / 4) * kChunksPerWarp;    // first of this warp's column chunks
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int et = threadIdx.x - 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t sig_n = 0;
    uint32_t blk = 0;
    bool aborted = false;
    PairWalk walk(args, num_pairs, cluster, nclusters);
    int p, kb0, kb1, jf;
    while (walk.next(args, p, kb0, kb1, jf)) {
      int pw, tn;
      pair_coords(args, pairs_w, p, pw, tn);
      const int tw = 2 * pw + static_cast<int>(half);
      const bool real = tw < args.tiles_w;
      const int tile = real ? tile_index(args, tw, tn) : 0;
      if constexpr (FUSED) {
        if (real) {
          int wn_;
          tile_rect<256, false>(args, tile, cur_m0, cur_hm, cur_n0, wn_);
          cur_tile = tile;
        }
      }
      const int row = tw * 128 + row_in_tile;
      // the tile's scales into shared memory (buffer blk & 1) before waiting;
      // the barrier below publishes them (see the single-CTA kernel)
      float* sbs = scale_stage + (blk & 1u) * 256;
      float* bss = scale_stage + 512 + (blk & 1u) * 256;
      const float sam = args.silu_i ? stage_tile_scales_silu(args, tn, et, real, row, sbs, bss)
                                    : stage_tile_scales(args, tn * 256, 256, et, real, row, sbs, bss);
      ++blk;
      const bool ok = dev::mbar_wait(dev::smem_u32(acc_full + acc), acc_phase, abort_flag, args.err, kErrGemmWait,
                                     tmo);
      if (dev::named_bar_or(1, kEpiThreads, !ok)) {
        aborted = true;
        break;
      }
      dev::tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_base + static_cast<uint32_t>(acc * T::kAccCols);
      if constexpr (!FUSED) {
        if (args.silu_i) {
          // SiLU epilogue: accumulator columns [0, 128) are the block's gate
          // features, [128, 256) their up features.  This warp takes features
          // [64 hh, 64 hh + 64) in two 32-feature chunks: gate and up chunk
          // dequantised to bf16 as the plain epilogue would write them, then
          // y = bf16(silu(g) * u) (the fused quantiser's arithmetic), staged and
          // written to C = y [M, I]; the row's max |y| goes to amax.
          const int hh = (warp - 2) >> 2;
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
              const uint32_t bar = dev::smem_u32(acc_empty + acc);
              if (half == 0) {
                dev::mbar_arrive(bar);
              } else {
                dev::mbar_arrive_cluster(dev::mapa(bar, 0));
              }
            }
            if (real) {
              uint4 pg[4], pu[4];
              dequant_pack32(args, sam, sbs + fc, bss + fc, vg, pg);
              dequant_pack32(args, sam, sbs + 128 + fc, bss + 128 + fc, vu, pu);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint4 y = act::silu_mul_vec8(pg[i], pu[i]);
                if (row < args.M) m2 = act::vec8_absmax2(y, m2);
                stg[stage_slot(lane, i)] = y;
              }
              store_staged_chunk(args, stg, lane, tw * 128 + quarter * 32, tn * 128 + fc, args.silu_i);
            }
          }
          if (real && row < args.M) atomicMax(args.amax + row, __float_as_uint(act::absmax_of(m2)));
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
          continue;
        }
      }
      if constexpr (!FUSED) {
        if (jf >= 0) {
          // A fragment of a last-wave block (split along K).  The CTA of each
          // half holds 128 rows x 256 columns of partial int32 sums.  Shares
          // j > 0 are parked in this CTA's slot (layout [chunk][quarter]
          // [8 column groups][lane][4 columns]: each warp store covers 512
          // contiguous bytes) and counted in the half's counter; the share
          // j = 0 (its pair is the block's owner) waits (bounded) for the
          // others' count, adds their slots (same half, CTAs of the next
          // pairs) and writes the block.  Shares never wait on anything, so
          // no pair waits on a pair that waits.
          int4* slots = reinterpret_cast<int4*>(args.ws);
          constexpr int kSlotInt4 = 128 * 256 / 4;
          uint32_t* counter = args.counters + 2 * p + static_cast<int>(half);
          if (jf > 0) {
            int4* mine = slots + static_cast<size_t>(blockIdx.x) * kSlotInt4;
#pragma unroll 1
            for (int c = c0; c < c0 + kChunksPerWarp; ++c) {
              uint32_t v[32];
              dev::tmem_ld32(t_acc + c * 32, v);
              dev::tmem_wait_ld(v);
              int4* dst = mine + ((c * 4 + quarter) * 8) * 32 + lane;
#pragma unroll
              for (int q = 0; q < 8; ++q)
                __stcg(dst + q * 32, make_int4(static_cast<int>(v[4 * q]), static_cast<int>(v[4 * q + 1]),
                                               static_cast<int>(v[4 * q + 2]), static_cast<int>(v[4 * q + 3])));
            }
            dev::tc_fence_before();
            const uint32_t bar = dev::smem_u32(acc_empty + acc);
            if (half == 0) {
              dev::mbar_arrive(bar);
            } else {
              dev::mbar_arrive_cluster(dev::mapa(bar, 0));
            }
            // one fence after the barrier orders every epilogue thread's slot
            // stores before the count
            dev::named_bar_sync(1, kEpiThreads);
            if (et == 0) {
              __threadfence();
              atomicAdd(counter, 1u);
            }
          } else {
            bool counted = true;
            if (et == 0)
              counted = dev::wait_counter(counter, static_cast<uint32_t>(args.pair_split - 1), abort_flag,
                                          args.err, kErrGemmWait, tmo);
            if (dev::named_bar_or(1, kEpiThreads, !counted)) {
              aborted = true;
              break;
            }
            const int first = cluster;  // this pair holds share 0; shares 1..s-1 are the next pairs
#pragma unroll 1
            for (int c = c0; c < c0 + kChunksPerWarp; ++c) {
              uint32_t v[32];
              dev::tmem_ld32(t_acc + c * 32, v);
              dev::tmem_wait_ld(v);
#pragma unroll 1
              for (int o = 1; o < args.pair_split; ++o) {
                const int cta = 2 * (first + o) + static_cast<int>(half);
                const int4* src = slots + static_cast<size_t>(cta) * kSlotInt4 + ((c * 4 + quarter) * 8) * 32 + lane;
                int4 qv[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) qv[q] = __ldcg(src + q * 32);
#pragma unroll
                for (int q = 0; q < 8; ++q) {  // two's-complement sums, as int32
                  v[4 * q] += static_cast<uint32_t>(qv[q].x);
                  v[4 * q + 1] += static_cast<uint32_t>(qv[q].y);
                  v[4 * q + 2] += static_cast<uint32_t>(qv[q].z);
                  v[4 * q + 3] += static_cast<uint32_t>(qv[q].w);
                }
              }
              if (c == c0 + kChunksPerWarp - 1) {
                dev::tc_fence_before();
                const uint32_t bar = dev::smem_u32(acc_empty + acc);
                if (half == 0) {
                  dev::mbar_arrive(bar);
                } else {
                  dev::mbar_arrive_cluster(dev::mapa(bar, 0));
                }
              }
              if (real) {
                store_chunk_smem(args, row, tn * 256 + c * 32, sam, sbs + c * 32, bss + c * 32, v, emit16);
                store_staged_chunk(args, stg, lane, tw * 128 + quarter * 32, tn * 256 + c * 32);
              }
            }
            if (et == 0) *counter = 0u;
          }
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
          continue;
        }
      }
      uint32_t vn[32];
      dev::tmem_ld32(t_acc + c0 * 32, vn);  // chunk c + 1 loads while chunk c is processed
#pragma unroll 1
      for (int c = c0; c < c0 + kChunksPerWarp; ++c) {
        uint32_t v[32];
        dev::tmem_wait_ld(vn);
#pragma unroll
        for (int q = 0; q < 32; ++q) v[q] = vn[q];
        const bool last = c == c0 + kChunksPerWarp - 1;
        if (!last) dev::tmem_ld32(t_acc + (c + 1) * 32, vn);
        if (last) {
          dev::tc_fence_before();
          const uint32_t bar = dev::smem_u32(acc_empty + acc);
          if (half == 0) {
            dev::mbar_arrive(bar);
          } else {
            dev::mbar_arrive_cluster(dev::mapa(bar, 0));
          }
        }
        if (real) {
          store_chunk_smem(args, row, tn * 256 + c * 32, sam, sbs + c * 32, bss + c * 32, v, emit16);
          if constexpr (FUSED) {
            push_chunk(c);
          } else {
            store_staged_chunk(args, stg, lane, tw * 128 + quarter * 32, tn * 256 + c * 32);
          }
        }
      }
      if constexpr (FUSED) {
        if (real) {
          // every epilogue thread's pushes of the tile precede the hand-over
          dev::named_bar_sync(1, kEpiThreads);
          if (et == 0 && !signal_handover(sigq, sig_n, tile, args.err, tmo)) *abort_flag = 1;
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    dev::tc_fence_before();
    if constexpr (FUSED) {
      if (aborted) *abort_flag = 1;
      if (et == 0) {
        *epoch_slot = epoch;
        dev::st_release_cta(&sigq->closed, 1u);
      }
    }
  } else {
    if constexpr (FUSED) {
      // ----------------------------------------------------------- reducers
      // Each CTA of the pair reduces its own share of the call's 128 x 256
      // tiles (t % gridDim.x == blockIdx.x) as the ranks' partials land, and
      // raises its own ready flags meanwhile and afterwards.
      dev::griddep_wait();
      const uint32_t ep = dev::ld_relaxed_gpu(dev::ctrl_ptr(cv.base[cv.rank])) + 1u;
      const ReduceGroup g{kReducerBar, kReduceThreads, static_cast<int>(threadIdx.x) - 32 * kGemmWarps, 0};
      fused_reduce_group<256, false>(args, cv, ep, g, abort_flag, sigq);
      if (g.tid == g.nthreads - 1) signal_drain(sigq, cv, ep, args.err, tmo);
    }
  }
  if constexpr (FUSED) {
    if (warp < kGemmWarps) {
      // The six GEMM warps, done with the GEMM, join the reduction.
      dev::named_bar_sync(kLateBar, 32 * kGemmWarps);
      if (*abort_flag == 0) {
        dev::griddep_wait();
        const ReduceGroup g{kLateBar, 32 * kGemmWarps, static_cast<int>(threadIdx.x), 1};
        fused_reduce_group<256, false>(args, cv, *epoch_slot, g, abort_flag, sigq);
      }
    }
  }

  __syncthreads();
  dev::cluster_sync();  // the pair is done with both CTAs' TMEM and shared memory
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc2(tmem_base, T::kTmemCols);
  }
  if constexpr (FUSED) {
    epoch = *epoch_slot;
    if (threadIdx.x == 0) {
      uint32_t* c = dev::ctrl_ptr(cv.base[cv.rank]);
      __threadfence();
      const uint32_t done = atomicAdd(c + 1, 1u);
      if (done == gridDim.x - 1) {
        c[1] = 0u;
        __threadfence();
        atomicExch(c, epoch);
      }
    }
  }
}

}  // namespace w8a8
