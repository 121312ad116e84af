// Kernel 2: W8A8 GEMM on 5th-generation tensor cores (tcgen05, kind::i8),
// optionally fused with the row-parallel all-reduce over NVLink peer memory.
//
//   C[M, N] = bf16( (f32(sum_k A[m,k] * B[n,k]) * sa[m]) * sb[n] + bias[n] )
//
// A: int8 activations [M, K] (K contiguous); B: int8 weight [N, K]
// (nn.Linear layout, K contiguous).  Both operands are K-major, which is the
// layout tcgen05 reads natively.
//
// Structure (one persistent CTA per SM, 6 warps, warp-specialised):
//   warp 0      TMA producer: 2-D tiled bulk-tensor loads of a 128-row tile of
//               the "wide" operand and a BN-row tile of the "narrow" operand,
//               128 K-bytes per stage, 128-byte swizzle, STAGES-deep mbarrier
//               ring.
//   warp 1      owns the TMEM allocation; lane 0 issues tcgen05.mma
//               (M=128, N=BN, K=32 per instruction, 4 per stage) into one of
//               two TMEM accumulators and commits stage releases and
//               accumulator-ready signals through tcgen05.commit.
//   warps 2-5   epilogue: tcgen05.ld of the int32 accumulator (warp w reads
//               TMEM lanes 32*(w%4)..+31), dequant in fp32 with separately
//               rounded multiplies, bf16 store; releases the accumulator so the
//               MMA of the next tile overlaps this epilogue.
//
// Orientation.  Normal: the 128-row side is A (tokens), the BN side is B
// (output channels).  Weight-stationary ("swap", small M): the 128-row side is
// B (output channels, filling the 128-lane MMA M slot), the BN side is the
// handful of tokens; the math is unchanged (C^T = B . A^T) and the epilogue
// writes C[m, n] with n along the 32 lanes of a warp.
//
// Schedule (hybrid data-parallel + stream-K).  With T tiles and G CTAs, whole
// tiles are dealt in grid-stride order first; when T is not a multiple of G,
// the last full wave is held back, and the k-block iterations of the held-back
// wave plus the remainder are laid end to end, CTA c taking the contiguous
// range [c*L/G, (c+1)*L/G) ("two-tile" stream-K: every CTA streams the same
// number of k blocks, between one and two tiles' worth, and no tile is cut
// between more than two CTAs).  A range cut inside a tile leaves a partial
// fragment: its int32 accumulator goes to a per-CTA workspace slot with
// coalesced 16-byte stores, the fragment's arrival is counted on the tile's
// counter, and the last arriving fragment adds the other slot(s) to its own
// accumulator, still in TMEM (int32, exact in any order), dequantises, writes
// the tile and resets the counter, so the counters stay zero between calls.
//
// Fused all-reduce (row-parallel layers, FUSED = true).  As each bf16 partial
// tile leaves the epilogue it is pushed over NVLink into the peers' receive
// slots (tile-blocked, 512-byte coalesced pieces through a per-warp shared
// memory transpose): one-shot pushes the whole tile to every rank, two-shot
// pushes each row share to the rank that owns it; then the tile's ready flag is
// raised on every rank.  After its GEMM work, CTA b reduces the tiles t with
// t % G == b from local memory only: it waits for every rank's ready(t), sums
// the ranks' partials in rank order (fp32, one rounding) into C, and, two-shot,
// pushes its reduced share into every peer's gather slot, raises gathered(t),
// then copies the other ranks' shares from its own gather slot.  Waits happen
// only after all of the CTA's own signals, so no wait can block a signal
// another rank needs.
//
// Every mbarrier / flag wait is bounded (%globaltimer); on expiry the CTA
// raises a shared abort flag and the device error word, drains its in-flight
// TMA loads and MMAs (bounded too), frees TMEM and exits.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdint>

#include "comm_dev.cuh"
#include "sm100.cuh"

namespace w8a8 {

struct GemmArgs {
  const float* sa;            // [M] activation scales
  const float* sb;            // [N] weight scales
  const __nv_bfloat16* bias;  // [N] or null
  __nv_bfloat16* C;           // [M, N] bf16 output (row stride ldc)
  int32_t* c_i32;             // [M, N] int32 accumulator output or null
  int32_t* ws;                // stream-K partial slots, 2 per CTA
  uint32_t* counters;         // per-tile fragment arrival counters (zeroed)
  unsigned int* err;          // device error word
  long long timeout_ns;
  int M, N, K;
  int ldc;
  int tiles_w, tiles_n;       // tiles along the 128-row side / the BN side
  int num_tiles, kblocks;
  int dp_tiles;               // leading tiles done whole, in grid-stride order
  int gran;                   // stream-K granularity in k blocks (1, or kblocks = whole tiles)
  long long units;            // (num_tiles - dp_tiles) * kblocks / gran
  int sk_ctas;                // CTAs sharing the stream-K part: min(G, units), >= 1
  int wide_fast;              // raster: 1 = consecutive tiles walk the 128-row side
  int vec_scales;             // 1: sb (and bias) are 16-byte aligned, read 8 columns per load
  // gate_up + SiLU epilogue (pair kernel, plain mode): silu_i = I > 0 when the
  // weight is [gate (I rows); up (I rows)] and C receives y = bf16(silu(g) * u)
  // [M, I] (ldc = I); amax[m] collects max |y| of row m as float bits.
  int silu_i;
  uint32_t* amax;
  // pair kernel: the blocks of the last, partial wave are split pair_split
  // ways along K (0: every block whole); slots in ws, counters per 128-row half
  int pair_split;
};

// Shared memory of the fused epilogue and reduction state (FusedState, below).
constexpr int kSignalBytes = 1088;

template <int BN, int STAGES, bool SWAP>
struct GemmTraits {
  static constexpr int kBM = 128;
  static constexpr int kBK = 128;  // bytes of K per stage (= int8 elements)
  static constexpr int kMmaK = 32;
  static constexpr int kTileWBytes = kBM * kBK;
  static constexpr int kTileNBytes = BN * kBK;
  static constexpr int kStageBytes = kTileWBytes + kTileNBytes;
  static constexpr int kAccCols = BN;
  static constexpr int kChunk = BN < 32 ? BN : 32;  // TMEM columns per epilogue load
  static constexpr int kChunks = BN / kChunk;
  static constexpr int kTmemCols = (2 * BN) <= 32 ? 32 : (2 * BN) <= 64 ? 64 : (2 * BN) <= 128 ? 128
                                   : (2 * BN) <= 256 ? 256 : 512;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kStagingBytes = 4 * 2048;  // fused epilogue: 2 KB transpose buffer per warp
  static constexpr int kTileOutBytes = 128 * BN * 2;  // one tile's bf16 block in a receive slot
  // The hand-over state exists only in fused mode.  The staging buffer serves
  // both modes in the normal orientation (the epilogue transposes each chunk
  // through it so that stores are row-contiguous); weight-stationary tiles
  // store token rows directly, so a plain swap launch has no staging.
  // double-buffered scales of the tile's BN columns (fp32): weight scales and
  // bias (normal orientation), token scales (weight-stationary)
  static constexpr int kScaleBytes = SWAP ? 2 * BN * 4 : 2 * 2 * BN * 4;
  // offset of the scales: a plain weight-stationary launch has no staging
  static constexpr int scale_offset(bool fused) { return (SWAP && !fused) ? 0 : kStagingBytes; }
  static constexpr int kSmemBytesPlain =
      1024 + STAGES * kStageBytes + kBarrierBytes + (SWAP ? 0 : kStagingBytes) + kScaleBytes;
  static constexpr int kSmemBytes =
      1024 + STAGES * kStageBytes + kBarrierBytes + kStagingBytes + kScaleBytes + kSignalBytes;
  static constexpr int smem_bytes(bool fused) { return fused ? kSmemBytes : kSmemBytesPlain; }
  static constexpr uint32_t kIdesc = dev::idesc_i8(kBM, BN);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "MMA N");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void tile_coords(const GemmArgs& a, int tile, int& tw, int& tn) {
  if (a.wide_fast) {
    tw = tile % a.tiles_w;
    tn = tile / a.tiles_w;
  } else {
    tn = tile % a.tiles_n;
    tw = tile / a.tiles_n;
  }
}

// Hybrid schedule: tiles [0, dp_tiles) are whole-tile work dealt out in
// grid-stride order (CTA c takes c, c+G, ...), which keeps the tiles in flight
// together adjacent for L2 reuse; the k-block iterations of the remaining
// tiles are split evenly (stream-K).  sk_begin(c) is the first stream-K
// iteration of CTA c (global iteration index).
// Only the first sk_ctas = min(G, units) CTAs take stream-K work, so every one
// of them has a non-empty range.
__device__ __forceinline__ long long sk_begin(const GemmArgs& a, int c) {
  const int cc = c < a.sk_ctas ? c : a.sk_ctas;
  return static_cast<long long>(a.dp_tiles) * a.kblocks + (static_cast<long long>(cc) * a.units / a.sk_ctas) * a.gran;
}

// The CTA whose stream-K range holds iteration x: max{c : sk_begin(c) <= x}.
__device__ __forceinline__ int sk_owner(const GemmArgs& a, long long x) {
  const long long rel = x - static_cast<long long>(a.dp_tiles) * a.kblocks;
  return static_cast<int>(((rel / a.gran + 1) * a.sk_ctas - 1) / a.units);
}

// Iterates the fragments (tile, [kb0, kb1)) of this CTA: its whole tiles of
// the data-parallel part, then its stream-K range.
struct FragmentWalk {
  int dp_tile, dp_tiles;
  long long it, end;
  int kblocks;
  __device__ __forceinline__ FragmentWalk(const GemmArgs& a)
      : dp_tile(blockIdx.x), dp_tiles(a.dp_tiles), it(sk_begin(a, blockIdx.x)),
        end(sk_begin(a, blockIdx.x + 1)), kblocks(a.kblocks) {}
  __device__ __forceinline__ bool next(int& tile, int& kb0, int& kb1) {
    if (dp_tile < dp_tiles) {
      tile = dp_tile;
      kb0 = 0;
      kb1 = kblocks;
      dp_tile += gridDim.x;
      return true;
    }
    if (it >= end) return false;
    tile = static_cast<int>(it / kblocks);
    kb0 = static_cast<int>(it - static_cast<long long>(tile) * kblocks);
    const long long left = end - it;
    kb1 = left < kblocks - kb0 ? kb0 + static_cast<int>(left) : kblocks;
    it += kb1 - kb0;
    return true;
  }
};

__device__ __forceinline__ float dequant1(int32_t acc, float sa, float sb) {
  return __fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sb);
}

// Weight-stationary dequantisation of CH accumulators of TMEM row `n` (a
// weight row): the values are tokens col0..col0+CH-1, with the row's scale
// and bias from registers and the tokens' scales from shared memory, staged
// before the accumulator wait (no global load after it).
template <int CH, class Emit2>
__device__ __forceinline__ void store_chunk_swap(const GemmArgs& a, int n, int col0, float sbn, float bnv,
                                                 const float* sas, const uint32_t (&v)[32], Emit2&& emit2) {
  if (n >= a.N) return;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int m = col0 + j;
    if (m >= a.M) break;
    float y = dequant1(static_cast<int32_t>(v[j]), sas[j], sbn);
    if (a.bias) y = __fadd_rn(y, bnv);
    emit2(m, n, __float2bfloat16_rn(y));
    if (a.c_i32) a.c_i32[static_cast<int64_t>(m) * a.N + n] = static_cast<int32_t>(v[j]);
  }
}


// Per-warp staging of one 32-row x 32-column bf16 chunk of the output tile
// (2 KB): row r (the lane that computed it), 16-byte piece g (8 columns) at
// slot r * 4 + (g ^ ((r >> 1) & 3)).  The XOR spreads both access patterns
// over distinct banks -- the writes (one lane per row, one piece each) and the
// reads (four lanes per row, so that a warp store covers 8 whole 64-byte row
// segments instead of 32 scattered 16-byte pieces).
__device__ __forceinline__ int stage_slot(int r, int g) { return r * 4 + (g ^ ((r >> 1) & 3)); }

// Write a staged chunk (rows m_base.., columns n0..n0+31) to C with
// row-contiguous 16-byte stores; rows >= M and columns >= n_limit are skipped.
__device__ __forceinline__ void store_staged_chunk(const GemmArgs& a, const uint4* stg, int lane, int m_base,
                                                   int n0, int n_limit) {
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = j * 8 + (lane >> 2), g = lane & 3;
    const int m = m_base + r, n = n0 + g * 8;
    if (m < a.M && n < n_limit)
      *reinterpret_cast<uint4*>(a.C + static_cast<size_t>(m) * a.ldc + n) = stg[stage_slot(r, g)];
  }
  __syncwarp();  // the next chunk may overwrite the staging buffer
}
__device__ __forceinline__ void store_staged_chunk(const GemmArgs& a, const uint4* stg, int lane, int m_base,
                                                   int n0) {
  store_staged_chunk(a, stg, lane, m_base, n0, a.N);
}

// The dequantised bf16 values of one 32-column chunk of row m, packed eight
// to a uint4 -- the same arithmetic as store_chunk_smem.
__device__ __forceinline__ void dequant_pack32(const GemmArgs& a, float sam, const float* sbs, const float* bss,
                                               const uint32_t (&v)[32], uint4 (&out)[4]) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float4 s0 = reinterpret_cast<const float4*>(sbs)[g * 2];
    const float4 s1 = reinterpret_cast<const float4*>(sbs)[g * 2 + 1];
    const float sb[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&out[g]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float y0 = dequant1(static_cast<int32_t>(v[g * 8 + 2 * j]), sam, sb[2 * j]);
      float y1 = dequant1(static_cast<int32_t>(v[g * 8 + 2 * j + 1]), sam, sb[2 * j + 1]);
      if (a.bias) {
        y0 = __fadd_rn(y0, bss[g * 8 + 2 * j]);
        y1 = __fadd_rn(y1, bss[g * 8 + 2 * j + 1]);
      }
      h[j] = __floats2bfloat162_rn(y0, y1);
    }
  }
}

// SiLU epilogue: stage the scales (and bias) of a block's 128 gate columns
// (tn * 128 ..) at [0, 128) and of the matching up columns (I + tn * 128 ..)
// at [128, 256), the order of the block's accumulator columns; thread t takes
// columns 2t and 2t + 1.  Returns row m's activation scale (0 past M).
__device__ __forceinline__ float stage_tile_scales_silu(const GemmArgs& a, int tn, int t, bool real, int m,
                                                        float* sbs, float* bss) {
  if (t < 128) {
    const int c = 2 * t;
    const int n = c < 128 ? tn * 128 + c : a.silu_i + tn * 128 + (c - 128);
    float2 sv = make_float2(0.0f, 0.0f), bv = make_float2(0.0f, 0.0f);
    if (real) {
      sv = make_float2(__ldg(a.sb + n), __ldg(a.sb + n + 1));
      if (a.bias) bv = make_float2(__bfloat162float(a.bias[n]), __bfloat162float(a.bias[n + 1]));
    }
    sbs[c] = sv.x;
    sbs[c + 1] = sv.y;
    bss[c] = bv.x;
    bss[c + 1] = bv.y;
  }
  return (real && m < a.M) ? __ldg(a.sa + m) : 0.0f;
}

// Normal orientation, with the tile's weight scales (and bias) staged in
// shared memory by the epilogue before it waited for the accumulator:
// dequantise one 32-column chunk of row m (activation scale sam) and emit it.
// Reading the scales as shared-memory broadcasts instead of global loads keeps
// an L2 round trip per chunk off the epilogue's critical path.
template <class Emit16>
__device__ __forceinline__ void store_chunk_smem(const GemmArgs& a, int m, int col0, float sam, const float* sbs,
                                                 const float* bss, const uint32_t (&v)[32], Emit16&& emit16) {
  if (m >= a.M) return;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int n = col0 + g * 8;
    if (n >= a.N) break;  // N % 16 == 0: granules are either fully in or out
    const float4 s0 = reinterpret_cast<const float4*>(sbs)[g * 2];
    const float4 s1 = reinterpret_cast<const float4*>(sbs)[g * 2 + 1];
    const float sb[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    uint4 pk;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float y0 = dequant1(static_cast<int32_t>(v[g * 8 + 2 * j]), sam, sb[2 * j]);
      float y1 = dequant1(static_cast<int32_t>(v[g * 8 + 2 * j + 1]), sam, sb[2 * j + 1]);
      if (a.bias) {
        y0 = __fadd_rn(y0, bss[g * 8 + 2 * j]);
        y1 = __fadd_rn(y1, bss[g * 8 + 2 * j + 1]);
      }
      h[j] = __floats2bfloat162_rn(y0, y1);
    }
    emit16(m, n, pk);
    if (a.c_i32) {
      int4* dst = reinterpret_cast<int4*>(a.c_i32 + static_cast<int64_t>(m) * a.N + n);
      dst[0] = make_int4(v[g * 8 + 0], v[g * 8 + 1], v[g * 8 + 2], v[g * 8 + 3]);
      dst[1] = make_int4(v[g * 8 + 4], v[g * 8 + 5], v[g * 8 + 6], v[g * 8 + 7]);
    }
  }
}

// Stage the weight scales (and bias, 0 without one) of output columns
// [n0, n0 + cols) into sbs / bss (cols <= 2 * nthreads), thread t taking
// columns 2t and 2t + 1; and return row m's activation scale (0 past M).
__device__ __forceinline__ float stage_tile_scales(const GemmArgs& a, int n0, int cols, int t, bool real, int m,
                                                   float* sbs, float* bss) {
  if (2 * t < cols) {
    const int n = n0 + 2 * t;
    float2 sv = make_float2(0.0f, 0.0f), bv = make_float2(0.0f, 0.0f);
    if (real && n < a.N) {  // N even: the pair is in or out together
      sv = make_float2(__ldg(a.sb + n), __ldg(a.sb + n + 1));
      if (a.bias) bv = make_float2(__bfloat162float(a.bias[n]), __bfloat162float(a.bias[n + 1]));
    }
    sbs[2 * t] = sv.x;
    sbs[2 * t + 1] = sv.y;
    bss[2 * t] = bv.x;
    bss[2 * t + 1] = bv.y;
  }
  return (real && m < a.M) ? __ldg(a.sa + m) : 0.0f;
}

// Fused mode: rank of the owner of row (m - m0) of a tile of hm rows when the
// rows are shared out evenly between the ranks (two-shot).
__device__ __forceinline__ int row_owner(int m, int m0, int hm, int world) {
  return ((m - m0 + 1) * world - 1) / hm;
}

// Output rectangle of a tile in C coordinates: rows [m0, m0+hm), columns
// [n0, n0+wn) with wn a multiple of 8.
template <int BN, bool SWAP>
__device__ __forceinline__ void tile_rect(const GemmArgs& a, int tile, int& m0, int& hm, int& n0, int& wn) {
  int tw, tn;
  tile_coords(a, tile, tw, tn);
  if (!SWAP) {
    m0 = tw * 128;
    hm = min(128, a.M - m0);
    n0 = tn * BN;
    wn = min(BN, a.N - n0);
  } else {
    m0 = tn * BN;
    hm = min(BN, a.M - m0);
    n0 = tw * 128;
    wn = min(128, a.N - n0);
  }
}

// Fused mode adds two reducer warps (warps 6-7) to the six GEMM warps.  They
// reduce the CTA's tiles across the ranks while the GEMM warps are still
// producing later tiles; once the GEMM warps are done they join in as a second
// group, and the two groups claim the CTA's tiles from shared counters.  The
// last thread of each group also raises the ready flags of the tiles the
// epilogue has pushed (FusedState).
constexpr int kGemmWarps = 6;
constexpr int kReduceThreads = 64;
template <bool FUSED>
constexpr int gemm_block_threads() { return 32 * kGemmWarps + (FUSED ? kReduceThreads : 0); }

// Threads of the CTA doing reduction work together.
struct ReduceGroup {
  int bar;       // named barrier of the group
  int nthreads;  // multiple of 32
  int tid;       // 0 .. nthreads-1
  int slot;      // the group's claim broadcast word
};
constexpr int kReducerBar = 2;  // warps 6-7
constexpr int kLateBar = 3;     // warps 0-5 once the GEMM work is done

// Shared state of the fused epilogue and the reduction.
//
// Hand-over of pushed tiles from the epilogue to the flag-raising threads.
// Raising a ready flag needs a system-scope fence that waits until the CTA's
// earlier peer stores have drained over NVLink (many microseconds when every
// SM is pushing), so the epilogue does not do it: it moves straight on to the
// next tile.  Epilogue thread 0 appends the tile id and publishes the count
// with a CTA-scope release after the epilogue's barrier; a reduce thread
// acquires the count, fences at system scope and stores the flags, which
// orders the whole epilogue's pushes before them (causality is transitive
// through the barrier and the CTA-scope release / acquire).  Raising a flag
// twice stores the same epoch again, so concurrent raisers are harmless.
constexpr int kSignalRing = 256;
struct FusedState {
  int tiles[kSignalRing];
  uint32_t count;     // tiles handed over
  uint32_t closed;    // 1 once the epilogue has handed over its last tile
  uint32_t taken;     // tiles whose flags are raised (monotonic)
  uint32_t claim[2];  // next tile index of this CTA to reduce, per phase
  int bcast[2];       // claimed index, broadcast within each group
};
static_assert(sizeof(FusedState) <= kSignalBytes, "fused state");

__device__ __forceinline__ void init_fused_state(FusedState* q) {
  q->count = 0u;
  q->closed = 0u;
  q->taken = 0u;
  q->claim[0] = q->claim[1] = 0u;
}

// Epilogue thread 0: append `tile` (n = tiles appended so far).  Bounded wait
// while the ring is full; false on timeout.
__device__ __forceinline__ bool signal_handover(FusedState* q, uint32_t& n, int tile, unsigned int* err,
                                                long long tmo) {
  if (n - dev::ld_acquire_cta(&q->taken) >= static_cast<uint32_t>(kSignalRing)) {
    const uint64_t t0 = dev::globaltimer_ns();
    while (n - dev::ld_acquire_cta(&q->taken) >= static_cast<uint32_t>(kSignalRing)) {
      if (dev::globaltimer_ns() - t0 > static_cast<uint64_t>(tmo)) {
        if (err) atomicOr(err, kErrGemmWait);
        return false;
      }
      __nanosleep(64);
    }
  }
  reinterpret_cast<volatile int*>(q->tiles)[n % kSignalRing] = tile;
  dev::st_release_cta(&q->count, ++n);
  return true;
}

// Raise ready(t) on every rank for each handed-over tile not yet raised.
// Returns true once the epilogue has closed the queue and every tile is raised.
__device__ __forceinline__ bool signal_pump(FusedState* q, const CommView& cv, uint32_t epoch) {
  const uint32_t closed = dev::ld_acquire_cta(&q->closed);  // before count: a closed queue's count is final
  const uint32_t n = dev::ld_acquire_cta(&q->count);
  const uint32_t d = dev::ld_acquire_cta(&q->taken);
  if (n != d) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (uint32_t i = d; i < n; ++i) {
      const int tile = reinterpret_cast<volatile int*>(q->tiles)[i % kSignalRing];
      for (int r = 0; r < cv.world; ++r) {
        uint32_t* f = dev::flag_ptr(cv.base[r], 0, tile, cv.rank);
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
      }
    }
    asm volatile("red.release.cta.shared::cta.max.u32 [%0], %1;" ::"r"(dev::smem_u32(&q->taken)), "r"(n)
                 : "memory");
  }
  return closed != 0;
}

// After its own work, a group's last thread keeps raising this CTA's ready
// flags until the epilogue closes the queue (bounded by tmo).
__device__ __forceinline__ void signal_drain(FusedState* q, const CommView& cv, uint32_t epoch, unsigned int* err,
                                             long long tmo) {
  const uint64_t t0 = dev::globaltimer_ns();
  for (uint32_t it = 0; !signal_pump(q, cv, epoch); ++it) {
    if ((it & 63u) == 63u && dev::globaltimer_ns() - t0 > static_cast<uint64_t>(tmo)) {
      if (err) atomicOr(err, kErrGemmWait);
      return;
    }
    __nanosleep(64);
  }
}

// The group waits (bounded) until every rank has raised flag (phase, slot) of
// call `epoch`; threads t < world poll rank t's flag and the group's last
// thread keeps this CTA's own ready flags moving meanwhile.  False on timeout
// or when the CTA's GEMM gave up.
__device__ __forceinline__ bool group_wait(const CommView& cv, int phase, int slot, uint32_t epoch,
                                           const ReduceGroup& g, FusedState* q, const volatile int* abort_flag) {
  const uint32_t* f = g.tid < cv.world ? dev::flag_ptr(cv.base[cv.rank], phase, slot, g.tid) : nullptr;
  const uint64_t t0 = dev::globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    const bool mine = f == nullptr || dev::ld_acquire_sys(f) == epoch;
    if (g.tid == g.nthreads - 1) signal_pump(q, cv, epoch);
    bool fail = false;
    if (!mine && (it & 15u) == 15u) {
      if (*abort_flag != 0) {
        fail = true;
      } else if (dev::globaltimer_ns() - t0 > static_cast<uint64_t>(cv.timeout_ns)) {
        if (cv.err) atomicOr(cv.err, kErrCommWait);
        uint32_t* c = dev::ctrl_ptr(cv.base[cv.rank]);
        c[2] = (static_cast<uint32_t>(phase) << 24) | static_cast<uint32_t>(slot);
        c[3] = static_cast<uint32_t>(g.tid);
        fail = true;
      }
    }
    if (dev::named_bar_or(g.bar, g.nthreads, fail)) return false;
    if (!dev::named_bar_or(g.bar, g.nthreads, !mine)) return true;
    if (it > 4) __nanosleep(32);
  }
}

// The group claims the next index from `counter` (same value in every thread).
__device__ __forceinline__ int group_claim(uint32_t* counter, const ReduceGroup& g, int* bcast) {
  if (g.tid == 0) *bcast = static_cast<int>(atomicAdd(counter, 1u));
  dev::named_bar_sync(g.bar, g.nthreads);
  const int i = *reinterpret_cast<volatile int*>(bcast);
  dev::named_bar_sync(g.bar, g.nthreads);  // every thread has read it before the next claim
  return i;
}

// Receive-slot layout of one tile (block of 128 x BN bf16 at t * kTileOutBytes):
//   normal: [chunk c = 0..BN/32)[row 0..127][32 columns]  (64-byte row pieces,
//           so the 128 rows of a chunk are 8 KB contiguous)
//   swap:   [token 0..BN)[128 channels]
// Vector (8 bf16) v of the block maps to tile row r / column col (in C).
template <int BN, bool SWAP>
__device__ __forceinline__ void block_vec_rc(int v, int& r, int& col) {
  if constexpr (!SWAP) {
    const int c = v >> 9;          // 512 vectors per chunk
    const int rem = v & 511;
    r = rem >> 2;
    col = c * 32 + (rem & 3) * 8;
  } else {
    r = v >> 4;                    // 16 vectors per token
    col = (v & 15) * 8;
  }
}

// Sum vectors `vec` (a batch of up to 8 / W block vectors per thread) of a
// tile block over the world receive slots of this rank (every rank's partial,
// pushed here by the epilogues): fp32 in rank order, one bf16 rounding; the
// result goes to C and, with push_gather, into every other rank's gather slot
// at the same block offset.  All loads are local; W = world at compile time
// keeps 8 independent 16-byte loads in flight per thread (W = 0: any world).
template <int W, int BN, bool SWAP, class VecOf>
__device__ __forceinline__ void reduce_block(const GemmArgs& a, const CommView& cv, uint32_t epoch, int t, int m0,
                                             int n0, int nvec, VecOf vec_of, int tid, int nt, bool push_gather) {
  constexpr int V = W > 0 ? 8 / W : 1;
  constexpr int TILE = 128 * BN * 2;
  const int world = W > 0 ? W : cv.world;
  const char* slot0 = dev::recv_slot(cv, cv.rank, 0, epoch) + static_cast<size_t>(t) * TILE;
  const size_t sstride = cv.slot_bytes;
  for (int base = tid; base < nvec; base += nt * V) {
    uint4 buf[V][W > 0 ? W : 1];
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int i = base + j * nt;
      if (i < nvec) {
        const size_t off = static_cast<size_t>(vec_of(i)) * 16;
        if constexpr (W > 0) {
#pragma unroll
          for (int q = 0; q < W; ++q) buf[j][q] = dev::ld_volatile_v4(slot0 + q * sstride + off);
        } else {
          buf[j][0] = dev::ld_volatile_v4(slot0 + off);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int i = base + j * nt;
      if (i >= nvec) continue;
      const int v = vec_of(i);
      const size_t off = static_cast<size_t>(v) * 16;
      float acc[8];
      {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&buf[j][0]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[2 * e] = f.x;
          acc[2 * e + 1] = f.y;
        }
      }
      for (int q = 1; q < world; ++q) {
        uint4 raw;
        if constexpr (W > 0) {
          raw = buf[j][q];
        } else {
          raw = dev::ld_volatile_v4(slot0 + q * sstride + off);
        }
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[2 * e] = __fadd_rn(acc[2 * e], f.x);
          acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], f.y);
        }
      }
      uint4 o;
      __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) ho[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
      int r, col;
      block_vec_rc<BN, SWAP>(v, r, col);
      const int m = m0 + r, n = n0 + col;
      if (m < a.M && n < a.N) *reinterpret_cast<uint4*>(a.C + static_cast<size_t>(m) * a.ldc + n) = o;
      if (push_gather) {
        for (int d = 0; d < world; ++d) {
          if (d == cv.rank) continue;
          *reinterpret_cast<uint4*>(dev::gather_slot(cv, d, epoch) + static_cast<size_t>(t) * TILE + off) = o;
        }
      }
    }
  }
}

template <int BN, bool SWAP, class VecOf>
__device__ __forceinline__ void reduce_block_any_world(const GemmArgs& a, const CommView& cv, uint32_t epoch, int t,
                                                       int m0, int n0, int nvec, VecOf vec_of, int tid, int nt,
                                                       bool push_gather) {
  switch (cv.world) {
    case 2: reduce_block<2, BN, SWAP>(a, cv, epoch, t, m0, n0, nvec, vec_of, tid, nt, push_gather); break;
    case 4: reduce_block<4, BN, SWAP>(a, cv, epoch, t, m0, n0, nvec, vec_of, tid, nt, push_gather); break;
    case 8: reduce_block<8, BN, SWAP>(a, cv, epoch, t, m0, n0, nvec, vec_of, tid, nt, push_gather); break;
    default: reduce_block<0, BN, SWAP>(a, cv, epoch, t, m0, n0, nvec, vec_of, tid, nt, push_gather); break;
  }
}

// Reduction of the tiles this CTA owns (t % gridDim.x == blockIdx.x) from the
// partials the epilogues of every rank pushed into this rank's receive slots,
// by one group; groups claim the tiles one at a time.
//   one-shot: wait for every rank's ready(t), reduce the whole tile into C.
//   two-shot: wait for ready(t), reduce this rank's row share into C and push
//             it into every other rank's gather slot, raise gathered(t);
//             then (second claim pass) wait for every rank's gathered(t) and
//             copy their shares from the local gather slot into C.
// Returns false if a flag wait timed out or the CTA's GEMM gave up (uniformly
// across the group).
template <int BN, bool SWAP>
__device__ bool fused_reduce_group(const GemmArgs& a, const CommView& cv, uint32_t epoch, const ReduceGroup& g,
                                   const volatile int* abort_flag, FusedState* q) {
  constexpr int TILE = 128 * BN * 2;
  constexpr int NV = TILE / 16;  // vectors per tile block
  const int G = static_cast<int>(gridDim.x), b = static_cast<int>(blockIdx.x);
  const int owned = (a.num_tiles - b + G - 1) / G;  // tiles b, b + G, ...
  for (;;) {
    const int i = group_claim(&q->claim[0], g, &q->bcast[g.slot]);
    if (i >= owned) break;
    const int t = b + i * G;
    if (!group_wait(cv, 0, t, epoch, g, q, abort_flag)) return false;
    int m0, hm, n0, wn;
    tile_rect<BN, SWAP>(a, t, m0, hm, n0, wn);
    if (!cv.two_shot) {
      reduce_block_any_world<BN, SWAP>(a, cv, epoch, t, m0, n0, NV, [](int v) { return v; }, g.tid, g.nthreads,
                                       false);
    } else if (cv.nvls) {
      // This rank's row share of tile t, summed over every rank's partial in
      // the switch (multimem.ld_reduce), written to C and multicast into every
      // rank's gather region; kInFlight reductions in flight per thread (each
      // is a round trip through the switch).
      const int r0 = (hm * cv.rank) / cv.world, r1 = (hm * (cv.rank + 1)) / cv.world;
      const int per_chunk = (r1 - r0) * 4;
      const int nv = per_chunk * (BN / 32);
      const char* mc_p = dev::nv_partials(cv, cv.mc_base, epoch) + static_cast<size_t>(t) * TILE;
      char* mc_g = dev::nv_gather(cv, cv.mc_base, epoch) + static_cast<size_t>(t) * TILE;
      dev::fence_proxy_alias();  // the peers' partials were written through their unicast mappings
      constexpr int kInFlight = 8;
      for (int base = g.tid; base < nv; base += kInFlight * g.nthreads) {
        uint4 sum[kInFlight];
        int vv[kInFlight];
#pragma unroll
        for (int j = 0; j < kInFlight; ++j) {
          const int i = base + j * g.nthreads;
          vv[j] = (i / per_chunk) * 512 + r0 * 4 + (i % per_chunk);
          if (i < nv) sum[j] = dev::mm_ld_reduce_bf16x8(mc_p + static_cast<size_t>(vv[j]) * 16);
        }
#pragma unroll
        for (int j = 0; j < kInFlight; ++j) {
          if (base + j * g.nthreads >= nv) continue;
          int r, col;
          block_vec_rc<BN, SWAP>(vv[j], r, col);
          const int m = m0 + r, n = n0 + col;
          if (m < a.M && n < a.N) *reinterpret_cast<uint4*>(a.C + static_cast<size_t>(m) * a.ldc + n) = sum[j];
          dev::mm_st_bf16x8(mc_g + static_cast<size_t>(vv[j]) * 16, sum[j]);
        }
      }
      dev::fence_proxy_alias();  // this thread's multicast stores before the group's gathered flag
      dev::named_bar_sync(g.bar, g.nthreads);
      dev::signal_peers(cv, 1, t, epoch, g.tid);
    } else {
      // rows [r0, r1) of every chunk: (r1 - r0) * 4 vectors per chunk
      const int r0 = (hm * cv.rank) / cv.world, r1 = (hm * (cv.rank + 1)) / cv.world;
      const int per_chunk = (r1 - r0) * 4;
      auto vec_of = [=](int v) { return (v / per_chunk) * 512 + r0 * 4 + (v % per_chunk); };
      reduce_block_any_world<BN, SWAP>(a, cv, epoch, t, m0, n0, per_chunk * (BN / 32), vec_of, g.tid, g.nthreads,
                                       true);
      dev::named_bar_sync(g.bar, g.nthreads);
      dev::signal_peers(cv, 1, t, epoch, g.tid);
    }
  }
  if (!cv.two_shot) return true;
  for (;;) {
    const int i = group_claim(&q->claim[1], g, &q->bcast[g.slot]);
    if (i >= owned) break;
    const int t = b + i * G;
    if (!group_wait(cv, 1, t, epoch, g, q, abort_flag)) return false;
    int m0, hm, n0, wn;
    tile_rect<BN, SWAP>(a, t, m0, hm, n0, wn);
    const char* from = (cv.nvls ? dev::nv_gather(cv, cv.nv_local, epoch) : dev::gather_slot(cv, cv.rank, epoch)) +
                       static_cast<size_t>(t) * TILE;
    if (cv.nvls) dev::fence_proxy_alias();  // the shares arrived through the multicast mapping
    // every vector outside this rank's own row share
    const int r0 = (hm * cv.rank) / cv.world, r1 = (hm * (cv.rank + 1)) / cv.world;
    for (int base = g.tid; base < NV; base += g.nthreads * 8) {
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = base + j * g.nthreads;
        int r, col;
        block_vec_rc<BN, SWAP>(k, r, col);
        if (k < NV && (r < r0 || r >= r1)) v[j] = dev::ld_volatile_v4(from + static_cast<size_t>(k) * 16);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = base + j * g.nthreads;
        int r, col;
        block_vec_rc<BN, SWAP>(k, r, col);
        const int m = m0 + r, n = n0 + col;
        if (k < NV && (r < r0 || r >= r1) && m < a.M && n < a.N)
          *reinterpret_cast<uint4*>(a.C + static_cast<size_t>(m) * a.ldc + n) = v[j];
      }
    }
  }
  return true;
}

template <int BN, int STAGES, bool SWAP, bool FUSED>
__global__ void __launch_bounds__(gemm_block_threads<FUSED>(), 1)
    w8a8_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_n,
                     const GemmArgs args, const CommView cv) {
  using T = GemmTraits<BN, STAGES, SWAP>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_w = smem;
  uint8_t* s_n = smem + STAGES * T::kTileWBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_n + STAGES * T::kTileNBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;
  volatile uint32_t* epoch_slot = reinterpret_cast<volatile uint32_t*>(last_flag + 1);
  uint8_t* staging = reinterpret_cast<uint8_t*>(bars) + T::kBarrierBytes;  // 16-byte aligned
  // [2][BN] sb, then [2][BN] bias (normal orientation); [2][BN] sa (weight-stationary)
  float* scale_stage = reinterpret_cast<float*>(staging + T::scale_offset(FUSED));
  FusedState* sigq = reinterpret_cast<FusedState*>(staging + T::kStagingBytes + T::kScaleBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    if constexpr (FUSED) init_fused_state(sigq);  // plain launches carry no staging / hand-over region
    for (int s = 0; s < STAGES; ++s) {
      dev::mbar_init(dev::smem_u32(full + s), 1);
      dev::mbar_init(dev::smem_u32(empty + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(dev::smem_u32(acc_full + s), 1);
      dev::mbar_init(dev::smem_u32(acc_empty + s), 128);
    }
    dev::mbar_init(dev::smem_u32(drain), 1);
    *abort_flag = 0;
    *last_flag = 0;
    dev::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    dev::prefetch_tmap(&tm_w);
    dev::prefetch_tmap(&tm_n);
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
  // This grid is resident (one CTA per SM): the next kernel may start its
  // prologue now; it waits for our completion before touching our data.
  dev::griddep_launch();

  // Fused mode: the call's epoch (published by the previous call's last CTA,
  // so read after griddep_wait) selects the data half; partial tiles go there
  // instead of C.
  uint32_t epoch = 0;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      // Weight-stationary tiles stream each weight byte once (evict first) and
      // re-read the few token rows (evict last); the normal orientation reuses
      // both operands across tiles and keeps the default policy.
      const uint64_t pol_w = dev::policy_evict_first();
      const uint64_t pol_n = dev::policy_evict_last();
      // The weight operand never depends on the previous kernel: the weight
      // half of the first stages is requested before griddep_wait.
      auto load_weights = [&](int stg, int kb, int tw, int tn) {
        const uint32_t fb = dev::smem_u32(full + stg);
        if constexpr (SWAP) {
          dev::tma_load_2d_hint(dev::smem_u32(s_w + stg * T::kTileWBytes), &tm_w, fb, kb * T::kBK, tw * T::kBM,
                                pol_w);
        } else {
          dev::tma_load_2d(dev::smem_u32(s_n + stg * T::kTileNBytes), &tm_n, fb, kb * T::kBK, tn * BN);
        }
      };
      auto load_tokens = [&](int stg, int kb, int tw, int tn) {
        const uint32_t fb = dev::smem_u32(full + stg);
        if constexpr (SWAP) {
          dev::tma_load_2d_hint(dev::smem_u32(s_n + stg * T::kTileNBytes), &tm_n, fb, kb * T::kBK, tn * BN,
                                pol_n);
        } else {
          dev::tma_load_2d(dev::smem_u32(s_w + stg * T::kTileWBytes), &tm_w, fb, kb * T::kBK, tw * T::kBM);
        }
      };
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      FragmentWalk walk(args);
      int tile, kb0, kb1;
      bool have = walk.next(tile, kb0, kb1);
      int pre = 0;
      if (have) {
        int tw, tn;
        tile_coords(args, tile, tw, tn);
        pre = min(STAGES, kb1 - kb0);
        for (int i = 0; i < pre; ++i) {
          dev::mbar_expect_tx(dev::smem_u32(full + i), T::kStageBytes);
          load_weights(i, kb0 + i, tw, tn);
        }
      }
      dev::griddep_wait();
      for (; ok && have; have = walk.next(tile, kb0, kb1)) {
        int tw, tn;
        tile_coords(args, tile, tw, tn);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (pre > 0) {
            // stage already armed with its weight half before griddep_wait
            --pre;
            load_tokens(stage, kb, tw, tn);
          } else {
            if (!dev::mbar_wait(dev::smem_u32(empty + stage), phase ^ 1u, abort_flag, args.err,
                                kErrGemmWait, tmo)) {
              ok = false;
              break;
            }
            dev::mbar_expect_tx(dev::smem_u32(full + stage), T::kStageBytes);
            load_weights(stage, kb, tw, tn);
            load_tokens(stage, kb, tw, tn);
          }
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
      dev::griddep_wait();
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      FragmentWalk walk(args);
      int tile, kb0, kb1;
      while (ok && walk.next(tile, kb0, kb1)) {
        if (!dev::mbar_wait(dev::smem_u32(acc_empty + acc), acc_phase ^ 1u, abort_flag, args.err,
                            kErrGemmWait, tmo)) {
          break;
        }
        dev::tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * T::kAccCols);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!dev::mbar_wait(dev::smem_u32(full + stage), phase, abort_flag, args.err, kErrGemmWait,
                              tmo)) {
            ok = false;
            break;
          }
          dev::tc_fence_after();
          const uint64_t dw = dev::sdesc_k_sw128(dev::smem_u32(s_w + stage * T::kTileWBytes));
          const uint64_t dn = dev::sdesc_k_sw128(dev::smem_u32(s_n + stage * T::kTileNBytes));
#pragma unroll
          for (int k = 0; k < T::kBK / T::kMmaK; ++k) {
            const uint64_t off = static_cast<uint64_t>((k * T::kMmaK) >> 4);
            dev::mma_i8(d_tmem, dw + off, dn + off, T::kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
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
  } else if (warp < kGemmWarps) {
    // ------------------------------------------------------------ epilogue
    dev::griddep_wait();
    if constexpr (FUSED) epoch = dev::ld_relaxed_gpu(dev::ctrl_ptr(cv.base[cv.rank])) + 1u;
    // Where a finished tile's bf16 values go.  Plain: C.  Fused: this rank's
    // receive slot (tile-blocked layout) on every rank (one-shot) or on the
    // rank owning the row (two-shot) -- remote stores over NVLink that overlap
    // the next tile's MMAs.  Normal-orientation values are transposed through
    // a 2 KB per-warp staging buffer so that every store instruction of a warp
    // writes 512 contiguous bytes; weight-stationary tiles (M <= 64, always
    // one-shot) store token rows of 64 contiguous bytes per warp directly.
    const size_t my_slot = kHeaderBytes + static_cast<size_t>(epoch & 1u) * cv.half_bytes +
                           static_cast<size_t>(cv.rank) * cv.slot_bytes;
    uint4* stg = reinterpret_cast<uint4*>(staging + (warp & 3) * 2048);
    int cur_m0 = 0, cur_hm = 1, cur_n0 = 0, cur_tile = 0;
    // normal orientation, both modes: [row in warp][16-byte piece] through the
    // staging buffer (chunks start at multiples of 32 columns)
    auto emit16 = [&](int, int n, const uint4& val) { stg[stage_slot(lane, (n & 31) >> 3)] = val; };
    auto emit2 = [&](int m, int n, __nv_bfloat16 val) {
      if constexpr (!FUSED) {
        args.C[static_cast<size_t>(m) * args.ldc + n] = val;
      } else {
        const size_t off = static_cast<size_t>(cur_tile) * T::kTileOutBytes +
                           (static_cast<size_t>(m - cur_m0) * 128 + (n - cur_n0)) * 2;
        for (int d = 0; d < cv.world; ++d) *reinterpret_cast<__nv_bfloat16*>(cv.base[d] + my_slot + off) = val;
      }
    };
    // Fused normal orientation: after a chunk's values are staged, the warp
    // pushes its 32 rows x 64 bytes (2 KB contiguous in the tile block).
    auto push_chunk = [&](int c) {
      if constexpr (FUSED && !SWAP) {
        __syncwarp();
        const size_t blk = static_cast<size_t>(cur_tile) * T::kTileOutBytes + static_cast<size_t>(c) * 8192 +
                           static_cast<size_t>(warp & 3) * 2048;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = lane + 32 * j;  // 16-byte piece k of the warp's 2 KB
          const int r = (warp & 3) * 32 + (k >> 2);
          if (r >= cur_hm) continue;    // padding rows of a bottom tile are never read: not pushed
          const uint4 val = stg[stage_slot(k >> 2, k & 3)];
          const size_t off = blk + static_cast<size_t>(k) * 16;
          if (cv.nvls) {
            // NVLS: the partial stays in this rank's buffer; the owner reads it through the switch
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
    const int quarter = warp & 3;
    // plain normal orientation: chunk c of tile (tw, tn) goes to C from the staging buffer
    auto out_chunk = [&](int tw, int tn, int c) {
      if constexpr (FUSED) {
        push_chunk(c);
      } else if constexpr (!SWAP) {
        store_staged_chunk(args, stg, lane, tw * T::kBM + quarter * 32, tn * BN + c * T::kChunk);
      }
    };
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int et = threadIdx.x - 64;  // 0..127 among the epilogue threads
    const long long my_begin = sk_begin(args, blockIdx.x);
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t sig_n = 0;
    bool aborted = false;
    FragmentWalk walk(args);
    int tile, kb0, kb1;
    uint32_t frag = 0;
    while (walk.next(tile, kb0, kb1)) {
      int tw, tn;
      tile_coords(args, tile, tw, tn);
      if constexpr (FUSED) {
        int wn_;
        tile_rect<BN, SWAP>(args, tile, cur_m0, cur_hm, cur_n0, wn_);
        cur_tile = tile;
      }
      const int row = tw * T::kBM + row_in_tile;
      // Normal orientation: the tile's scales into shared memory (buffer
      // frag & 1) before waiting; the barrier below publishes them, and no
      // warp still reads this buffer (it belonged to fragment frag - 2).
      float* sbs = scale_stage + (frag & 1u) * BN;
      float* bss = scale_stage + 2 * BN + (frag & 1u) * BN;
      float sam = 0.0f;
      // weight-stationary: this thread's weight-row scale and bias in
      // registers, the tile's token scales staged in shared memory (sbs)
      float sbn = 0.0f, bnv = 0.0f;
      if constexpr (!SWAP) {
        sam = stage_tile_scales(args, tn * BN, BN, et, true, row, sbs, bss);
      } else {
        if (et < BN) {
          const int m = tn * BN + et;
          sbs[et] = m < args.M ? __ldg(args.sa + m) : 0.0f;
        }
        if (row < args.N) {
          sbn = __ldg(args.sb + row);
          if (args.bias) bnv = __bfloat162float(args.bias[row]);
        }
      }
      ++frag;
      const bool ok = dev::mbar_wait(dev::smem_u32(acc_full + acc), acc_phase, abort_flag, args.err,
                                     kErrGemmWait, tmo);
      if (dev::named_bar_or(1, 128, !ok)) {  // uniform exit of all epilogue threads
        aborted = true;
        break;
      }
      dev::tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_base + static_cast<uint32_t>(acc * T::kAccCols);
      // normal orientation from the staged scales, weight-stationary as before
      auto dequant_chunk = [&](int c, const uint32_t (&v)[32]) {
        if constexpr (!SWAP) {
          store_chunk_smem(args, row, tn * BN + c * T::kChunk, sam, sbs + c * T::kChunk, bss + c * T::kChunk, v,
                           emit16);
        } else {
          store_chunk_swap<T::kChunk>(args, row, tn * BN + c * T::kChunk, sbn, bnv, sbs + c * T::kChunk, v, emit2);
        }
      };
      bool wrote_tile = true;
      if (kb0 == 0 && kb1 == args.kblocks) {
        // whole tile in this CTA: dequantise straight from TMEM, the next
        // chunk's columns loading while this one is processed
        uint32_t vn[32];
        dev::tmem_ld<T::kChunk>(t_acc, vn);
#pragma unroll 1
        for (int c = 0; c < T::kChunks; ++c) {
          uint32_t v[32];
          dev::tmem_wait_ld(vn);
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = vn[q];
          if (c + 1 < T::kChunks) {
            dev::tmem_ld<T::kChunk>(t_acc + (c + 1) * T::kChunk, vn);
          } else {
            dev::tc_fence_before();
            dev::mbar_arrive(dev::smem_u32(acc_empty + acc));
          }
          dequant_chunk(c, v);
          out_chunk(tw, tn, c);
        }
      } else {
        // Partial fragment of a tile cut between CTAs c_first..c_last.  The
        // tile's owner is c_first: it holds the tile's first k-blocks at the
        // END of its stream-K range, so it is the last to finish the tile,
        // while every other CTA holds the tile as its FIRST fragment (or as
        // its whole range) and never waits for anything.  A non-owner parks its
        // int32 values in its slot (layout [chunk][warp][column group j][lane]
        // [4 columns]: a thread moves its chunk as kChunk/4 16-byte stores, each
        // warp instruction covers 512 contiguous bytes) and counts itself in
        // the tile's counter; the owner waits (bounded) for the count, adds the
        // slots to its own values, still in TMEM, and writes the tile.  The
        // owner thus never parks its own share nor takes the counter atomic:
        // its tail after the last MMA is one counter read and one batch of
        // slot loads.
        const long long tile_begin = static_cast<long long>(tile) * args.kblocks;
        const int c_first = sk_owner(args, tile_begin);
        const int c_last = sk_owner(args, tile_begin + args.kblocks - 1);
        const int me = static_cast<int>(blockIdx.x);
        constexpr int kVec = T::kChunk / 4;
        if (me != c_first) {
          const int slot = 2 * me + (my_begin < tile_begin ? 1 : 0);
          int4* wslot = reinterpret_cast<int4*>(args.ws + static_cast<int64_t>(slot) * (T::kBM * BN));
#pragma unroll 1
          for (int c = 0; c < T::kChunks; ++c) {
            uint32_t v[32];
            dev::tmem_ld<T::kChunk>(t_acc + c * T::kChunk, v);
            dev::tmem_wait_ld(v);
            int4* p = wslot + ((c * 4 + quarter) * kVec) * 32 + lane;
#pragma unroll
            for (int j = 0; j < kVec; ++j)
              __stcg(p + j * 32, make_int4(static_cast<int>(v[4 * j]), static_cast<int>(v[4 * j + 1]),
                                      static_cast<int>(v[4 * j + 2]), static_cast<int>(v[4 * j + 3])));
          }
          dev::tc_fence_before();
          dev::mbar_arrive(dev::smem_u32(acc_empty + acc));
          // one fence after the barrier orders every epilogue thread's slot
          // stores (ordered before it by the barrier) before the count
          dev::named_bar_sync(1, 128);
          if (et == 0) {
            __threadfence();
            atomicAdd(args.counters + tile, 1u);
          }
          wrote_tile = false;
        } else {
          bool counted = true;
          if (et == 0)
            counted = dev::wait_counter(args.counters + tile, static_cast<uint32_t>(c_last - c_first), abort_flag,
                                        args.err, kErrGemmWait, tmo);
          // et == 0's acquire of the count, then the barrier, order every
          // epilogue thread's slot loads (L2, .cg) after the other CTAs' stores
          if (dev::named_bar_or(1, 128, !counted)) {
            aborted = true;
            break;
          }
          // The slots' loads are issued in batches of kBatch CTAs, all in
          // flight together (a tile of a decode GEMM spans up to ~5 CTAs).
          constexpr int kBatch = kVec <= 4 ? 4 : 2;
#pragma unroll 1
          for (int c = 0; c < T::kChunks; ++c) {
            uint32_t v[32];
            dev::tmem_ld<T::kChunk>(t_acc + c * T::kChunk, v);
            dev::tmem_wait_ld(v);
#pragma unroll 1
            for (int cta0 = c_first + 1; cta0 <= c_last; cta0 += kBatch) {
              int4 q[kBatch][kVec];
#pragma unroll
              for (int b = 0; b < kBatch; ++b) {
                const int cta = cta0 + b;
                if (cta > c_last) continue;
                const int s = 2 * cta + (sk_begin(args, cta) < tile_begin ? 1 : 0);
                const int4* p = reinterpret_cast<const int4*>(args.ws + static_cast<int64_t>(s) * (T::kBM * BN)) +
                                ((c * 4 + quarter) * kVec) * 32 + lane;
#pragma unroll
                for (int j = 0; j < kVec; ++j) q[b][j] = __ldcg(p + j * 32);
              }
#pragma unroll
              for (int b = 0; b < kBatch; ++b) {
                if (cta0 + b > c_last) continue;
#pragma unroll
                for (int j = 0; j < kVec; ++j) {  // two's-complement sums, as int32
                  v[4 * j] += static_cast<uint32_t>(q[b][j].x);
                  v[4 * j + 1] += static_cast<uint32_t>(q[b][j].y);
                  v[4 * j + 2] += static_cast<uint32_t>(q[b][j].z);
                  v[4 * j + 3] += static_cast<uint32_t>(q[b][j].w);
                }
              }
            }
            if (c == T::kChunks - 1) {
              dev::tc_fence_before();
              dev::mbar_arrive(dev::smem_u32(acc_empty + acc));
            }
            dequant_chunk(c, v);
            out_chunk(tw, tn, c);
          }
          if (et == 0) args.counters[tile] = 0u;
        }
      }
      if constexpr (FUSED) {
        if (wrote_tile) {
          // every epilogue thread's pushes of the tile precede the hand-over
          dev::named_bar_sync(1, 128);
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
      // Reduce this CTA's tiles across the ranks as every rank's partial of
      // each lands, overlapping the GEMM of the later tiles; raise this CTA's
      // own ready flags meanwhile and afterwards.
      dev::griddep_wait();
      const uint32_t ep = dev::ld_relaxed_gpu(dev::ctrl_ptr(cv.base[cv.rank])) + 1u;
      const ReduceGroup g{kReducerBar, kReduceThreads, static_cast<int>(threadIdx.x) - 32 * kGemmWarps, 0};
      fused_reduce_group<BN, SWAP>(args, cv, ep, g, abort_flag, sigq);
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
        fused_reduce_group<BN, SWAP>(args, cv, *epoch_slot, g, abort_flag, sigq);
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem_base, T::kTmemCols);
  }
  if constexpr (FUSED) {
    epoch = *epoch_slot;
    // The last CTA of the call publishes the epoch for the next call.
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
