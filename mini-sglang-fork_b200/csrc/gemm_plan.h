// Tile-configuration planner of the W8A8 GEMM (host only, no CUDA calls, so
// it is unit-testable without a GPU through w8a8_gemm_plan()).
//
// Variants (BM = 128 rows of the "wide" operand per tile, BK = 128):
//   1: normal, BN = 256   2: normal, BN = 128
//   3..6: weight-stationary (swap), BN = 16 / 32 / 64 / 128 token columns
//   7: CTA pairs with the 2-SM MMA, 256 x 256 blocks (two 128 x 256 tiles),
//      whole blocks in grid-stride order over SM pairs (prefill shapes); a
//      last wave at most half full is split along K over the idle pairs
// Schedule: stream-K over G persistent CTAs (one per SM by default).  The
// k-block iterations of all tiles are split evenly between the CTAs; tiles cut
// by a CTA boundary are finished through the workspace (two int32 tile slots
// per CTA plus one counter per tile).  Without room for that workspace the
// ranges are rounded to whole tiles (no cut tiles, no workspace).
#pragma once

#include <cstddef>
#include <cstdint>

namespace w8a8 {

struct GemmPlan {
  int variant;
  int bn;
  bool swap;
  int tiles_w, tiles_n, num_tiles;
  int kblocks;
  int dp_tiles;             // leading whole tiles in grid-stride order
  int gran;                 // stream-K granularity in k blocks: 1 or kblocks
  long long units;          // (num_tiles - dp_tiles) * kblocks / gran
  int sk_ctas;              // CTAs sharing the stream-K part: min(grid, units), >= 1
  int grid;                 // persistent CTAs
  int wide_fast;
  bool cut_tiles;           // some tile is shared by two or more CTAs
  size_t ws_counter_bytes;  // tile counters at the workspace head
  size_t ws_bytes;          // total workspace bytes needed (0 if no tile is cut)
  int pair_split;           // pair variant: the last, partial wave's blocks split this many ways along K (0: none)
};

constexpr int kMaxVariant = 7;

inline int variant_bn(int v) {
  static const int kBn[] = {0, 256, 128, 16, 32, 64, 128, 256};
  return (v >= 1 && v <= kMaxVariant) ? kBn[v] : 0;
}

inline bool variant_swap(int v) { return v >= 3 && v <= 6; }

// Share of SM pairs kept busy when 256 x 256 blocks are dealt whole.
inline int64_t pair_blocks(int64_t M, int64_t N) { return ((M + 255) / 256) * ((N + 255) / 256); }

inline const char* plan_error(int rc) {
  switch (rc) {
    case 1: return "invalid shape or variant";
    default: return "unknown planning error";
  }
}

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// The workspace starts with a counter region of fixed size, whatever the
// shape, so counters left at zero by one call are never overlapped by another
// call's partial tiles.
constexpr int kMaxCounterTiles = 65536;
constexpr size_t kCounterBytes = static_cast<size_t>(kMaxCounterTiles) * 4;

// Counter words a plan uses at the workspace head: one per tile, or for the
// pair variant one per 128-row half of each 256 x 256 block.
inline size_t plan_counter_words(const GemmPlan& p) {
  if (p.variant == 7) return 2 * static_cast<size_t>((p.tiles_w + 1) / 2) * p.tiles_n;
  return static_cast<size_t>(p.num_tiles);
}

// Returns 0 and fills *p; nonzero on invalid input.  ctas_req = 0 picks one
// CTA per SM.
inline int plan_gemm(int64_t M, int64_t N, int64_t K, int variant, int ctas_req, size_t ws_avail, int nsm,
                     GemmPlan* p) {
  if (M <= 0 || N <= 0 || K <= 0 || nsm <= 0 || ctas_req < 0) return 1;
  int v = variant;
  if (v == 0) {
    if (M <= 16) {
      v = 3;
    } else if (M <= 32) {
      v = 4;
    } else if (M <= 64) {
      v = 5;
    } else if (M > 128 && pair_blocks(M, N) * 2 >= nsm / 2) {
      // 256 x 256 blocks on SM pairs whenever at least half of the pairs get
      // a block: the pair kernel moves 128 int8 MACs per staged operand byte
      // (128 x 256 tiles: 85), which outweighs its coarser tail.
      v = 7;
    } else {
      // 128 x 128 tiles + stream-K: measured faster than 128 x 256 tiles at
      // every shape the pair kernel does not take
      v = 2;
    }
  }
  if (v < 1 || v > kMaxVariant) return 1;
  p->variant = v;
  p->bn = variant_bn(v);
  p->swap = variant_swap(v);
  const int64_t rows_w = p->swap ? N : M;
  const int64_t rows_n = p->swap ? M : N;
  p->tiles_w = static_cast<int>((rows_w + 127) / 128);
  p->tiles_n = static_cast<int>((rows_n + p->bn - 1) / p->bn);
  p->num_tiles = p->tiles_w * p->tiles_n;
  p->kblocks = static_cast<int>((K + 127) / 128);
  p->pair_split = 0;
  if (v == 7) {
    // whole 256 x 256 blocks over SM pairs in grid-stride order
    const int64_t pairs = static_cast<int64_t>((p->tiles_w + 1) / 2) * p->tiles_n;
    int64_t clusters = ctas_req > 0 ? ctas_req / 2 : nsm / 2;
    if (clusters > nsm / 2) clusters = nsm / 2;
    if (clusters < 1) clusters = 1;
    if (clusters > pairs) clusters = pairs;
    p->grid = static_cast<int>(2 * clusters);
    p->dp_tiles = p->num_tiles;
    p->gran = p->kblocks;
    p->units = 0;
    p->sk_ctas = 1;
    p->cut_tiles = false;
    p->ws_counter_bytes = 0;
    p->ws_bytes = 0;
    p->wide_fast = (rows_w <= rows_n) ? 1 : 0;
    // A last wave at most half full (e.g. 320 blocks on 74 pairs: 4 full
    // waves and 24 blocks) is split along K: each of its blocks goes to
    // `split` pairs, each taking a contiguous share of the k blocks (at least
    // 8), and the pair holding the first share adds the others' int32 shares
    // (one slot of 128 x 256 int32 per CTA, one counter per 128-row half).
    const int64_t rem = pairs % clusters;
    if (pairs >= clusters && rem > 0 && 2 * rem <= clusters) {
      int split = static_cast<int>(clusters / rem);
      if (split > 4) split = 4;
      while (split > 1 && p->kblocks / split < 8) --split;
      const size_t need = kCounterBytes + static_cast<size_t>(2 * clusters) * 128 * 256 * 4;
      if (split >= 2 && need <= ws_avail && 2 * pairs <= kMaxCounterTiles) {
        p->pair_split = split;
        p->cut_tiles = true;
        p->ws_counter_bytes = kCounterBytes;
        p->ws_bytes = need;
      }
    }
    return 0;
  }
  const long long total_iters = static_cast<long long>(p->num_tiles) * p->kblocks;
  long long g = ctas_req > 0 ? (ctas_req < nsm ? ctas_req : nsm) : nsm;
  if (g > total_iters) g = total_iters;
  // Whole tiles for every CTA first, stream-K over the rest.  With a
  // remainder and at least one full wave, the last full wave joins the
  // stream-K region ("two-tile" stream-K): every CTA then takes between one
  // and two tiles of iterations, so no tile is cut between more than two CTAs
  // and a fix-up adds at most one other CTA's partial.
  const long long full_waves = p->num_tiles / g;
  const bool remainder = (p->num_tiles % g) != 0;
  p->dp_tiles = static_cast<int>((remainder && full_waves >= 1 ? full_waves - 1 : full_waves) * g);
  const long long iters = static_cast<long long>(p->num_tiles - p->dp_tiles) * p->kblocks;

  // Does an even split of the remaining iterations over min(g, iters) CTAs
  // cut any tile?
  const long long gs = iters < g ? iters : g;
  bool cut = false;
  for (long long c = 1; c < gs && !cut; ++c) cut = ((c * iters / gs) % p->kblocks) != 0;
  const size_t need = kCounterBytes + 2 * static_cast<size_t>(g) * 128 * p->bn * 4;
  if (cut && (need > ws_avail || p->num_tiles > kMaxCounterTiles)) {
    // no room to finish cut tiles: whole-tile ranges (plain data-parallel waves)
    p->gran = p->kblocks;
    p->dp_tiles = static_cast<int>(full_waves * g);
    if (g > p->num_tiles) {
      g = p->num_tiles;
      p->dp_tiles = p->num_tiles;
    }
    cut = false;
  } else {
    p->gran = 1;
  }
  p->grid = static_cast<int>(g);
  p->units = (static_cast<long long>(p->num_tiles - p->dp_tiles) * p->kblocks) / p->gran;
  p->sk_ctas = static_cast<int>(p->units < g ? (p->units > 0 ? p->units : 1) : g);
  p->cut_tiles = cut;
  p->ws_counter_bytes = cut ? kCounterBytes : 0;
  p->ws_bytes = cut ? need : 0;
  // Keep the smaller operand L2-resident: walk it fastest.
  p->wide_fast = (rows_w <= rows_n) ? 1 : 0;
  return 0;
}

}  // namespace w8a8
