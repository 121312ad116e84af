// Tile-configuration planner of the W8A8 GEMM (host only, no CUDA calls, so
// it is unit-testable without a GPU through w8a8_gemm_plan()).
//
// Variants (BM = 128 rows of the "wide" operand per tile, BK = 128):
//   1: normal, BN = 256   2: normal, BN = 128
//   3..6: weight-stationary (swap), BN = 16 / 32 / 64 / 128 token columns
// Split-K factor: the smallest-penalty factor maximising the share of busy
// CTAs in the last round of the persistent schedule.
#pragma once

#include <cstddef>
#include <cstdint>

namespace w8a8 {

struct GemmPlan {
  int variant;
  int bn;
  bool swap;
  int tiles_w, tiles_n, num_tiles;
  int kblocks, splits, kb_per_split;
  int units, grid;
  int wide_fast;
  size_t ws_counter_bytes;  // tile counters at the workspace head
  size_t ws_bytes;          // total workspace bytes needed (0 if splits == 1)
};

inline int variant_bn(int v) {
  static const int kBn[] = {0, 256, 128, 16, 32, 64, 128};
  return (v >= 1 && v <= 6) ? kBn[v] : 0;
}

inline bool variant_swap(int v) { return v >= 3; }

inline const char* plan_error(int rc) {
  switch (rc) {
    case 1: return "invalid shape or variant";
    case 2: return "split-K workspace too small for the requested split factor";
    default: return "unknown planning error";
  }
}

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Returns 0 and fills *p; nonzero on invalid input.
inline int plan_gemm(int64_t M, int64_t N, int64_t K, int variant, int splits_req, size_t ws_avail, int nsm,
                     GemmPlan* p) {
  if (M <= 0 || N <= 0 || K <= 0 || nsm <= 0) return 1;
  int v = variant;
  if (v == 0) {
    if (M <= 16) {
      v = 3;
    } else if (M <= 32) {
      v = 4;
    } else if (M <= 64) {
      v = 5;
    } else {
      const int64_t tiles256 = ((M + 127) / 128) * ((N + 255) / 256);
      v = tiles256 >= nsm ? 1 : 2;
    }
  }
  if (v < 1 || v > 6) return 1;
  p->variant = v;
  p->bn = variant_bn(v);
  p->swap = variant_swap(v);
  const int64_t rows_w = p->swap ? N : M;
  const int64_t rows_n = p->swap ? M : N;
  p->tiles_w = static_cast<int>((rows_w + 127) / 128);
  p->tiles_n = static_cast<int>((rows_n + p->bn - 1) / p->bn);
  p->num_tiles = p->tiles_w * p->tiles_n;
  p->kblocks = static_cast<int>((K + 127) / 128);

  auto ws_need = [&](int s) -> size_t {
    if (s <= 1) return 0;
    const size_t counters = round_up(static_cast<size_t>(p->num_tiles) * 4, 256);
    return counters + static_cast<size_t>(p->num_tiles) * 128 * p->bn * 4;
  };

  int s = 1;
  if (splits_req > 0) {
    s = splits_req < p->kblocks ? splits_req : p->kblocks;
    if (s > 1 && ws_need(s) > ws_avail) return 2;
  } else {
    // Each split keeps >= 4 K blocks (512 bytes of K) so the pipeline fills.
    const int smax = p->kblocks / 4 < 16 ? p->kblocks / 4 : 16;
    double best = -1.0;
    for (int c = 1; c <= (smax > 1 ? smax : 1); ++c) {
      if (c > 1 && ws_need(c) > ws_avail) break;
      const int64_t units = static_cast<int64_t>(p->num_tiles) * c;
      const int64_t rounds = (units + nsm - 1) / nsm;
      const double eff = static_cast<double>(units) / static_cast<double>(rounds * nsm);
      const double score = eff - 0.01 * (c - 1);
      if (score > best + 1e-9) {
        best = score;
        s = c;
      }
    }
  }
  p->kb_per_split = (p->kblocks + s - 1) / s;
  p->splits = (p->kblocks + p->kb_per_split - 1) / p->kb_per_split;
  p->units = p->num_tiles * p->splits;
  p->grid = p->units < nsm ? p->units : nsm;
  // Keep the smaller operand L2-resident: walk it fastest.
  p->wide_fast = (rows_w <= rows_n) ? 1 : 0;
  p->ws_counter_bytes = p->splits > 1 ? round_up(static_cast<size_t>(p->num_tiles) * 4, 256) : 0;
  p->ws_bytes = ws_need(p->splits);
  return 0;
}

}  // namespace w8a8
