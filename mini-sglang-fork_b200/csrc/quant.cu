// Kernel 1: per-token symmetric absmax int8 quantiser, and its fusion with
// SiLU*mul (the silu_and_mul step between gate_up and down in GatedMLP,
// M/models/utils.py:44-50 and M/layers/activation.py:9-12 of mini-sglang).
//
// Every row is read once from HBM with 128-bit loads (or 1-D bulk copies),
// reduced to its absmax and quantised from on-chip storage, with 64-bit int8
// stores, so HBM traffic is exactly the algorithmic 2K (or 4I) bytes in and
// K (+4) bytes out per row.  Paths, by shape:
//   few rows (decode):        one row per cluster of 2..8 CTAs, the absmax
//                             meeting in distributed shared memory;
//   many plain rows          1, 2 or 4 warps per row in registers, no
//   (<= 16384 wide):          CTA-wide barrier, persistent grid;
//   otherwise (SiLU*mul       one CTA per row, in registers (<= 1024 vectors)
//   rows among them):         or staged in shared memory.
// Arithmetic convention (bit-exact with the CPU oracle):
//   s = fp32(amax) / 127.0f (IEEE divide), q = clamp(rint_even(x / s), +-127),
//   q = 0 for an all-zero row.
#include <cuda_bf16.h>

#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "silu.cuh"
#include "sm100.cuh"

namespace {

using namespace w8a8::act;  // SiLU*mul arithmetic and the bf16-pair absmax (silu.cuh)

constexpr int kRegThreads = 256;
constexpr int kSmemThreads = 512;
constexpr int kMaxVec = 4096;  // 16-byte vectors per row (K <= 32768)

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide max; every thread gets the result.
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float r = (lane < nw) ? red[lane] : 0.0f;
  return warp_max(r);
}

// q = clamp(rint_even(fl(v / s)), -127, 127) without an IEEE divide on the
// common path.  With Q = v/s exact (|Q| < 127.5), inv = fl(1/s) = (1/s)(1+d1)
// and p = v * inv taken UNROUNDED inside a fused multiply-add: p = Q(1+d1),
// |p - Q| <= 127.5 * 2^-24, and |fl(Q) - Q| <= 127.5 * 2^-24, so
// |p - fl(v/s)| <= 1.52e-5.  If rint(p) and rint(fl(v/s)) differed, a
// half-integer would lie within 1.52e-5 of p; so outside a 6.1e-5 band
// around half-integers rint(p) is exact, and inside it the quotient is taken
// with the IEEE divide.
//
// rint(p) itself uses no conversion-unit instruction (those issue at a
// quarter of the FP32 rate): for |p| < 2^22 the sum p + 1.5 * 2^23 lies in
// [2^23, 2^24), where the float spacing is 1, so t = fma(v, inv, 1.5 * 2^23)
// rounds p to the nearest integer, ties to even, and that integer is the low
// mantissa field of t: its low byte is the two's-complement int8 of rint(p)
// (bits(1.5 * 2^23) has a zero low byte), which the byte permutes pick
// directly.  -rint(p) = 1.5 * 2^23 - t exactly (Sterbenz), and
// f = fma(v, inv, -rint(p)) = p - rint(p) with one rounding (|f| <= 0.5, error
// <= 2^-25); p lies in the band exactly when |f| > 0.5 - 6.1e-5.
// Three packed f32x2 operations per two values and one branch per vector of
// eight, which sends a vector with any value in the band to the exact path,
// kept out of line so that it costs nothing when not taken.
// The clamp to +-127 never binds for finite inputs: |v| <= amax, so
// |p| <= 127 (1 + 2^-23) < 127.5 and rint(p) <= 127 (likewise for fl(v/s)).
// A scale below 2^-126 (a row whose absmax is below ~1.5e-36) may have an
// infinite reciprocal: such a row takes the IEEE divide for every value.
constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
constexpr float kBand = 0.5f - 6.1e-5f;

// Row scale of the quantiser: s = fl(amax / 127) (IEEE divide), inv = fl(1/s)
// (0 for an all-zero row, whose values are all zero and quantise to 0).
struct RowScale {
  float s;
  float inv;
  bool exact;  // s in (0, 2^-126): every value takes the IEEE divide
};

__device__ __forceinline__ RowScale row_scale(float amax) {
  RowScale r;
  r.s = __fdiv_rn(amax, 127.0f);
  r.inv = r.s > 0.0f ? __frcp_rn(r.s) : 0.0f;
  r.exact = r.s > 0.0f && r.s < 0x1p-126f;
  return r;
}

// Low bytes of four words, packed little-endian.
__device__ __forceinline__ uint32_t pack4_s8(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Every value through the IEEE divide (s > 0).
__device__ __noinline__ uint2 quant_vec8_div(uint4 raw, float s) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  uint32_t q[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 v = __bfloat1622float2(h[j]);
    const int a = __float2int_rn(__fdiv_rn(v.x, s)), b = __float2int_rn(__fdiv_rn(v.y, s));
    q[2 * j] = static_cast<uint32_t>(a < -127 ? -127 : (a > 127 ? 127 : a));
    q[2 * j + 1] = static_cast<uint32_t>(b < -127 ? -127 : (b > 127 ? 127 : b));
  }
  return make_uint2(pack4_s8(q[0], q[1], q[2], q[3]), pack4_s8(q[4], q[5], q[6], q[7]));
}

// Eight bf16 values -> eight int8 (packed little-endian in a uint2), without
// a branch: `band` is set when a value lies in the band (the result must then
// be replaced by quant_vec8_div's).  Two lanes at a time in packed f32x2
// arithmetic (each lane correctly rounded, as the scalar operations are).
__device__ __forceinline__ uint2 quant_vec8_fast(const uint4& raw, float inv, bool& band) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  const float2 inv2 = make_float2(inv, inv);
  const float2 rnd = make_float2(kRound, kRound), m1 = make_float2(-1.0f, -1.0f);
  uint32_t q[8];
  band = false;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 v = __bfloat1622float2(h[j]);
    const float2 t = __ffma2_rn(v, inv2, rnd);    // 1.5 * 2^23 + rint(p)
    const float2 nr = __ffma2_rn(t, m1, rnd);     // -rint(p), exact
    const float2 f = __ffma2_rn(v, inv2, nr);     // p - rint(p)
    band |= (fabsf(f.x) > kBand) | (fabsf(f.y) > kBand);
    q[2 * j] = __float_as_uint(t.x);
    q[2 * j + 1] = __float_as_uint(t.y);
  }
  return make_uint2(pack4_s8(q[0], q[1], q[2], q[3]), pack4_s8(q[4], q[5], q[6], q[7]));
}

__device__ __forceinline__ uint2 quant_vec8(const uint4& raw, const RowScale& rs) {
  if (rs.exact) return quant_vec8_div(raw, rs.s);
  bool band;
  const uint2 r = quant_vec8_fast(raw, rs.inv, band);
  return band ? quant_vec8_div(raw, rs.s) : r;
}

// max |x| over eight bf16 values, compared as bf16 pairs (exact: a maximum
// involves no rounding) and widened once.
__device__ __forceinline__ float vec8_absmax(const uint4& raw) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  const __nv_bfloat162 m = __hmax2(__hmax2(__habs2(h[0]), __habs2(h[1])), __hmax2(__habs2(h[2]), __habs2(h[3])));
  return fmaxf(__low2float(m), __high2float(m));
}

// bf16-only silu_and_mul (M/layers/activation.py:9-12): y = bf16(silu(g) * u)
// with no quantisation, element-parallel over [M, I] in 16-byte vectors, two
// vectors per thread with both loads in flight.  nv = I / 8 vectors per row.
constexpr int kEltThreads = 256;
__global__ void __launch_bounds__(kEltThreads) silu_mul_kernel(const __nv_bfloat16* __restrict__ in, int64_t ld,
                                                               __nv_bfloat16* __restrict__ y, int64_t ldy, int64_t nv,
                                                               int64_t total) {
  w8a8::dev::griddep_launch();  // the next kernel may start its prologue now (see rows_reg_kernel)
  w8a8::dev::griddep_wait();
  const int64_t step = static_cast<int64_t>(gridDim.x) * kEltThreads;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * kEltThreads + threadIdx.x; v < total; v += 2 * step) {
    uint4 g[2], u[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int64_t w = v + j * step;
      if (w < total) {
        const int64_t row = w / nv, c = w - row * nv;
        const uint4* src = reinterpret_cast<const uint4*>(in + row * ld);
        g[j] = __ldcs(src + c);
        u[j] = __ldcs(src + nv + c);
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int64_t w = v + j * step;
      if (w < total) {
        const int64_t row = w / nv, c = w - row * nv;
        reinterpret_cast<uint4*>(y + row * ldy)[c] = silu_mul_vec8(g[j], u[j]);
      }
    }
  }
}

// Row source: the plain bf16 row (SILU = false) or SiLU*mul of the gate / up
// halves of a gate_up row (SILU = true).
template <bool SILU>
struct RowSrc {
  const uint4* a;
  const uint4* b;
  __device__ __forceinline__ RowSrc(const __nv_bfloat16* base, int64_t row, int64_t ld, int width) {
    a = reinterpret_cast<const uint4*>(base + row * ld);
    b = reinterpret_cast<const uint4*>(base + row * ld + width);
  }
  // Issue the HBM load(s) of vector vi; combine() turns them into the value.
  // Kept apart so a thread can have all of its loads in flight before it
  // consumes the first one.
  __device__ __forceinline__ void fetch(int vi, uint4& x, uint4& y) const {
    x = __ldcs(a + vi);
    if constexpr (SILU) y = __ldcs(b + vi);
  }
  __device__ __forceinline__ uint4 combine(const uint4& x, const uint4& y) const {
    if constexpr (SILU) {
      return silu_mul_vec8(x, y);
    } else {
      return x;
    }
  }
};

// Register path: VPT vectors per thread held in registers.
template <int VPT, bool SILU>
__global__ void __launch_bounds__(kRegThreads) rows_reg_kernel(const __nv_bfloat16* __restrict__ in, int64_t ld,
                                                               int8_t* __restrict__ q, float* __restrict__ scale,
                                                               __nv_bfloat16* __restrict__ y_out, int width) {
  __shared__ float red[32];
  // Dependent launch is triggered before waiting for this kernel's own input:
  // the next kernel (typically a GEMM) may then start its prologue and weight
  // prefetch while the kernel before this one drains.  That is safe because
  // the next kernel waits for this grid's completion (which follows the wait
  // below) before it reads anything this grid writes.
  w8a8::dev::griddep_launch();
  w8a8::dev::griddep_wait();  // the row is the previous kernel's output
  const int64_t row = blockIdx.x;
  const int nvec = width >> 3;
  const RowSrc<SILU> src(in, row, ld, width);
  uint4 buf[VPT], aux[VPT];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) src.fetch(vi, buf[i], aux[i]);
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      buf[i] = src.combine(buf[i], aux[i]);
      amax = fmaxf(amax, vec8_absmax(buf[i]));
    }
  }
  amax = block_max(amax, red);
  const RowScale rs = row_scale(amax);
  uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(width));
  uint4* yr = y_out ? reinterpret_cast<uint4*>(y_out + row * static_cast<int64_t>(width)) : nullptr;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      qr[vi] = quant_vec8(buf[i], rs);
      if (SILU && yr) yr[vi] = buf[i];
    }
  }
  if (threadIdx.x == 0) scale[row] = rs.s;
}

// Shared-memory path: the row (or the SiLU*mul product) is staged on chip.
template <bool SILU>
__global__ void __launch_bounds__(kSmemThreads, 2) rows_smem_kernel(const __nv_bfloat16* __restrict__ in, int64_t ld,
                                                                 int8_t* __restrict__ q, float* __restrict__ scale,
                                                                 __nv_bfloat16* __restrict__ y_out, int width) {
  extern __shared__ uint4 stage[];
  __shared__ float red[32];
  w8a8::dev::griddep_launch();  // early trigger, as in rows_reg_kernel
  w8a8::dev::griddep_wait();    // the row is the previous kernel's output
  const int64_t row = blockIdx.x;
  const int nvec = width >> 3;
  const RowSrc<SILU> src(in, row, ld, width);
  float amax = 0.0f;
  int vi = threadIdx.x;
  // four independent loads in flight per thread
  for (; vi + 3 * kSmemThreads < nvec; vi += 4 * kSmemThreads) {
    uint4 x0, y0, x1, y1, x2, y2, x3, y3;
    src.fetch(vi, x0, y0);
    src.fetch(vi + kSmemThreads, x1, y1);
    src.fetch(vi + 2 * kSmemThreads, x2, y2);
    src.fetch(vi + 3 * kSmemThreads, x3, y3);
    const uint4 v0 = src.combine(x0, y0), v1 = src.combine(x1, y1);
    const uint4 v2 = src.combine(x2, y2), v3 = src.combine(x3, y3);
    stage[vi] = v0;
    stage[vi + kSmemThreads] = v1;
    stage[vi + 2 * kSmemThreads] = v2;
    stage[vi + 3 * kSmemThreads] = v3;
    amax = fmaxf(fmaxf(amax, vec8_absmax(v0)), fmaxf(vec8_absmax(v1), fmaxf(vec8_absmax(v2), vec8_absmax(v3))));
  }
  for (; vi < nvec; vi += kSmemThreads) {
    uint4 x, y;
    src.fetch(vi, x, y);
    const uint4 v = src.combine(x, y);
    stage[vi] = v;
    amax = fmaxf(amax, vec8_absmax(v));
  }
  amax = block_max(amax, red);  // its __syncthreads also publishes `stage`
  const RowScale rs = row_scale(amax);
  uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(width));
  uint4* yr = y_out ? reinterpret_cast<uint4*>(y_out + row * static_cast<int64_t>(width)) : nullptr;
  for (int i = threadIdx.x; i < nvec; i += kSmemThreads) {
    const uint4 v = stage[i];
    qr[i] = quant_vec8(v, rs);
    if (SILU && yr) yr[i] = v;
  }
  if (threadIdx.x == 0) scale[row] = rs.s;
}

// Warp-group path (the plain quantiser, many rows of at most 16384 values):
// G warps (G = 1, 2 or 4) own a row, lane t of the group (t < 32 G) holding
// vectors t + 32 G j, j < VPT, in registers, so every load is a coalesced
// 128-bit access and all of a lane's loads are in flight together.  Each
// group loops over rows g, g + groups, ... (persistent grid; a second row
// buffer in registers, to load the next row while one is computed, measured
// slower: the extra registers cost more resident groups than the overlap
// gains).  The row's absmax is a warp-shuffle reduction plus,
// for G > 1, one exchange through shared memory under a named barrier of the
// group's own warps: no CTA-wide barrier, so rows never wait for one another.
constexpr int kWarpThreads = 128;  // 4 warps: groups of G = 1, 2 or 4 (at most 2 groups take a barrier)
#ifndef W8A8_WARP_MAX_VPT
#define W8A8_WARP_MAX_VPT 10  // vectors per lane before G doubles
#endif

template <int VPT, int G, bool SCATTER = false>
__global__ void __launch_bounds__(kWarpThreads) rows_warp_kernel(const __nv_bfloat16* __restrict__ in, int64_t ld,
                                                                 int8_t* __restrict__ q, float* __restrict__ scale,
                                                                 int64_t M, int width,
                                                                 const int32_t* __restrict__ dst_rows = nullptr,
                                                                 int fanout = 0) {
  constexpr int kGroups = kWarpThreads / 32 / G;
  __shared__ float part[2][kWarpThreads / 32];  // per-warp maxima, by row parity
  w8a8::dev::griddep_launch();  // early trigger, as in rows_reg_kernel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / G;
  const int t = (warp % G) * 32 + lane;
  const int nvec = width >> 3;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kGroups;
  auto load = [&](int64_t r, uint4 (&dst)[VPT]) {
    const uint4* src = reinterpret_cast<const uint4*>(in + r * ld);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int vi = t + j * 32 * G;
      dst[j] = vi < nvec ? __ldcs(src + vi) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  w8a8::dev::griddep_wait();  // the rows are the previous kernel's output
  int it = 0;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kGroups + grp; row < M; row += stride, ++it) {
    uint4 v[VPT];
    load(row, v);
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.0f);
#pragma unroll
    for (int j = 0; j < VPT; ++j)
      if (t + j * 32 * G < nvec) m2 = vec8_absmax2(v[j], m2);
    float amax = warp_max(absmax_of(m2));
    if constexpr (G > 1) {
      float* p = &part[it & 1][grp * G];
      if (lane == 0) p[warp % G] = amax;
      // constant barrier ids (one per group of the CTA)
      if (kGroups == 1 || grp == 0)
        w8a8::dev::named_bar_sync(1, 32 * G);
      else
        w8a8::dev::named_bar_sync(2, 32 * G);
#pragma unroll
      for (int k = 0; k < G; ++k) amax = fmaxf(amax, p[k]);
    }
    const RowScale rs = row_scale(amax);
    if constexpr (SCATTER) {
      // mixture of experts: the row's int8 values and scale go to each of
      // the rows dst_rows[row * fanout + f] (skipped when negative)
      uint2 qv[VPT];
#pragma unroll
      for (int j = 0; j < VPT; ++j)
        if (t + j * 32 * G < nvec) qv[j] = quant_vec8(v[j], rs);
      for (int f = 0; f < fanout; ++f) {
        const int d = __ldg(dst_rows + row * fanout + f);
        if (d < 0) continue;
        uint2* qr = reinterpret_cast<uint2*>(q + static_cast<int64_t>(d) * width);
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const int vi = t + j * 32 * G;
          if (vi < nvec) qr[vi] = qv[j];
        }
        if (t == 0) scale[d] = rs.s;
      }
    } else {
      uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(width));
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int vi = t + j * 32 * G;
        if (vi < nvec) qr[vi] = quant_vec8(v[j], rs);
      }
      if (t == 0) scale[row] = rs.s;
    }
  }
}

// Quantiser with a known row absmax (the gate_up GEMM's SiLU epilogue has
// already folded every row's max |y| into amax, as float bits): no reduction
// is left, so the rows are quantised element-parallel.  Block (x, y) takes
// vectors [1024 x, 1024 x + 1024) of rows y, y + gridDim.y, ...; thread 0
// computes the row's scale once for the block.
constexpr int kAmaxThreads = 256;
constexpr int kAmaxVpt = 4;
__global__ void __launch_bounds__(kAmaxThreads) rows_amax_kernel(const __nv_bfloat16* __restrict__ y, int64_t ld,
                                                                 const uint32_t* __restrict__ amax,
                                                                 int8_t* __restrict__ q, float* __restrict__ scale,
                                                                 int64_t M, int width,
                                                                 const int32_t* __restrict__ num_blocks) {
  __shared__ float s_s, s_inv;
  __shared__ int s_exact;
  w8a8::dev::griddep_launch();  // early trigger, as in rows_reg_kernel
  w8a8::dev::griddep_wait();    // y and amax are the previous kernel's output
  if (num_blocks != nullptr) {  // rows in use: the 128-row blocks of the expert-sorted layout
    const int64_t used = static_cast<int64_t>(max(*num_blocks, 0)) * 128;
    if (used < M) M = used;
  }
  const int nvec = width >> 3;
  const int v0 = blockIdx.x * (kAmaxThreads * kAmaxVpt) + threadIdx.x;
  for (int64_t row = blockIdx.y; row < M; row += gridDim.y) {
    if (threadIdx.x == 0) {
      const RowScale rs = row_scale(__uint_as_float(amax[row]));
      s_s = rs.s;
      s_inv = rs.inv;
      s_exact = rs.exact ? 1 : 0;
      if (blockIdx.x == 0) scale[row] = rs.s;
    }
    __syncthreads();
    RowScale rs;
    rs.s = s_s;
    rs.inv = s_inv;
    rs.exact = s_exact != 0;
    const uint4* src = reinterpret_cast<const uint4*>(y + row * ld);
    uint2* dst = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(width));
    uint4 v[kAmaxVpt];
#pragma unroll
    for (int j = 0; j < kAmaxVpt; ++j) {
      const int i = v0 + j * kAmaxThreads;
      if (i < nvec) v[j] = __ldcs(src + i);
    }
#pragma unroll
    for (int j = 0; j < kAmaxVpt; ++j) {
      const int i = v0 + j * kAmaxThreads;
      if (i < nvec) dst[i] = quant_vec8(v[j], rs);
    }
    __syncthreads();  // the row's scale in shared memory is rewritten for the next row
  }
}

// Narrow rows (at most 256 vectors, K <= 2048) with a known absmax: one warp
// per row, every lane's VPT vector loads issued before any is converted, the
// warps of the grid striding over the rows (with num_blocks the row count is
// read on the device).  The same arithmetic as rows_amax_kernel.
constexpr int kAmaxWarpThreads = 256;
template <int VPT>
__global__ void __launch_bounds__(kAmaxWarpThreads) rows_amax_warp_kernel(
    const __nv_bfloat16* __restrict__ y, int64_t ld, const uint32_t* __restrict__ amax, int8_t* __restrict__ q,
    float* __restrict__ scale, int64_t M, int width, const int32_t* __restrict__ num_blocks) {
  w8a8::dev::griddep_launch();  // early trigger, as in rows_reg_kernel
  w8a8::dev::griddep_wait();    // y and amax are the previous kernel's output
  if (num_blocks != nullptr) {
    const int64_t used = static_cast<int64_t>(max(*num_blocks, 0)) * 128;
    if (used < M) M = used;
  }
  const int lane = threadIdx.x & 31;
  const int nvec = width >> 3;
  constexpr int kWarps = kAmaxWarpThreads / 32;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); row < M; row += stride) {
    const uint4* src = reinterpret_cast<const uint4*>(y + row * ld);
    uint4 v[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int vi = lane + 32 * j;
      if (vi < nvec) v[j] = __ldcs(src + vi);
    }
    const RowScale rs = row_scale(__uint_as_float(__ldg(amax + row)));
    uint2* dst = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(width));
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int vi = lane + 32 * j;
      if (vi < nvec) dst[vi] = quant_vec8(v[j], rs);
    }
    if (lane == 0) scale[row] = rs.s;
  }
}

// Cluster path (few rows): one row per cluster of C CTAs (C = the cluster
// size, 2..8), CTA c taking vectors [c*nvec/C, (c+1)*nvec/C) of the row in
// registers (VPT per thread).  Each CTA reduces its share's absmax, publishes
// it in its shared memory, and after a cluster barrier reads all C values
// through distributed shared memory (ld.shared::cluster), so every CTA
// quantises its share with the row's scale.  At decode sizes (M of 1..64)
// that spreads the row's HBM traffic and SiLU arithmetic over M*C SMs instead
// of M.  Same arithmetic as the one-CTA paths, so the results are identical.
__device__ __forceinline__ float cluster_max(float v, float* slot) {
  *slot = v;
  w8a8::dev::cluster_sync();  // every CTA's slot written (release / acquire at cluster scope)
  uint32_t n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  const uint32_t local = w8a8::dev::smem_u32(slot);
  float m = 0.0f;
  for (uint32_t r = 0; r < n; ++r) {
    float x;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(x) : "r"(w8a8::dev::mapa(local, r)) : "memory");
    m = fmaxf(m, x);
  }
  return m;
}

template <int VPT, bool SILU>
__global__ void __launch_bounds__(kRegThreads) rows_cluster_kernel(const __nv_bfloat16* __restrict__ in, int64_t ld,
                                                                   int8_t* __restrict__ q, float* __restrict__ scale,
                                                                   __nv_bfloat16* __restrict__ y_out, int width) {
  __shared__ float red[32];
  __shared__ float share_max;
  w8a8::dev::griddep_launch();  // early trigger, as in rows_reg_kernel
  w8a8::dev::griddep_wait();
  uint32_t c, nc;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(c));
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(nc));
  const int64_t row = blockIdx.x / nc;
  const int nvec = width >> 3;
  const int lo = static_cast<int>((static_cast<int64_t>(nvec) * c) / nc);
  const int hi = static_cast<int>((static_cast<int64_t>(nvec) * (c + 1)) / nc);
  const RowSrc<SILU> src(in, row, ld, width);
  uint4 buf[VPT], aux[VPT];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = lo + threadIdx.x + i * kRegThreads;
    if (vi < hi) src.fetch(vi, buf[i], aux[i]);
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = lo + threadIdx.x + i * kRegThreads;
    if (vi < hi) {
      buf[i] = src.combine(buf[i], aux[i]);
      amax = fmaxf(amax, vec8_absmax(buf[i]));
    }
  }
  amax = block_max(amax, red);
  amax = cluster_max(amax, &share_max);
  const RowScale rs = row_scale(amax);
  uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(width));
  uint4* yr = y_out ? reinterpret_cast<uint4*>(y_out + row * static_cast<int64_t>(width)) : nullptr;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = lo + threadIdx.x + i * kRegThreads;
    if (vi < hi) {
      qr[vi] = quant_vec8(buf[i], rs);
      if (SILU && yr) yr[vi] = buf[i];
    }
  }
  if (c == 0 && threadIdx.x == 0) scale[row] = rs.s;
  w8a8::dev::cluster_sync();  // no CTA leaves while a peer may still read its share_max
}

// ------------------------------------------------------------------ RMSNorm
// RMSNorm (optionally after a residual add) fused with the per-token quantiser:
// the input side of qkv and gate_up (RMSNorm / RMSNormFused,
// M/layers/norm.py:8-38, whose flashinfer kernels compute in fp32):
//   v = x (+ residual, fp32 add);  residual_out = bf16(v) when a residual is given
//   r = 1 / sqrt(sum(v*v) / K + eps)   (correctly rounded sqrt and divide)
//   y = bf16((v * r) * w)              (the normalised row, never written unless y_out)
//   q, s = per-token quantisation of y (the rule above)
// One CTA per row, the row in registers (K <= 8192), two block reductions.
constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 4 * kNormThreads;  // K <= 8192

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float r = (lane < nw) ? red[lane] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  __syncthreads();  // `red` is reused by the next reduction
  return r;
}

template <int VPT, bool ADD>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_quant_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* residual, int64_t ldr,
    const __nv_bfloat16* __restrict__ w, float eps, int8_t* __restrict__ q, float* __restrict__ scale,
    __nv_bfloat16* residual_out, __nv_bfloat16* __restrict__ y_out, int width) {
  __shared__ float red[32];
  w8a8::dev::griddep_launch();  // early trigger, as in rows_reg_kernel
  w8a8::dev::griddep_wait();    // x / residual are the previous kernel's output
  const int64_t row = blockIdx.x;
  const int nvec = width >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  const uint4* rr = ADD ? reinterpret_cast<const uint4*>(residual + row * ldr) : nullptr;
  uint4 xa[VPT], ra[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      xa[i] = __ldcs(xr + vi);
      if constexpr (ADD) ra[i] = __ldcs(rr + vi);
    }
  }
  float v[VPT][8];
  float ss = 0.0f;
  uint4* ro = ADD && residual_out ? reinterpret_cast<uint4*>(residual_out + row * ldr) : nullptr;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi >= nvec) continue;
    const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&xa[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(hx[j]);
      if constexpr (ADD) {
        const float2 g = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&ra[i])[j]);
        f.x = __fadd_rn(f.x, g.x);
        f.y = __fadd_rn(f.y, g.y);
      }
      v[i][2 * j] = f.x;
      v[i][2 * j + 1] = f.y;
      ss = __fmaf_rn(f.x, f.x, ss);
      ss = __fmaf_rn(f.y, f.y, ss);
    }
    if (ro) {
      uint4 o;
      __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) ho[j] = __floats2bfloat162_rn(v[i][2 * j], v[i][2 * j + 1]);
      ro[vi] = o;
    }
  }
  ss = block_sum(ss, red);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(width)), eps)));
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4 ya[VPT];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi >= nvec) continue;
    const uint4 wv = __ldg(wr + vi);
    const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&wv);
    __nv_bfloat162* hy = reinterpret_cast<__nv_bfloat162*>(&ya[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 wf = __bfloat1622float2(hw[j]);
      hy[j] = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(v[i][2 * j], r), wf.x),
                                    __fmul_rn(__fmul_rn(v[i][2 * j + 1], r), wf.y));
    }
    amax = fmaxf(amax, vec8_absmax(ya[i]));
  }
  amax = block_max(amax, red);
  const RowScale rs = row_scale(amax);
  uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(width));
  uint4* yr = y_out ? reinterpret_cast<uint4*>(y_out + row * static_cast<int64_t>(width)) : nullptr;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi >= nvec) continue;
    qr[vi] = quant_vec8(ya[i], rs);
    if (yr) yr[vi] = ya[i];
  }
  if (threadIdx.x == 0) scale[row] = rs.s;
}

// Resident CTAs per SM of a kernel at a given block size and dynamic shared
// memory, queried once per device and kernel instance.
template <typename Kernel>
int resident_ctas(Kernel kernel, int threads, size_t smem) {
  static int cached[64] = {0};
  const int dev = w8a8::current_device();
  if (dev < 0 || dev >= 64) return 1;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess || n < 1) n = 1;
    cached[dev] = n;
  }
  return cached[dev];
}

// Warp-group RMSNorm + quantiser (many rows of at most 8192 values): G warps
// own a row, lane t of the group holding vectors t + 32 G j of x (and of the
// residual) as raw bf16 in registers; v = x (+ residual) in fp32 is computed
// again in the second pass instead of being kept (8 fp32 per vector would
// cost the occupancy the one-CTA-per-row kernel loses).  Both reductions
// (sum of squares, absmax) are warp shuffles plus one shared-memory exchange
// under the group's named barrier; the same arithmetic as rmsnorm_quant_kernel
// (its sum of squares is accumulated in another order: the fp32 rounding of
// the sum, hence r, may differ in the last bit, within the tolerance the y
// output is held to).  Persistent grid, group g taking rows g, g + groups, ...
template <int VPT, int G, bool ADD>
__global__ void __launch_bounds__(kWarpThreads) rmsnorm_warp_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* residual, int64_t ldr,
    const __nv_bfloat16* __restrict__ w, float eps, int8_t* __restrict__ q, float* __restrict__ scale,
    __nv_bfloat16* residual_out, __nv_bfloat16* __restrict__ y_out, int64_t M, int width) {
  constexpr int kGroups = kWarpThreads / 32 / G;
  __shared__ float part_ss[2][kWarpThreads / 32], part_mx[2][kWarpThreads / 32];
  w8a8::dev::griddep_launch();  // early trigger, as in rows_reg_kernel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / G;
  const int t = (warp % G) * 32 + lane;
  const int nvec = width >> 3;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kGroups;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  auto group_bar = [&]() {
    if (kGroups == 1 || grp == 0)
      w8a8::dev::named_bar_sync(1, 32 * G);
    else
      w8a8::dev::named_bar_sync(2, 32 * G);
  };
  w8a8::dev::griddep_wait();  // x / residual are the previous kernel's output
  int it = 0;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kGroups + grp; row < M; row += stride, ++it) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
    const uint4* rr = ADD ? reinterpret_cast<const uint4*>(residual + row * ldr) : nullptr;
    uint4 xa[VPT], ra[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int vi = t + j * 32 * G;
      if (vi < nvec) {
        xa[j] = __ldcs(xr + vi);
        if constexpr (ADD) ra[j] = __ldcs(rr + vi);
      }
    }
    auto value = [&](int j, int e) {  // v of element e (0..7) of vector j, fp32
      const __nv_bfloat162 hx = reinterpret_cast<const __nv_bfloat162*>(&xa[j])[e >> 1];
      float f = (e & 1) ? __high2float(hx) : __low2float(hx);
      if constexpr (ADD) {
        const __nv_bfloat162 hr = reinterpret_cast<const __nv_bfloat162*>(&ra[j])[e >> 1];
        f = __fadd_rn(f, (e & 1) ? __high2float(hr) : __low2float(hr));
      }
      return f;
    };
    float ss = 0.0f;
    uint4* ro = ADD && residual_out ? reinterpret_cast<uint4*>(residual_out + row * ldr) : nullptr;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int vi = t + j * 32 * G;
      if (vi >= nvec) continue;
      uint4 o;
      __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float a = value(j, e), b = value(j, e + 1);
        ss = __fmaf_rn(a, a, ss);
        ss = __fmaf_rn(b, b, ss);
        ho[e >> 1] = __floats2bfloat162_rn(a, b);
      }
      if (ro) ro[vi] = o;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if constexpr (G > 1) {
      float* p = &part_ss[it & 1][grp * G];
      if (lane == 0) p[warp % G] = ss;
      group_bar();
      ss = p[0];
#pragma unroll
      for (int k = 1; k < G; ++k) ss += p[k];
    }
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(width)), eps)));
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.0f);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int vi = t + j * 32 * G;
      if (vi >= nvec) continue;
      const uint4 wv = __ldg(wr + vi);
      const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&wv);
      uint4 yv;
      __nv_bfloat162* hy = reinterpret_cast<__nv_bfloat162*>(&yv);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float2 wf = __bfloat1622float2(hw[e >> 1]);
        hy[e >> 1] = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(value(j, e), r), wf.x),
                                           __fmul_rn(__fmul_rn(value(j, e + 1), r), wf.y));
      }
      xa[j] = yv;  // x of this vector is no longer needed: keep y in its place
      m2 = vec8_absmax2(yv, m2);
    }
    float amax = warp_max(absmax_of(m2));
    if constexpr (G > 1) {
      float* p = &part_mx[it & 1][grp * G];
      if (lane == 0) p[warp % G] = amax;
      group_bar();
#pragma unroll
      for (int k = 0; k < G; ++k) amax = fmaxf(amax, p[k]);
    }
    const RowScale rs = row_scale(amax);
    uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(width));
    uint4* yr = y_out ? reinterpret_cast<uint4*>(y_out + row * static_cast<int64_t>(width)) : nullptr;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int vi = t + j * 32 * G;
      if (vi >= nvec) continue;
      qr[vi] = quant_vec8(xa[j], rs);
      if (yr) yr[vi] = xa[j];
    }
    if (t == 0) scale[row] = rs.s;
  }
}

template <int VPT, int G, bool ADD>
cudaError_t launch_rmsnorm_warp(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* res, int64_t ldr,
                                const __nv_bfloat16* w, float eps, int8_t* q, float* scale,
                                __nv_bfloat16* res_out, __nv_bfloat16* y, int64_t M, int width, int nsm,
                                cudaStream_t s) {
  constexpr int kGroups = kWarpThreads / 32 / G;
  const int per_sm = resident_ctas(rmsnorm_warp_kernel<VPT, G, ADD>, kWarpThreads, 0);
  int64_t grid = (M + kGroups - 1) / kGroups;
  const int64_t cap = static_cast<int64_t>(nsm) * per_sm;
  if (grid > cap) grid = cap;
  return w8a8::launch_pdl(rmsnorm_warp_kernel<VPT, G, ADD>, dim3(static_cast<unsigned>(grid)), dim3(kWarpThreads),
                          0, s, x, ldx, res, ldr, w, eps, q, scale, res_out, y, M, width);
}

// The warp-group RMSNorm for `nvec` vectors per row: the fewest warps (1, 2
// or 4) that keep a lane's vectors at 6 or fewer (x and the residual are both
// held); not launched when 4 warps are not enough.  Measured against the
// one-CTA-per-row kernel: faster at K = 5120 (6 vectors per lane, 4 warps),
// slower at 8 vectors per lane (K = 8192, 4 warps; K = 4096, 2 warps), where
// the registers leave too few groups resident.
template <bool ADD>
int launch_rmsnorm_warp_any(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* res, int64_t ldr,
                            const __nv_bfloat16* w, float eps, int8_t* q, float* scale, __nv_bfloat16* res_out,
                            __nv_bfloat16* y, int64_t M, int width, int nsm, cudaStream_t s, bool* launched) {
  const int nvec = width / 8;
  *launched = false;
  int g = 0;
  for (int c = 1; c <= 4 && g == 0; c *= 2)
    if ((nvec + 32 * c - 1) / (32 * c) <= 6) g = c;
  if (g == 0) return W8A8_OK;
  const int vpt = (nvec + 32 * g - 1) / (32 * g);
#define W8A8_RMS(V, GG)                                                                                        \
  W8A8_CUDA_TRY((launch_rmsnorm_warp<V, GG, ADD>(x, ldx, res, ldr, w, eps, q, scale, res_out, y, M, width, nsm, s)))
  if (g == 1) {
    if (vpt <= 4) W8A8_RMS(4, 1); else if (vpt <= 6) W8A8_RMS(6, 1); else W8A8_RMS(8, 1);
  } else if (g == 2) {
    if (vpt <= 4) W8A8_RMS(4, 2); else if (vpt <= 6) W8A8_RMS(6, 2); else W8A8_RMS(8, 2);
  } else {
    if (vpt <= 4) W8A8_RMS(4, 4); else if (vpt <= 6) W8A8_RMS(6, 4); else W8A8_RMS(8, 4);
  }
#undef W8A8_RMS
  *launched = true;
  return W8A8_OK;
}

template <bool ADD>
int launch_rmsnorm(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* res, int64_t ldr,
                   const __nv_bfloat16* w, float eps, int8_t* q, float* scale, __nv_bfloat16* res_out,
                   __nv_bfloat16* y, int64_t M, int width, cudaStream_t s) {
  const int nvec = width / 8;
  int nsm = w8a8::sm_count();
  if (nsm <= 0) nsm = 148;
  if (M >= 2LL * nsm && nvec >= 32) {  // many rows: warp groups per row
    bool launched = false;
    const int rc = launch_rmsnorm_warp_any<ADD>(x, ldx, res, ldr, w, eps, q, scale, res_out, y, M, width, nsm, s,
                                                &launched);
    if (rc != W8A8_OK || launched) return rc;
  }
  const int vpt = nvec <= kNormThreads ? 1 : (nvec <= 2 * kNormThreads ? 2 : 4);
  const int need = (nvec + vpt - 1) / vpt;
  const int threads = need < 32 ? 32 : ((need + 31) / 32) * 32;
  const dim3 grid(static_cast<unsigned>(M)), block(threads);
  switch (vpt) {
    case 1: W8A8_CUDA_TRY(w8a8::launch_pdl(rmsnorm_quant_kernel<1, ADD>, grid, block, 0, s, x, ldx, res, ldr, w, eps,
                                           q, scale, res_out, y, width)); break;
    case 2: W8A8_CUDA_TRY(w8a8::launch_pdl(rmsnorm_quant_kernel<2, ADD>, grid, block, 0, s, x, ldx, res, ldr, w, eps,
                                           q, scale, res_out, y, width)); break;
    default: W8A8_CUDA_TRY(w8a8::launch_pdl(rmsnorm_quant_kernel<4, ADD>, grid, block, 0, s, x, ldx, res, ldr, w,
                                            eps, q, scale, res_out, y, width)); break;
  }
  return W8A8_OK;
}

// Cluster size for the split-row path: the smallest power of two (2..8) that
// gives at least two CTAs per SM over the M rows and at most four vectors per
// thread; 0 = use the one-CTA-per-row paths (enough rows, or short rows).
inline int row_cluster_size(int64_t M, int nvec, int nsm) {
  if (nvec < 2 * kRegThreads || M >= 2LL * nsm) return 0;
  for (int c = 2; c <= 8; c *= 2)
    if (M * c >= 2LL * nsm && (nvec + c - 1) / c <= 4 * kRegThreads) return c;
  return (nvec + 7) / 8 <= 4 * kRegThreads ? 8 : 0;
}

template <int VPT, bool SILU>
cudaError_t launch_cluster_rows(const __nv_bfloat16* in, int64_t ld, int8_t* q, float* scale, __nv_bfloat16* y,
                                int64_t M, int width, int csize, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(M * csize));
  cfg.blockDim = dim3(kRegThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(csize);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, rows_cluster_kernel<VPT, SILU>, in, ld, q, scale, y, width);
}

template <int VPT, int G, bool SCATTER>
cudaError_t launch_warp_rows(const __nv_bfloat16* in, int64_t ld, int8_t* q, float* scale, int64_t M, int width,
                             int nsm, cudaStream_t s, const int32_t* dst, int fanout) {
  constexpr int kGroups = kWarpThreads / 32 / G;
  const int per_sm = resident_ctas(rows_warp_kernel<VPT, G, SCATTER>, kWarpThreads, 0);
  int64_t grid = (M + kGroups - 1) / kGroups;
  const int64_t cap = static_cast<int64_t>(nsm) * per_sm;
  if (grid > cap) grid = cap;
  return w8a8::launch_pdl(rows_warp_kernel<VPT, G, SCATTER>, dim3(static_cast<unsigned>(grid)), dim3(kWarpThreads),
                          0, s, in, ld, q, scale, M, width, dst, fanout);
}

// Vectors per lane rounded up to an instantiated count (2, 4, 6, 8, 10, 12, 16).
template <int G, bool SCATTER>
cudaError_t launch_warp_rows_vpt(int vpt, const __nv_bfloat16* in, int64_t ld, int8_t* q, float* scale, int64_t M,
                                 int width, int nsm, cudaStream_t s, const int32_t* dst, int fanout) {
  if (vpt <= 2) return launch_warp_rows<2, G, SCATTER>(in, ld, q, scale, M, width, nsm, s, dst, fanout);
  if (vpt <= 4) return launch_warp_rows<4, G, SCATTER>(in, ld, q, scale, M, width, nsm, s, dst, fanout);
  if (vpt <= 6) return launch_warp_rows<6, G, SCATTER>(in, ld, q, scale, M, width, nsm, s, dst, fanout);
  if (vpt <= 8) return launch_warp_rows<8, G, SCATTER>(in, ld, q, scale, M, width, nsm, s, dst, fanout);
  if (vpt <= 10) return launch_warp_rows<10, G, SCATTER>(in, ld, q, scale, M, width, nsm, s, dst, fanout);
  if (vpt <= 12) return launch_warp_rows<12, G, SCATTER>(in, ld, q, scale, M, width, nsm, s, dst, fanout);
  return launch_warp_rows<16, G, SCATTER>(in, ld, q, scale, M, width, nsm, s, dst, fanout);
}

// Warps per row for the warp-group path: the fewest (1, 2 or 4) that keep a
// lane's vectors within the target; 0 when the row is too wide for 4 warps.
inline int warp_group_size(int nvec) {
  for (int g = 1; g <= 4; g *= 2)
    if ((nvec + 32 * g - 1) / (32 * g) <= W8A8_WARP_MAX_VPT) return g;
  return (nvec + 127) / 128 <= 16 ? 4 : 0;
}

template <bool SCATTER>
int launch_warp_group_t(const __nv_bfloat16* in, int64_t ld, int8_t* q, float* scale, int64_t M, int width, int g,
                        int nsm, cudaStream_t s, const int32_t* dst, int fanout) {
  const int nvec = width / 8;
  const int vpt = (nvec + 32 * g - 1) / (32 * g);
  switch (g) {
    case 1: W8A8_CUDA_TRY((launch_warp_rows_vpt<1, SCATTER>(vpt, in, ld, q, scale, M, width, nsm, s, dst, fanout))); break;
    case 2: W8A8_CUDA_TRY((launch_warp_rows_vpt<2, SCATTER>(vpt, in, ld, q, scale, M, width, nsm, s, dst, fanout))); break;
    default: W8A8_CUDA_TRY((launch_warp_rows_vpt<4, SCATTER>(vpt, in, ld, q, scale, M, width, nsm, s, dst, fanout))); break;
  }
  return W8A8_OK;
}

int launch_warp_group(const __nv_bfloat16* in, int64_t ld, int8_t* q, float* scale, int64_t M, int width, int g,
                      int nsm, cudaStream_t s) {
  return launch_warp_group_t<false>(in, ld, q, scale, M, width, g, nsm, s, nullptr, 0);
}

template <bool SILU>
int launch_rows(const __nv_bfloat16* in, int64_t ld, int8_t* q, float* scale, __nv_bfloat16* y, int64_t M,
                int width, cudaStream_t s) {
  const int nvec = width / 8;
  const dim3 grid(static_cast<unsigned>(M));
  int nsm = w8a8::sm_count();
  if (nsm <= 0) nsm = 148;
  const int csize = row_cluster_size(M, nvec, nsm);
  const bool aligned = (reinterpret_cast<uintptr_t>(in) & 15u) == 0 && ld % 8 == 0;
  if (!SILU && csize == 0 && aligned) {
    // many plain rows: warp groups per row
    const int g = warp_group_size(nvec);
    if (g > 0) return launch_warp_group(in, ld, q, scale, M, width, g, nsm, s);
  }
  if (csize > 0) {
    const int per = (nvec + csize - 1) / csize;
    const int vpt = per <= kRegThreads ? 1 : (per <= 2 * kRegThreads ? 2 : 4);
    switch (vpt) {
      case 1: W8A8_CUDA_TRY((launch_cluster_rows<1, SILU>(in, ld, q, scale, y, M, width, csize, s))); break;
      case 2: W8A8_CUDA_TRY((launch_cluster_rows<2, SILU>(in, ld, q, scale, y, M, width, csize, s))); break;
      default: W8A8_CUDA_TRY((launch_cluster_rows<4, SILU>(in, ld, q, scale, y, M, width, csize, s))); break;
    }
    return W8A8_OK;
  }
  if (nvec <= 4 * kRegThreads) {
    const int vpt = nvec <= kRegThreads ? 1 : (nvec <= 2 * kRegThreads ? 2 : 4);
    const int need = (nvec + vpt - 1) / vpt;
    const int threads = need < 32 ? 32 : ((need + 31) / 32) * 32;
    switch (vpt) {
      case 1: W8A8_CUDA_TRY(w8a8::launch_pdl(rows_reg_kernel<1, SILU>, grid, dim3(threads), 0, s, in, ld, q, scale, y,
                                             width)); break;
      case 2: W8A8_CUDA_TRY(w8a8::launch_pdl(rows_reg_kernel<2, SILU>, grid, dim3(threads), 0, s, in, ld, q, scale, y,
                                             width)); break;
      default: W8A8_CUDA_TRY(w8a8::launch_pdl(rows_reg_kernel<4, SILU>, grid, dim3(threads), 0, s, in, ld, q, scale,
                                              y, width)); break;
    }
  } else {
    static std::mutex mu;
    static bool configured[64] = {false};
    const int dev = w8a8::current_device();
    W8A8_REQUIRE(dev >= 0 && dev < 64, W8A8_ERR_CUDA, "no current device");
    {
      std::lock_guard<std::mutex> lk(mu);
      if (!configured[dev]) {
        W8A8_CUDA_TRY(cudaFuncSetAttribute(rows_smem_kernel<SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kMaxVec * 16));
        configured[dev] = true;
      }
    }
    W8A8_CUDA_TRY(w8a8::launch_pdl(rows_smem_kernel<SILU>, grid, dim3(kSmemThreads), static_cast<size_t>(nvec) * 16, s,
                                   in, ld, q, scale, y, width));
  }
  W8A8_CUDA_TRY(cudaGetLastError());
  return W8A8_OK;
}

template <int VPT>
cudaError_t launch_rows_amax_warp(const __nv_bfloat16* y, int64_t ld, const uint32_t* amax, int8_t* q,
                                  float* scale, int64_t M, int width, const int32_t* num_blocks, cudaStream_t s) {
  constexpr int kWarps = kAmaxWarpThreads / 32;
  const int per_sm = resident_ctas(rows_amax_warp_kernel<VPT>, kAmaxWarpThreads, 0);
  int64_t grid = (M + kWarps - 1) / kWarps;
  const int64_t cap = static_cast<int64_t>(w8a8::sm_count()) * per_sm;
  if (grid > cap) grid = cap;
  return w8a8::launch_pdl(rows_amax_warp_kernel<VPT>, dim3(static_cast<unsigned>(grid)), dim3(kAmaxWarpThreads), 0,
                          s, y, ld, amax, q, scale, M, width, num_blocks);
}

}  // namespace

namespace w8a8 {

// rows_amax_kernel over rows [0, M) (with num_blocks: [0, min(M, 128 *
// *num_blocks)), the bound read on the device).
int launch_rows_amax(const __nv_bfloat16* y, int64_t ld, const uint32_t* amax, int8_t* q, float* scale, int64_t M,
                     int width, const int32_t* num_blocks, cudaStream_t s) {
  const int64_t nvec = width / 8;
  if (nvec <= 256) {
    const int vpt = static_cast<int>((nvec + 31) / 32);
    cudaError_t e;
    if (vpt <= 1) e = launch_rows_amax_warp<1>(y, ld, amax, q, scale, M, width, num_blocks, s);
    else if (vpt <= 2) e = launch_rows_amax_warp<2>(y, ld, amax, q, scale, M, width, num_blocks, s);
    else if (vpt <= 3) e = launch_rows_amax_warp<3>(y, ld, amax, q, scale, M, width, num_blocks, s);
    else if (vpt <= 4) e = launch_rows_amax_warp<4>(y, ld, amax, q, scale, M, width, num_blocks, s);
    else if (vpt <= 6) e = launch_rows_amax_warp<6>(y, ld, amax, q, scale, M, width, num_blocks, s);
    else e = launch_rows_amax_warp<8>(y, ld, amax, q, scale, M, width, num_blocks, s);
    W8A8_CUDA_TRY(e);
    return W8A8_OK;
  }
  const int64_t gx = (nvec + kAmaxThreads * kAmaxVpt - 1) / (kAmaxThreads * kAmaxVpt);
  int64_t gy = M < 65535 ? M : 65535;
  if (num_blocks != nullptr) {
    // the rows in use are known on the device only: cover the bound with
    // about four CTAs per SM (the kernel strides over rows)
    const int64_t cap = 4LL * w8a8::sm_count() / (gx > 0 ? gx : 1);
    if (gy > cap && cap > 0) gy = cap;
  }
  W8A8_REQUIRE(gx <= 0x7fffffff, W8A8_ERR_UNSUPPORTED, "quant_rows_amax: K too large");
  W8A8_CUDA_TRY(w8a8::launch_pdl(rows_amax_kernel, dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)),
                                 dim3(kAmaxThreads), 0, s, y, ld, amax, q, scale, M, width, num_blocks));
  return W8A8_OK;
}

}  // namespace w8a8

extern "C" {

int w8a8_quant_rows_amax(const void* y, int64_t ldy, const uint32_t* amax, int8_t* q, float* scale, int64_t M,
                         int64_t K, void* stream) {
  W8A8_REQUIRE(M >= 0 && K >= 0, W8A8_ERR_INVALID_ARG, "quant_rows_amax: negative shape");
  if (M == 0) return W8A8_OK;
  W8A8_REQUIRE(y && amax && q && scale, W8A8_ERR_INVALID_ARG, "quant_rows_amax: null pointer");
  W8A8_REQUIRE(K > 0 && K % 8 == 0 && K <= 0x7fffffff, W8A8_ERR_INVALID_ARG,
               "quant_rows_amax: K=%lld must be a positive multiple of 8", (long long)K);
  W8A8_REQUIRE(ldy >= K && ldy % 8 == 0, W8A8_ERR_INVALID_ARG,
               "quant_rows_amax: row stride %lld must be >= K and a multiple of 8", (long long)ldy);
  W8A8_REQUIRE(W8A8_ALIGNED16(y) && W8A8_ALIGNED16(q), W8A8_ERR_ALIGNMENT,
               "quant_rows_amax: y and q must be 16-byte aligned");
  return w8a8::launch_rows_amax(static_cast<const __nv_bfloat16*>(y), ldy, amax, q, scale, M, static_cast<int>(K),
                                nullptr, static_cast<cudaStream_t>(stream));
}

int w8a8_quant_per_token(const void* x, int64_t ldx, int8_t* q, float* scale, int64_t M, int64_t K,
                         void* stream) {
  W8A8_REQUIRE(M >= 0 && K >= 0, W8A8_ERR_INVALID_ARG, "quant_per_token: negative shape M=%lld K=%lld",
               (long long)M, (long long)K);
  if (M == 0) return W8A8_OK;
  W8A8_REQUIRE(x && q && scale, W8A8_ERR_INVALID_ARG, "quant_per_token: null pointer");
  W8A8_REQUIRE(K > 0 && K % 8 == 0, W8A8_ERR_INVALID_ARG, "quant_per_token: K=%lld must be a positive multiple of 8",
               (long long)K);
  W8A8_REQUIRE(ldx >= K && ldx % 8 == 0, W8A8_ERR_INVALID_ARG,
               "quant_per_token: row stride %lld must be >= K and a multiple of 8", (long long)ldx);
  W8A8_REQUIRE(M <= 0x7fffffff, W8A8_ERR_UNSUPPORTED, "quant_per_token: M=%lld too large", (long long)M);
  W8A8_REQUIRE(W8A8_ALIGNED16(x) && W8A8_ALIGNED16(q), W8A8_ERR_ALIGNMENT,
               "quant_per_token: x and q must be 16-byte aligned");
  W8A8_REQUIRE(K / 8 <= kMaxVec, W8A8_ERR_UNSUPPORTED, "quant_per_token: K=%lld exceeds the 32768 limit",
               (long long)K);
  return launch_rows<false>(static_cast<const __nv_bfloat16*>(x), ldx, q, scale, nullptr, M, static_cast<int>(K),
                            static_cast<cudaStream_t>(stream));
}

int w8a8_moe_quant_scatter(const void* x, int64_t ldx, int64_t T, int64_t K, const int32_t* inv_pos, int topk,
                           int8_t* q_sorted, float* sa_sorted, void* stream) {
  W8A8_REQUIRE(T >= 0 && K >= 0, W8A8_ERR_INVALID_ARG, "moe_quant_scatter: negative shape T=%lld K=%lld",
               (long long)T, (long long)K);
  if (T == 0) return W8A8_OK;
  W8A8_REQUIRE(x && inv_pos && q_sorted && sa_sorted, W8A8_ERR_INVALID_ARG, "moe_quant_scatter: null pointer");
  W8A8_REQUIRE(topk >= 1 && topk <= 64, W8A8_ERR_UNSUPPORTED, "moe_quant_scatter: top-k %d (1..64 supported)", topk);
  W8A8_REQUIRE(K > 0 && K % 8 == 0, W8A8_ERR_INVALID_ARG, "moe_quant_scatter: K=%lld must be a positive multiple of 8",
               (long long)K);
  W8A8_REQUIRE(ldx >= K && ldx % 8 == 0, W8A8_ERR_INVALID_ARG,
               "moe_quant_scatter: row stride %lld must be >= K and a multiple of 8", (long long)ldx);
  W8A8_REQUIRE(T * topk <= 0x7fffffff, W8A8_ERR_UNSUPPORTED, "moe_quant_scatter: too many slots");
  W8A8_REQUIRE(W8A8_ALIGNED16(x) && W8A8_ALIGNED16(q_sorted), W8A8_ERR_ALIGNMENT,
               "moe_quant_scatter: x and q_sorted must be 16-byte aligned");
  const int g = warp_group_size(static_cast<int>(K / 8));
  W8A8_REQUIRE(g > 0, W8A8_ERR_UNSUPPORTED, "moe_quant_scatter: K=%lld exceeds the 16384 limit", (long long)K);
  const int nsm = w8a8::sm_count();
  W8A8_REQUIRE(nsm > 0, W8A8_ERR_CUDA, "moe_quant_scatter: no CUDA device");
  return launch_warp_group_t<true>(static_cast<const __nv_bfloat16*>(x), ldx, q_sorted, sa_sorted, T,
                                   static_cast<int>(K), g, nsm, static_cast<cudaStream_t>(stream), inv_pos, topk);
}

int w8a8_silu_mul_quant(const void* gate_up, int64_t ld, int8_t* q, float* scale, void* y_out,
                        int64_t M, int64_t I, void* stream) {
  W8A8_REQUIRE(M >= 0 && I >= 0, W8A8_ERR_INVALID_ARG, "silu_mul_quant: negative shape");
  if (M == 0) return W8A8_OK;
  W8A8_REQUIRE(gate_up != nullptr, W8A8_ERR_INVALID_ARG, "silu_mul_quant: null gate_up");
  W8A8_REQUIRE((q == nullptr) == (scale == nullptr), W8A8_ERR_INVALID_ARG,
               "silu_mul_quant: q and scale are given together (or both null for the bf16-only form)");
  W8A8_REQUIRE(q != nullptr || y_out != nullptr, W8A8_ERR_INVALID_ARG,
               "silu_mul_quant: nothing to write (q, scale and y_out all null)");
  W8A8_REQUIRE(I > 0 && I % 8 == 0, W8A8_ERR_INVALID_ARG, "silu_mul_quant: I=%lld must be a positive multiple of 8",
               (long long)I);
  W8A8_REQUIRE(ld >= 2 * I && ld % 8 == 0, W8A8_ERR_INVALID_ARG,
               "silu_mul_quant: row stride %lld must be >= 2I and a multiple of 8", (long long)ld);
  W8A8_REQUIRE(M <= 0x7fffffff, W8A8_ERR_UNSUPPORTED, "silu_mul_quant: M too large");
  W8A8_REQUIRE(W8A8_ALIGNED16(gate_up) && W8A8_ALIGNED16(q) && W8A8_ALIGNED16(y_out), W8A8_ERR_ALIGNMENT,
               "silu_mul_quant: gate_up, q and y_out must be 16-byte aligned");
  if (q == nullptr) {
    // bf16-only silu_and_mul: no reduction, no quantisation
    const int64_t nv = I / 8, total = M * nv;
    int nsm = w8a8::sm_count();
    if (nsm <= 0) nsm = 148;
    int64_t grid = (total + 2 * kEltThreads - 1) / (2 * kEltThreads);
    if (grid > 8LL * nsm) grid = 8LL * nsm;
    W8A8_CUDA_TRY(w8a8::launch_pdl(silu_mul_kernel, dim3(static_cast<unsigned>(grid)), dim3(kEltThreads), 0,
                                   static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(gate_up), ld,
                                   static_cast<__nv_bfloat16*>(y_out), I, nv, total));
    return W8A8_OK;
  }
  W8A8_REQUIRE(I / 8 <= kMaxVec, W8A8_ERR_UNSUPPORTED, "silu_mul_quant: I=%lld exceeds the 32768 limit",
               (long long)I);
  return launch_rows<true>(static_cast<const __nv_bfloat16*>(gate_up), ld, q, scale,
                           static_cast<__nv_bfloat16*>(y_out), M, static_cast<int>(I),
                           static_cast<cudaStream_t>(stream));
}

int w8a8_rmsnorm_quant(const void* x, int64_t ldx, const void* residual, int64_t ldr, const void* weight,
                       float eps, int8_t* q, float* scale, void* residual_out, void* y_out, int64_t M, int64_t K,
                       void* stream) {
  W8A8_REQUIRE(M >= 0 && K >= 0, W8A8_ERR_INVALID_ARG, "rmsnorm_quant: negative shape");
  if (M == 0) return W8A8_OK;
  W8A8_REQUIRE(x && weight && q && scale, W8A8_ERR_INVALID_ARG, "rmsnorm_quant: null pointer (x, weight, q, scale)");
  W8A8_REQUIRE(K > 0 && K % 8 == 0, W8A8_ERR_INVALID_ARG, "rmsnorm_quant: K=%lld must be a positive multiple of 8",
               (long long)K);
  W8A8_REQUIRE(K / 8 <= kNormMaxVec, W8A8_ERR_UNSUPPORTED, "rmsnorm_quant: K=%lld exceeds the 8192 limit",
               (long long)K);
  W8A8_REQUIRE(ldx >= K && ldx % 8 == 0, W8A8_ERR_INVALID_ARG,
               "rmsnorm_quant: row stride %lld must be >= K and a multiple of 8", (long long)ldx);
  W8A8_REQUIRE(!(eps < 0.0f) && eps == eps, W8A8_ERR_INVALID_ARG, "rmsnorm_quant: eps must be >= 0");
  W8A8_REQUIRE(M <= 0x7fffffff, W8A8_ERR_UNSUPPORTED, "rmsnorm_quant: M too large");
  W8A8_REQUIRE(W8A8_ALIGNED16(x) && W8A8_ALIGNED16(weight) && W8A8_ALIGNED16(q) && W8A8_ALIGNED16(y_out),
               W8A8_ERR_ALIGNMENT, "rmsnorm_quant: x, weight, q and y_out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(weight);
  auto* yb = static_cast<__nv_bfloat16*>(y_out);
  if (residual == nullptr) {
    W8A8_REQUIRE(residual_out == nullptr, W8A8_ERR_INVALID_ARG,
                 "rmsnorm_quant: residual_out needs a residual (without one the residual is x itself)");
    return launch_rmsnorm<false>(xb, ldx, nullptr, K, wb, eps, q, scale, nullptr, yb, M, static_cast<int>(K), s);
  }
  W8A8_REQUIRE(residual_out != nullptr, W8A8_ERR_INVALID_ARG,
               "rmsnorm_quant: with a residual, residual_out (may be the residual itself) is required");
  W8A8_REQUIRE(ldr >= K && ldr % 8 == 0, W8A8_ERR_INVALID_ARG,
               "rmsnorm_quant: residual row stride %lld must be >= K and a multiple of 8", (long long)ldr);
  W8A8_REQUIRE(W8A8_ALIGNED16(residual) && W8A8_ALIGNED16(residual_out), W8A8_ERR_ALIGNMENT,
               "rmsnorm_quant: residual and residual_out must be 16-byte aligned");
  return launch_rmsnorm<true>(xb, ldx, static_cast<const __nv_bfloat16*>(residual), ldr, wb, eps, q, scale,
                              static_cast<__nv_bfloat16*>(residual_out), yb, M, static_cast<int>(K), s);
}

}  // extern "C"
