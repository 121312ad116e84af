// SiLU*mul arithmetic shared by the fused quantiser (quant.cu) and the
// gate_up GEMM's SiLU epilogue (gemm2_sm100.cuh), so that both produce the
// same bf16 product bit for bit; and the bf16-pair running absmax.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

namespace w8a8 {
namespace act {

// Running max |x| over vectors, kept as a bf16 pair (exact: a maximum
// involves no rounding) and widened once per row by absmax_of.
__device__ __forceinline__ __nv_bfloat162 vec8_absmax2(const uint4& raw, __nv_bfloat162 m) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  m = __hmax2(m, __habs2(h[0]));
  m = __hmax2(m, __habs2(h[1]));
  m = __hmax2(m, __habs2(h[2]));
  return __hmax2(m, __habs2(h[3]));
}

__device__ __forceinline__ float absmax_of(__nv_bfloat162 m) { return fmaxf(__low2float(m), __high2float(m)); }

// silu(g) = g / (1 + exp(-g)) in fp32, y = bf16(silu(g) * u).  The fast
// divide (g * rcp.approx(d)) is within a couple of fp32 ulps for
// denominators up to 2^126, but
// returns 0 for denominators in (2^126, 2^128) (g in about [-88.7, -87.3],
// where the true value is a normal ~1e-36); a vector with such a denominator,
// or an overflowed exp (denominator inf: the IEEE quotient is -0, as on the
// CPU), is recomputed out of line with the IEEE divide.  The fp32 value is
// rounded to bf16 (8 significand bits) at the end, so the fast divide's couple
// of fp32 ulps almost never reach the bf16 result; the quantiser then works on
// the bf16 values exactly.

// 1/x with the MUFU rcp unit (the reciprocal step of the fast divide).
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x with the MUFU ex2 unit (relative error ~2^-22 over the range used
// here), subnormal inputs and results flushed to zero: d = 1 + 2^x rounds to
// 1 for any 2^x below 2^-24 and for any |x| below 2^-24, so the flush never
// changes d.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kNegLog2e = -1.4426950408889634f;

// The same values as the fast path below, with the quotient of a lane whose
// denominator exceeds 2^126 taken by the IEEE divide.
static __device__ __noinline__ uint4 silu_mul_vec8_exact(uint4 graw, uint4 uraw) {
  const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&graw);
  const __nv_bfloat162* u = reinterpret_cast<const __nv_bfloat162*>(&uraw);
  uint4 out;
  __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 gf = __bfloat1622float2(g[j]);
    const float2 uf = __bfloat1622float2(u[j]);
    const float gv[2] = {gf.x, gf.y}, uv[2] = {uf.x, uf.y};
    float y[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float d = __fadd_rn(ex2_approx(__fmul_rn(gv[e], kNegLog2e)), 1.0f);
      const float sl = d > 0x1p126f ? __fdiv_rn(gv[e], d) : __fmul_rn(gv[e], rcp_approx(d));
      y[e] = __fmul_rn(sl, uv[e]);
    }
    o[j] = __floats2bfloat162_rn(y[0], y[1]);
  }
  return out;
}

// Fast path: exp(-g) from the identity e^x = 2^(x * log2 e), one multiply and
// one ex2 per value; with |g| of a few units the argument's rounding adds
// ~1e-7 relative error, and in all ~1e-6 at |g| = 20, far below the bf16
// rounding step (2^-8) -- the fused product differs from the CPU's in the last
// bf16 bit on a small fraction of elements, never by more.  Then the fast
// divide, and the two multiplies as packed f32x2 arithmetic.  The fast divide
// is safe when every gate value of the vector is >= -87: then
// -g log2 e <= 125.52 and d < 2^126; the vector's minimum gate is taken on the
// bf16 pairs (three min instructions and one compare per eight values).
__device__ __forceinline__ uint4 silu_mul_vec8(const uint4& graw, const uint4& uraw) {
  const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&graw);
  const __nv_bfloat162* u = reinterpret_cast<const __nv_bfloat162*>(&uraw);
  uint4 out;
  __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
  const __nv_bfloat162 gmin = __hmin2(__hmin2(g[0], g[1]), __hmin2(g[2], g[3]));
  // (a NaN gate drops out of the minimum; both paths give NaN for it)
  const bool safe = __hbge2(gmin, __float2bfloat162_rn(-87.0f));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 gf = __bfloat1622float2(g[j]);
    const float2 uf = __bfloat1622float2(u[j]);
    const float2 a = __fmul2_rn(gf, make_float2(kNegLog2e, kNegLog2e));
    const float2 d = __fadd2_rn(make_float2(ex2_approx(a.x), ex2_approx(a.y)), make_float2(1.0f, 1.0f));
    const float2 y = __fmul2_rn(__fmul2_rn(gf, make_float2(rcp_approx(d.x), rcp_approx(d.y))), uf);
    o[j] = __floats2bfloat162_rn(y.x, y.y);
  }
  if (!safe) return silu_mul_vec8_exact(graw, uraw);
  return out;
}

}  // namespace act
}  // namespace w8a8
