// Kernel 1: per-token symmetric absmax int8 quantiser, and its fusion with
// SiLU*mul (the silu_and_mul step between gate_up and down in GatedMLP,
// M/models/utils.py:44-50 and M/layers/activation.py:9-12 of mini-sglang).
//
// One CTA per row.  The row is read once with 128-bit loads into registers
// (VPT 16-byte vectors per thread), reduced to its absmax with warp shuffles
// plus one shared-memory step, then quantised from registers and written with
// 64-bit stores — HBM traffic is exactly 2K bytes in + K bytes + 4 out per
// row.  Arithmetic convention (bit-exact with the CPU oracle):
//   s = fp32(amax) / 127.0f (IEEE divide), q = clamp(rint_even(x / s), +-127),
//   q = 0 for an all-zero row.
#include <cuda_bf16.h>

#include <cstdint>

#include "common.cuh"

namespace {

constexpr int kMaxThreads = 512;

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
  r = warp_max(r);
  return r;
}

__device__ __forceinline__ int8_t quant_one(float v, float s) {
  if (s == 0.0f) return 0;
  int q = __float2int_rn(__fdiv_rn(v, s));
  q = q > 127 ? 127 : (q < -127 ? -127 : q);
  return static_cast<int8_t>(q);
}

__device__ __forceinline__ uint2 quant_vec8(const uint4& raw, float s) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __bfloat1622float2(h[j]);
    uint32_t b0 = static_cast<uint8_t>(quant_one(f.x, s));
    uint32_t b1 = static_cast<uint8_t>(quant_one(f.y, s));
    uint32_t pair = b0 | (b1 << 8);
    if (j < 2)
      lo |= pair << (16 * j);
    else
      hi |= pair << (16 * (j - 2));
  }
  return make_uint2(lo, hi);
}

__device__ __forceinline__ float vec8_absmax(const uint4& raw) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __bfloat1622float2(h[j]);
    m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  return m;
}

template <int VPT>
__global__ void __launch_bounds__(kMaxThreads) quant_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                                 int64_t ldx, int8_t* __restrict__ q,
                                                                 float* __restrict__ scale, int K) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = K >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  uint4 buf[VPT];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      buf[i] = __ldcs(xr + vi);
      amax = fmaxf(amax, vec8_absmax(buf[i]));
    }
  }
  amax = block_max(amax, red);
  const float s = __fdiv_rn(amax, 127.0f);
  uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(K));
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) qr[vi] = quant_vec8(buf[i], s);
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// y = bf16(silu(g) * u) for 8 lanes, silu(g) = g / (1 + exp(-g)) in fp32.
__device__ __forceinline__ uint4 silu_mul_vec8(const uint4& graw, const uint4& uraw) {
  const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&graw);
  const __nv_bfloat162* u = reinterpret_cast<const __nv_bfloat162*>(&uraw);
  uint4 out;
  __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 gf = __bfloat1622float2(g[j]);
    float2 uf = __bfloat1622float2(u[j]);
    float y0 = __fmul_rn(__fdiv_rn(gf.x, __fadd_rn(1.0f, expf(-gf.x))), uf.x);
    float y1 = __fmul_rn(__fdiv_rn(gf.y, __fadd_rn(1.0f, expf(-gf.y))), uf.y);
    o[j] = __floats2bfloat162_rn(y0, y1);
  }
  return out;
}

template <int VPT>
__global__ void __launch_bounds__(kMaxThreads) silu_mul_quant_kernel(
    const __nv_bfloat16* __restrict__ gu, int64_t ld, int8_t* __restrict__ q,
    float* __restrict__ scale, __nv_bfloat16* __restrict__ y_out, int I) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = I >> 3;
  const uint4* gr = reinterpret_cast<const uint4*>(gu + row * ld);
  const uint4* ur = reinterpret_cast<const uint4*>(gu + row * ld + I);
  uint4 buf[VPT];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      buf[i] = silu_mul_vec8(__ldcs(gr + vi), __ldcs(ur + vi));
      amax = fmaxf(amax, vec8_absmax(buf[i]));
    }
  }
  amax = block_max(amax, red);
  const float s = __fdiv_rn(amax, 127.0f);
  uint2* qr = reinterpret_cast<uint2*>(q + row * static_cast<int64_t>(I));
  uint4* yr = y_out ? reinterpret_cast<uint4*>(y_out + row * static_cast<int64_t>(I)) : nullptr;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      qr[vi] = quant_vec8(buf[i], s);
      if (yr) yr[vi] = buf[i];
    }
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// Vectors per thread and block size for a row of `nvec` 16-byte vectors:
// the fewest vectors per thread that keep the CTA at <= 256 threads, else 8
// vectors per thread with up to kMaxThreads threads.
bool pick_row_shape(int nvec, int* vpt, int* threads) {
  static const int kVpt[] = {1, 2, 4, 8};
  for (int v : kVpt) {
    const int need = (nvec + v - 1) / v;
    if (need <= 256 || (v == 8 && need <= kMaxThreads)) {
      *vpt = v;
      *threads = need < 32 ? 32 : ((need + 31) / 32) * 32;
      return true;
    }
  }
  return false;
}

}  // namespace

extern "C" {

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
  int vpt = 0, threads = 0;
  W8A8_REQUIRE(pick_row_shape(static_cast<int>(K / 8), &vpt, &threads), W8A8_ERR_UNSUPPORTED,
               "quant_per_token: K=%lld exceeds the 32768 limit", (long long)K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const dim3 grid(static_cast<unsigned>(M));
  switch (vpt) {
    case 1: quant_rows_kernel<1><<<grid, threads, 0, s>>>(xb, ldx, q, scale, (int)K); break;
    case 2: quant_rows_kernel<2><<<grid, threads, 0, s>>>(xb, ldx, q, scale, (int)K); break;
    case 4: quant_rows_kernel<4><<<grid, threads, 0, s>>>(xb, ldx, q, scale, (int)K); break;
    default: quant_rows_kernel<8><<<grid, threads, 0, s>>>(xb, ldx, q, scale, (int)K); break;
  }
  W8A8_CUDA_TRY(cudaGetLastError());
  return W8A8_OK;
}

int w8a8_silu_mul_quant(const void* gate_up, int64_t ld, int8_t* q, float* scale, void* y_out,
                        int64_t M, int64_t I, void* stream) {
  W8A8_REQUIRE(M >= 0 && I >= 0, W8A8_ERR_INVALID_ARG, "silu_mul_quant: negative shape");
  if (M == 0) return W8A8_OK;
  W8A8_REQUIRE(gate_up && q && scale, W8A8_ERR_INVALID_ARG, "silu_mul_quant: null pointer");
  W8A8_REQUIRE(I > 0 && I % 8 == 0, W8A8_ERR_INVALID_ARG, "silu_mul_quant: I=%lld must be a positive multiple of 8",
               (long long)I);
  W8A8_REQUIRE(ld >= 2 * I && ld % 8 == 0, W8A8_ERR_INVALID_ARG,
               "silu_mul_quant: row stride %lld must be >= 2I and a multiple of 8", (long long)ld);
  W8A8_REQUIRE(M <= 0x7fffffff, W8A8_ERR_UNSUPPORTED, "silu_mul_quant: M too large");
  W8A8_REQUIRE(W8A8_ALIGNED16(gate_up) && W8A8_ALIGNED16(q) && W8A8_ALIGNED16(y_out), W8A8_ERR_ALIGNMENT,
               "silu_mul_quant: gate_up, q and y_out must be 16-byte aligned");
  int vpt = 0, threads = 0;
  W8A8_REQUIRE(pick_row_shape(static_cast<int>(I / 8), &vpt, &threads), W8A8_ERR_UNSUPPORTED,
               "silu_mul_quant: I=%lld exceeds the 32768 limit", (long long)I);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* g = static_cast<const __nv_bfloat16*>(gate_up);
  auto* y = static_cast<__nv_bfloat16*>(y_out);
  const dim3 grid(static_cast<unsigned>(M));
  switch (vpt) {
    case 1: silu_mul_quant_kernel<1><<<grid, threads, 0, s>>>(g, ld, q, scale, y, (int)I); break;
    case 2: silu_mul_quant_kernel<2><<<grid, threads, 0, s>>>(g, ld, q, scale, y, (int)I); break;
    case 4: silu_mul_quant_kernel<4><<<grid, threads, 0, s>>>(g, ld, q, scale, y, (int)I); break;
    default: silu_mul_quant_kernel<8><<<grid, threads, 0, s>>>(g, ld, q, scale, y, (int)I); break;
  }
  W8A8_CUDA_TRY(cudaGetLastError());
  return W8A8_OK;
}

}  // extern "C"
