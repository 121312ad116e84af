// Internal host entry of the GEMM launcher, shared by the plain GEMM entry
// points (gemm.cu) and the fused row-parallel GEMM + all-reduce (comm.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "comm_dev.cuh"

namespace w8a8 {

// comm == nullptr: plain GEMM into C.  comm != nullptr: every rank's partial
// goes through the communicator's buffers and C receives the all-reduced sum.
// silu_amax != nullptr: B is a merged [gate; up] weight of N = 2I rows, C
// receives y = bf16(silu(gate) * up) [M, I] and silu_amax[m] max |y| of row m
// (float bits, atomic max; the caller zeroes it); 2-SM pair plans only.
int run_gemm(const int8_t* A, const int8_t* B, const float* sa, const float* sb, const void* bias, void* C,
             int32_t* c_i32, int64_t M, int64_t N, int64_t K, int variant, int ctas, void* workspace,
             size_t workspace_bytes, cudaStream_t stream, long long timeout_ns, const CommView* comm,
             uint32_t* silu_amax = nullptr);

// Tensor map over a row-major int8 matrix [rows, K] (row stride K) read as
// boxes of box_rows x 128 bytes with the 128-byte swizzle; out-of-range rows
// and columns read as zero.
int encode_operand(CUtensorMap* tm, const void* base, int64_t rows, int64_t K, int box_rows);

// Host-side checks of a GEMM call (shape limits, null pointers, 16-byte
// alignment) that run_gemm makes before any launch; 0 or a status code.
int validate_gemm_args(const int8_t* A, const int8_t* B, const float* sa, const float* sb, const void* C,
                       int64_t M, int64_t N, int64_t K);

}  // namespace w8a8
