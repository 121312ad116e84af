/*
 * w8a8_tp.h — C ABI of the B200 (sm_100a) W8A8 tensor-parallel linear path.
 *
 * One shared library (mini-sglang-fork_b200/_w8a8_tp.so) exports these
 * entry points.  Plain pointers and sizes only: device pointers are raw CUDA
 * device addresses, `stream` is a cudaStream_t passed as void*.  The caller
 * owns every tensor; the library owns only a communicator's IPC-shared
 * buffers.  Apart from w8a8_comm_create (which allocates those buffers) and
 * the calls documented as synchronising (w8a8_device_error,
 * w8a8_comm_status, w8a8_comm_destroy, and the first call of
 * w8a8_gemm_static_scratch on a device), no call allocates device memory or
 * synchronises the device.  No call throws; all of them return an int status
 * (0 = W8A8_OK) and leave a message for w8a8_last_error() on failure.  Shapes
 * and alignment are validated on the host before any launch.
 *
 * Reference interfaces replaced (paths inside mini-sglang, M/ = python/minisgl/):
 *   - _LinearTPImpl.forward = F.linear(x, W, b)          M/layers/linear.py:31-32
 *   - LinearOProj / LinearRowParallel forward + all_reduce M/layers/linear.py:102-106,123-127
 *   - silu_and_mul(x, out)                                 M/layers/activation.py:9-12
 *   - RMSNorm / RMSNormFused forward (+ the quantiser)     M/layers/norm.py:8-38
 *   - NCCLWrapper(rank, world, max_bytes, uid)             M/kernel/csrc/src/pynccl.cu:74-91
 *   - NCCLWrapper::all_reduce(t, "sum")                    M/kernel/csrc/src/pynccl.cu:93-134
 *   - init_pynccl (UID broadcast over the CPU group)       M/kernel/pynccl.py:45-78
 *   - host::RuntimeCheck / PanicError message channel      M/kernel/csrc/include/minisgl/utils.h:40-88
 */
#ifndef W8A8_TP_H_
#define W8A8_TP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum w8a8_status {
  W8A8_OK = 0,
  W8A8_ERR_INVALID_ARG = 1, /* bad shape, null pointer, bad rank/world     */
  W8A8_ERR_ALIGNMENT = 2,   /* pointer / stride not 16-byte aligned        */
  W8A8_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed           */
  W8A8_ERR_UNSUPPORTED = 4, /* device is not sm_100 or size beyond limits  */
  W8A8_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up          */
  W8A8_ERR_WORKSPACE = 6,   /* workspace missing or too small              */
  W8A8_ERR_STATE = 7        /* communicator used before its peers were opened */
};

/* Last error message of the calling thread ("" if none).  Replaces the
 * PanicError text channel of M/kernel/csrc/include/minisgl/utils.h:40-88. */
const char* w8a8_last_error(void);

/* ABI version (bumped on any signature change). */
int w8a8_abi_version(void);

/* Reads (and optionally clears) the device-side error word the kernels set
 * when a bounded wait gives up (W8A8_ERR_TIMEOUT) — synchronises the current
 * device.  *code receives the bitwise OR of the kernel error bits. */
int w8a8_device_error(int* code, int clear);

/* ---------------------------------------------------------------- kernel 1
 * Per-token symmetric absmax quantiser: x[M, K] bf16 (row stride ldx
 * elements) -> q[M, K] int8 (contiguous) + scale[M] fp32,
 * scale = amax/127, q = clamp(rint(x/scale), -127, 127), q = 0 if scale = 0.
 * No reference counterpart (the reference feeds bf16 to F.linear,
 * M/layers/linear.py:31-32); it is the input side of every W8A8 linear.
 * Needs K % 8 == 0, ldx % 8 == 0, 16-byte aligned x and q. */
int w8a8_quant_per_token(const void* x, int64_t ldx, int8_t* q, float* scale,
                         int64_t M, int64_t K, void* stream);

/* Fused SiLU*mul + per-token quantiser.  gate_up[M, 2I] bf16 (row stride ld
 * elements); y = bf16(silu(gate) * up) as silu_and_mul computes it
 * (M/layers/activation.py:9-12), then q/scale of y as above.  y_out[M, I]
 * (nullable) receives the bf16 y.  With q and scale both null (y_out then
 * required) only the bf16 y is computed, with no quantisation: the plain
 * silu_and_mul(x, out).  Needs I % 8 == 0, ld % 8 == 0. */
int w8a8_silu_mul_quant(const void* gate_up, int64_t ld, int8_t* q, float* scale,
                        void* y_out, int64_t M, int64_t I, void* stream);

/* The per-token quantiser for rows whose absmax is already known: amax[M]
 * holds max |y| of each row as float bits (as w8a8_gemm_silu leaves it);
 * scale = amax/127 and q follow w8a8_quant_per_token's rule exactly.  The
 * second half of the gate_up + SiLU*mul + quantiser fusion (the reference's
 * gate_up F.linear and silu_and_mul, M/models/utils.py:44-50).  Needs
 * K % 8 == 0, ldy % 8 == 0, 16-byte aligned y and q. */
int w8a8_quant_rows_amax(const void* y, int64_t ldy, const uint32_t* amax, int8_t* q,
                         float* scale, int64_t M, int64_t K, void* stream);

/* RMSNorm fused with the per-token quantiser: the input side of qkv and
 * gate_up.  Replaces RMSNorm.forward / RMSNormFused.forward
 * (M/layers/norm.py:8-38) followed by the quantiser.  x[M, K] bf16 (row stride
 * ldx), weight[K] bf16.  With residual[M, K] (row stride ldr, nullable):
 * v = x + residual (fp32), residual_out = bf16(v) (required; may be the
 * residual itself); without: v = x and residual_out must be null.  Then
 * y = bf16((v * r) * weight) with r = 1 / sqrt(sum(v*v)/K + eps) (correctly
 * rounded), and q/scale are y's per-token quantisation.  y_out[M, K]
 * (nullable) receives y.  Needs K % 8 == 0, K <= 8192, 16-byte alignment. */
int w8a8_rmsnorm_quant(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                       const void* weight, float eps, int8_t* q, float* scale, void* residual_out,
                       void* y_out, int64_t M, int64_t K, void* stream);

/* ---------------------------------------------------------------- kernel 2
 * W8A8 GEMM on tcgen05 tensor cores: C[M, N] bf16 =
 *   bf16((f32(A[M,K] . B[N,K]^T) * sa[m]) * sb[n] + bias[n])
 * A = int8 activations [M, K] row-major, B = int8 weight [N, K] row-major
 * (nn.Linear layout), sa[M] / sb[N] fp32 scales, bias[N] bf16 (nullable).
 * c_i32 (nullable) receives the exact int32 accumulator [M, N].
 * Replaces F.linear in _LinearTPImpl.forward (M/layers/linear.py:31-32).
 * Needs K % 16 == 0, N % 16 == 0, 16-byte aligned A, B, C.
 * Schedule: stream-K over one persistent CTA per SM.  `workspace` holds the
 * int32 partial tiles of tiles cut between two CTAs plus one counter per tile;
 * the caller zero-initialises it once and every successful call leaves the
 * counters zero again.  w8a8_gemm_workspace_size() gives the bytes a shape
 * needs (0 = none); with less, ranges are rounded to whole tiles. */
size_t w8a8_gemm_workspace_size(int64_t M, int64_t N, int64_t K);
int w8a8_gemm(const int8_t* A, const int8_t* B, const float* sa, const float* sb,
              const void* bias, void* C, int32_t* c_i32, int64_t M, int64_t N, int64_t K,
              void* workspace, size_t workspace_bytes, void* stream);

/* gate_up GEMM with the SiLU*mul in its epilogue: B = [gate (I rows); up
 * (I rows)] int8 [2I, K] (the merged gate_up weight of
 * LinearColParallelMerged, M/layers/linear.py:56-71), bias [2I] or null;
 * Y[M, I] bf16 receives y = bf16(silu(g) * u), g and u the bf16 values
 * w8a8_gemm would write, and amax[M] (uint32, zeroed by the caller) the
 * float bits of every row's max |y| -- the gate_up linear and silu_and_mul
 * of GatedMLP (M/models/utils.py:44-50) without the [M, 2I] tensor in HBM.
 * Runs on the 2-SM pair kernel: M > 128 and 2I % 256 == 0, else
 * W8A8_ERR_UNSUPPORTED (take w8a8_gemm + w8a8_silu_mul_quant then). */
int w8a8_gemm_silu(const int8_t* A, const int8_t* B, const float* sa, const float* sb,
                   const void* bias, void* Y, uint32_t* amax, int64_t M, int64_t N2, int64_t K,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Same as w8a8_gemm with an explicit configuration (for tests and tuning):
 * variant 0 = auto, 1 = 128x256 tiles, 2 = 128x128 tiles, 3..6 =
 * weight-stationary (swap-AB) 128 x {16,32,64,128}, 7 = 256x256 blocks on
 * SM pairs (2-CTA clusters sharing one tcgen05 MMA, whole blocks, no
 * workspace); ctas = 0 for one CTA per SM, else the number of persistent
 * CTAs (at most one per SM; rounded down to an even count for variant 7). */
int w8a8_gemm_config(const int8_t* A, const int8_t* B, const float* sa, const float* sb,
                     const void* bias, void* C, int32_t* c_i32, int64_t M, int64_t N,
                     int64_t K, int variant, int ctas, void* workspace,
                     size_t workspace_bytes, void* stream);

/* w8a8_gemm without a caller workspace and without any allocation: the
 * stream-K scratch is a fixed 20 MiB device array in the library, one per
 * device.  No counterpart in the reference (its F.linear path allocates
 * through torch).  For callers that cannot allocate at call time: an engine
 * whose KV-cache pool holds the HBM left after the weights, and FFI callers
 * without a caching allocator, for which cudaMalloc/cudaFree mid-step would
 * synchronise the device.  Same plan and results as w8a8_gemm; a shape whose
 * plan needs more than 20 MiB of scratch returns W8A8_ERR_WORKSPACE before
 * any launch.  The first accepted non-empty call on a device (device current)
 * does the set-up (cudaGetSymbolAddress, counters cleared synchronously):
 * make it before any stream capture.  Overlapping calls on one device share
 * the scratch and race. */
int w8a8_gemm_static_scratch(const int8_t* A, const int8_t* B, const float* sa, const float* sb,
                             const void* bias, void* C, int32_t* c_i32, int64_t M, int64_t N,
                             int64_t K, void* stream);

/* Measurement only, no counterpart in the reference: the int8 tensor-core
 * ceiling of the current device.  Launches an MMA-only loop (operands
 * resident in shared memory, no global-memory traffic) of `iters` x 4
 * tcgen05.mma kind::i8 per CTA: pair = 0 one CTA per SM with 128 x 256 x 32
 * MMAs, pair = 1 CTA pairs with 256 x 256 x 32 MMAs (cta_group::2, the
 * prefill kernel's shape).  *ops_out receives the integer ops the launch
 * performs (2 x MACs); the caller times the launch on `stream` with events. */
int w8a8_mma_peak_probe(int pair, int64_t iters, int64_t* ops_out, void* stream);

/* Host-only planner query (no GPU needed): the configuration w8a8_gemm would
 * use for a shape on a device with num_sms SMs.  out[8] receives
 * {variant, BN, swap, tiles, CTAs, k-blocks per tile, partition granularity
 * in k-blocks, workspace bytes}. */
int w8a8_gemm_plan(int64_t M, int64_t N, int64_t K, int variant, int ctas, size_t workspace_bytes,
                   int num_sms, int64_t* out);

/* ------------------------------------------------------ mixture of experts
 * The expert path of fused_experts_impl (M/moe/fused.py:135-215) with int8
 * expert weights: w1 [E, 2I, H] ([gate; up] per expert) and w2 [E, H, I],
 * per-channel fp32 scales [E, 2I] / [E, H].  A slot s = t * topk + j is
 * token t's j-th choice (topk_ids / topk_weights [T, topk], row-major).
 * Sorted buffers have P = 128 * w8a8_moe_max_blocks(T * topk, E) rows; the
 * calls chain on one stream with no host sync (CUDA-graph capturable):
 *   w8a8_moe_align -> w8a8_moe_quant_scatter -> w8a8_moe_gemm (w1, SiLU)
 *   -> w8a8_moe_quant_rows -> w8a8_moe_gemm (w2, routed) -> w8a8_moe_sum */

/* Bound on the 128-row expert blocks of T * topk slots over E experts. */
int64_t w8a8_moe_max_blocks(int64_t num_slots, int64_t num_experts);

/* moe_align_block_size (M/moe/fused.py:32-83) with 128-row blocks: expert e
 * gets ceil(c_e / 128) consecutive blocks, its c_e slots first (order within
 * an expert unspecified), padding after.  Writes sorted_ids[P] (slot of each
 * row; num_slots on padding), block_expert[max_blocks], num_blocks[1],
 * inv_pos[num_slots] (row of each slot; -1 for an expert id outside [0, E),
 * which then contributes nothing) and 0 to sa_sorted on padding rows.
 * E <= 1024. */
int w8a8_moe_align(const int32_t* topk_ids, int64_t num_slots, int num_experts, int32_t* sorted_ids,
                   int32_t* block_expert, int32_t* num_blocks, int32_t* inv_pos, float* sa_sorted,
                   void* stream);

/* Per-token quantiser (w8a8_quant_per_token's rule) of x[T, K] whose int8 row
 * and scale are written to rows inv_pos[t * topk + j] (skipped when < 0) of
 * q_sorted[P, K] / sa_sorted[P].  K % 8 == 0, K <= 16384. */
int w8a8_moe_quant_scatter(const void* x, int64_t ldx, int64_t T, int64_t K, const int32_t* inv_pos, int topk,
                           int8_t* q_sorted, float* sa_sorted, void* stream);

/* Grouped W8A8 GEMM over the expert-sorted rows (tcgen05, 128 x 256 tiles of
 * one expert each; the blocks in use are read from num_blocks on the
 * device).  w [E * N, K] int8, sw [E * N].
 *  - silu_amax != null: w holds [gate; up] (N = 2I, N % 32 == 0); C [P, I]
 *    receives y = bf16(silu(g) * u), g and u the bf16 dequantised gate and
 *    up values, and silu_amax[P] (zeroed by the caller) each row's max |y|
 *    as float bits -- fused_moe_kernel on w1 plus silu_and_mul.
 *  - otherwise C [P, N] = bf16(((f32(acc) * sa) * sw) * route_w[slot]),
 *    route_w (nullable; needs sorted_ids) the slot's routing weight --
 *    fused_moe_kernel on w2 with MUL_ROUTED_WEIGHT.
 * K % 16 == 0, N % 16 == 0, 16-byte aligned a_sorted, w, sw and C. */
int w8a8_moe_gemm(const int8_t* a_sorted, const int8_t* w, const float* sa_sorted, const float* sw,
                  const int32_t* block_expert, const int32_t* num_blocks, int64_t max_blocks,
                  const int32_t* sorted_ids, const float* route_w, int64_t num_slots, void* C,
                  uint32_t* silu_amax, int num_experts, int64_t N, int64_t K, void* stream);

/* w8a8_quant_rows_amax over the rows in use (128 * *num_blocks, read on the
 * device) of y[P, K]. */
int w8a8_moe_quant_rows(const void* y, int64_t ldy, const uint32_t* amax, int8_t* q, float* scale,
                        const int32_t* num_blocks, int64_t max_blocks, int64_t K, void* stream);

/* moe_sum_reduce (M/kernel/triton/fused_moe.py:5-48): out[t] = bf16(sum over
 * j = 0..topk-1 of f32(c_sorted[inv_pos[t * topk + j]])), an fp32 sum from
 * zero in choice order; dropped choices add nothing.  H % 8 == 0. */
int w8a8_moe_sum(const void* c_sorted, int64_t ldc, const int32_t* inv_pos, int64_t T, int topk, int64_t H,
                 void* out, int64_t ldo, void* stream);

/* ---------------------------------------------------------------- kernel 3
 * Tensor-parallel communicator over NVLink / NVSwitch peer memory.
 * Replaces NCCLWrapper (M/kernel/csrc/src/pynccl.cu:74-91) + init_pynccl
 * (M/kernel/pynccl.py:45-78): each rank creates its buffers, exports an
 * opaque handle blob of w8a8_comm_handle_bytes() bytes, the blobs are
 * all-gathered over the CPU group (rank order), then every rank opens its
 * peers. */
typedef struct w8a8_comm w8a8_comm;
size_t w8a8_comm_handle_bytes(void);
int w8a8_comm_create(int rank, int world, int device, size_t max_bytes, w8a8_comm** comm,
                     void* handle_out);
int w8a8_comm_open_peers(w8a8_comm* comm, const void* all_handles);
/* Algorithm: 0 = automatic (one-shot for world 2 or small tensors, two-shot
 * with peer stores otherwise), 1 = always one-shot, 2 = always two-shot (peer
 * stores), 3 = the fused GEMM's two-shot through NVLS (needs the multicast
 * buffer; opt-in: measured slower than peer stores at world 2). */
int w8a8_comm_set_mode(w8a8_comm* comm, int mode);

/* Attach an NVSwitch multicast (NVLS) buffer for the fused row-parallel
 * reduce: `mc` its multicast address, `uc` this rank's unicast address of the
 * same memory, `bytes` >= 4 x max_bytes (rounded up to 4 KiB): two halves of
 * [partials | gathered shares].  Every rank attaches its own mapping of one
 * multicast object (the caller allocates it, e.g. with torch's symmetric
 * memory).  With it, each rank keeps its partial tiles local and the owner of
 * a row share reads their sum through the switch (multimem.ld_reduce, fp32
 * accumulation) and multicasts the result (multimem.st).  No counterpart in
 * NCCLWrapper, whose symmetric window (M/kernel/csrc/src/pynccl.cu:74-91)
 * lets NCCL do the same inside ncclAllReduce. */
int w8a8_comm_attach_multicast(w8a8_comm* comm, void* mc, void* uc, size_t bytes);
/* Bounded-wait budget of every device-side flag wait (default 10 s). */
int w8a8_comm_set_timeout_ms(w8a8_comm* comm, int64_t timeout_ms);

/* In-place sum all-reduce of a bf16 tensor across the ranks; every rank gets
 * the fp32 sum of the ranks' values in rank order, rounded once to bf16.
 * Replaces NCCLWrapper::all_reduce(t, "sum") (M/kernel/csrc/src/pynccl.cu:93-134)
 * and PyNCCLDistributedImpl.all_reduce (M/distributed/impl.py:44-50). */
int w8a8_all_reduce(w8a8_comm* comm, void* x, int64_t numel, void* stream);

/* In-place broadcast of nbytes (a multiple of 16, at most max_bytes) from
 * rank `root` to every rank over NVLink peer loads.  No counterpart in
 * NCCLWrapper (the reference's ranks each copy their own host input in); it
 * lets one rank copy a step's host input in once and hand it to the other
 * ranks on the device. */
int w8a8_broadcast(w8a8_comm* comm, void* x, int64_t nbytes, int root, void* stream);

/* Row-parallel W8A8 linear with the all-reduce fused into the GEMM: every
 * rank passes its K-shard (A[M, K_local], B[N, K_local]) and receives the
 * all-reduced C[M, N] on every rank.  Replaces LinearOProj.forward /
 * LinearRowParallel.forward (M/layers/linear.py:102-106,123-127). */
int w8a8_gemm_allreduce(w8a8_comm* comm, const int8_t* A, const int8_t* B, const float* sa,
                        const float* sb, const void* bias, void* C, int64_t M, int64_t N,
                        int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* Device-side status of the communicator: *device_error != 0 once a bounded
 * flag wait gave up (a peer that never arrived); synchronises the device. */
int w8a8_comm_status(w8a8_comm* comm, int* device_error);
void w8a8_comm_destroy(w8a8_comm* comm);

#ifdef __cplusplus
}
#endif

#endif /* W8A8_TP_H_ */
