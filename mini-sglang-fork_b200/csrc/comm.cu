// Kernel 3: tensor-parallel communicator over NVLink / NVSwitch peer memory.
//
// Host side: one IPC-exportable buffer per rank (flags + control words + two
// data halves), handle blobs exchanged by the caller over its CPU group
// (rank order), peers opened with cudaIpcOpenMemHandle.  Replaces
// mini-sglang's NCCLWrapper (M/kernel/csrc/src/pynccl.cu:74-134) for the
// row-parallel all-reduce.
//
// Device side (standalone in-place all-reduce of a bf16 tensor):
//   one-shot  (world 2 or small messages): every rank stages its tensor in its
//             buffer, one cross-rank barrier, then sums all ranks' copies of
//             its share of vectors straight into the output;
//   two-shot  (large messages): stage, barrier, reduce-scatter (rank r sums
//             chunk r from every rank into its own buffer), barrier,
//             all-gather (rank r copies chunk c from rank c).
// CTA b owns sub-range b of every chunk, so the barriers are per CTA (flag
// slot b) — no grid-wide synchronisation.  Every flag wait is bounded.
#include <cuda_bf16.h>

#include <cstring>
#include <mutex>

#include "comm_dev.cuh"
#include "common.cuh"
#include "gemm_api.h"
#include "gemm_plan.h"

namespace {

constexpr uint32_t kBlobMagic = 0x57384138u;  // "W8A8"

struct HandleBlob {
  uint32_t magic;
  int32_t rank;
  int32_t world;
  int32_t device;
  uint64_t half_bytes;
  uint64_t total_bytes;
  cudaIpcMemHandle_t handle;
};

}  // namespace

struct w8a8_comm {
  int rank = 0;
  int world = 1;
  int device = 0;
  size_t slot_bytes = 0;   // max_bytes rounded up
  size_t half_bytes = 0;   // (world + 1) * slot_bytes
  size_t total_bytes = 0;
  char* local = nullptr;
  char* peers[w8a8::kMaxWorld] = {nullptr};
  bool opened = false;
  long long timeout_ns = 10000000000LL;  // 10 s
  int mode = 0;                           // 0 auto, 1 one-shot, 2 two-shot, 3 NVLS two-shot (fused GEMM)
  char* nv_mc = nullptr;                  // attached multicast buffer (NVLS), or null
  char* nv_uc = nullptr;
  size_t nv_bytes = 0;
};

namespace w8a8 {

namespace {

constexpr int kArThreads = 512;

__device__ __forceinline__ void finish_call(const CommView& v, uint32_t epoch) {
  // The last CTA of the call publishes the epoch for the next call (which is
  // stream-ordered after this kernel, so it sees the update).
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* c = dev::ctrl_ptr(v.base[v.rank]);
    __threadfence();
    const uint32_t done = atomicAdd(c + 1, 1u);
    if (done == gridDim.x - 1) {
      c[1] = 0u;
      __threadfence();
      atomicExch(c, epoch);
    }
  }
}

// Cross-rank barrier of this CTA at (phase, slot): signal every rank, then
// wait for every rank.  Returns false (uniformly across the CTA) on timeout.
__device__ __forceinline__ bool cta_barrier(const CommView& v, int phase, int slot, uint32_t epoch) {
  __syncthreads();
  dev::signal_peers(v, phase, slot, epoch, threadIdx.x);
  const bool ok = dev::wait_peer(v, phase, slot, epoch, threadIdx.x);
  return __syncthreads_and(ok) != 0;
}

// Copy vectors [lo, hi) of `src` to `dst`, four per thread in flight.
template <class Load>
__device__ __forceinline__ void copy_vectors(uint4* dst, Load load, long long lo, long long hi) {
  const long long s = blockDim.x;
  for (long long i = lo + threadIdx.x; i < hi; i += 4 * s) {
    uint4 t[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i + u * s < hi) t[u] = load(i + u * s);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i + u * s < hi) dst[i + u * s] = t[u];
  }
}

// fp32 rank-order sum (rank 0's value, then ranks 1..W-1 added in order, one
// bf16 rounding) of vectors i and i + s (those below hi) over every rank's
// staged copy.  All 2 * W loads are issued before the first add.
template <int W>
__device__ __forceinline__ void sum_ranks_pair(const CommView& v, uint32_t epoch, long long i, long long s,
                                               long long hi, uint4 (&out)[2]) {
  uint4 raw[2][W];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const long long k = i + u * s;
    if (k < hi) {
#pragma unroll
      for (int r = 0; r < W; ++r) raw[u][r] = dev::ld_volatile_v4(dev::half_ptr(v, r, epoch) + static_cast<size_t>(k) * 16);
    }
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    if (i + u * s >= hi) continue;
    float acc[8];
    const __nv_bfloat162* h0 = reinterpret_cast<const __nv_bfloat162*>(&raw[u][0]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h0[j]);
      acc[2 * j] = f.x;
      acc[2 * j + 1] = f.y;
    }
#pragma unroll
    for (int r = 1; r < W; ++r) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[u][r]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] = __fadd_rn(acc[2 * j], f.x);
        acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], f.y);
      }
    }
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out[u]);
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
  }
}

// Reduce vectors [lo, hi) into x (and into this rank's staged copy when
// `mine` is set).  W = world at compile time (0: any world, one vector at a
// time).
template <int W>
__device__ __forceinline__ void reduce_range(const CommView& v, uint32_t epoch, uint4* x, uint4* mine, long long lo,
                                             long long hi) {
  const long long s = blockDim.x;
  if constexpr (W > 0) {
    for (long long i = lo + threadIdx.x; i < hi; i += 2 * s) {
      uint4 out[2];
      sum_ranks_pair<W>(v, epoch, i, s, hi, out);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (i + u * s >= hi) continue;
        if (mine) mine[i + u * s] = out[u];
        x[i + u * s] = out[u];
      }
    }
  } else {
    for (long long i = lo + threadIdx.x; i < hi; i += s) {
      const uint4 o = dev::sum_ranks_vec8(v, epoch, static_cast<size_t>(i) * 16);
      if (mine) mine[i] = o;
      x[i] = o;
    }
  }
}

// x: nvec 16-byte vectors (8 bf16 each), in place.
template <int W>
__global__ void __launch_bounds__(kArThreads) allreduce_kernel(CommView v, uint4* x, long long nvec, int two_shot) {
  dev::griddep_wait();  // x and the epoch word come from earlier kernels
  dev::griddep_launch();
  const uint32_t epoch = dev::ld_relaxed_gpu(dev::ctrl_ptr(v.base[v.rank])) + 1u;
  uint4* mine = reinterpret_cast<uint4*>(dev::half_ptr(v, v.rank, epoch));
  const int slot = blockIdx.x;
  // chunk c = [c*cv, min(nvec, (c+1)*cv)); CTA b owns [b*sub, (b+1)*sub) of each
  const long long chunks = two_shot ? v.world : 1;
  const long long cv = (nvec + chunks - 1) / chunks;
  const long long sub = (cv + gridDim.x - 1) / gridDim.x;
  auto range = [&](long long c, long long& lo, long long& hi) {
    const long long c0 = c * cv, c1 = min(nvec, c0 + cv);
    lo = c0 + blockIdx.x * sub;
    hi = min(c1, lo + sub);
  };
  // stage
  for (long long c = 0; c < chunks; ++c) {
    long long lo, hi;
    range(c, lo, hi);
    copy_vectors(mine, [&](long long i) { return x[i]; }, lo, hi);
  }
  bool ok = cta_barrier(v, 0, slot, epoch);
  if (ok) {
    long long lo, hi;
    if (!two_shot) {
      range(0, lo, hi);
      reduce_range<W>(v, epoch, x, nullptr, lo, hi);
    } else {
      range(v.rank, lo, hi);
      reduce_range<W>(v, epoch, x, mine, lo, hi);
      ok = cta_barrier(v, 1, slot, epoch);
      if (ok) {
        for (int c = 0; c < v.world; ++c) {
          if (c == v.rank) continue;
          range(c, lo, hi);
          const char* src = dev::half_ptr(v, c, epoch);
          copy_vectors(x, [&](long long i) { return dev::ld_volatile_v4(src + static_cast<size_t>(i) * 16); }, lo, hi);
        }
      }
    }
  }
  finish_call(v, epoch);
}

// Broadcast of `nvec` 16-byte vectors from rank `root` to every rank, in
// place: the root stages its tensor in its own buffer, one cross-rank barrier
// per CTA, then every other rank pulls CTA b's sub-range from the root's
// buffer over NVLink.
__global__ void __launch_bounds__(kArThreads) broadcast_kernel(CommView v, uint4* x, long long nvec, int root) {
  dev::griddep_wait();
  dev::griddep_launch();
  const uint32_t epoch = dev::ld_relaxed_gpu(dev::ctrl_ptr(v.base[v.rank])) + 1u;
  const long long sub = (nvec + gridDim.x - 1) / gridDim.x;
  const long long lo = blockIdx.x * sub, hi = min(nvec, lo + sub);
  if (v.rank == root) {
    uint4* mine = reinterpret_cast<uint4*>(dev::half_ptr(v, v.rank, epoch));
    copy_vectors(mine, [&](long long i) { return x[i]; }, lo, hi);
  }
  if (cta_barrier(v, 0, blockIdx.x, epoch) && v.rank != root) {
    const char* src = dev::half_ptr(v, root, epoch);
    copy_vectors(x, [&](long long i) { return dev::ld_volatile_v4(src + static_cast<size_t>(i) * 16); }, lo, hi);
  }
  finish_call(v, epoch);
}

}  // namespace

CommView make_view(const w8a8_comm* c, unsigned int* err) {
  CommView v;
  std::memset(&v, 0, sizeof(v));
  for (int r = 0; r < c->world; ++r) v.base[r] = (r == c->rank) ? c->local : c->peers[r];
  v.rank = c->rank;
  v.world = c->world;
  v.half_bytes = c->half_bytes;
  v.slot_bytes = c->slot_bytes;
  v.two_shot = 0;
  v.err = err;
  v.timeout_ns = c->timeout_ns;
  v.mc_base = c->nv_mc;
  v.nv_local = c->nv_uc;
  v.nvls = 0;
  return v;
}

// One-shot when the extra traffic of reading every peer's whole tensor is
// small (or equal, at world 2); two-shot otherwise.
bool use_one_shot(int world, size_t bytes) { return world <= 2 || bytes * (world - 1) <= (size_t(1) << 20); }

int comm_ready(const w8a8_comm* c) {
  W8A8_REQUIRE(c != nullptr, W8A8_ERR_INVALID_ARG, "comm is null");
  W8A8_REQUIRE(c->opened || c->world == 1, W8A8_ERR_STATE, "comm: peers not opened (call w8a8_comm_open_peers)");
  int dev = current_device();
  W8A8_REQUIRE(dev == c->device, W8A8_ERR_STATE, "comm: current device %d is not the comm's device %d", dev,
               c->device);
  return W8A8_OK;
}

}  // namespace w8a8

extern "C" {

size_t w8a8_comm_handle_bytes(void) { return sizeof(HandleBlob); }

int w8a8_comm_create(int rank, int world, int device, size_t max_bytes, w8a8_comm** out, void* handle_out) {
  using namespace w8a8;
  W8A8_REQUIRE(out && handle_out, W8A8_ERR_INVALID_ARG, "comm_create: null output pointer");
  *out = nullptr;
  W8A8_REQUIRE(world >= 1 && world <= kMaxWorld, W8A8_ERR_INVALID_ARG, "comm_create: world %d not in [1, %d]",
               world, kMaxWorld);
  W8A8_REQUIRE(rank >= 0 && rank < world, W8A8_ERR_INVALID_ARG, "comm_create: rank %d not in [0, %d)", rank, world);
  W8A8_REQUIRE(max_bytes > 0 && max_bytes <= (size_t(8) << 30), W8A8_ERR_INVALID_ARG,
               "comm_create: max_bytes %zu not in (0, 8 GiB]", max_bytes);
  int prev = -1;
  W8A8_CUDA_TRY(cudaGetDevice(&prev));
  W8A8_CUDA_TRY(cudaSetDevice(device));
  auto* c = new w8a8_comm();
  c->rank = rank;
  c->world = world;
  c->device = device;
  c->slot_bytes = round_up(max_bytes, 4096);
  c->half_bytes = static_cast<size_t>(world + 1) * c->slot_bytes;
  c->total_bytes = kHeaderBytes + 2 * c->half_bytes;
  cudaError_t e = cudaMalloc(&c->local, c->total_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, kHeaderBytes);
  HandleBlob blob;
  std::memset(&blob, 0, sizeof(blob));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&blob.handle, c->local);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return fail(W8A8_ERR_CUDA, "comm_create: %s", cudaGetErrorString(e));
  }
  blob.magic = kBlobMagic;
  blob.rank = rank;
  blob.world = world;
  blob.device = device;
  blob.half_bytes = c->half_bytes;
  blob.total_bytes = c->total_bytes;
  std::memcpy(handle_out, &blob, sizeof(blob));
  *out = c;
  return W8A8_OK;
}

int w8a8_comm_open_peers(w8a8_comm* c, const void* all_handles) {
  using namespace w8a8;
  W8A8_REQUIRE(c && all_handles, W8A8_ERR_INVALID_ARG, "comm_open_peers: null argument");
  W8A8_REQUIRE(!c->opened, W8A8_ERR_STATE, "comm_open_peers: already opened");
  const auto* blobs = static_cast<const HandleBlob*>(all_handles);
  for (int r = 0; r < c->world; ++r) {
    const HandleBlob& b = blobs[r];
    W8A8_REQUIRE(b.magic == kBlobMagic && b.rank == r && b.world == c->world, W8A8_ERR_INVALID_ARG,
                 "comm_open_peers: handle %d is not rank %d's blob of a world-%d communicator", r, r, c->world);
    W8A8_REQUIRE(b.half_bytes == c->half_bytes, W8A8_ERR_INVALID_ARG,
                 "comm_open_peers: rank %d was created with a different max_bytes", r);
    W8A8_REQUIRE(r == c->rank || b.device != c->device, W8A8_ERR_INVALID_ARG,
                 "comm_open_peers: ranks %d and %d share device %d (one rank per GPU required)", r, c->rank,
                 c->device);
  }
  int prev = -1;
  W8A8_CUDA_TRY(cudaGetDevice(&prev));
  W8A8_CUDA_TRY(cudaSetDevice(c->device));
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, blobs[r].handle, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (c->peers[q]) {
          cudaIpcCloseMemHandle(c->peers[q]);
          c->peers[q] = nullptr;
        }
      cudaSetDevice(prev);
      return fail(W8A8_ERR_CUDA, "comm_open_peers: opening rank %d's buffer failed: %s", r, cudaGetErrorString(e));
    }
    c->peers[r] = static_cast<char*>(p);
  }
  cudaSetDevice(prev);
  c->opened = true;
  return W8A8_OK;
}

int w8a8_comm_set_mode(w8a8_comm* c, int mode) {
  W8A8_REQUIRE(c != nullptr, W8A8_ERR_INVALID_ARG, "comm_set_mode: null comm");
  W8A8_REQUIRE(mode >= 0 && mode <= 3, W8A8_ERR_INVALID_ARG, "comm_set_mode: mode %d not in {0, 1, 2, 3}", mode);
  W8A8_REQUIRE(mode != 3 || c->nv_mc != nullptr, W8A8_ERR_STATE,
               "comm_set_mode: mode 3 (NVLS) needs a multicast buffer (w8a8_comm_attach_multicast)");
  c->mode = mode;
  return W8A8_OK;
}

int w8a8_comm_attach_multicast(w8a8_comm* c, void* mc, void* uc, size_t bytes) {
  using namespace w8a8;
  W8A8_REQUIRE(c != nullptr && mc != nullptr && uc != nullptr, W8A8_ERR_INVALID_ARG,
               "comm_attach_multicast: null argument");
  W8A8_REQUIRE(W8A8_ALIGNED16(mc) && W8A8_ALIGNED16(uc), W8A8_ERR_ALIGNMENT,
               "comm_attach_multicast: addresses must be 16-byte aligned");
  W8A8_REQUIRE(bytes >= 4 * c->slot_bytes, W8A8_ERR_INVALID_ARG,
               "comm_attach_multicast: %zu bytes, need 2 halves x (partials + gather) = %zu", bytes,
               4 * c->slot_bytes);
  c->nv_mc = static_cast<char*>(mc);
  c->nv_uc = static_cast<char*>(uc);
  c->nv_bytes = bytes;
  return W8A8_OK;
}

int w8a8_comm_set_timeout_ms(w8a8_comm* c, int64_t timeout_ms) {
  W8A8_REQUIRE(c != nullptr, W8A8_ERR_INVALID_ARG, "comm_set_timeout_ms: null comm");
  W8A8_REQUIRE(timeout_ms > 0 && timeout_ms <= 600000, W8A8_ERR_INVALID_ARG,
               "comm_set_timeout_ms: %lld ms not in (0, 600000]", (long long)timeout_ms);
  c->timeout_ns = timeout_ms * 1000000LL;
  return W8A8_OK;
}

int w8a8_all_reduce(w8a8_comm* c, void* x, int64_t numel, void* stream) {
  using namespace w8a8;
  int rc = comm_ready(c);
  if (rc) return rc;
  W8A8_REQUIRE(numel >= 0, W8A8_ERR_INVALID_ARG, "all_reduce: negative numel");
  if (numel == 0 || c->world == 1) return W8A8_OK;
  W8A8_REQUIRE(x != nullptr, W8A8_ERR_INVALID_ARG, "all_reduce: null tensor");
  W8A8_REQUIRE(numel % 8 == 0, W8A8_ERR_INVALID_ARG, "all_reduce: numel %lld must be a multiple of 8",
               (long long)numel);
  W8A8_REQUIRE(W8A8_ALIGNED16(x), W8A8_ERR_ALIGNMENT, "all_reduce: tensor must be 16-byte aligned");
  const size_t bytes = static_cast<size_t>(numel) * 2;
  W8A8_REQUIRE(bytes <= c->slot_bytes, W8A8_ERR_INVALID_ARG,
               "all_reduce: %zu bytes exceed the communicator's max_bytes %zu", bytes, c->slot_bytes);
  unsigned int* err = device_error_word();
  if (!err) return W8A8_ERR_CUDA;
  const CommView v = make_view(c, err);
  const long long nvec = numel / 8;
  const bool one = c->mode == 1 || (c->mode == 0 && use_one_shot(c->world, bytes));
  const long long per_chunk = one ? nvec : (nvec + c->world - 1) / c->world;
  int nsm = sm_count();
  if (nsm <= 0) nsm = 148;
  long long grid = (per_chunk + kArThreads * 2 - 1) / (kArThreads * 2);
  grid = grid < 1 ? 1 : (grid > 2 * nsm ? 2 * nsm : grid);
  const dim3 g(static_cast<unsigned>(grid)), b(kArThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint4* xv = static_cast<uint4*>(x);
  const int two = one ? 0 : 1;
  switch (c->world) {
    case 2: W8A8_CUDA_TRY(launch_pdl(allreduce_kernel<2>, g, b, 0, st, v, xv, nvec, two)); break;
    case 4: W8A8_CUDA_TRY(launch_pdl(allreduce_kernel<4>, g, b, 0, st, v, xv, nvec, two)); break;
    case 8: W8A8_CUDA_TRY(launch_pdl(allreduce_kernel<8>, g, b, 0, st, v, xv, nvec, two)); break;
    default: W8A8_CUDA_TRY(launch_pdl(allreduce_kernel<0>, g, b, 0, st, v, xv, nvec, two)); break;
  }
  return W8A8_OK;
}

int w8a8_broadcast(w8a8_comm* c, void* x, int64_t nbytes, int root, void* stream) {
  using namespace w8a8;
  int rc = comm_ready(c);
  if (rc) return rc;
  W8A8_REQUIRE(nbytes >= 0, W8A8_ERR_INVALID_ARG, "broadcast: negative size");
  W8A8_REQUIRE(root >= 0 && root < c->world, W8A8_ERR_INVALID_ARG, "broadcast: root %d not in [0, %d)", root,
               c->world);
  if (nbytes == 0 || c->world == 1) return W8A8_OK;
  W8A8_REQUIRE(x != nullptr, W8A8_ERR_INVALID_ARG, "broadcast: null tensor");
  W8A8_REQUIRE(nbytes % 16 == 0, W8A8_ERR_INVALID_ARG, "broadcast: %lld bytes is not a multiple of 16",
               (long long)nbytes);
  W8A8_REQUIRE(W8A8_ALIGNED16(x), W8A8_ERR_ALIGNMENT, "broadcast: tensor must be 16-byte aligned");
  W8A8_REQUIRE(static_cast<size_t>(nbytes) <= c->slot_bytes, W8A8_ERR_INVALID_ARG,
               "broadcast: %lld bytes exceed the communicator's max_bytes %zu", (long long)nbytes, c->slot_bytes);
  unsigned int* err = device_error_word();
  if (!err) return W8A8_ERR_CUDA;
  const CommView v = make_view(c, err);
  const long long nvec = nbytes / 16;
  int nsm = sm_count();
  if (nsm <= 0) nsm = 148;
  long long grid = (nvec + kArThreads * 4 - 1) / (kArThreads * 4);
  grid = grid < 1 ? 1 : (grid > 2 * nsm ? 2 * nsm : grid);
  W8A8_CUDA_TRY(launch_pdl(broadcast_kernel, dim3(static_cast<unsigned>(grid)), dim3(kArThreads), 0,
                           static_cast<cudaStream_t>(stream), v, static_cast<uint4*>(x), nvec, root));
  return W8A8_OK;
}

int w8a8_gemm_allreduce(w8a8_comm* c, const int8_t* A, const int8_t* B, const float* sa, const float* sb,
                        const void* bias, void* C, int64_t M, int64_t N, int64_t K, void* workspace,
                        size_t workspace_bytes, void* stream) {
  using namespace w8a8;
  int rc = comm_ready(c);
  if (rc) return rc;
  if (c->world == 1)
    return run_gemm(A, B, sa, sb, bias, C, nullptr, M, N, K, 0, 0, workspace, workspace_bytes,
                    static_cast<cudaStream_t>(stream), kDefaultGemmTimeoutNs, nullptr);
  unsigned int* err = device_error_word();
  if (!err) return W8A8_ERR_CUDA;
  CommView v = make_view(c, err);
  // One-shot push (every rank receives every partial row and reduces the whole
  // tile itself: one flag hop) unless the extra (world - 2) copies of the
  // output would cost more NVLink time than a second hop: two-shot for large
  // outputs at world >= 4 (tiles in the normal orientation, M > 64).
  const size_t bytes = static_cast<size_t>(M) * N * 2;
  const bool big = c->world >= 4 && M > 64 && bytes * (c->world - 1) > (4u << 20);
  const bool two = c->mode == 2 || c->mode == 3 || (c->mode == 0 && big);
  v.two_shot = (two && M > 64) ? 1 : 0;
  // NVLS two-shot only when asked for (mode 3, with a multicast buffer
  // attached).  It moves ~(1 + 1/p) x the output per rank and direction
  // against 2 (p - 1) / p x for peer stores, but measured at world 2 its
  // switch-reduced loads (few in flight per thread, each a round trip through
  // the switch) left the reduce ~4x longer than the peer-store path, so the
  // automatic mode keeps peer stores.
  v.nvls = (v.two_shot && c->nv_mc != nullptr && c->mode == 3) ? 1 : 0;
  return run_gemm(A, B, sa, sb, bias, C, nullptr, M, N, K, 0, 0, workspace, workspace_bytes,
                  static_cast<cudaStream_t>(stream), c->timeout_ns, &v);
}

int w8a8_comm_status(w8a8_comm* c, int* device_error) {
  using namespace w8a8;
  W8A8_REQUIRE(c && device_error, W8A8_ERR_INVALID_ARG, "comm_status: null argument");
  int prev = -1;
  W8A8_CUDA_TRY(cudaGetDevice(&prev));
  W8A8_CUDA_TRY(cudaSetDevice(c->device));
  int code = 0;
  int rc = w8a8_device_error(&code, 0);
  cudaSetDevice(prev);
  if (rc) return rc;
  *device_error = code & static_cast<int>(kErrCommWait);
  return W8A8_OK;
}

void w8a8_comm_destroy(w8a8_comm* c) {
  if (!c) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < c->world; ++r)
    if (c->peers[r]) cudaIpcCloseMemHandle(c->peers[r]);
  if (c->local) cudaFree(c->local);
  if (prev >= 0) cudaSetDevice(prev);
  delete c;
}

}  // extern "C"
