// Device side of the tensor-parallel communicator: layout of the IPC-shared
// buffer, cross-rank flags with release/acquire at system scope, and the
// bounded flag wait.
//
// Every rank owns one cudaMalloc'd buffer, mapped into its peers with CUDA
// IPC (peer loads/stores travel over NVLink / NVSwitch):
//
//   [flags: 2 phases x kMaxSlots x kMaxWorld u32][ctrl: 1 KB][half 0][half 1]
//
// flags[phase][slot][src] on rank r is written by rank `src` (a peer store)
// and polled by rank r (local loads).  A flag holds the epoch of the call
// that last signalled it; waits compare for equality, epochs only grow.
// ctrl[0] = epoch of the last completed call, ctrl[1] = CTAs finished in the
// current call, ctrl[2..3] = where the last bounded wait gave up.  Calls use
// data half (epoch & 1): a rank can only start writing a half again after
// every peer has passed a barrier of the next call, i.e. after every peer has
// finished reading that half, so no end-of-call barrier is needed.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

#include "sm100.cuh"

namespace w8a8 {

constexpr int kMaxWorld = 8;
constexpr int kMaxSlots = 8192;
constexpr size_t kFlagBytes = 2ull * kMaxSlots * kMaxWorld * sizeof(uint32_t);
constexpr size_t kCtrlBytes = 1024;
constexpr size_t kHeaderBytes = kFlagBytes + kCtrlBytes;

struct CommView {
  char* base[kMaxWorld];  // every rank's buffer, as mapped in this process
  int rank;
  int world;
  unsigned long long half_bytes;  // (world + 1) * slot_bytes
  unsigned long long slot_bytes;  // one [M, N] bf16 tensor of at most max_bytes
  int two_shot;                   // fused GEMM reduce: 1 = two-shot, 0 = one-shot
  unsigned int* err;              // device error word
  long long timeout_ns;
  // NVLS (NVSwitch multicast) two-shot: a buffer of 2 halves x [partials P |
  // gather G] (slot_bytes each), bound to a multicast object on every rank.
  // nvls = 1: partial tiles stay in this rank's P; the row share's owner reads
  // the sum over all ranks with multimem.ld_reduce and multimem.st's it into
  // every rank's G.
  char* mc_base;                  // the buffer's multicast address (same on every rank's mapping)
  char* nv_local;                 // this rank's unicast address of the same buffer
  int nvls;
};

namespace dev {

__device__ __forceinline__ uint32_t* flag_ptr(char* base, int phase, int slot, int src) {
  return reinterpret_cast<uint32_t*>(base) + (static_cast<size_t>(phase) * kMaxSlots + slot) * kMaxWorld + src;
}

__device__ __forceinline__ uint32_t* ctrl_ptr(char* base) {
  return reinterpret_cast<uint32_t*>(base + kFlagBytes);
}

__device__ __forceinline__ char* half_ptr(const CommView& v, int r, uint32_t epoch) {
  return v.base[r] + kHeaderBytes + static_cast<size_t>(epoch & 1u) * v.half_bytes;
}

// Inside a data half, the fused GEMM reduce uses world receive slots (slot s
// holds source rank s's bf16 partial tiles, in the tile-blocked layout the
// fused epilogue pushes: tile t at t * 128 * BN * 2 bytes) followed by one
// gather slot (reduced row shares pushed by their owners, two-shot only, same
// layout).  The standalone all-reduce uses the start of the half (slot 0).
__device__ __forceinline__ char* recv_slot(const CommView& v, int at_rank, int src, uint32_t epoch) {
  return half_ptr(v, at_rank, epoch) + static_cast<size_t>(src) * v.slot_bytes;
}

__device__ __forceinline__ char* gather_slot(const CommView& v, int at_rank, uint32_t epoch) {
  return half_ptr(v, at_rank, epoch) + static_cast<size_t>(v.world) * v.slot_bytes;
}

// NVLS buffer regions of call `epoch` (half epoch & 1): P (partials) and G
// (gathered shares), at a unicast or multicast base.
__device__ __forceinline__ char* nv_partials(const CommView& v, char* base, uint32_t epoch) {
  return base + static_cast<size_t>(epoch & 1u) * 2 * v.slot_bytes;
}
__device__ __forceinline__ char* nv_gather(const CommView& v, char* base, uint32_t epoch) {
  return base + static_cast<size_t>(epoch & 1u) * 2 * v.slot_bytes + v.slot_bytes;
}

// Orders this thread's accesses through one virtual alias of a location
// (unicast or multicast) with its accesses through the other.
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// Sum over every rank of 8 bf16 at multicast address `mc`, reduced in the
// switch with fp32 accumulation, rounded once to bf16.
__device__ __forceinline__ uint4 mm_ld_reduce_bf16x8(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}

// Store 8 bf16 to the multicast address `mc`: every rank's copy receives them.
__device__ __forceinline__ void mm_st_bf16x8(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread `t` (< world) of the calling group tells rank t that this rank has
// reached (phase, slot) of call `epoch`.  The caller has synchronised the
// group after its data stores; the system-scope fence makes those stores
// (cumulatively) visible before the flag.
__device__ __forceinline__ void signal_peers(const CommView& v, int phase, int slot, uint32_t epoch, int t) {
  if (t < v.world) {
    if (v.nvls) fence_proxy_alias();  // the group's multimem stores precede the flag
    __threadfence_system();
    st_release_sys(flag_ptr(v.base[t], phase, slot, v.rank), epoch);
  }
}

// Thread `t` (< world) waits until rank t has signalled (phase, slot) of call
// `epoch`.  Bounded by v.timeout_ns; on expiry records where and returns false.
// Polls back off with a short sleep after the first few.
__device__ __forceinline__ bool wait_peer(const CommView& v, int phase, int slot, uint32_t epoch, int t) {
  if (t >= v.world) return true;
  const uint32_t* f = flag_ptr(v.base[v.rank], phase, slot, t);
  if (ld_acquire_sys(f) == epoch) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ld_acquire_sys(f) == epoch) return true;
    if ((it & 255u) == 0) {
      if (globaltimer_ns() - t0 > static_cast<uint64_t>(v.timeout_ns)) {
        if (v.err) atomicOr(v.err, 2u /* kErrCommWait */);
        uint32_t* c = ctrl_ptr(v.base[v.rank]);
        c[2] = (static_cast<uint32_t>(phase) << 24) | static_cast<uint32_t>(slot);
        c[3] = static_cast<uint32_t>(t);
        return false;
      }
    }
    if (it > 32) __nanosleep(32);
  }
}

// 16-byte load of data another rank (or another call) wrote: cached at L2
// only (.cg), never in this SM's L1, so no stale line can be hit.  Ordering
// comes from the flag protocol: the polling thread's acquire load of the flag,
// then a barrier of the reading threads, precede every such load.
__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}

// fp32 rank-order sum of 8 bf16 lanes from every rank's copy of one 16-byte
// vector, rounded once to bf16 (the oracle's all_reduce_sum: start from rank
// 0's value, add ranks 1..p-1 in order).
__device__ __forceinline__ uint4 sum_ranks_vec8(const CommView& v, uint32_t epoch, size_t byte_off) {
  float acc[8];
  {
    const uint4 raw = ld_volatile_v4(half_ptr(v, 0, epoch) + byte_off);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      acc[2 * j] = f.x;
      acc[2 * j + 1] = f.y;
    }
  }
  for (int r = 1; r < v.world; ++r) {
    const uint4 raw = ld_volatile_v4(half_ptr(v, r, epoch) + byte_off);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      acc[2 * j] = __fadd_rn(acc[2 * j], f.x);
      acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], f.y);
    }
  }
  uint4 out;
  __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
  return out;
}

}  // namespace dev
}  // namespace w8a8
