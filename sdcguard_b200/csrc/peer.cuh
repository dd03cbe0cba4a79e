// Peer-memory synchronisation shared by the NVLink collectives (tensor-parallel reduce-scatter / all-gather,
// expert-parallel dispatch / combine): symmetric buffers are addressed through a table of every rank's base
// pointer, and one collective step is a generation flag that every rank publishes to every peer.
//
//   signal : gen += 1 on this rank; store gen into flags[my_rank] of every peer (release, system scope).
//   wait   : spin (bounded by wait_limit_ns() of %globaltimer) until every flags[r] of this rank >= gen (acquire).
//
// Every rank calls signal/wait the same number of times in the same order, so the generations agree; the
// counter lives on the device, which keeps the sequence valid inside CUDA graphs.
#pragma once

#include "common.cuh"

namespace sdc {
namespace peer {

constexpr int MAXW = 8;

struct Peers {
  const void* ptr[MAXW];    // per rank: base of that rank's copy of a symmetric buffer
};

inline Peers make_peers(const unsigned long long* ptrs, int world) {
  Peers p;
  for (int i = 0; i < MAXW; ++i) p.ptr[i] = i < world ? reinterpret_cast<const void*>(ptrs[i]) : nullptr;
  return p;
}

__device__ __forceinline__ long long ld_acquire_sys(const long long* p) {
  long long v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(long long* p, long long v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// one thread: bump the generation and publish it to every peer's flag slot for this rank
static __global__ void signal_kernel(long long* gen, Peers flags, int world, int rank) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const long long g = *gen + 1;
  *gen = g;
  __threadfence_system();
  for (int r = 0; r < world; ++r) st_release_sys(static_cast<long long*>(const_cast<void*>(flags.ptr[r])) + rank, g);
}

// every CTA's thread 0 waits for all peers to reach this rank's generation; returns false on timeout
__device__ inline bool wait_all(const long long* gen, const long long* my_flags, int world, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const long long g = *gen;
    ok = 1;
    const unsigned long long t0 = globaltimer();
    for (int r = 0; r < world && ok; ++r) {
      while (ld_acquire_sys(my_flags + r) < g) {
        if (globaltimer() - t0 > wait_limit_ns()) {
          ok = 0;
          record_error(err, ERR_TIMEOUT_PEER);
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

}  // namespace peer
}  // namespace sdc
