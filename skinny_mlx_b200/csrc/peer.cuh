// Synchronisation of the sharded step's producers and consumers through peer memory (one GPU
// per rank, peers' buffers mapped with CUDA IPC over NVLink; plain loads and stores only).
//
// A producer launch (a kernel that writes this rank's slice of a buffer the other ranks read)
// ends with peer_signal_done: every CTA fences its writes at system scope and counts itself on a
// local counter; the last one resets the counter and stores the step's epoch into this rank's
// flag word in every rank's flag array.  A consumer launch (one that reads other ranks' slices)
// starts with peer_wait_all: one thread waits, bounded, until every rank's flag for this launch
// holds the epoch, and the CTA proceeds (or records an error and skips its reads).
//
// The epoch is a device counter the caller advances once per step, so one captured graph serves
// every step; flags only grow, so a flag is never reset while a peer may still read it.
#pragma once
#include <cstdint>

#include "../../include/skinny_b200.h"
#include "ptx.cuh"
#include "skinny_status.h"

namespace skinny {

constexpr int kMaxPeers = 8;

struct PeerSync {
  const uint32_t* epoch;        // null: no peer synchronisation in this launch
  const uint32_t* wait_flags;   // [n_ranks] local flags to wait for, or null
  uint32_t* counter;            // local completion counter of this launch, or null (no signal)
  uint32_t* signal_flags[kMaxPeers];
  uint32_t* err;
  int n_ranks;
  uint8_t* mirror[kMaxPeers];  // other ranks' copies of the launch's digit output (xq)
  int n_mirror;
};

inline PeerSync peer_sync_from(const skinny_peer_sync* s) {
  PeerSync p{};
  if (!s) return p;
  p.epoch = s->epoch;
  p.wait_flags = s->wait_flags;
  p.counter = s->counter;
  for (int i = 0; i < kMaxPeers; ++i) p.signal_flags[i] = s->signal_flags[i];
  p.err = s->err;
  p.n_ranks = s->n_ranks;
  p.n_mirror = s->epoch ? s->n_mirror : 0;
  for (int i = 0; i < kMaxPeers; ++i) p.mirror[i] = i < p.n_mirror ? static_cast<uint8_t*>(s->mirror[i]) : nullptr;
  return p;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Called by one thread.  True when every rank's flag reached the epoch; false (error bit set)
// after SKINNY_WAIT_NS.
__device__ __forceinline__ bool peer_wait_flags(const PeerSync& s) {
  if (!s.epoch || !s.wait_flags) return true;
  const uint32_t e = *s.epoch;
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < s.n_ranks; ++r) {
    while (static_cast<int32_t>(ld_acquire_sys(s.wait_flags + r) - e) < 0) {
      if (globaltimer_ns() - t0 > SKINNY_WAIT_NS) {
        atomicOr(s.err, kErrBitWaitPeer);
        return false;
      }
    }
  }
  return true;
}

// Every thread of the CTA: thread 0 waits, the CTA learns the outcome.
__device__ __forceinline__ bool peer_wait_all(const PeerSync& s, int* flag_smem) {
  if (!s.epoch || !s.wait_flags) return true;
  if (threadIdx.x == 0) *flag_smem = peer_wait_flags(s) ? 1 : 0;
  __syncthreads();
  return *flag_smem != 0;
}

// Every thread of the CTA, after its last write of the launch.
__device__ __forceinline__ void peer_signal_done(const PeerSync& s, int* flag_smem) {
  if (!s.epoch || !s.counter) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this CTA's writes (ordered before by the barrier) reach every rank
    const uint32_t n = gridDim.x * gridDim.y * gridDim.z;
    const uint32_t prev = atomicAdd(s.counter, 1u);
    *flag_smem = prev == n - 1;
  }
  __syncthreads();
  if (*flag_smem && threadIdx.x == 0) {
    *s.counter = 0u;
    __threadfence_system();  // every CTA's writes: they fenced before counting
    const uint32_t e = *s.epoch;
    for (int r = 0; r < s.n_ranks; ++r) st_release_sys(s.signal_flags[r], e);
  }
}

}  // namespace skinny
