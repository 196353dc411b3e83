// Synchronisation of the sharded step's producers and consumers through peer memory (one GPU
// per rank, peers' buffers mapped with CUDA IPC over NVLink; plain loads and stores only).
//
// A producer launch (a kernel that writes this rank's slice of a buffer the other ranks read)
// ends with peer_signal_done: every CTA counts itself on a local counter with a GPU-scope
// acquire-release atomic (releasing the CTA's writes, its local ones and those into the other
// ranks' buffers alike); the last one, which thereby acquired every CTA's writes, resets the
// counter, issues ONE system-scope fence and stores the step's epoch into this rank's flag word
// in every rank's flag array.  By the PTX memory model's causality order (release / acquire at
// GPU scope between the CTAs, then the system-scope fence and flag store, then the consumer's
// system-scope acquire) every write of the launch is visible to a consumer that saw the flag.
// A system-scope fence costs microseconds: with one in every CTA before the counting, the 2-GPU
// config-5 step took 8.92 ms, against 6.54 ms with this protocol.
//
// A consumer launch (one that reads other ranks' slices) starts with peer_wait_all: warp 0 waits,
// bounded, until every rank's flag for this launch holds the epoch (one lane per rank), and the
// CTA proceeds (or records an error and skips its reads).
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
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Called by all 32 lanes of one warp: lane r < n_ranks waits (bounded) until rank r's flag
// reached the epoch, with system-scope acquire loads; the ranks' flags are thus polled in
// parallel, not one acquire after another.  The warp then synchronises, which orders every lane's
// acquire before the warp's later reads.  True when every flag reached the epoch; false (error
// bit set) after SKINNY_WAIT_NS.
__device__ __forceinline__ bool peer_wait_flags_warp(const PeerSync& s, int lane) {
  if (!s.epoch || !s.wait_flags) return true;
  bool ok = true;
  if (lane < s.n_ranks) {
    const uint32_t e = *s.epoch;
    const uint64_t t0 = globaltimer_ns();
    while (static_cast<int32_t>(ld_acquire_sys(s.wait_flags + lane) - e) < 0) {
      if (globaltimer_ns() - t0 > SKINNY_WAIT_NS) {
        atomicOr(s.err, kErrBitWaitPeer);
        ok = false;
        break;
      }
    }
  }
  ok = __all_sync(0xFFFFFFFFu, ok);
  __syncwarp();
  return ok;
}

// Every thread of the CTA: warp 0 waits, the CTA learns the outcome.
__device__ __forceinline__ bool peer_wait_all(const PeerSync& s, int* flag_smem) {
  if (!s.epoch || !s.wait_flags) return true;
  if (threadIdx.x < 32) {
    const bool ok = peer_wait_flags_warp(s, threadIdx.x);
    if (threadIdx.x == 0) *flag_smem = ok ? 1 : 0;
  }
  __syncthreads();
  return *flag_smem != 0;
}

// Every thread of the CTA, after its last write of the launch.
__device__ __forceinline__ void peer_signal_done(const PeerSync& s, int* flag_smem) {
  if (!s.epoch || !s.counter) return;
  __syncthreads();  // the CTA's writes, observed by thread 0 through the barrier
  if (threadIdx.x == 0) {
    const uint32_t n = gridDim.x * gridDim.y * gridDim.z;
    const uint32_t prev = atom_add_acq_rel_gpu(s.counter, 1u);  // release ours, acquire the earlier CTAs'
    *flag_smem = prev == n - 1;
  }
  __syncthreads();
  if (*flag_smem && threadIdx.x == 0) {
    *s.counter = 0u;  // (the next launch's atomics come after this kernel in stream order)
    asm volatile("fence.acq_rel.sys;" ::: "memory");  // with the relaxed stores: a system-scope release
    const uint32_t e = *s.epoch;
    for (int r = 0; r < s.n_ranks; ++r) st_relaxed_sys(s.signal_flags[r], e);
  }
}

}  // namespace skinny
