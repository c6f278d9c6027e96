// qw_exchange.cuh -- the peer-memory exchange protocol of a communicator
// (qw_allreduce), shared by the allreduce and greedy-token kernels and by the
// decode kernel's fused row-parallel epilogue.
//
// Each rank owns one buffer that every rank maps (CUDA IPC):
//   [flags: 2 parities x 8 ranks x 1024 chunks of uint32]
//   [data:  2 parities x P ranks x n_max floats]
// A call with epoch e (parity e & 1) stores rank `rank`'s values into slot
// (parity, rank) of every rank's data, then flags (parity, rank, chunk) = e
// in every rank's flags with system-scope release; a reader waits (bounded)
// until flag (parity, r, chunk) of its own buffer reaches e for every rank r
// (acquire) and reads the slots.  A call's epoch is the number of calls
// before it plus one, kept on the device: every CTA reads it after the
// previous kernel of the stream completed, and the call's last CTA to finish
// publishes it (ar_finish), so a call captured in a CUDA graph advances on
// every replay and ranks running the same sequence of calls agree without a
// host exchange.  Two parities make slot reuse safe: a rank stores call
// e + 2 only after its call e + 1 completed, which needed every rank's flag
// of call e + 1, and a rank flags call e + 1 only after its whole call e
// (its reads of the slots included) completed.
#pragma once

#include <cstdint>

#include "qw_internal.h"
#include "qw_ptx.cuh"

namespace qw {

constexpr int kArMaxChunks = 1024;
constexpr size_t kArFlagBytes = (size_t)2 * kArMaxRanks * kArMaxChunks * sizeof(unsigned int);

struct ArParams {
  float* data[kArMaxRanks];  // each rank's data area (mapped here)
  unsigned int* flags[kArMaxRanks];
  unsigned int* epochs;  // local: [0] the last finished call's epoch, [1] CTAs done in this call
  unsigned int* status;
  int P, rank;  // P = 0: no exchange
  long long n_max;
};

inline ArParams ar_params(const ArComm& c) {
  ArParams p{};
  for (int r = 0; r < c.P; ++r) {
    p.data[r] = reinterpret_cast<float*>(static_cast<uint8_t*>(c.peer_bufs[r]) + kArFlagBytes);
    p.flags[r] = static_cast<unsigned int*>(c.peer_bufs[r]);
  }
  p.epochs = c.counters;
  p.status = c.status;
  p.P = c.P;
  p.rank = c.rank;
  p.n_max = c.n_max;
  return p;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Slot (par, src) of rank dst's data area.
__device__ __forceinline__ float* ar_slot(const ArParams& p, int dst, int par, int src) {
  return p.data[dst] + ((long long)par * p.P + src) * p.n_max;
}
// Flag (par, src, chunk b) in rank dst's buffer.
__device__ __forceinline__ unsigned int* ar_flag_ptr(const ArParams& p, int dst, int par, int src, int b) {
  return p.flags[dst] + ((size_t)par * kArMaxRanks + src) * kArMaxChunks + b;
}
// The epoch of the call this kernel belongs to (read after the previous
// kernel of the stream completed, before this CTA counts itself done).
__device__ __forceinline__ unsigned int ar_next_epoch(const ArParams& p) {
  return *(volatile const unsigned int*)p.epochs + 1u;
}
// One thread: waits, bounded, until flag f reaches epoch e.  Returns false
// (and records a peer timeout) when the wait runs out, and at once when an
// earlier call already gave up: the status stays set until the host clears
// it, so a broken job ends in its own time instead of 2 s per call.
__device__ __forceinline__ bool ar_wait_flag(const ArParams& p, const unsigned int* f, unsigned int e) {
  if (*(volatile unsigned int*)p.status == kDevTimeoutPeer) return false;
  if ((int)(ld_acquire_sys(f) - e) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  while ((int)(ld_acquire_sys(f) - e) < 0) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_status(p.status, kDevTimeoutPeer);
      return false;
    }
  }
  return true;
}
// One thread per CTA: counts this CTA done; the call's last CTA publishes
// the call's epoch.
__device__ __forceinline__ void ar_count_done(const ArParams& p, unsigned int e) {
  __threadfence();  // this CTA's read of the epoch precedes its count
  if (atomicAdd(p.epochs + 1, 1u) == gridDim.x - 1) {
    p.epochs[1] = 0u;
    *(volatile unsigned int*)p.epochs = e;
  }
}

}  // namespace qw
