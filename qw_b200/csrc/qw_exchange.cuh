// qw_exchange.cuh -- the peer-memory exchange protocol of a communicator
// (qw_allreduce), shared by the allreduce and greedy-token kernels and by the
// decode kernel's fused row-parallel epilogue.
//
// Each rank owns one buffer that every rank maps (CUDA IPC):
//   [flags: 2 parities x 8 ranks x 1024 chunks of uint32]
//   [data:  2 parities x P ranks x n_max floats]
//   [ll:    2 parities x P ranks x n_ll 64-bit words]
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
//
// The ll slots carry the fused row-parallel exchange with no flags and no
// fences: every value travels with its call's epoch in one 64-bit word
// (value bits low, epoch high), written with one single-copy-atomic store,
// so a reader that sees the epoch sees the value.  Epochs grow by one per
// call, so a word left from call e - 2 in the same parity never matches.
#pragma once

#include <cstdint>

#include "qw_internal.h"
#include "qw_ptx.cuh"

namespace qw {

constexpr int kArMaxChunks = 1024;
constexpr size_t kArFlagBytes = (size_t)2 * kArMaxRanks * kArMaxChunks * sizeof(unsigned int);
// Words per ll slot: 16 rows of up to 131072 outputs at most.
constexpr long long kArLLMax = 1ll << 21;
inline long long ar_ll_elems(long long n_max) { return n_max < kArLLMax ? n_max : kArLLMax; }

struct ArParams {
  float* data[kArMaxRanks];  // each rank's data area (mapped here)
  unsigned int* flags[kArMaxRanks];
  unsigned long long* ll[kArMaxRanks];  // each rank's ll area
  unsigned int* epochs;  // local: [0] the last finished call's epoch, [1] CTAs done in this call
  unsigned int* status;
  int P, rank;  // P = 0: no exchange
  long long n_max;
  long long n_ll;
};

inline ArParams ar_params(const ArComm& c) {
  ArParams p{};
  for (int r = 0; r < c.P; ++r) {
    p.data[r] = reinterpret_cast<float*>(static_cast<uint8_t*>(c.peer_bufs[r]) + kArFlagBytes);
    p.flags[r] = static_cast<unsigned int*>(c.peer_bufs[r]);
    p.ll[r] = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(c.peer_bufs[r]) + kArFlagBytes +
                                                    (size_t)2 * c.P * c.n_max * sizeof(float));
  }
  p.n_ll = ar_ll_elems(c.n_max);
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
// ll slot (par, src) of rank dst.
__device__ __forceinline__ unsigned long long* ar_ll_slot(const ArParams& p, int dst, int par, int src) {
  return p.ll[dst] + ((long long)par * p.P + src) * p.n_ll;
}
__device__ __forceinline__ void ar_ll_store(unsigned long long* a, float v, unsigned int e) {
  const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}
// The value of ll word a once it carries epoch e; false (and a recorded peer
// timeout) when it does not within the wait bound, or at once after an
// earlier call gave up.
__device__ __forceinline__ bool ar_ll_load(const ArParams& p, const unsigned long long* a, unsigned int e,
                                           float* v) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
  if ((unsigned int)(w >> 32) != e) {
    if (*(volatile unsigned int*)p.status == kDevTimeoutPeer) return false;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
      if ((unsigned int)(w >> 32) == e) break;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_status(p.status, kDevTimeoutPeer);
        return false;
      }
    }
  }
  *v = __uint_as_float((unsigned int)w);
  return true;
}
// Two adjacent ll words (16-byte aligned) once both carry epoch e, summed
// over the P ranks' slots (slot r at a + r * stride) in rank order: all P
// loads are in flight before any is checked, and only words still without
// the epoch are read again.  False (and a recorded peer timeout) when the
// wait bound runs out, or at once after an earlier call gave up.
__device__ __forceinline__ bool ar_ll_sum2(const ArParams& p, const unsigned long long* a, long long stride,
                                           unsigned int e, float* s0, float* s1) {
  ulonglong2 w[kArMaxRanks];
#pragma unroll
  for (int r = 0; r < kArMaxRanks; ++r)
    if (r < p.P)
      asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                   : "=l"(w[r].x), "=l"(w[r].y)
                   : "l"(a + r * stride)
                   : "memory");
  uint64_t t0 = 0;
#pragma unroll
  for (int r = 0; r < kArMaxRanks; ++r) {
    if (r >= p.P) break;
    while ((unsigned int)(w[r].x >> 32) != e || (unsigned int)(w[r].y >> 32) != e) {
      if (t0 == 0) {
        if (*(volatile unsigned int*)p.status == kDevTimeoutPeer) return false;
        t0 = globaltimer_ns();
      } else if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_status(p.status, kDevTimeoutPeer);
        return false;
      }
      asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                   : "=l"(w[r].x), "=l"(w[r].y)
                   : "l"(a + r * stride)
                   : "memory");
    }
  }
  float x0 = 0.f, x1 = 0.f;
#pragma unroll
  for (int r = 0; r < kArMaxRanks; ++r)
    if (r < p.P) {
      x0 += __uint_as_float((unsigned int)w[r].x);
      x1 += __uint_as_float((unsigned int)w[r].y);
    }
  *s0 = x0;
  *s1 = x1;
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
