// qw_allreduce.cu -- one-shot sum of the row-parallel projections' fp32
// partials across the GPUs of one node, over NVLink peer memory, with the
// fp16 rounding of the sum fused (the o and down projections of a
// tensor-parallel layer: each rank holds y_r = x_r W_r^T over its K-slice,
// and y = fp16(sum_r y_r)), and the greedy-token exchange of a vocabulary-
// sharded LM head.  The buffers, epochs and flags are qw_exchange.cuh's.
//
// CTA b of every rank handles chunk b of the vector (every rank launches the
// same grid for the same n), so the exchange is per chunk and needs no
// grid-wide step.  CTA b with epoch e (parity e & 1):
//   1. stores its chunk of the local partial into slot (parity, rank) of
//      every rank's buffer (plain stores over NVLink), then, after a CTA
//      barrier, writes flag (parity, rank, b) = e into every rank's buffer;
//   2. waits, bounded, until flags (parity, r, b) of its own buffer reach e
//      for every rank r, then sums its chunk over the P slots in rank order
//      (every rank gets identical y) and writes fp16 (or fp32).
// The grid, and so each chunk's range, depends on n, so calls of different
// sizes cut the vector differently; the call-wide epoch and parity keep that
// safe.  No multicast, no NVLS: plain loads and stores to mapped peer
// memory.  A rank whose peers never flag gives up after the wait bound,
// records a status and returns (its output is then incomplete).
#include <cuda_fp16.h>

#include "qw_exchange.cuh"
#include "qw_internal.h"
#include "qw_ptx.cuh"

namespace qw {

namespace {

constexpr int kArThreads = 256;
constexpr int kArVec = 4;  // floats per thread per step

// --- the exchange protocol for kernels whose whole CTA takes part.
// A call's epoch: every CTA reads it before it counts itself done in
// ar_finish, and the last CTA to count writes the next one, so all CTAs of
// a call see the same.
__device__ __forceinline__ unsigned int ar_epoch(const ArParams& p) {
  __shared__ unsigned int s_e;
  if (threadIdx.x == 0) s_e = ar_next_epoch(p);
  __syncthreads();
  return s_e;
}
// After a CTA barrier that orders every thread's stores to the slots before
// it: flag (parity, rank, chunk b) = e in every rank's buffer.
__device__ __forceinline__ void ar_flag(const ArParams& p, int par, int b, unsigned int e) {
  if (threadIdx.x < p.P) {
    __threadfence_system();
    st_release_sys(ar_flag_ptr(p, threadIdx.x, par, p.rank, b), e);
  }
}
// Waits, bounded, for every rank's flag of chunk b in this rank's buffer.
// Returns (to every thread) whether the chunk's slots may be read.
__device__ __forceinline__ bool ar_wait(const ArParams& p, int par, int b, unsigned int e) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < p.P && !ar_wait_flag(p, ar_flag_ptr(p, p.rank, par, threadIdx.x, b), e)) s_ok = 0;
  __syncthreads();
  return s_ok != 0;
}
// Counts this CTA done; the call's last CTA publishes its epoch.
__device__ __forceinline__ void ar_finish(const ArParams& p, unsigned int e) {
  if (threadIdx.x == 0) ar_count_done(p, e);
}

template <bool OUT_F32>
__global__ void __launch_bounds__(kArThreads) allreduce_kernel(const ArParams p, const float* __restrict__ partial,
                                                               void* __restrict__ out, long long n, int vec_ok) {
  const int b = blockIdx.x;
  // this CTA's chunk: contiguous, in units of 4 floats
  const long long nv = (n + kArVec - 1) / kArVec;
  const long long per = (nv + gridDim.x - 1) / gridDim.x;
  const long long v0 = (long long)b * per;
  const long long v1 = v0 + per < nv ? v0 + per : nv;
  // The partial is the previous kernel's output, and the epoch was written by
  // the previous call of this kernel: both complete once the wait returns
  // (every kernel of these streams waits on its predecessor before it ends).
  pdl_wait();
  pdl_launch_dependents();
  const unsigned int e = ar_epoch(p);
  const int par = (int)(e & 1u);

  // 1. scatter into slot (par, rank) of every rank, then flag the chunk
  for (long long v = v0 + threadIdx.x; v < v1; v += kArThreads) {
    const long long i = v * kArVec;
    if (vec_ok) {
      const float4 x = *reinterpret_cast<const float4*>(partial + i);
      for (int r = 0; r < p.P; ++r)
        *reinterpret_cast<float4*>(ar_slot(p, r, par, p.rank) + i) = x;
    } else {
      for (int j = 0; j < kArVec && i + j < n; ++j) {
        const float x = partial[i + j];
        for (int r = 0; r < p.P; ++r) ar_slot(p, r, par, p.rank)[i + j] = x;
      }
    }
  }
  __syncthreads();  // every thread's stores precede the flags
  ar_flag(p, par, b, e);

  // 2. wait for every rank's flag of this chunk, then sum it
  if (ar_wait(p, par, b, e)) {
    const float* mine = ar_slot(p, p.rank, par, 0);
    for (long long v = v0 + threadIdx.x; v < v1; v += kArThreads) {
      const long long i = v * kArVec;
      if (vec_ok) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < p.P; ++r) {  // rank order: every rank sums identically
          const float4 x = __ldcg(reinterpret_cast<const float4*>(mine + (long long)r * p.n_max + i));
          s.x += x.x;
          s.y += x.y;
          s.z += x.z;
          s.w += x.w;
        }
        if (OUT_F32) {
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + i) = s;
        } else {
          __half2* o = reinterpret_cast<__half2*>(reinterpret_cast<__half*>(out) + i);
          o[0] = __floats2half2_rn(s.x, s.y);
          o[1] = __floats2half2_rn(s.z, s.w);
        }
      } else {
        for (int j = 0; j < kArVec && i + j < n; ++j) {
          float s = 0.f;
          for (int r = 0; r < p.P; ++r) s += __ldcg(mine + (long long)r * p.n_max + i + j);
          if (OUT_F32) reinterpret_cast<float*>(out)[i + j] = s;
          else reinterpret_cast<__half*>(out)[i + j] = __float2half_rn(s);
        }
      }
    }
  }
  ar_finish(p, e);
}

// Greedy token across vocabulary shards: keys[m] is this rank's best logit of
// row m as (order-preserving fp16 value << 32) | (2^32 - 1 - local index); the
// global index is index_base + local index, so the global key is keys[m] -
// index_base.  One CTA stores its M global keys (as pairs of floats) into
// slot (parity, rank) of every rank's buffer, flags chunk 0, waits for every
// rank, and takes the largest key of each row: the largest logit, and among
// equal logits the lowest global index.
__global__ void __launch_bounds__(kArThreads) argmax_exchange_kernel(const ArParams p,
                                                                     const unsigned long long* __restrict__ keys,
                                                                     unsigned long long index_base,
                                                                     uint32_t* __restrict__ idx, int M) {
  pdl_wait();
  pdl_launch_dependents();
  const unsigned int e = ar_epoch(p);
  const int par = (int)(e & 1u);
  for (int m = threadIdx.x; m < M; m += kArThreads) {
    const unsigned long long k = keys[m] - index_base;
    for (int r = 0; r < p.P; ++r)
      reinterpret_cast<unsigned long long*>(ar_slot(p, r, par, p.rank))[m] = k;
  }
  __syncthreads();
  ar_flag(p, par, 0, e);
  if (ar_wait(p, par, 0, e)) {
    const float* mine = ar_slot(p, p.rank, par, 0);
    for (int m = threadIdx.x; m < M; m += kArThreads) {
      unsigned long long best = 0ull;
      for (int r = 0; r < p.P; ++r) {
        const unsigned long long k = __ldcg(reinterpret_cast<const unsigned long long*>(mine + (long long)r * p.n_max) + m);
        best = k > best ? k : best;
      }
      idx[m] = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull);
    }
  }
  ar_finish(p, e);
}

}  // namespace

size_t allreduce_buffer_bytes(int P, int64_t n_max) {
  return kArFlagBytes + (size_t)2 * P * (size_t)n_max * sizeof(float) +
         (size_t)2 * P * (size_t)ar_ll_elems(n_max) * sizeof(unsigned long long);
}

int64_t allreduce_ll_elems(int64_t n_max) { return ar_ll_elems(n_max); }

size_t allreduce_epoch_bytes() { return 2 * sizeof(unsigned int); }


cudaError_t launch_argmax_exchange(const ArComm& c, const unsigned long long* keys, int64_t index_base,
                                   uint32_t* idx, int64_t M, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  const ArParams p = ar_params(c);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, argmax_exchange_kernel, p, keys, (unsigned long long)index_base, idx, (int)M);
}

cudaError_t launch_allreduce(const ArComm& c, const float* partial, void* out, bool out_f32, bool vec, int64_t n,
                             int sm_count, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const ArParams p = ar_params(c);
  // chunks of about 2 float4 per thread; the grid depends on n only, so
  // every rank splits a call identically
  const long long nv = (n + kArVec - 1) / kArVec;
  long long grid = (nv + kArThreads * 2 - 1) / (kArThreads * 2);
  if (grid > sm_count) grid = sm_count;
  if (grid > kArMaxChunks) grid = kArMaxChunks;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int v = vec ? 1 : 0;
  return out_f32 ? cudaLaunchKernelEx(&cfg, allreduce_kernel<true>, p, partial, out, (long long)n, v)
                 : cudaLaunchKernelEx(&cfg, allreduce_kernel<false>, p, partial, out, (long long)n, v);
}

}  // namespace qw
