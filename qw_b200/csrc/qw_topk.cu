// qw_topk.cu -- the k largest fp16 logits of each row and their indices:
// the candidate step after the LM-head projection (argpartition(logits, -k)
// then take_along_axis, as the reference's DFlash2 candidate selector does).
//
// One thread-block cluster of 8 CTAs (1024 threads each) per row.  Each CTA
// owns a contiguous eighth of the row, streamed from L2 in rounds of 8192
// logits (8 per thread, one 16-byte load when the row allows).  Exact radix
// select on 16-bit keys (the fp16 bit pattern made order-preserving):
//   1. histogram of the keys' high byte, summed over the cluster through
//      distributed shared memory; the bin H holding the k-th largest;
//   2. the same for the low byte among keys in H: the exact k-th key T, the
//      count of keys above T, and the number `need` of keys equal to T that
//      complete the k;
//   3. every key above T goes to CTA 0's candidate list (remote atomics and
//      stores); so do the equal keys, all of them when just `need` exist,
//      else the `need` lowest indices: each CTA counts its equal keys, the
//      CTAs before it in row order tell it how many are still wanted, and it
//      takes its first ones in index order;
//   4. CTA 0 sorts the k candidates by value, descending, lower index first
//      among equal values, and writes them out.
// Every CTA of a cluster takes the same branches (the totals it decides on
// are the cluster's), so the cluster barriers always pair up; the cluster's
// CTAs are co-scheduled, so those barriers cannot wait on an absent CTA.
// Histograms are kept per warp (shared-memory atomics then contend only
// within a warp) and summed per CTA.  A CTA's share of a row of up to
// 262,144 logits stays in registers (4 rounds) after its first read.
#include <cuda_fp16.h>

#include "qw_internal.h"
#include "qw_ptx.cuh"

namespace qw {

namespace {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMax = 1024;  // largest k
constexpr int kPer = 8;         // logits per thread per round
constexpr int kRound = kTopkThreads * kPer;
constexpr int kCluster = 8;     // CTAs per row
constexpr int kCache = 4;       // rounds a thread keeps in registers

__device__ __forceinline__ uint32_t order_key(uint32_t b) {
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

// Raw fp16 bits of logits i0 .. i0+7 (unspecified past the end of the row:
// every use checks the index against N).
template <bool VEC>
__device__ __forceinline__ uint4 load_raw(const __half* row, int i0, int N) {
  if constexpr (VEC) {  // N % 8 == 0 and the row 16-byte aligned: a vector is wholly in or out of range
    return i0 < N ? __ldcg(reinterpret_cast<const uint4*>(row + i0)) : make_uint4(0u, 0u, 0u, 0u);
  } else {
    uint32_t h[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) h[j] = (i0 + j < N) ? __half_as_ushort(row[i0 + j]) : 0u;
    return make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
  }
}

__device__ __forceinline__ void keys_of(uint4 v, uint32_t (&key)[kPer]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    key[2 * j] = order_key(w[j] & 0xFFFFu);
    key[2 * j + 1] = order_key(w[j] >> 16);
  }
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of this CTA's shared variable `p` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t remote(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ uint32_t ld_remote(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_remote(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_remote(uint32_t addr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.shared::cluster.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(addr), "r"(v) : "memory");
  return old;
}

// Bin b (scanning down from the top of nbins) where the running count from
// the top first reaches `want`; *above = the count in bins above b.
__device__ __forceinline__ int bin_from_top(const uint32_t* hist, int nbins, uint32_t want, uint32_t* above) {
  uint32_t acc = 0;
  for (int b = nbins - 1; b >= 0; --b) {
    if (acc + hist[b] >= want) {
      *above = acc;
      return b;
    }
    acc += hist[b];
  }
  *above = acc;
  return 0;
}

// Exclusive prefix of `cnt` over the CTA's threads in thread order, and the
// CTA's total; uses `warp_tot` (32 words) and two barriers.
__device__ __forceinline__ uint32_t block_prefix(uint32_t cnt, uint32_t* warp_tot, uint32_t* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint32_t incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_tot[wid] = incl;
  __syncthreads();
  uint32_t before = 0, all = 0;
  for (int w = 0; w < kTopkThreads / 32; ++w) {
    const uint32_t t = warp_tot[w];
    before += (w < wid) ? t : 0u;
    all += t;
  }
  __syncthreads();
  *total = all;
  return before + incl - cnt;
}

template <bool VEC>
__global__ void __launch_bounds__(kTopkThreads, 1)
    topk_rows_kernel(const __half* __restrict__ logits, int64_t ld, int N, int k, uint32_t* __restrict__ idx_out,
                     __half* __restrict__ val_out) {
  __shared__ uint32_t whist[kTopkThreads / 32][256];  // per-warp histograms
  __shared__ uint32_t hist[256];      // this CTA's histogram (read by the whole cluster)
  __shared__ uint32_t tot[256];       // the cluster's
  __shared__ uint32_t rcount[1024];   // equal keys per round of this CTA
  __shared__ uint32_t warp_tot[32];
  __shared__ uint32_t cand_key[kTopkMax];  // CTA 0: the candidates
  __shared__ uint32_t cand_idx[kTopkMax];
  __shared__ uint32_t ncand;
  __shared__ uint32_t n_equal;        // equal keys in this CTA's share

  const uint32_t crank = cluster_rank();
  const int rowi = blockIdx.x / kCluster;
  const __half* row = logits + (size_t)rowi * ld;
  const int tid = threadIdx.x, wid = tid >> 5;
  const int rounds = (N + kRound - 1) / kRound;
  // this CTA's rounds: a contiguous share, so row order is CTA order
  const int r0 = (int)(((int64_t)rounds * crank) / kCluster);
  const int r1 = (int)(((int64_t)rounds * (crank + 1)) / kCluster);
  auto first = [&](int rd) { return rd * kRound + tid * kPer; };
  const uint32_t ncand0 = remote(&ncand, 0), ckey0 = remote(cand_key, 0), cidx0 = remote(cand_idx, 0);
  auto append = [&](uint32_t key, uint32_t i) {  // into CTA 0's list
    const uint32_t slot = atom_add_remote(ncand0, 1u);
    st_remote(ckey0 + 4 * slot, key);
    st_remote(cidx0 + 4 * slot, i);
  };
  // A pass over this CTA's rounds: body(rd, keys) per round, from the
  // register copy when the share fits in it.
  const bool cached = r1 - r0 <= kCache;
  uint4 cache[kCache];
#pragma unroll
  for (int q = 0; q < kCache; ++q)
    cache[q] = (cached && r0 + q < r1) ? load_raw<VEC>(row, first(r0 + q), N) : make_uint4(0u, 0u, 0u, 0u);
  auto for_rounds = [&](auto&& body) {
    if (cached) {
#pragma unroll
      for (int q = 0; q < kCache; ++q) {
        if (r0 + q < r1) {
          uint32_t key[kPer];
          keys_of(cache[q], key);
          body(r0 + q, key);
        }
      }
    } else {
      for (int rd = r0; rd < r1; ++rd) {
        uint32_t key[kPer];
        keys_of(load_raw<VEC>(row, first(rd), N), key);
        body(rd, key);
      }
    }
  };
  auto clear_whist = [&]() {
    for (int b = tid; b < (kTopkThreads / 32) * 256; b += kTopkThreads) (&whist[0][0])[b] = 0;
  };
  // this CTA's histogram from the warps', then the cluster's sum into `tot`
  auto reduce_hist = [&]() {
    __syncthreads();
    for (int b = tid; b < 256; b += kTopkThreads) {
      uint32_t v = 0;
      for (int w = 0; w < kTopkThreads / 32; ++w) v += whist[w][b];
      hist[b] = v;
    }
    cluster_sync();  // every CTA's histogram is complete
    for (int b = tid; b < 256; b += kTopkThreads) {
      uint32_t v[kCluster];
#pragma unroll
      for (int c = 0; c < kCluster; ++c) v[c] = ld_remote(remote(&hist[b], (uint32_t)c));
      uint32_t sum = 0;
#pragma unroll
      for (int c = 0; c < kCluster; ++c) sum += v[c];
      tot[b] = sum;
    }
    cluster_sync();  // every CTA has read every histogram (they may be cleared now)
  };

  // 1. high byte
  clear_whist();
  for (int b = tid; b < 1024; b += kTopkThreads) rcount[b] = 0;
  if (tid == 0) {
    ncand = 0;
    n_equal = 0;
  }
  __syncthreads();
  for_rounds([&](int rd, const uint32_t (&key)[kPer]) {
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (first(rd) + j < N) atomicAdd(&whist[wid][key[j] >> 8], 1u);
  });
  reduce_hist();
  uint32_t above_h;
  const uint32_t H = (uint32_t)bin_from_top(tot, 256, (uint32_t)k, &above_h);

  // 2. low byte within H
  clear_whist();
  __syncthreads();
  for_rounds([&](int rd, const uint32_t (&key)[kPer]) {
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (first(rd) + j < N && (key[j] >> 8) == H) atomicAdd(&whist[wid][key[j] & 255u], 1u);
  });
  uint32_t above_l;
  reduce_hist();
  const uint32_t L = (uint32_t)bin_from_top(tot, 256, (uint32_t)k - above_h, &above_l);
  const uint32_t T = (H << 8) | L;
  const uint32_t n_gt = above_h + above_l;   // keys above T (< k)
  const uint32_t n_eq = tot[L];
  const uint32_t need = (uint32_t)k - n_gt;  // 1 <= need <= n_eq
  const bool take_all_eq = n_eq == need;

  // 3. collect into CTA 0: keys above T, and the equal keys when all are taken;
  //    otherwise count this CTA's equal keys per round
  for_rounds([&](int rd, const uint32_t (&key)[kPer]) {
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = first(rd) + j;
      if (i < N && (key[j] > T || (take_all_eq && key[j] == T))) append(key[j], (uint32_t)i);
      c += (i < N && key[j] == T) ? 1u : 0u;
    }
    if (!take_all_eq) {
      c += __shfl_xor_sync(0xffffffffu, c, 1);
      c += __shfl_xor_sync(0xffffffffu, c, 2);
      c += __shfl_xor_sync(0xffffffffu, c, 4);
      c += __shfl_xor_sync(0xffffffffu, c, 8);
      c += __shfl_xor_sync(0xffffffffu, c, 16);
      if ((tid & 31) == 0 && c) {
        atomicAdd(&rcount[rd - r0], c);
        atomicAdd(&n_equal, c);
      }
    }
  });
  if (!take_all_eq) {
    // The `need` lowest indices among the keys equal to T: the CTAs before
    // this one (in row order) hold `before` of them; this CTA takes its
    // first need - before in index order, round by round.
    cluster_sync();  // every CTA's n_equal is final
    uint32_t before = 0;
    for (uint32_t c = 0; c < crank; ++c) before += ld_remote(remote(&n_equal, c));
    for (int rd = r0; rd < r1 && before < need; ++rd) {
      const uint32_t in_round = rcount[rd - r0];
      if (in_round) {
        uint32_t key[kPer];
        keys_of(load_raw<VEC>(row, first(rd), N), key);
        uint32_t c = 0;
#pragma unroll
        for (int j = 0; j < kPer; ++j) c += (first(rd) + j < N && key[j] == T) ? 1u : 0u;
        uint32_t total;
        uint32_t rank = before + block_prefix(c, warp_tot, &total);
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          if (first(rd) + j < N && key[j] == T) {
            if (rank < need) append(T, (uint32_t)(first(rd) + j));
            ++rank;
          }
        }
      }
      before += in_round;
    }
  }
  cluster_sync();  // all candidates are in CTA 0
  if (crank != 0) return;

  // 4. sort the k candidates: larger key first, lower index first among equals
  int P = 1;
  while (P < k) P <<= 1;
  for (int j = tid + k; j < P; j += kTopkThreads) {  // padding sorts last
    cand_key[j] = 0u;
    cand_idx[j] = 0xFFFFFFFFu;
  }
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int j = tid; j < P; j += kTopkThreads) {
        const int partner = j ^ stride;
        if (partner > j) {
          const uint64_t a = ((uint64_t)cand_key[j] << 32) | (0xFFFFFFFFu - cand_idx[j]);
          const uint64_t c = ((uint64_t)cand_key[partner] << 32) | (0xFFFFFFFFu - cand_idx[partner]);
          const bool descending = (j & size) == 0;
          if (descending ? (a < c) : (a > c)) {
            const uint32_t tk = cand_key[j], ti = cand_idx[j];
            cand_key[j] = cand_key[partner];
            cand_idx[j] = cand_idx[partner];
            cand_key[partner] = tk;
            cand_idx[partner] = ti;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int j = tid; j < k; j += kTopkThreads) {
    const uint32_t key = cand_key[j];
    const uint32_t bits = (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
    idx_out[(size_t)rowi * k + j] = cand_idx[j];
    if (val_out) val_out[(size_t)rowi * k + j] = __ushort_as_half((unsigned short)bits);
  }
}

}  // namespace

int topk_max_k() { return kTopkMax; }

// A CTA counts its equal keys per round in a 1024-word array: rows of at
// most 1024 rounds of 8192 per CTA of the cluster.
int64_t topk_max_n() { return (int64_t)1024 * kRound * kCluster; }

cudaError_t launch_topk_rows(const void* logits, int64_t ld, int64_t M, int64_t N, int k, uint32_t* idx,
                             void* values, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  const bool vec = (N % kPer == 0) && (ld % kPer == 0) && (reinterpret_cast<uintptr_t>(logits) % 16 == 0);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(M * kCluster));
  cfg.blockDim = dim3(kTopkThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const __half* lp = (const __half*)logits;
  __half* vp = (__half*)values;
  return vec ? cudaLaunchKernelEx(&cfg, topk_rows_kernel<true>, lp, ld, (int)N, k, idx, vp)
             : cudaLaunchKernelEx(&cfg, topk_rows_kernel<false>, lp, ld, (int)N, k, idx, vp);
}

}  // namespace qw
