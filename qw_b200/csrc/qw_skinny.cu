// qw_skinny.cu -- affine 4-bit group-64 quantized matmul for M <= 16 rows of x
// (decode M=1, MTP verify M=4, DFlash2 block M=16).  HBM-bound: the packed
// weights are streamed once.
//
// Work decomposition ("stream-K"): the weight matrix is cut into row tiles of
// BN rows and the K axis into 512-wide chunks (8 groups).  The T*C
// (tile, chunk) units are dealt out as contiguous ranges to a persistent grid
// of G CTAs, so every CTA streams the same number of bytes whatever N and K
// are.  A tile whose chunks are split between CTAs is combined through fp32
// partial slots in scratch memory: every contributor writes its slot, bumps
// the tile's counter, and the last one to arrive adds the slots in CTA order
// (deterministic) and writes y.
//
// CTA roles (warp-specialised):
//   warp 0      TMA producer: packed W (two 128-byte SW128 boxes per stage),
//               scales, biases, then the x boxes (issued only after
//               griddepcontrol.wait, so the weight stream of this launch
//               overlaps the tail of the previous kernel under PDL).
//   warp 1      x-sum warp: X[g][m] = sum of the 64 x values of group g, in
//               fp32, for the per-group fold below.
//   warps 2..   consumers, 16 weight rows each.
//
// Consumer arithmetic (no per-element dequantisation): a packed word w holds
// 8 nibbles; lop3((w >> 4j) & 0x000F000F | 0x64006400) is an fp16 pair
// (1024 + q_j, 1024 + q_{j+4}), exact.  Those pairs feed mma.sync m16n8k16
// directly as the A operand (16 weight rows), with x as B (one column per
// token) permuted in registers to the same (k, k+4) pairing.  One group's four
// MMAs give acc = sum_k x_k (1024 + q_k) in fp32; the group is folded into the
// output as  y += s * acc + (b - 1024 s) * X,  which equals
// sum_k x_k (s q_k + b) with the weight formed in fp32 (the reference
// semantics) and fp32 accumulation.
#include <cuda_fp16.h>

#include "qw_internal.h"
#include "qw_ptx.cuh"

namespace qw {

namespace {

constexpr int kGroup = 64;
constexpr int kGroupsPerStage = 8;
constexpr size_t kMaxCounters = 1u << 16;  // row tiles per launch (N <= 8M rows)
constexpr size_t kCounterBytes = kMaxCounters * sizeof(unsigned int);
constexpr int kChunkK = kGroup * kGroupsPerStage;  // 512

template <int NT, int WARPS, int STAGES>
struct SkinnyCfg {
  static constexpr int BN = WARPS * 16;
  static constexpr int W_BOX = BN * 128;
  static constexpr int W_BYTES = 2 * W_BOX;
  static constexpr int SB_BYTES = BN * 16;
  static constexpr int XROWS = 8 * NT;
  static constexpr int X_GROUP = XROWS * 128;
  static constexpr int X_BYTES = kGroupsPerStage * X_GROUP;
  static constexpr int XS_BYTES = kGroupsPerStage * XROWS * 4;
  static constexpr int OFF_W = 0;
  static constexpr int OFF_X = W_BYTES;  // multiple of 1024
  static constexpr int OFF_S = OFF_X + X_BYTES;
  static constexpr int OFF_B = OFF_S + SB_BYTES;
  static constexpr int OFF_XS = OFF_B + SB_BYTES;
  static constexpr int STAGE = ((OFF_XS + XS_BYTES) + 1023) / 1024 * 1024;
  static constexpr int NBAR = 4 * STAGES;  // wfull, xfull, xready, empty
  static constexpr int SMEM = STAGES * STAGE + NBAR * 8 + 16 + 1024;
  static constexpr int THREADS = (WARPS + 2) * 32;
  static constexpr int MPAD = 8 * NT;
  static constexpr int PART = BN * MPAD;  // floats per partial slot
};

struct SkinnyParams {
  int M, N, K;
  int C;          // chunks along K
  int T;          // row tiles
  long long U;    // T * C
  int G;          // CTAs
  int xrows_box;  // rows of x in each x TMA box (min(M, XROWS))
  int sb_tma;     // scales/biases through TMA (needs K % 512 == 0)
  int y_f32;
  void* y;
  const __half* scales;
  const __half* biases;
  float* part;            // [G][2][PART]
  unsigned int* counter;  // [T]
  unsigned int* status;   // device status word
};

__device__ __forceinline__ long long unit_begin(long long i, long long U, int G) { return (i * U) / G; }
// CTA whose range [unit_begin(i), unit_begin(i+1)) contains unit u.
__device__ __forceinline__ int cta_of_unit(long long u, long long U, int G) {
  return (int)(((u + 1) * (long long)G - 1) / U);
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ float sum8_f16(uint4 v) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
  float2 a = __half22float2(h[0]);
  float2 b = __half22float2(h[1]);
  float2 c = __half22float2(h[2]);
  float2 d = __half22float2(h[3]);
  return ((a.x + a.y) + (b.x + b.y)) + ((c.x + c.y) + (d.x + d.y));
}

template <int NT, int WARPS, int STAGES>
__global__ void __launch_bounds__((WARPS + 2) * 32, 1)
    qmm_skinny_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                      const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_x,
                      const SkinnyParams p) {
  using Cfg = SkinnyCfg<NT, WARPS, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE);
  uint64_t* wfull = bars;
  uint64_t* xfull = bars + STAGES;
  uint64_t* xready = bars + 2 * STAGES;
  uint64_t* empty = bars + 3 * STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + Cfg::NBAR);
  volatile int* fin_flag = abort_flag + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const long long u0 = unit_begin(blockIdx.x, p.U, p.G);
  const long long u1 = unit_begin(blockIdx.x + 1, p.U, p.G);
  const int nunits = (int)(u1 - u0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&xfull[s], 1);
      mbar_init(&xready[s], 1);
      mbar_init(&empty[s], WARPS);
    }
    *abort_flag = 0;
    *fin_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  const uint32_t w_bytes = Cfg::W_BYTES + (p.sb_tma ? 2 * Cfg::SB_BYTES : 0);
  const uint32_t x_bytes = kGroupsPerStage * 128 * p.xrows_box;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&tm_w);
      prefetch_tensormap(&tm_x);
      if (p.sb_tma) {
        prefetch_tensormap(&tm_s);
        prefetch_tensormap(&tm_b);
      }
      const uint64_t pol_w = l2_policy_evict_first();
      auto issue_w = [&](int j) {
        const long long u = u0 + j;
        const int t = (int)(u / p.C), c = (int)(u % p.C);
        const int slot = j % STAGES;
        uint8_t* st = smem + slot * Cfg::STAGE;
        mbar_arrive_expect_tx(&wfull[slot], w_bytes);
        tma_load_2d_hint(st + Cfg::OFF_W, &tm_w, &wfull[slot], c * 256, t * Cfg::BN, pol_w);
        tma_load_2d_hint(st + Cfg::OFF_W + Cfg::W_BOX, &tm_w, &wfull[slot], c * 256 + 128, t * Cfg::BN, pol_w);
        if (p.sb_tma) {
          tma_load_2d_hint(st + Cfg::OFF_S, &tm_s, &wfull[slot], c * kGroupsPerStage, t * Cfg::BN, pol_w);
          tma_load_2d_hint(st + Cfg::OFF_B, &tm_b, &wfull[slot], c * kGroupsPerStage, t * Cfg::BN, pol_w);
        }
      };
      auto issue_x = [&](int j) {
        const long long u = u0 + j;
        const int c = (int)(u % p.C);
        const int slot = j % STAGES;
        uint8_t* st = smem + slot * Cfg::STAGE;
        mbar_arrive_expect_tx(&xfull[slot], x_bytes);
        for (int gi = 0; gi < kGroupsPerStage; ++gi)
          tma_load_2d(st + Cfg::OFF_X + gi * Cfg::X_GROUP, &tm_x, &xfull[slot], c * kChunkK + gi * kGroup, 0);
      };
      const int npre = nunits < STAGES ? nunits : STAGES;
      // Weights do not depend on the previous kernel: start streaming them
      // before waiting on it.
      for (int j = 0; j < npre; ++j) issue_w(j);
      pdl_wait();
      for (int j = 0; j < npre; ++j) issue_x(j);
      int issued = npre;
      for (int j = npre; j < nunits; ++j) {
        const int slot = j % STAGES;
        const int round = j / STAGES;
        if (!*abort_flag) {
          if (!mbar_wait(&empty[slot], (round - 1) & 1, p.status, kDevTimeoutEmpty)) *abort_flag = 1;
        }
        if (*abort_flag) break;
        issue_w(j);
        issue_x(j);
        issued = j + 1;
      }
      if (*abort_flag) {
        // Let the copies already in flight land before the CTA retires.
        const int first = issued > STAGES ? issued - STAGES : 0;
        for (int j = first; j < issued; ++j) {
          const int slot = j % STAGES;
          mbar_wait(&wfull[slot], (j / STAGES) & 1, p.status, kDevTimeoutFull);
          mbar_wait(&xfull[slot], (j / STAGES) & 1, p.status, kDevTimeoutFull);
        }
      }
    }
    return;
  }

  if (warp == 1) {
    // -------------------------------------------------------------- x sums
    pdl_wait();
    for (int j = 0; j < nunits; ++j) {
      const long long u = u0 + j;
      const int t = (int)(u / p.C), c = (int)(u % p.C);
      const int slot = j % STAGES;
      uint8_t* st = smem + slot * Cfg::STAGE;
      if (!*abort_flag && !mbar_wait(&xfull[slot], (j / STAGES) & 1, p.status, kDevTimeoutFull)) *abort_flag = 1;
      const uint32_t xbase = smem_u32(st + Cfg::OFF_X);
      float* xs = reinterpret_cast<float*>(st + Cfg::OFF_XS);
      const int ntask = kGroupsPerStage * p.M;
      for (int t0 = 0; t0 < ntask; t0 += 4) {
        const int task = t0 + lane / 8;
        const int sub = lane % 8;
        float v = 0.f;
        int gi = 0, n = 0;
        if (task < ntask) {
          gi = task / p.M;
          n = task - gi * p.M;
          v = sum8_f16(lds128(xbase + gi * Cfg::X_GROUP + n * 128 + ((sub ^ (n & 7)) << 4)));
        }
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        if (sub == 0 && task < ntask) xs[gi * Cfg::XROWS + n] = v;
      }
      if (!p.sb_tma) {
        // Scales/biases rows are not 16-byte strided (K % 512 != 0): stage
        // them with plain loads, zero beyond the matrix edge.
        __half* ss = reinterpret_cast<__half*>(st + Cfg::OFF_S);
        __half* sb = reinterpret_cast<__half*>(st + Cfg::OFF_B);
        const int G = p.K / kGroup;
        for (int e = lane; e < Cfg::BN * kGroupsPerStage; e += 32) {
          const int r = e / kGroupsPerStage, g = e % kGroupsPerStage;
          const int row = t * Cfg::BN + r, grp = c * kGroupsPerStage + g;
          __half sv = __float2half(0.f), bv = __float2half(0.f);
          if (row < p.N && grp < G) {
            sv = p.scales[(size_t)row * G + grp];
            bv = p.biases[(size_t)row * G + grp];
          }
          ss[e] = sv;
          sb[e] = bv;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&xready[slot]);
    }
    return;
  }

  // ----------------------------------------------------------------- consumers
  const int cw = warp - 2;
  const int wrow = cw * 16;          // first row of this warp inside the tile
  const int r = lane / 4, s4 = lane % 4;
  pdl_wait();

  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[t][e] = 0.f;

  const int first_tile = (int)(u0 / p.C);
  int seg_begin = (int)(u0 % p.C);

  // ldmatrix lane addressing: matrix mi = lane/8 covers rows 8*(mi&1).. of
  // chunk (mi>>1) of the group.
  const int lm_mi = lane / 8;
  const int lm_row = wrow + (lane % 8) + 8 * (lm_mi & 1);
  const int lm_sw = lm_row & 7;

  for (int j = 0; j < nunits; ++j) {
    const long long u = u0 + j;
    const int t = (int)(u / p.C), c = (int)(u % p.C);
    const int slot = j % STAGES;
    const uint32_t parity = (j / STAGES) & 1;
    uint8_t* st = smem + slot * Cfg::STAGE;
    if (!*abort_flag) {
      if (!mbar_wait(&wfull[slot], parity, p.status, kDevTimeoutFull)) *abort_flag = 1;
      else if (!mbar_wait(&xready[slot], parity, p.status, kDevTimeoutFull)) *abort_flag = 1;
    }
    if (!*abort_flag) {
      const uint32_t wbase = smem_u32(st + Cfg::OFF_W);
      const uint32_t xbase = smem_u32(st + Cfg::OFF_X);
      const uint4 sv_lo = *reinterpret_cast<const uint4*>(st + Cfg::OFF_S + (wrow + r) * 16);
      const uint4 sv_hi = *reinterpret_cast<const uint4*>(st + Cfg::OFF_S + (wrow + r + 8) * 16);
      const uint4 bv_lo = *reinterpret_cast<const uint4*>(st + Cfg::OFF_B + (wrow + r) * 16);
      const uint4 bv_hi = *reinterpret_cast<const uint4*>(st + Cfg::OFF_B + (wrow + r + 8) * 16);
      const float* xs = reinterpret_cast<const float*>(st + Cfg::OFF_XS);
#pragma unroll
      for (int gi = 0; gi < kGroupsPerStage; ++gi) {
        const int box = gi / 4;
        const int chunk = (gi % 4) * 2 + (lm_mi >> 1);
        uint32_t A0, A1, A2, A3;
        ldmatrix_x4(wbase + box * Cfg::W_BOX + lm_row * 128 + ((chunk ^ lm_sw) << 4), A0, A1, A2, A3);

        uint32_t bfr[NT][4][2];
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
          const int n = tt * 8 + r;
          uint4 xv0 = make_uint4(0, 0, 0, 0), xv1 = make_uint4(0, 0, 0, 0);
          if (n < p.M) {
            const uint32_t rowaddr = xbase + gi * Cfg::X_GROUP + n * 128;
            xv0 = lds128(rowaddr + ((s4 ^ (n & 7)) << 4));
            xv1 = lds128(rowaddr + (((4 + s4) ^ (n & 7)) << 4));
          }
          bfr[tt][0][0] = prmt(xv0.x, xv0.z, 0x5410);
          bfr[tt][1][0] = prmt(xv0.x, xv0.z, 0x7632);
          bfr[tt][2][0] = prmt(xv0.y, xv0.w, 0x5410);
          bfr[tt][3][0] = prmt(xv0.y, xv0.w, 0x7632);
          bfr[tt][0][1] = prmt(xv1.x, xv1.z, 0x5410);
          bfr[tt][1][1] = prmt(xv1.x, xv1.z, 0x7632);
          bfr[tt][2][1] = prmt(xv1.y, xv1.w, 0x5410);
          bfr[tt][3][1] = prmt(xv1.y, xv1.w, 0x7632);
        }
        float d[NT][4];
#pragma unroll
        for (int tt = 0; tt < NT; ++tt)
#pragma unroll
          for (int e = 0; e < 4; ++e) d[tt][e] = 0.f;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint32_t a0 = lop3_expand(A0 >> (4 * jj));
          const uint32_t a1 = lop3_expand(A1 >> (4 * jj));
          const uint32_t a2 = lop3_expand(A2 >> (4 * jj));
          const uint32_t a3 = lop3_expand(A3 >> (4 * jj));
#pragma unroll
          for (int tt = 0; tt < NT; ++tt) mma_16816(d[tt], a0, a1, a2, a3, bfr[tt][jj][0], bfr[tt][jj][1]);
        }
        // fold the group: y += s*acc + (b - 1024 s) * X
        const __half* slo = reinterpret_cast<const __half*>(&sv_lo);
        const __half* shi = reinterpret_cast<const __half*>(&sv_hi);
        const __half* blo = reinterpret_cast<const __half*>(&bv_lo);
        const __half* bhi = reinterpret_cast<const __half*>(&bv_hi);
        const float s_r = __half2float(slo[gi]);
        const float s_r8 = __half2float(shi[gi]);
        const float c_r = __half2float(blo[gi]) - 1024.f * s_r;
        const float c_r8 = __half2float(bhi[gi]) - 1024.f * s_r8;
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
          const float2 X = *reinterpret_cast<const float2*>(xs + gi * Cfg::XROWS + tt * 8 + 2 * s4);
          acc[tt][0] += s_r * d[tt][0] + c_r * X.x;
          acc[tt][1] += s_r * d[tt][1] + c_r * X.y;
          acc[tt][2] += s_r8 * d[tt][2] + c_r8 * X.x;
          acc[tt][3] += s_r8 * d[tt][3] + c_r8 * X.y;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);

    const bool seg_end = (c == p.C - 1) || (j == nunits - 1);
    if (!seg_end) continue;

    const int row0 = t * Cfg::BN + wrow + r;
    const bool whole = (seg_begin == 0) && (c == p.C - 1);
    if (whole) {
      if (!*abort_flag) {
#pragma unroll
        for (int tt = 0; tt < NT; ++tt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int n = tt * 8 + 2 * s4 + (e & 1);
            const int row = row0 + ((e & 2) ? 8 : 0);
            if (n < p.M && row < p.N) {
              const size_t idx = (size_t)n * p.N + row;
              if (p.y_f32) reinterpret_cast<float*>(p.y)[idx] = acc[tt][e];
              else reinterpret_cast<__half*>(p.y)[idx] = __float2half_rn(acc[tt][e]);
            }
          }
      }
    } else {
      // split tile: publish this CTA's partial, last contributor reduces.
      const int slot_idx = (t == first_tile) ? 0 : 1;
      float* mine = p.part + ((size_t)blockIdx.x * 2 + slot_idx) * Cfg::PART;
#pragma unroll
      for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = tt * 8 + 2 * s4 + (e & 1);
          const int rl = wrow + r + ((e & 2) ? 8 : 0);
          mine[rl * Cfg::MPAD + n] = acc[tt][e];
        }
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"r"(WARPS * 32) : "memory");
      const long long tu0 = (long long)t * p.C;
      const int i_first = cta_of_unit(tu0, p.U, p.G);
      const int i_last = cta_of_unit(tu0 + p.C - 1, p.U, p.G);
      if (cw == 0 && lane == 0) {
        const unsigned int ncontrib = (unsigned int)(i_last - i_first + 1);
        const unsigned int old = atomicAdd(&p.counter[t], 1u);
        const int last = (old == ncontrib - 1) ? 1 : 0;
        if (last) atomicExch(&p.counter[t], 0u);
        *fin_flag = last;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(WARPS * 32) : "memory");
      const int last = *fin_flag;
      if (last) {
        __threadfence();
        float tot[NT][4];
#pragma unroll
        for (int tt = 0; tt < NT; ++tt)
#pragma unroll
          for (int e = 0; e < 4; ++e) tot[tt][e] = 0.f;
        for (int i = i_first; i <= i_last; ++i) {
          const int ft = (int)(unit_begin(i, p.U, p.G) / p.C);
          const float* src = p.part + ((size_t)i * 2 + (t == ft ? 0 : 1)) * Cfg::PART;
#pragma unroll
          for (int tt = 0; tt < NT; ++tt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int n = tt * 8 + 2 * s4 + (e & 1);
              const int rl = wrow + r + ((e & 2) ? 8 : 0);
              tot[tt][e] += __ldcg(src + rl * Cfg::MPAD + n);
            }
        }
        if (!*abort_flag) {
#pragma unroll
          for (int tt = 0; tt < NT; ++tt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int n = tt * 8 + 2 * s4 + (e & 1);
              const int row = row0 + ((e & 2) ? 8 : 0);
              if (n < p.M && row < p.N) {
                const size_t idx = (size_t)n * p.N + row;
                if (p.y_f32) reinterpret_cast<float*>(p.y)[idx] = tot[tt][e];
                else reinterpret_cast<__half*>(p.y)[idx] = __float2half_rn(tot[tt][e]);
              }
            }
        }
      }
      // the flag is rewritten by the next split tile only after this barrier
      asm volatile("bar.sync 1, %0;" ::"r"(WARPS * 32) : "memory");
    }
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[tt][e] = 0.f;
    seg_begin = 0;
  }
}

template <int NT, int WARPS, int STAGES>
cudaError_t launch_cfg(const SkinnyArgs& a, const Scratch& scratch, cudaStream_t stream, bool pdl,
                       std::string* err) {
  using Cfg = SkinnyCfg<NT, WARPS, STAGES>;
  auto kern = qmm_skinny_kernel<NT, WARPS, STAGES>;
  int dev = 0;
  cudaGetDevice(&dev);
  const DeviceInfo& di = device_info(dev);
  static thread_local int configured_dev = -1;
  // cudaFuncSetAttribute is per device; cheap enough to repeat on change.
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  SkinnyParams p{};
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.C = (int)((a.K + kChunkK - 1) / kChunkK);
  p.T = (int)((a.N + Cfg::BN - 1) / Cfg::BN);
  p.U = (long long)p.T * p.C;
  static thread_local int occ_dev = -1, occ = 1;
  if (occ_dev != dev) {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, Cfg::THREADS, Cfg::SMEM);
    if (occ < 1) occ = 1;
    occ_dev = dev;
  }
  long long G = (long long)di.sm_count * occ;
  if (a.max_ctas > 0 && G > a.max_ctas) G = a.max_ctas;
  if (G > p.U) G = p.U;
  p.G = (int)G;
  p.xrows_box = (int)(a.M < Cfg::XROWS ? a.M : Cfg::XROWS);
  p.sb_tma = (a.K % kChunkK == 0) ? 1 : 0;
  p.y_f32 = a.y_f32 ? 1 : 0;
  p.y = a.y;
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.biases = reinterpret_cast<const __half*>(a.biases);
  // Scratch layout: the split-tile counters at a fixed offset (they are zero
  // between launches, whatever grid the previous launch used), then the
  // partial slots, which need no initialisation.
  if ((size_t)p.T > kMaxCounters) {
    *err = "too many row tiles for the skinny path's counter block";
    return cudaErrorInvalidValue;
  }
  const size_t need = kCounterBytes + (size_t)p.G * 2 * Cfg::PART * sizeof(float);
  if (scratch.bytes < need || scratch.base == nullptr) {
    *err = "scratch too small for the skinny path";
    return cudaErrorInvalidValue;
  }
  p.status = a.status;
  p.counter = reinterpret_cast<unsigned int*>(scratch.base);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scratch.base) + kCounterBytes);

  CUtensorMap tw, ts, tb, tx;
  if (!encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, (uint64_t)(a.K / 2), (uint64_t)a.N,
                      (uint64_t)(a.K / 2), 128, Cfg::BN, CU_TENSOR_MAP_SWIZZLE_128B, err))
    return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, (uint64_t)a.K, (uint64_t)a.M,
                      (uint64_t)a.K * 2, kGroup, (uint32_t)p.xrows_box, CU_TENSOR_MAP_SWIZZLE_128B, err))
    return cudaErrorInvalidValue;
  if (p.sb_tma) {
    const uint64_t G64 = (uint64_t)(a.K / kGroup);
    if (!encode_tmap_2d(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.scales, G64, (uint64_t)a.N, G64 * 2,
                        kGroupsPerStage, Cfg::BN, CU_TENSOR_MAP_SWIZZLE_NONE, err))
      return cudaErrorInvalidValue;
    if (!encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.biases, G64, (uint64_t)a.N, G64 * 2,
                        kGroupsPerStage, Cfg::BN, CU_TENSOR_MAP_SWIZZLE_NONE, err))
      return cudaErrorInvalidValue;
  } else {
    ts = tw;  // unused
    tb = tw;
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.G);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, tw, ts, tb, tx, p);
}

// Configuration table: (NT, consumer warps, stages).
constexpr int kWarpsDefault = 8;

}  // namespace

size_t skinny_scratch_bytes(const SkinnyArgs& a, int device) {
  const DeviceInfo& di = device_info(device);
  const int NT = a.M <= 8 ? 1 : 2;
  const int BN = kWarpsDefault * 16;
  const long long T = (a.N + BN - 1) / BN;
  (void)T;
  const long long G = (long long)di.sm_count * 2;  // upper bound on resident CTAs
  return kCounterBytes + (size_t)G * 2 * BN * 8 * NT * sizeof(float);
}

cudaError_t launch_skinny(const SkinnyArgs& a, const Scratch& scratch, cudaStream_t stream, bool pdl,
                          std::string* err) {
  if (a.M <= 8) return launch_cfg<1, kWarpsDefault, 4>(a, scratch, stream, pdl, err);
  return launch_cfg<2, kWarpsDefault, 3>(a, scratch, stream, pdl, err);
}

}  // namespace qw
