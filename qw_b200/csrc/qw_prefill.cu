// qw_prefill.cu -- affine 4-bit group-64 quantized matmul for prefill-sized
// M (>= 17 rows of x) on the 5th-generation tensor cores.  Compute-bound.
//
// One CTA per SM walks output tiles of 128 weight rows x 256 tokens
// (persistent, token tiles fastest so a weight tile is reused from L2):
//
//   warp 0      TMA producer, per 64-wide k group: the x box (256 tokens x
//               64 halves, 128-byte swizzle, K-major: the UMMA B operand) and
//               the packed weights of the group (128 rows x 32 bytes).
//   warp 1      allocates TMEM and issues tcgen05.mma (one thread):
//               D[128 x 256, fp32, TMEM] += A[128 x 64, TMEM] * x^T, four
//               K=16 instructions per group, tcgen05.commit releasing stages.
//   warps 2-9   dequantize: the two warps of a TMEM lane quarter own its 32
//               weight rows (one row per lane) and take alternate groups, all
//               64 codes of each; they write fp16 weights to a TMEM A stage
//               with tcgen05.st.  After the last group of a tile they read D
//               back (tcgen05.ld, half of the tokens each) and store y.
//
// SwiGLU (gate and up projections with the activation fused): a tile is 64
// gate rows and the same 64 up rows, staged so that TMEM lanes l and l + 16
// of each lane quarter hold one output's gate and up sums; the epilogue pairs
// them with one shuffle per token and writes silu(gate) * up (64 outputs per
// tile, each op rounded to fp16).
//
// The weights the MMA consumes are exactly qw_dequantize's (fp16(fp16(s*q)
// + b)): pairs (1024 + q_even, 1024 + 16 q_odd) come from one prmt and one
// and, fma.rn.f16x2 with (s, s/16) and (-1024 s, -64 s) gives fp16(s*q)
// rounded once from the exact product, and add.rn.f16x2 adds b.  Scales too
// small for s/16 to be exact, or too large for 1024 s, take an exact
// per-element path.  Accumulation is fp32 in the tensor cores.
#include <cuda_fp16.h>

#include "qw_internal.h"
#include "qw_ptx.cuh"

namespace qw {

namespace {

constexpr int kGroup = 64;
constexpr int BM = 128;       // weight rows per tile (UMMA M, TMEM lanes)
// Packed codes of one 64-wide k block: BITS/2 words (4-bit: 8, 8-bit: 16) per
// row.  BT tokens per tile (UMMA N): 256 for prefill; 32 for calls of at most
// 32 rows of x (the configurations without the decode kernel: 8-bit codes,
// groups of 128, and 17..32 rows), whose narrow x tiles leave room for a
// deeper pipeline of weight blocks.
template <int BITS, int BT_>
struct PfCfg {
  static constexpr int BT = BT_;
  static constexpr int STAGES = BT >= 128 ? 4 : 8;  // pipeline depth (x box, packed W, TMEM A)
  static constexpr int X_STAGE = BT * 128;          // 64 halves of k per token row
  static constexpr int WP_ROW = kGroup * BITS / 8;   // bytes per row per k block
  static constexpr int WORDS = kGroup * BITS / 32;   // packed words per row per k block
  static constexpr int WP_STAGE = BM * WP_ROW;
  static constexpr int OFF_X = 0;
  static constexpr int OFF_WP = STAGES * X_STAGE;
  // barriers: xfull, wpfull, wpempty, afull, aempty (per stage), dfull, dempty
  static constexpr int NBAR = 5 * STAGES + 2;
  static constexpr int OFF_BAR = OFF_WP + STAGES * WP_STAGE;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 64 + 1024;
  // TMEM: D (BT fp32 columns) at 0, then the A stages (32 columns each)
  static constexpr uint32_t D_COL = 0;
  static constexpr uint32_t A_COL = BT >= 128 ? BT : 128;
  static constexpr uint32_t TMEM_COLS = A_COL + 32 * STAGES <= 256 ? 256 : 512;
  static_assert(A_COL + 32 * STAGES <= 512, "TMEM columns");
  static_assert(SMEM <= 232448, "shared memory budget");
};
constexpr int DQW = 8;             // dequant / epilogue warps: 2 per TMEM lane quarter
constexpr int THREADS = (2 + DQW) * 32;

struct PrefillParams {
  int M, N, K;
  int n_tiles, m_tiles, groups;  // groups: 64-wide k blocks
  int gsh;                       // k blocks per quantization group (group_size / 64)
  int sb_groups;                 // quantization groups per row (K / group_size)
  int y_f32;
  int swiglu;      // gate (tm_w, scales, biases) and up (tm_w2, scales2, biases2), 64 rows of each per tile
  int tile_rows;   // output rows per tile: 128, or 64 with swiglu
  void* y;
  const __half* scales;
  const __half* biases;
  const __half* scales2;
  const __half* biases2;
  unsigned int* status;
};

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  // K-major, 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart.
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, M x N.
constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Exact per-element dequantization, for scales outside the fast path's range.
// Inlined and fully unrolled so that `out` stays in registers on both paths.
__device__ __forceinline__ void dequant_group_slow(const uint32_t (&wd)[4], __half s, __half b, uint32_t (&out)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      const uint32_t q0 = (wd[i] >> (8 * pp)) & 0xFu, q1 = (wd[i] >> (8 * pp + 4)) & 0xFu;
      const __half t0 = __hmul_rn(s, __uint2half_rn(q0));
      const __half t1 = __hmul_rn(s, __uint2half_rn(q1));
      out[4 * i + pp] = h2_bits(__halves2half2(__hadd_rn(t0, b), __hadd_rn(t1, b)));
    }
  }
}

template <int BITS, int BT_>
__global__ void __launch_bounds__(THREADS, 1)
    qmm_prefill_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                       const __grid_constant__ CUtensorMap tm_w2, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  using Cfg = PfCfg<BITS, BT_>;
  constexpr int BT = Cfg::BT;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int X_STAGE = Cfg::X_STAGE;
  constexpr int OFF_X = Cfg::OFF_X;
  constexpr uint32_t D_COL = Cfg::D_COL, A_COL = Cfg::A_COL, TMEM_COLS = Cfg::TMEM_COLS;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* xfull = bars;
  uint64_t* wpfull = bars + STAGES;
  uint64_t* wpempty = bars + 2 * STAGES;
  uint64_t* afull = bars + 3 * STAGES;
  uint64_t* aempty = bars + 4 * STAGES;  // arrived by tcgen05.commit: x slot and A stage are free
  uint64_t* dfull = bars + 5 * STAGES;
  uint64_t* dempty = dfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dempty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int total_tiles = p.n_tiles * p.m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&wpfull[s], 1);
      mbar_init(&wpempty[s], DQW / 2);  // the four warps (lane quarters) that own the group
      mbar_init(&afull[s], DQW / 2);
      mbar_init(&aempty[s], 1);
    }
    mbar_init(dfull, 1);
    mbar_init(dempty, DQW);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&tm_x);
      prefetch_tensormap(&tm_w);
      if (p.swiglu) prefetch_tensormap(&tm_w2);
      pdl_wait();
      const uint64_t pol_w = l2_policy_evict_last();
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort_flag; tile += gridDim.x) {
        const int nt = tile / p.m_tiles, mt = tile % p.m_tiles;
        for (int g = 0; g < p.groups; ++g, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (it >= STAGES) {
            // x slot s is free once the MMAs that read it completed; the
            // packed-weight slot once the dequant warps read it.
            if (!mbar_wait(&aempty[s], ph ^ 1, p.status, kDevTimeoutEmpty) ||
                !mbar_wait(&wpempty[s], ph ^ 1, p.status, kDevTimeoutEmpty)) {
              *abort_flag = 1;
              break;
            }
          }
          mbar_arrive_expect_tx(&xfull[s], X_STAGE);
          tma_load_2d(smem + OFF_X + s * X_STAGE, &tm_x, &xfull[s], g * kGroup, mt * BT);
          mbar_arrive_expect_tx(&wpfull[s], Cfg::WP_STAGE);
          uint8_t* wp = smem + Cfg::OFF_WP + s * Cfg::WP_STAGE;
          if (!p.swiglu) {
            tma_load_2d_hint(wp, &tm_w, &wpfull[s], g * Cfg::WP_ROW, nt * BM, pol_w);
          } else {  // 64 gate rows, then the same 64 up rows
            tma_load_2d_hint(wp, &tm_w, &wpfull[s], g * Cfg::WP_ROW, nt * (BM / 2), pol_w);
            tma_load_2d_hint(wp + (BM / 2) * Cfg::WP_ROW, &tm_w2, &wpfull[s], g * Cfg::WP_ROW, nt * (BM / 2), pol_w);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = idesc_f16(BM, BT);
    uint32_t it = 0, tile_count = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++tile_count) {
      // the epilogue has drained D from the previous tile
      if (tile_count > 0 && !*abort_flag &&
          !mbar_wait(dempty, (tile_count - 1) & 1, p.status, kDevTimeoutAccum))
        *abort_flag = 1;
      tc_fence_after();
      for (int g = 0; g < p.groups; ++g, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!*abort_flag) {
          if (!mbar_wait(&xfull[s], ph, p.status, kDevTimeoutFull) ||
              !mbar_wait(&afull[s], ph, p.status, kDevTimeoutFull))
            *abort_flag = 1;
        }
        tc_fence_after();
        if (lane == 0 && !*abort_flag) {
          const uint64_t bdesc = smem_desc_sw128(smem_u32(smem + OFF_X + s * X_STAGE));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            tc_mma_ts(tmem + D_COL, tmem + A_COL + s * 32 + kk * 8, bdesc + (uint64_t)(2 * kk), idesc,
                      (g > 0 || kk > 0) ? 1u : 0u);
          }
        }
        __syncwarp();
        if (lane == 0) tc_commit(&aempty[s]);  // frees x slot s and A stage s when these MMAs finish
        __syncwarp();
      }
      if (lane == 0) tc_commit(dfull);
      __syncwarp();
    }
  } else {
    // ---------------------------------------------- dequant + epilogue
    const int dw = warp - 2;                 // 0..7
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int khalf = dw >> 2;               // which groups (even / odd) / which 128 tokens
    // The weight row this lane dequantizes into its TMEM lane (quarter * 32 +
    // lane): the tile's row quarter * 32 + lane, or with SwiGLU, lanes 0-15
    // of a quarter take gate rows 16 quarter + lane and lanes 16-31 the same
    // rows' up projection (staged 64 rows further on), so lanes l and l + 16
    // hold the two halves of one output.
    const bool up_lane = p.swiglu && lane >= 16;
    const int row_in_tile = p.swiglu ? quarter * 16 + (lane & 15) : quarter * 32 + lane;  // output row
    const int smem_row = p.swiglu ? row_in_tile + (up_lane ? BM / 2 : 0) : row_in_tile;
    const __half* scales = up_lane ? p.scales2 : p.scales;
    const __half* biases = up_lane ? p.biases2 : p.biases;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    pdl_wait();
    uint32_t tile_count = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++tile_count) {
      const int nt = tile / p.m_tiles, mt = tile % p.m_tiles;
      const int row = nt * p.tile_rows + row_in_tile;
      const bool row_ok = row < p.N;
      const __half* srow = scales + (size_t)(row_ok ? row : 0) * p.sb_groups;
      const __half* brow = biases + (size_t)(row_ok ? row : 0) * p.sb_groups;
      // This warp dequantizes every other k block of the tile in full (the
      // other warp of its lane quarter takes the rest), so each warp has two
      // MMA block-times per block of its own.
      __half s_next = (row_ok && khalf < p.groups) ? srow[khalf / p.gsh] : __float2half(0.f);
      __half b_next = (row_ok && khalf < p.groups) ? brow[khalf / p.gsh] : __float2half(0.f);
      for (int g = khalf; g < p.groups; g += 2) {
        const uint32_t it = tile_count * (uint32_t)p.groups + (uint32_t)g;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const __half sc = s_next, bi = b_next;
        if (g + 2 < p.groups && row_ok) {  // prefetch this warp's next block's scale/bias
          s_next = srow[(g + 2) / p.gsh];
          b_next = brow[(g + 2) / p.gsh];
        }
        if (!*abort_flag && !mbar_wait(&wpfull[s], ph, p.status, kDevTimeoutFull)) *abort_flag = 1;
        uint32_t wd[Cfg::WORDS];
        {
          const uint4* src =
              reinterpret_cast<const uint4*>(smem + Cfg::OFF_WP + s * Cfg::WP_STAGE + smem_row * Cfg::WP_ROW);
#pragma unroll
          for (int i = 0; i < Cfg::WORDS / 4; ++i) {
            const uint4 a = src[i];
            wd[4 * i] = a.x; wd[4 * i + 1] = a.y; wd[4 * i + 2] = a.z; wd[4 * i + 3] = a.w;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&wpempty[s]);
        // dequantize the block's 64 codes into 32 fp16 pairs (k ascending)
        uint32_t out[2][16];
        const float sf = __half2float(sc);
        const uint32_t b2 = h2_bits(__halves2half2(bi, bi));
        if (BITS == 4) {
          const bool fast = fabsf(sf) >= 0.0009765625f && fabsf(sf) < 63.0f;  // s/16 exact, 1024 s finite
          if (fast) {
            const __half s16 = __float2half_rn(sf * 0.0625f);  // exact: s >= 2^-10
            const uint32_t s2 = h2_bits(__halves2half2(sc, s16));
            const uint32_t c2 =
                h2_bits(__halves2half2(__float2half_rn(-1024.f * sf), __float2half_rn(-64.f * sf)));
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
#pragma unroll
                for (int pp = 0; pp < 4; ++pp) {
                  const uint32_t t = prmt(wd[4 * hh + i], 0x64646464u, 0x4040u + 0x0101u * pp) & 0xFFF0FF0Fu;
                  out[hh][4 * i + pp] = hadd2_rn(hfma2_rn(t, s2, c2), b2);
                }
              }
          } else {
            uint32_t w0[4] = {wd[0], wd[1], wd[2], wd[3]}, w1[4] = {wd[4], wd[5], wd[6], wd[7]};
            dequant_group_slow(w0, sc, bi, out[0]);
            dequant_group_slow(w1, sc, bi, out[1]);
          }
        } else {
          // 8-bit: a word holds 4 codes; prmt pairs them with 0x64 into
          // (1024 + q_even, 1024 + q_odd), and fma with (s, s), (-1024 s,
          // -1024 s) rounds s*q once from the exact product.
          const bool fast = fabsf(sf) < 63.0f;  // 1024 s finite
          if (fast) {
            const uint32_t s2 = h2_bits(__halves2half2(sc, sc));
            const __half c = __float2half_rn(-1024.f * sf);
            const uint32_t c2 = h2_bits(__halves2half2(c, c));
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const uint32_t t0 = prmt(wd[i], 0x64646464u, 0x5140u);
              const uint32_t t1 = prmt(wd[i], 0x64646464u, 0x5342u);
              out[i / 8][2 * (i % 8)] = hadd2_rn(hfma2_rn(t0, s2, c2), b2);
              out[i / 8][2 * (i % 8) + 1] = hadd2_rn(hfma2_rn(t1, s2, c2), b2);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
#pragma unroll
              for (int pp = 0; pp < 2; ++pp) {
                const uint32_t q0 = (wd[i] >> (16 * pp)) & 0xFFu, q1 = (wd[i] >> (16 * pp + 8)) & 0xFFu;
                const __half t0 = __hmul_rn(sc, __uint2half_rn(q0));
                const __half t1 = __hmul_rn(sc, __uint2half_rn(q1));
                out[i / 8][2 * (i % 8) + pp] = h2_bits(__halves2half2(__hadd_rn(t0, bi), __hadd_rn(t1, bi)));
              }
          }
        }
        // write A stage s once the MMAs that read it last have completed
        if (it >= STAGES && !*abort_flag && !mbar_wait(&aempty[s], ph ^ 1, p.status, kDevTimeoutEmpty))
          *abort_flag = 1;
        tc_fence_after();
        tmem_st_x16(tmem + lane_base + A_COL + s * 32, out[0]);
        tmem_st_x16(tmem + lane_base + A_COL + s * 32 + 16, out[1]);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[s]);
      }
      // ---------------------------------------------------------- epilogue
      if (!*abort_flag && !mbar_wait(dfull, tile_count & 1, p.status, kDevTimeoutAccum)) *abort_flag = 1;
      tc_fence_after();
#pragma unroll 1
      for (int cb = khalf * (BT / 32); cb < (khalf + 1) * (BT / 32); ++cb) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(tmem + lane_base + D_COL + cb * 16, v);
        tmem_wait_ld();
        if (p.swiglu) {
          // lane l < 16 finishes tokens 0-7 of the block and lane l + 16
          // tokens 8-15: each sends its partner the half the partner needs
          float g[8], u[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float mine_lo = __uint_as_float(v[q]), mine_hi = __uint_as_float(v[q + 8]);
            const float other = __shfl_xor_sync(0xffffffffu, up_lane ? mine_lo : mine_hi, 16);
            g[q] = up_lane ? other : mine_lo;
            u[q] = up_lane ? mine_hi : other;
          }
          if (!row_ok || *abort_flag) continue;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int tok = mt * BT + cb * 16 + (up_lane ? 8 : 0) + q;
            if (tok < p.M) {
              const size_t idx = (size_t)tok * p.N + row;
              const float h = swiglu_f16(g[q], u[q]);
              if (p.y_f32) reinterpret_cast<float*>(p.y)[idx] = h;
              else reinterpret_cast<__half*>(p.y)[idx] = __float2half_rn(h);
            }
          }
          continue;
        }
        if (!row_ok || *abort_flag) continue;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int tok = mt * BT + cb * 16 + q;
          if (tok < p.M) {
            const size_t idx = (size_t)tok * p.N + row;
            const float f = __uint_as_float(v[q]);
            if (p.y_f32) reinterpret_cast<float*>(p.y)[idx] = f;
            else reinterpret_cast<__half*>(p.y)[idx] = __float2half_rn(f);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dempty);
    }
  }

  // everyone: make sure all tcgen05 work is finished before freeing TMEM
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

bool prefill_available() { return true; }

namespace {
template <int BITS, int BT>
cudaError_t launch_cfg(const PrefillArgs& a, cudaStream_t stream, bool pdl, std::string* err) {
  using Cfg = PfCfg<BITS, BT>;
  int dev = 0;
  cudaGetDevice(&dev);
  const DeviceInfo& di = device_info(dev);
  static thread_local int configured_dev = -1;
  if (configured_dev != dev) {
    cudaError_t e =
        cudaFuncSetAttribute(qmm_prefill_kernel<BITS, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  PrefillParams p{};
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.groups = (int)(a.K / kGroup);
  p.gsh = a.group_size / kGroup;
  p.sb_groups = (int)(a.K / a.group_size);
  p.swiglu = a.swiglu ? 1 : 0;
  p.tile_rows = a.swiglu ? BM / 2 : BM;
  p.n_tiles = (int)((a.N + p.tile_rows - 1) / p.tile_rows);
  p.m_tiles = (int)((a.M + BT - 1) / BT);
  p.y_f32 = a.y_f32 ? 1 : 0;
  p.y = a.y;
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.biases = reinterpret_cast<const __half*>(a.biases);
  p.scales2 = reinterpret_cast<const __half*>(a.swiglu ? a.scales2 : a.scales);
  p.biases2 = reinterpret_cast<const __half*>(a.swiglu ? a.biases2 : a.biases);
  p.status = a.status;
  CUtensorMap tx, tw, tw2;
  if (!encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, (uint64_t)a.K, (uint64_t)a.M,
                      (uint64_t)(a.x_ld ? a.x_ld : a.K) * 2, kGroup, BT, CU_TENSOR_MAP_SWIZZLE_128B, err))
    return cudaErrorInvalidValue;
  const uint64_t row_bytes = (uint64_t)a.K * BITS / 8;
  if (!encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, row_bytes, (uint64_t)a.N, row_bytes, Cfg::WP_ROW,
                      p.tile_rows, CU_TENSOR_MAP_SWIZZLE_NONE, err))
    return cudaErrorInvalidValue;
  tw2 = tw;  // unused unless SwiGLU
  if (a.swiglu && !encode_tmap_2d(&tw2, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w2, row_bytes, (uint64_t)a.N, row_bytes,
                                  Cfg::WP_ROW, p.tile_rows, CU_TENSOR_MAP_SWIZZLE_NONE, err))
    return cudaErrorInvalidValue;
  const int tiles = p.n_tiles * p.m_tiles;
  int grid = di.sm_count < tiles ? di.sm_count : tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, qmm_prefill_kernel<BITS, BT>, tx, tw, tw2, p);
}
}  // namespace

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream, bool pdl, std::string* err) {
  if ((a.bits != 4 && a.bits != 8) || (a.group_size != 64 && a.group_size != 128) || a.K % a.group_size) {
    *err = "the prefill kernel takes 4- or 8-bit codes in groups of 64 or 128";
    return cudaErrorInvalidValue;
  }
  // narrow token tiles for at most 32 rows of x
  if (a.M <= 32) return a.bits == 4 ? launch_cfg<4, 32>(a, stream, pdl, err) : launch_cfg<8, 32>(a, stream, pdl, err);
  return a.bits == 4 ? launch_cfg<4, 256>(a, stream, pdl, err) : launch_cfg<8, 256>(a, stream, pdl, err);
}

}  // namespace qw
