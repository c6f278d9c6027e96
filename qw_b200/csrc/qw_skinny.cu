// qw_skinny.cu -- affine 4- or 8-bit quantized matmul (groups of 64 or 128)
// for M <= 16 rows of x (decode M=1, MTP verify M=4, DFlash2 block M=16).
// HBM-bound: the packed weights are streamed once.
//
// Work decomposition ("stream-K"): the weight matrix is cut into row tiles of
// BN = 128 rows and the K axis into 512-wide chunks (8 groups).  The T*C
// (tile, chunk) units are dealt out as contiguous ranges to a persistent grid
// of one CTA per SM, so every CTA streams the same number of bytes whatever N
// and K are.  A tile whose chunks are split between CTAs is combined through
// fp32 partial slots in scratch memory: every contributor writes its slot,
// bumps the tile's counter, and the last one to arrive adds the slots in CTA
// order (deterministic) and writes y.
//
// CTA roles (warp-specialised), per pipeline stage of 128 rows x 512 k:
//   warp 0        TMA producer of packed W (two 128-byte SW128 boxes, 32 KB;
//                 four, 64 KB, with 8-bit codes),
//                 scales and biases (one box each); it does not wait for the
//                 previous kernel, so under PDL this launch's weight stream
//                 starts while the previous kernel finishes.
//   warp 1        TMA producer of x (one 3-D box of 8 groups x M rows), after
//                 griddepcontrol.wait (x is the previous kernel's output).
//   helper warps  turn the stage's x into the MMA B fragments every consumer
//                 warp needs (permuted, odd k pre-scaled by 1/16) and the
//                 per-group sums X and Z of the fold below.
//   8 consumers   16 weight rows and all 8 groups of a unit each (rows
//                 8c..8c+7 of each 64-row half of the tile for consumer c).
//                 With up to 8 tokens a consumer copies unit j+1's weights
//                 out of the ring group by group while it computes unit j,
//                 so a weight slot is released one unit earlier.
//
// SwiGLU ops (an MLP's gate and up projections, activation fused): the top
// half of a tile is 64 gate rows and the bottom half the same 64 up rows, so
// each consumer lane ends with a gate sum and its up sum in registers and
// writes silu(gate) * up, rounded to fp16 after each op as the reference's
// fp16 arrays are; the 2I projection outputs are never stored.
//
// One token with 4-bit codes: the 8 groups of a unit are the 8 columns of
// the MMAs (group gi's B fragment is x in the lanes of column gi and zero in
// the others), so one accumulator pair collects the whole unit and the fold
// below runs once per unit instead of once per group.  This path also comes
// with 16-group units (1024 k, four boxes a stage, a fold per 8 groups):
// 512 contiguous bytes per weight row per stage and half the units, chosen
// per shape by the host.
//
// Row-parallel exchange (a separate instantiation, XCHG): the launch is one
// rank's K-slice of a tensor-parallel projection, and y is the sum over the
// ranks.  Finished tiles go to this rank's slot of the communicator's buffer
// (qw_exchange.cuh); after its last unit a CTA copies its tiles into every
// peer's buffer, flags them, waits (bounded) for every rank's flags of the
// same tiles, and sums them in rank order into y.
//
// Consumer arithmetic (no per-element dequantisation): a packed word w holds
// nibbles q0..q7 (k ascending).  lop3(w & 0x000F000F | 0x64006400) is the fp16
// pair (1024 + q0, 1024 + q4) and lop3(w & 0x00F000F0 | 0x64006400) is
// (1024 + 16 q1, 1024 + 16 q5), both exact; the same on w >> 8 gives q2/q6 and
// q3/q7.  These feed mma.sync m16n8k16 directly as the A operand (16 weight
// rows) against x as B (one column per token, odd k scaled by 1/16), so one
// group's four MMAs give d = 1024 X_even + 64 X_odd + sum_k x_k q_k in fp32.
// The group is folded into the output as
//     y += s * (d - Z) + b * X,   Z = 1024 X_even + 64 X_odd,
// which is sum_k x_k (s q_k + b): the weight formed in fp32 and accumulated in
// fp32 (the reference semantics).
//
// 8-bit codes: a stage's chunk is four SW128 boxes (512 bytes per row), a
// word holds codes q0..q3, and prmt(w, 0x64646464) pairs each byte with 0x64
// into the exact fp16 1024 + q, so the MMAs see x unscaled (the helpers only
// reorder it) and Z = 1024 X.
#include <cuda_fp16.h>

#include <mutex>

#include "qw_exchange.cuh"
#include "qw_internal.h"
#include "qw_ptx.cuh"

namespace qw {

namespace {

constexpr int kGroup = 64;
constexpr int kGroupsPerStage = 8;
constexpr size_t kMaxCounters = kSkinnyMaxCounters;  // row tiles per launch (N <= 8M rows)
constexpr size_t kCounterBytes = kSkinnyCounterBytes;

constexpr int align1k(int v) { return (v + 1023) / 1024 * 1024; }

// MT: most tokens (rows of x) a launch of this configuration handles.
//
// Shared memory holds two rings:
//   weight ring (WST stages): packed W (two SW128 boxes) + scales + biases of
//     one unit.  Consumers copy what they need into registers (ldmatrix and
//     the group's scale/bias pairs) and release the slot before computing, so
//     a slot is busy only while its copy is in flight: the ring is the
//     kernel's bytes-in-flight budget against HBM latency.
//   small ring (SST stages): the unit's x box and what the helper warps derive
//     from it (MMA B fragments, per-group X / Z sums).  x comes from L2.
// WIDE: 16 groups (1024 k) per unit instead of 8, for the one-token 4-bit
// column scheme: 512 contiguous bytes per weight row per stage, half the
// units and so half the per-unit fixed costs.  The host picks it per shape
// (launch_skinny), since larger units leave a short launch less balanced.
template <int MT, int BITS = 4, bool WIDE = false>
struct SkinnyCfg {
  static constexpr int NT = (MT + 7) / 8;       // n8 MMA column tiles
  static constexpr int MPAD_ = 8 * NT;
  static constexpr int CW = 8;                  // consumer warps: 16 rows x all 8 groups of a unit each
  static constexpr int HW = MT == 1 ? 1 : (MT <= 8 ? 2 : 3);  // helper warps
  static constexpr int BN = 128;                // rows per tile
  // A stage's 512-wide chunk is 256 bytes of 4-bit codes per row (two SW128
  // boxes of 128 bytes) or 512 bytes of 8-bit codes (four boxes), so 8-bit
  // stages are twice as large and the rings shallower.
  // Column scheme (4-bit codes, one to four tokens): the MMA's 8 columns hold
  // (token, group) pairs, TPC token columns for each of GPC groups, so one
  // accumulator chain collects GPC groups and the fold runs once per GPC
  // groups.  Group gi's B fragment is x in the lanes of its columns and zero
  // in the others.  One token: 8 groups a chain; up to four: 2 groups a chain.
  static constexpr bool COLS = BITS == 4 && (MT == 1 || MT == 4);
  static constexpr int TPC = MT == 4 ? 4 : 1;  // token columns per group
  static constexpr int GPC = 8 / TPC;          // groups per accumulator chain
  static_assert(!WIDE || (COLS && TPC == 1), "16-group units are built for the one-token column scheme");
  // 64-wide groups per unit (per pipeline stage): the unit is 128 rows x 64 GPS k
  static constexpr int GPS = WIDE ? 16 : 8;
  static constexpr int CK = kGroup * GPS;       // k per unit
  static constexpr int NBOX = GPS * kGroup * BITS / 8 / 128;  // 128-byte TMA boxes of a unit's codes
  // Ring depths: the one-token 4-bit path measured fastest with two weight
  // stages (13.4 us at 17408 x 5120 against 13.8 to 14.2 with 3 to 5).
  static constexpr int WST = BITS == 8 ? (MT == 1 ? 3 : 2) : (COLS ? 2 : (MT <= 8 ? 4 : 3));
  static constexpr int SST = BITS == 8 ? 2 : (COLS ? 2 : (MT <= 8 ? 3 : 2));
  static constexpr int W_BOX = BN * 128;
  static constexpr int SB_BYTES = BN * 2 * GPS;
  static constexpr int W_STAGE = NBOX * W_BOX + 2 * SB_BYTES;  // W boxes, scales, biases
  static constexpr int OFF_WS = NBOX * W_BOX;
  static constexpr int OFF_WB = OFF_WS + SB_BYTES;
  static constexpr int X_BYTES = GPS * MT * 128;
  static constexpr int BF_TOK = MT;
  // COLS: per group a 1 KB block [b0 | b1][32 lanes][16 bytes], zero except
  // the lanes of group gi's columns.  Otherwise per group
  // [b0 | b1][token][lane column][16 bytes]: a warp's lanes read consecutive
  // 16-byte words, free of bank conflicts.
  static constexpr int BF_GROUP = BF_TOK * 4 * 32;
  static constexpr int BF_BYTES = COLS ? GPS * 1024 : GPS * BF_GROUP;
  // (X, Z) per group and token column: with COLS entry (gi, t) is at gi * TPC + t
  static constexpr int XZ_COLS = COLS ? TPC : 8 * NT;
  static constexpr int XZ_BYTES = GPS * XZ_COLS * 8;
  static constexpr int OFF_X = 0;  // within a small stage (1024-aligned for SW128)
  static constexpr int OFF_BF = align1k(X_BYTES);
  static constexpr int OFF_XZ = OFF_BF + BF_BYTES;
  static constexpr int S_STAGE = align1k(OFF_XZ + XZ_BYTES);
  static constexpr int OFF_WRING = 0;
  static constexpr int OFF_SRING = WST * W_STAGE;
  static constexpr int OFF_COMB = OFF_SRING + SST * S_STAGE;
  static constexpr int COMB_BYTES = 0;
  // Cluster split-K: the leader CTA of a tile receives the other CTAs'
  // partials here (distributed shared memory).
  static constexpr int SPLIT_MAX = MT <= 8 ? 4 : 2;
  static constexpr int RECV_BYTES = (SPLIT_MAX - 1) * BN * MPAD_ * 4;
  static constexpr int OFF_RECV = OFF_COMB + COMB_BYTES;
  static constexpr int OFF_BAR = OFF_RECV + RECV_BYTES;
  static constexpr int NBAR = 2 * WST + 3 * SST + 1;  // wfull, wempty | sfull, ready, sempty | recv
  // after the barriers: MISC_INTS words (abort, two finish flags, the
  // exchange's epoch)
  static constexpr int MISC_INTS = 4;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + MISC_INTS * 4 + 1024;
  static constexpr int THREADS = (2 + HW + CW) * 32;
  // registers per thread: the whole register file over the CTA's warps
  static constexpr int MAXREG = (65536 / THREADS) & ~7;
  static constexpr int MPAD = 8 * NT;
  static constexpr int PART = BN * MPAD;  // floats per partial slot
  static_assert(W_STAGE % 1024 == 0, "weight stages stay 1024-aligned");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// One quantized matmul of a launch.  The tensor maps live in the kernel's
// parameter space (__grid_constant__), where TMA may read them.
//
// A SwiGLU op (swiglu = 1) is the gate and up projections of an MLP with the
// activation fused into the epilogue: a tile is 64 gate rows (tm_w, tm_s,
// tm_b) above the same 64 up rows (tm_w2, tm_s2, tm_b2), so the thread that
// holds gate row i also holds up row i, and y = silu(gate) * up has N (the
// intermediate width) columns.
struct SkinnyOp {
  CUtensorMap tm_w, tm_s, tm_b, tm_x;
  CUtensorMap tm_w2, tm_s2, tm_b2;  // SwiGLU: the up projection
  int N, K;
  int C;          // chunks along K
  int T;          // row tiles
  long long U;    // T * C
  int G;          // CTAs that take units of this matmul: the first min(grid, U)
  int sb_tma;     // scales/biases through TMA (needs K % 512 == 0 and groups of 64)
  int gsh;        // 64-wide groups per quantization group (1: groups of 64, 2: of 128)
  int y_f32;
  int swiglu;
  void* y;
  const __half* scales;
  const __half* biases;
  const __half* scales2;  // SwiGLU: the up projection's
  const __half* biases2;
};

// A launch runs OPS_MAX >= n_ops matmuls in order, every CTA taking its share
// of each.  With several, matmul o+1 may read what matmul o wrote: a CTA
// counts itself in gbar[o] once all its writes for o are done, and loads x
// for o+1 only when all G CTAs have (the weight ring runs ahead regardless).
template <int OPS_MAX>
struct SkinnyLaunch {
  SkinnyOp op[OPS_MAX];
  int n_ops;
  int M;
  int G;                  // CTAs (all resident at once when n_ops > 1)
  int split;              // > 1 (one matmul only): each tile split over a cluster of `split` CTAs
  float* part;            // [G][2][PART]
  unsigned int* counter;  // [T], zero between launches
  unsigned int* gbar;     // [n_ops]: CTAs done with each matmul, zero at launch (n_ops > 1)
  unsigned long long* amax;  // one matmul only, may be null: [M] greedy-token keys (atomicMax)
  unsigned int* status;   // device status word
  ArParams ar;            // one matmul only: ar.P > 0 sums y over the ranks in the epilogue
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
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void sts_f32x2(uint32_t addr, float a, float b) {
  asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t w, uint32_t mask) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "r"(mask), "r"(0x64006400u));
  return r;
}
__device__ __forceinline__ float half_lo(uint32_t h2) { return __half2float(__ushort_as_half((uint16_t)(h2 & 0xffffu))); }
__device__ __forceinline__ float half_hi(uint32_t h2) { return __half2float(__ushort_as_half((uint16_t)(h2 >> 16))); }

// Greedy-token key of logit `v` at `row`: the fp16 logit as an order-
// preserving unsigned integer above, the complement of the row below, so the
// largest key is the largest logit and, among equal logits, the lowest row.
__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}
__device__ __forceinline__ unsigned long long amax_key(float v, int row) {
  uint32_t b = __float_as_uint(__half2float(__float2half_rn(v)));
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}

// Grid-wide wait of a chained launch: all `target` CTAs have finished the
// matmul whose tally `gbar` is.
__device__ __forceinline__ bool wait_matmuls_done(const unsigned int* gbar, unsigned int target,
                                                  unsigned int* status) {
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(gbar) : "memory");
    if (v >= target) break;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_status(status, kDevTimeoutAccum);
      return false;
    }
    __nanosleep(64);
  }
  // x is read by TMA (async proxy) after other CTAs' generic stores
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// XCHG: the row-parallel exchange in the epilogue (p.ar); a separate
// instantiation, so the plain kernel carries none of its code.
template <int MT, int OPS_MAX, int BITS, bool WIDE, bool XCHG>
__global__ void __launch_bounds__((SkinnyCfg<MT, BITS, WIDE>::THREADS), 1)
    __maxnreg__((SkinnyCfg<MT, BITS, WIDE>::MAXREG))
        qmm_skinny_kernel(const __grid_constant__ SkinnyLaunch<OPS_MAX> p) {
  using Cfg = SkinnyCfg<MT, BITS, WIDE>;
  static_assert(!XCHG || OPS_MAX == 1, "the exchange takes single-matmul launches");
  constexpr int NT = Cfg::NT;
  constexpr int WST = Cfg::WST;
  constexpr int SST = Cfg::SST;
  extern __shared__ uint8_t smem_raw[];
  // Align to 1024 bytes by pointer arithmetic on the shared array itself, so
  // the compiler keeps treating every access through `smem` as shared memory.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* wfull = bars;
  uint64_t* wempty = bars + WST;
  uint64_t* sfull = bars + 2 * WST;
  uint64_t* ready = sfull + SST;
  uint64_t* sempty = ready + SST;
  uint64_t* recv_bar = sempty + SST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + Cfg::NBAR);
  volatile int* fin_flag = abort_flag + 1;  // [2]: tile+1 to finish per partial slot, 0 = none
  volatile unsigned int* xepoch = reinterpret_cast<volatile unsigned int*>(abort_flag + 3);  // exchange epoch
  uint8_t* wring = smem + Cfg::OFF_WRING;
  uint8_t* sring = smem + Cfg::OFF_SRING;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  // This CTA's contiguous range of (tile, chunk) units of matmul o.
  auto units_of = [&](int o, long long* u0) -> int {
    const SkinnyOp& op = p.op[OPS_MAX == 1 ? 0 : o];
    if ((int)blockIdx.x >= op.G) {
      *u0 = 0;
      return 0;
    }
    *u0 = unit_begin(blockIdx.x, op.U, op.G);
    return (int)(unit_begin(blockIdx.x + 1, op.U, op.G) - *u0);
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < WST; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], Cfg::CW);
    }
    for (int i = 0; i < SST; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&ready[i], Cfg::HW);
      mbar_init(&sempty[i], Cfg::CW);
    }
    mbar_init(recv_bar, (p.split - 1) * Cfg::CW);
    *abort_flag = 0;
    fin_flag[0] = 0;
    fin_flag[1] = 0;
    fence_barrier_init();
  }
  if (p.split > 1) {
    // every CTA's barriers are initialised before any remote arrival
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  } else {
    __syncthreads();
  }
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------------------------------------------- weight producer
    // Weights, scales and biases are constants of the launch: this ring does
    // not wait for the previous kernel, nor for the previous matmul of a
    // chain, so their tails overlap the next weights' stream.
    const uint64_t pol_w = l2_policy_evict_first();
    int slot = 0, issued = 0;
    uint32_t phase = 0;
    for (int o = 0; o < (OPS_MAX == 1 ? 1 : p.n_ops); ++o) {
      const SkinnyOp& op = p.op[OPS_MAX == 1 ? 0 : o];
      const uint32_t w_bytes = Cfg::NBOX * Cfg::W_BOX + (op.sb_tma ? 2 * Cfg::SB_BYTES : 0);
      if (lane == 0) {
        prefetch_tensormap(&op.tm_w);
        if (op.sb_tma) {
          prefetch_tensormap(&op.tm_s);
          prefetch_tensormap(&op.tm_b);
        }
        if (op.swiglu) {
          prefetch_tensormap(&op.tm_w2);
          if (op.sb_tma) {
            prefetch_tensormap(&op.tm_s2);
            prefetch_tensormap(&op.tm_b2);
          }
        }
      }
      long long u0;
      const int nunits = units_of(o, &u0);
      const int G = op.K / kGroup;  // 64-wide groups of a row
      const int Gs = G / op.gsh;    // scale and bias columns of a row
      int t = (int)(u0 / op.C), c = (int)(u0 % op.C);
      for (int j = 0; j < nunits; ++j, ++issued) {
        if (issued >= WST && !*abort_flag) {
          if (!mbar_wait(&wempty[slot], phase ^ 1u, p.status, kDevTimeoutEmpty)) *abort_flag = 1;
        }
        if (*abort_flag) break;
        uint8_t* st = wring + slot * Cfg::W_STAGE;
        if (lane == 0) {
          if (op.sb_tma) mbar_arrive_expect_tx(&wfull[slot], w_bytes);
          else mbar_expect_tx(&wfull[slot], w_bytes);
          // byte column of the chunk: 512 codes of BITS bits
          const int cx = c * (Cfg::NBOX * 128);
          if (!op.swiglu) {
#pragma unroll
            for (int bx = 0; bx < Cfg::NBOX; ++bx)
              tma_load_2d_hint(st + bx * Cfg::W_BOX, &op.tm_w, &wfull[slot], cx + bx * 128, t * Cfg::BN, pol_w);
            if (op.sb_tma) {
              tma_load_2d_hint(st + Cfg::OFF_WS, &op.tm_s, &wfull[slot], c * Cfg::GPS, t * Cfg::BN, pol_w);
              tma_load_2d_hint(st + Cfg::OFF_WB, &op.tm_b, &wfull[slot], c * Cfg::GPS, t * Cfg::BN, pol_w);
            }
          } else {
            // 64 gate rows, then the same 64 up rows (boxes of 64 rows; the
            // up half starts on a 1024-byte boundary, so the 128-byte swizzle
            // pattern is the one a 128-row box would have)
            constexpr int H = Cfg::BN / 2;
            const int r0 = t * H;
#pragma unroll
            for (int bx = 0; bx < Cfg::NBOX; ++bx) {
              tma_load_2d_hint(st + bx * Cfg::W_BOX, &op.tm_w, &wfull[slot], cx + bx * 128, r0, pol_w);
              tma_load_2d_hint(st + bx * Cfg::W_BOX + H * 128, &op.tm_w2, &wfull[slot], cx + bx * 128, r0, pol_w);
            }
            if (op.sb_tma) {
              tma_load_2d_hint(st + Cfg::OFF_WS, &op.tm_s, &wfull[slot], c * Cfg::GPS, r0, pol_w);
              tma_load_2d_hint(st + Cfg::OFF_WS + H * 2 * Cfg::GPS, &op.tm_s2, &wfull[slot], c * Cfg::GPS, r0, pol_w);
              tma_load_2d_hint(st + Cfg::OFF_WB, &op.tm_b, &wfull[slot], c * Cfg::GPS, r0, pol_w);
              tma_load_2d_hint(st + Cfg::OFF_WB + H * 2 * Cfg::GPS, &op.tm_b2, &wfull[slot], c * Cfg::GPS, r0, pol_w);
            }
          }
        }
        if (!op.sb_tma) {
          // Scales/biases staged with plain loads (rows not 16-byte strided
          // when K is not a multiple of the unit's k; groups of 128, whose
          // scale serves both 64-wide groups it covers), zero beyond the
          // matrix edge, after the weight boxes are on their way; the stage's
          // arrival follows them.  The stage holds GPS halves per row, filled
          // eight groups (16 bytes) at a time.
          for (int sc = 0; sc < Cfg::GPS / kGroupsPerStage; ++sc) {
            __half* ss = reinterpret_cast<__half*>(st + Cfg::OFF_WS) + sc * kGroupsPerStage;
            __half* sb = reinterpret_cast<__half*>(st + Cfg::OFF_WB) + sc * kGroupsPerStage;
            const int g0 = c * Cfg::GPS + sc * kGroupsPerStage;  // first 64-wide group of these eight
            if (op.gsh == 2 && op.K % Cfg::CK == 0) {
              // Groups of 128 with 16-byte strided rows: a chunk holds 4 per
              // row, one 8-byte load per row each for scales and biases (all in
              // flight together), each value written for both 64-wide groups.
              uint2 sv4[Cfg::BN / 32], bv4[Cfg::BN / 32];
#pragma unroll
              for (int i = 0; i < Cfg::BN / 32; ++i) {
                const int r = lane + 32 * i;
                const bool up = op.swiglu && r >= Cfg::BN / 2;
                const int row = op.swiglu ? t * (Cfg::BN / 2) + (r % (Cfg::BN / 2)) : t * Cfg::BN + r;
                sv4[i] = bv4[i] = make_uint2(0u, 0u);
                if (row < op.N) {
                  const size_t off = (size_t)row * Gs + (size_t)g0 / 2;
                  sv4[i] = *reinterpret_cast<const uint2*>((up ? op.scales2 : op.scales) + off);
                  bv4[i] = *reinterpret_cast<const uint2*>((up ? op.biases2 : op.biases) + off);
                }
              }
#pragma unroll
              for (int i = 0; i < Cfg::BN / 32; ++i) {
                const int r = lane + 32 * i;
                // halves (h0 h1 h2 h3) -> (h0 h0 h1 h1 h2 h2 h3 h3)
                *reinterpret_cast<uint4*>(ss + r * Cfg::GPS) =
                    make_uint4(prmt(sv4[i].x, 0u, 0x1010u), prmt(sv4[i].x, 0u, 0x3232u), prmt(sv4[i].y, 0u, 0x1010u),
                               prmt(sv4[i].y, 0u, 0x3232u));
                *reinterpret_cast<uint4*>(sb + r * Cfg::GPS) =
                    make_uint4(prmt(bv4[i].x, 0u, 0x1010u), prmt(bv4[i].x, 0u, 0x3232u), prmt(bv4[i].y, 0u, 0x1010u),
                               prmt(bv4[i].y, 0u, 0x3232u));
              }
            } else {
              // One row per lane and step, the loads of all four steps in flight
              // together: the eight 64-wide groups of the chunk as two 8-byte
              // loads when the row allows (groups of 64, 8-byte aligned, not past
              // the row's end), one 8-byte load of four group-128 values written
              // twice each, or element by element at a ragged edge.
              uint32_t sw[Cfg::BN / 32][4], bw[Cfg::BN / 32][4];
#pragma unroll
              for (int i = 0; i < Cfg::BN / 32; ++i) {
                const int r = lane + 32 * i;
                const bool up = op.swiglu && r >= Cfg::BN / 2;
                const int row = op.swiglu ? t * (Cfg::BN / 2) + (r % (Cfg::BN / 2)) : t * Cfg::BN + r;
                const __half* srow = (up ? op.scales2 : op.scales) + (size_t)row * Gs;
                const __half* brow = (up ? op.biases2 : op.biases) + (size_t)row * Gs;
#pragma unroll
                for (int q = 0; q < 4; ++q) sw[i][q] = bw[i][q] = 0u;
                if (row >= op.N) continue;
                if (op.gsh == 1 && g0 + kGroupsPerStage <= G && (((size_t)row * Gs + g0) & 3) == 0) {
                  const uint2 s0 = *reinterpret_cast<const uint2*>(srow + g0);
                  const uint2 s1 = *reinterpret_cast<const uint2*>(srow + g0 + 4);
                  const uint2 b0 = *reinterpret_cast<const uint2*>(brow + g0);
                  const uint2 b1 = *reinterpret_cast<const uint2*>(brow + g0 + 4);
                  sw[i][0] = s0.x; sw[i][1] = s0.y; sw[i][2] = s1.x; sw[i][3] = s1.y;
                  bw[i][0] = b0.x; bw[i][1] = b0.y; bw[i][2] = b1.x; bw[i][3] = b1.y;
                } else if (op.gsh == 2 && g0 + kGroupsPerStage <= G && (((size_t)row * Gs + g0 / 2) & 3) == 0) {
                  const uint2 s4 = *reinterpret_cast<const uint2*>(srow + g0 / 2);
                  const uint2 b4 = *reinterpret_cast<const uint2*>(brow + g0 / 2);
                  // halves (h0 h1 h2 h3) -> (h0 h0 h1 h1 h2 h2 h3 h3)
                  sw[i][0] = prmt(s4.x, 0u, 0x1010u); sw[i][1] = prmt(s4.x, 0u, 0x3232u);
                  sw[i][2] = prmt(s4.y, 0u, 0x1010u); sw[i][3] = prmt(s4.y, 0u, 0x3232u);
                  bw[i][0] = prmt(b4.x, 0u, 0x1010u); bw[i][1] = prmt(b4.x, 0u, 0x3232u);
                  bw[i][2] = prmt(b4.y, 0u, 0x1010u); bw[i][3] = prmt(b4.y, 0u, 0x3232u);
                } else {
#pragma unroll
                  for (int g = 0; g < kGroupsPerStage; ++g) {
                    const int grp = g0 + g;
                    if (grp < G) {
                      const uint32_t sv = __half_as_ushort(srow[grp / op.gsh]);
                      const uint32_t bv = __half_as_ushort(brow[grp / op.gsh]);
                      sw[i][g / 2] |= sv << (16 * (g & 1));
                      bw[i][g / 2] |= bv << (16 * (g & 1));
                    }
                  }
                }
              }
#pragma unroll
              for (int i = 0; i < Cfg::BN / 32; ++i) {
                const int r = lane + 32 * i;
                *reinterpret_cast<uint4*>(ss + r * Cfg::GPS) = make_uint4(sw[i][0], sw[i][1], sw[i][2], sw[i][3]);
                *reinterpret_cast<uint4*>(sb + r * Cfg::GPS) = make_uint4(bw[i][0], bw[i][1], bw[i][2], bw[i][3]);
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&wfull[slot]);
        }
        __syncwarp();
        if (++slot == WST) {
          slot = 0;
          phase ^= 1u;
        }
        if (++c == op.C) {
          c = 0;
          ++t;
        }
      }
    }
    return;
  }

  if (warp == 1) {
    // ------------------------------------------------------- x producer
    if (lane == 0) {
      const uint32_t x_bytes = Cfg::GPS * 128 * p.M;
      pdl_wait();  // x is the previous kernel's output
      int slot = 0, issued = 0;
      uint32_t phase = 0;
      for (int o = 0; o < (OPS_MAX == 1 ? 1 : p.n_ops) && !*abort_flag; ++o) {
        const SkinnyOp& op = p.op[OPS_MAX == 1 ? 0 : o];
        prefetch_tensormap(&op.tm_x);
        // matmul o's x may be matmul o-1's y: wait until every CTA is done with it
        if (o > 0 && !wait_matmuls_done(p.gbar + (o - 1), (unsigned int)p.G, p.status)) {
          *abort_flag = 1;
          break;
        }
        long long u0;
        const int nunits = units_of(o, &u0);
        int c = (int)(u0 % op.C);
        for (int j = 0; j < nunits; ++j, ++issued) {
          if (issued >= SST && !*abort_flag) {
            if (!mbar_wait(&sempty[slot], phase ^ 1u, p.status, kDevTimeoutEmpty)) *abort_flag = 1;
          }
          if (*abort_flag) break;
          mbar_arrive_expect_tx(&sfull[slot], x_bytes);
          tma_load_3d(sring + slot * Cfg::S_STAGE + Cfg::OFF_X, &op.tm_x, &sfull[slot], 0, 0, c * Cfg::GPS);
          if (++slot == SST) {
            slot = 0;
            phase ^= 1u;
          }
          if (++c == op.C) c = 0;
        }
      }
    }
    return;
  }

  if (warp < 2 + Cfg::HW) {
    // ------------------------------------------------------------- helpers
    const int h = warp - 2;
    pdl_wait();
    // COLS: the B blocks are zero outside the lanes of their own group's
    // column, for the whole launch; only those lanes are written per unit.
    if (Cfg::COLS) {
      for (int e = h * 32 + lane; e < SST * (Cfg::BF_BYTES / 16); e += Cfg::HW * 32)
        sts128(smem_u32(sring + (e / (Cfg::BF_BYTES / 16)) * Cfg::S_STAGE + Cfg::OFF_BF) +
                   (e % (Cfg::BF_BYTES / 16)) * 16,
               make_uint4(0u, 0u, 0u, 0u));
    }
    // (X, Z) of token columns >= M stay zero for the whole launch.
    for (int e = h * 32 + lane; e < SST * Cfg::GPS * Cfg::XZ_COLS; e += Cfg::HW * 32) {
      const int slot = e / (Cfg::GPS * Cfg::XZ_COLS);
      const int col = e % Cfg::XZ_COLS;
      if (col >= p.M) {
        const int gi = (e / Cfg::XZ_COLS) % Cfg::GPS;
        sts_f32x2(smem_u32(sring + slot * Cfg::S_STAGE + Cfg::OFF_XZ) + (gi * Cfg::XZ_COLS + col) * 8, 0.f, 0.f);
      }
    }
    int slot = 0;
    uint32_t phase = 0;
    for (int o = 0; o < (OPS_MAX == 1 ? 1 : p.n_ops); ++o) {
      long long u0;
      const int nunits = units_of(o, &u0);
      for (int j = 0; j < nunits; ++j) {
        if (!*abort_flag && !mbar_wait(&sfull[slot], phase, p.status, kDevTimeoutFull)) *abort_flag = 1;
        uint8_t* st = sring + slot * Cfg::S_STAGE;
        const uint32_t xbase = smem_u32(st + Cfg::OFF_X);
        const uint32_t bf = smem_u32(st + Cfg::OFF_BF);
        const uint32_t xz = smem_u32(st + Cfg::OFF_XZ);
        // task = ((gi * M + n) * 4 + s): lanes 4k..4k+3 share one (group, token)
        for (int base = h * 32; base < 4 * Cfg::GPS * p.M; base += Cfg::HW * 32) {
          const int task = base + lane;
          const int s = task & 3;
          const int gn = task >> 2;
          const int gi = MT == 1 ? gn : gn / p.M;
          const int n = MT == 1 ? 0 : gn - gi * p.M;
          const int line = gn;  // box layout [group][token][64 halves]
          if (BITS == 8) {
            // Byte codes: MMA block q of the group (k 16q..16q+15) takes, in
            // lane (token, s), x[16q + 4s .. 16q + 4s + 3] as its two B words,
            // unscaled; the four blocks' words are stored in q order.
            uint2 xb[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              xb[q] = lds64(xbase + line * 128 + (((2 * q + (s >> 1)) ^ (line & 7)) << 4) + 8 * (s & 1));
            const uint32_t fa = bf + gi * Cfg::BF_GROUP + (n * 4 + s) * 16;
            sts128(fa, make_uint4(xb[0].x, xb[0].y, xb[1].x, xb[1].y));
            sts128(fa + Cfg::BF_GROUP / 2, make_uint4(xb[2].x, xb[2].y, xb[3].x, xb[3].y));
            float xs = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&xb[q].x));
              const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&xb[q].y));
              xs += (f0.x + f0.y) + (f1.x + f1.y);
            }
            xs += __shfl_xor_sync(0xffffffffu, xs, 1);
            xs += __shfl_xor_sync(0xffffffffu, xs, 2);
            if (s == 0) sts_f32x2(xz + (gi * Cfg::XZ_COLS + n) * 8, xs, 1024.f * xs);
            continue;
          }
          const uint4 xv0 = lds128(xbase + line * 128 + ((s ^ (line & 7)) << 4));
          const uint4 xv1 = lds128(xbase + line * 128 + (((4 + s) ^ (line & 7)) << 4));
          // B fragment of MMA jj: (x[8s+jj], x[8s+jj+4]) and the same 32 further
          // on; odd jj scaled by 1/16 to match the in-place odd nibbles.
          uint4 f0, f1;
          f0.x = prmt(xv0.x, xv0.z, 0x5410);
          f0.y = prmt(xv1.x, xv1.z, 0x5410);
          f0.z = hmul2_rn(prmt(xv0.x, xv0.z, 0x7632), 0x2C002C00u);
          f0.w = hmul2_rn(prmt(xv1.x, xv1.z, 0x7632), 0x2C002C00u);
          f1.x = prmt(xv0.y, xv0.w, 0x5410);
          f1.y = prmt(xv1.y, xv1.w, 0x5410);
          f1.z = hmul2_rn(prmt(xv0.y, xv0.w, 0x7632), 0x2C002C00u);
          f1.w = hmul2_rn(prmt(xv1.y, xv1.w, 0x7632), 0x2C002C00u);
          if (Cfg::COLS) {
            // lane (row n + TPC (gi % GPC), column s) of group gi's block:
            // token n's column among the group's
            const int lr = n + Cfg::TPC * (gi % Cfg::GPC);
            sts128(bf + gi * 1024 + (lr * 4 + s) * 16, f0);
            sts128(bf + gi * 1024 + 512 + (lr * 4 + s) * 16, f1);
          } else {
            const uint32_t fa = bf + gi * Cfg::BF_GROUP + (n * 4 + s) * 16;
            sts128(fa, f0);
            sts128(fa + Cfg::BF_GROUP / 2, f1);
          }
          // sums over even and odd k of the 16 x values this lane holds
          float xe = 0.f, xo = 0.f;
          const uint32_t wv[8] = {xv0.x, xv0.y, xv0.z, xv0.w, xv1.x, xv1.y, xv1.z, xv1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[i]));
            xe += f.x;
            xo += f.y;
          }
          xe += __shfl_xor_sync(0xffffffffu, xe, 1);
          xo += __shfl_xor_sync(0xffffffffu, xo, 1);
          xe += __shfl_xor_sync(0xffffffffu, xe, 2);
          xo += __shfl_xor_sync(0xffffffffu, xo, 2);
          if (s == 0)
            sts_f32x2(xz + (gi * Cfg::XZ_COLS + n) * 8, xe + xo, 1024.f * xe + 64.f * xo);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready[slot]);
        if (++slot == SST) {
          slot = 0;
          phase ^= 1u;
        }
      }
    }
    return;
  }

  // ----------------------------------------------------------------- consumers
  const int cw = warp - 2 - Cfg::HW;
  // This warp's 16 rows of a tile: rows wrow..wrow+7 of each half (MMA rows
  // r and r + 8 of a lane are tile rows wrow + r and 64 + wrow + r), so in a
  // SwiGLU tile a lane holds a gate row and its up row.
  const int wrow = cw * 8;
  const int r = lane / 4, s4 = lane % 4;
  pdl_wait();
  // Row-parallel exchange: this call's epoch, read once the previous kernel
  // of the stream (the previous call's last CTA included) has completed;
  // kept in shared memory, not in registers across the main loop.
  if constexpr (XCHG) {
    if (cw == 0 && lane == 0) *xepoch = ar_next_epoch(p.ar);
    asm volatile("bar.sync 1, %0;" ::"r"(Cfg::CW * 32) : "memory");
  }

  float acc[NT][4];
#pragma unroll
  for (int q = 0; q < NT; ++q)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[q][e] = 0.f;
  // greedy-token keys of the logits this thread writes: tokens tt*8 + 2*s4 + j
  unsigned long long best[NT][2];
#pragma unroll
  for (int q = 0; q < NT; ++q) best[q][0] = best[q][1] = 0ull;

  // y (and the greedy-token keys) of this lane's outputs of row tile `tile`
  auto store_tile = [&](const SkinnyOp& op, int tile, const float (&v)[NT][4]) {
    if (op.swiglu) {
      const int row = tile * (Cfg::BN / 2) + wrow + r;  // gate in v[.][0..1], up in v[.][2..3]
#pragma unroll
      for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int n = tt * 8 + 2 * s4 + j;
          if (n < p.M && row < op.N && op.y) {
            const float h = swiglu_f16(v[tt][j], v[tt][j + 2]);
            const size_t idx = (size_t)n * op.N + row;
            if (op.y_f32) reinterpret_cast<float*>(op.y)[idx] = h;
            else reinterpret_cast<__half*>(op.y)[idx] = __float2half_rn(h);
          }
        }
      return;
    }
    // row-parallel exchange: this rank's fp32 products go, each with the
    // call's epoch, into ll slot (parity, rank) of every rank
    const unsigned int xe = XCHG ? *xepoch : 0u;
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int n = tt * 8 + 2 * s4 + (e & 1);
        const int row = tile * Cfg::BN + wrow + r + ((e & 2) ? Cfg::BN / 2 : 0);
        if (n < p.M && row < op.N) {
          const size_t idx = (size_t)n * op.N + row;
          if (XCHG) {
            for (int q = 0; q < p.ar.P; ++q)
              ar_ll_store(ar_ll_slot(p.ar, q, (int)(xe & 1u), p.ar.rank) + idx, v[tt][e], xe);
          } else if (!op.y) {
          } else if (op.y_f32) reinterpret_cast<float*>(op.y)[idx] = v[tt][e];
          else reinterpret_cast<__half*>(op.y)[idx] = __float2half_rn(v[tt][e]);
          if (p.amax) best[tt][e & 1] = umax64(best[tt][e & 1], amax_key(v[tt][e], row));
        }
      }
  };

  // ldmatrix lane addressing: matrix mi = lane/8 covers rows 8*(mi&1).. of
  // chunk (mi>>1) of the group; per-lane offsets (groups 0-3 of box 0; box 1
  // adds W_BOX) hoisted out of the loop.
  const int lm_mi = lane / 8;
  const int lm_row = wrow + (lane % 8) + (Cfg::BN / 2) * (lm_mi & 1);
  const int lm_sw = lm_row & 7;
  uint32_t lm_off[4];
#pragma unroll
  for (int g4 = 0; g4 < 4; ++g4) lm_off[g4] = lm_row * 128 + (((g4 * 2 + (lm_mi >> 1)) ^ lm_sw) << 4);
  // scale/bias rows of MMA rows r and r+8 of this warp, all 8 groups (16 bytes each)
  const uint32_t sb_off = (wrow + r) * 2 * Cfg::GPS;
  constexpr uint32_t kSbHi = (Cfg::BN / 2) * 2 * Cfg::GPS;
  // B fragments: a lane whose token column is >= M reads token M-1's (a
  // shared-memory broadcast).  MMA output columns depend only on their own B
  // column, so those columns are never mixed into a written result.
  uint32_t bf_off[NT];
#pragma unroll
  for (int tt = 0; tt < NT; ++tt) {
    const int tok = (tt * 8 + r) < p.M ? (tt * 8 + r) : (p.M - 1);
    bf_off[tt] = Cfg::OFF_BF + (tok * 4 + s4) * 16;
  }
  const uint32_t xz_off = Cfg::OFF_XZ + 2 * s4 * 8;
  const uint32_t wring_u = smem_u32(wring);

  int wslot = 0, sslot = 0;
  uint32_t wphase = 0, sphase = 0;
  // units of every matmul this CTA takes, in ring order
  int total = 0;
  for (int o = 0; o < (OPS_MAX == 1 ? 1 : p.n_ops); ++o) {
    long long u0;
    total += units_of(o, &u0);
  }
  int done = 0;

  // This warp's share of a unit's weights, scales and biases lives in
  // registers: A (ldmatrix fragments of 8 groups) and the rows' scale/bias
  // words.  The next unit's fragments (of this matmul or the next) are loaded
  // group by group while a unit is computed (A[gi] is free once group gi has
  // been expanded), so the weight slot goes back to the producer one unit
  // earlier and the shared-memory latency of the copy is hidden behind the
  // MMAs.  (With 16 tokens the register file has no room for this overlap:
  // those warps copy each unit's share when they start it.)
  //
  // 8-bit codes take twice the registers per unit, so their warps hold two
  // groups at a time instead: a group is two ldmatrix.x4 loads (64 bytes of
  // each of 16 rows; load li of the unit covers 16-byte chunks 2(li % 4) and
  // 2(li % 4) + 1 of box li / 4), group gi + 1 is loaded while group gi is
  // computed, and the slot is released once the last group's loads are
  // issued.
  constexpr bool kRoll = BITS == 4 && MT <= 8;
  uint32_t A[BITS == 8 ? 4 : Cfg::GPS][4];
  uint4 sv_lo, sv_hi, bv_lo, bv_hi;
  uint32_t wb_cur = 0;  // 8-bit: the slot of the unit being computed
  auto release_wslot = [&]() {
    __syncwarp();
    if (lane == 0) mbar_arrive(&wempty[wslot]);
    if (++wslot == WST) {
      wslot = 0;
      wphase ^= 1u;
    }
  };
  // Scales and biases of this lane's rows: all 8 groups (16 bytes a row), or
  // for one token the two groups 2 s4, 2 s4 + 1 of its MMA columns (4 bytes).
  auto load_sb = [&](uint32_t wb) {
    if (Cfg::COLS && Cfg::TPC == 1) {
      // word q (q < GPS / 8) of each: groups 8 q + 2 s4 and 8 q + 2 s4 + 1
      sv_lo.x = lds32(wb + Cfg::OFF_WS + sb_off + 4 * s4);
      sv_hi.x = lds32(wb + Cfg::OFF_WS + sb_off + kSbHi + 4 * s4);
      bv_lo.x = lds32(wb + Cfg::OFF_WB + sb_off + 4 * s4);
      bv_hi.x = lds32(wb + Cfg::OFF_WB + sb_off + kSbHi + 4 * s4);
      if (Cfg::GPS > 8) {
        sv_lo.y = lds32(wb + Cfg::OFF_WS + sb_off + 16 + 4 * s4);
        sv_hi.y = lds32(wb + Cfg::OFF_WS + sb_off + kSbHi + 16 + 4 * s4);
        bv_lo.y = lds32(wb + Cfg::OFF_WB + sb_off + 16 + 4 * s4);
        bv_hi.y = lds32(wb + Cfg::OFF_WB + sb_off + kSbHi + 16 + 4 * s4);
      }
    } else {
      sv_lo = lds128(wb + Cfg::OFF_WS + sb_off);
      sv_hi = lds128(wb + Cfg::OFF_WS + sb_off + kSbHi);
      bv_lo = lds128(wb + Cfg::OFF_WB + sb_off);
      bv_hi = lds128(wb + Cfg::OFF_WB + sb_off + kSbHi);
    }
  };
  auto copy_unit = [&]() {
    if (!*abort_flag && !mbar_wait(&wfull[wslot], wphase, p.status, kDevTimeoutFull)) *abort_flag = 1;
    const uint32_t wb = wring_u + wslot * Cfg::W_STAGE;
    if (BITS == 8) {
      wb_cur = wb;
#pragma unroll
      for (int li = 0; li < 2; ++li)  // group 0
        ldmatrix_x4(wb + lm_off[li], A[li][0], A[li][1], A[li][2], A[li][3]);
    } else {
#pragma unroll
      for (int gi = 0; gi < Cfg::GPS; ++gi)
        ldmatrix_x4(wb + (gi / 4) * Cfg::W_BOX + lm_off[gi % 4], A[gi][0], A[gi][1], A[gi][2], A[gi][3]);
    }
    load_sb(wb);
    if (BITS != 8) release_wslot();
  };
  if (total > 0) copy_unit();

  for (int o = 0; o < (OPS_MAX == 1 ? 1 : p.n_ops); ++o) {
    const SkinnyOp& op = p.op[OPS_MAX == 1 ? 0 : o];
    long long u0;
    const int nunits = units_of(o, &u0);
    const int first_tile = (int)(u0 / op.C);
    int t = first_tile, c = (int)(u0 % op.C);
    int seg_begin = c;
    for (int j = 0; j < nunits; ++j, ++done) {
      if (!kRoll && done > 0) copy_unit();
      const bool has_next = kRoll && done + 1 < total;
      const uint32_t wb_next = wring_u + wslot * Cfg::W_STAGE;
      // compute against the unit's x fragments, refilling A with the next unit
      if (!*abort_flag && !mbar_wait(&ready[sslot], sphase, p.status, kDevTimeoutFull)) *abort_flag = 1;
      if constexpr (Cfg::COLS) {
        // 4-bit codes, one to four tokens.  MMA column c of group gi is token
        // c % TPC of group gi - gi % GPC + c / TPC: group gi's B block is x's
        // fragment in the lanes of its TPC columns and zero in the others, so
        // one accumulator pair collects GPC groups, each in its own columns
        // (d = 1024 X_even + 64 X_odd + sum_k x_k q_k of that group and
        // token), and the fold runs once per GPC groups.  Lane (r, s4) folds
        // columns 2 s4 and 2 s4 + 1 of rows r and r + 8; the lanes of a row
        // that hold the same tokens are summed when the row's segment ends.
        const uint32_t stu = smem_u32(sring + sslot * Cfg::S_STAGE);
        float dA[4] = {0.f, 0.f, 0.f, 0.f}, dB[4] = {0.f, 0.f, 0.f, 0.f};  // set by each chain's first MMAs
        auto b_addr = [&](int g) { return stu + Cfg::OFF_BF + g * 1024 + lane * 16; };
        // The next unit's fragments are copied in the unit's second half
        // (groups 0-7 of the next unit while groups 4-7 of this one compute),
        // so its data has the longest time to land before the wait.
        auto roll = [&](int g) {
          ldmatrix_x4(wb_next + (g / 4) * Cfg::W_BOX + lm_off[g % 4], A[g][0], A[g][1], A[g][2], A[g][3]);
        };
        auto word = [](const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; };
        // fold of the chain ending at group block q: y += s (d - Z) + b X
        auto fold = [&](int q) {
          // (X, Z) of this lane's two columns: entries 8 q + 2 s4 and 8 q + 2 s4 + 1
          const float4 v =
              *reinterpret_cast<const float4*>(sring + sslot * Cfg::S_STAGE + Cfg::OFF_XZ + (q * 8 + 2 * s4) * 8);
          if constexpr (Cfg::TPC == 1) {
            // one token: the columns are groups 8 q + 2 s4 and 8 q + 2 s4 + 1
            const uint32_t sl = word(sv_lo, q), sh = word(sv_hi, q), bl = word(bv_lo, q), bh = word(bv_hi, q);
            acc[0][0] = fmaf(half_lo(sl), (dA[0] + dB[0]) - v.y, fmaf(half_lo(bl), v.x, acc[0][0]));
            acc[0][0] = fmaf(half_hi(sl), (dA[1] + dB[1]) - v.w, fmaf(half_hi(bl), v.z, acc[0][0]));
            acc[0][2] = fmaf(half_lo(sh), (dA[2] + dB[2]) - v.y, fmaf(half_lo(bh), v.x, acc[0][2]));
            acc[0][2] = fmaf(half_hi(sh), (dA[3] + dB[3]) - v.w, fmaf(half_hi(bh), v.z, acc[0][2]));
          } else {
            // both columns belong to group GPC q + s4 / 2 (word q of the row's scales)
            const bool hi = (s4 & 2) != 0;
            const float s_r = hi ? half_hi(word(sv_lo, q)) : half_lo(word(sv_lo, q));
            const float s_r8 = hi ? half_hi(word(sv_hi, q)) : half_lo(word(sv_hi, q));
            const float b_r = hi ? half_hi(word(bv_lo, q)) : half_lo(word(bv_lo, q));
            const float b_r8 = hi ? half_hi(word(bv_hi, q)) : half_lo(word(bv_hi, q));
            acc[0][0] = fmaf(s_r, (dA[0] + dB[0]) - v.y, fmaf(b_r, v.x, acc[0][0]));
            acc[0][1] = fmaf(s_r, (dA[1] + dB[1]) - v.w, fmaf(b_r, v.z, acc[0][1]));
            acc[0][2] = fmaf(s_r8, (dA[2] + dB[2]) - v.y, fmaf(b_r8, v.x, acc[0][2]));
            acc[0][3] = fmaf(s_r8, (dA[3] + dB[3]) - v.w, fmaf(b_r8, v.z, acc[0][3]));
          }
        };
#pragma unroll
        for (int gi = 0; gi < Cfg::GPS; ++gi) {
          const uint4 b0 = lds128(b_addr(gi));
          const uint4 b1 = lds128(b_addr(gi) + 512);
          uint32_t e[4][4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t w8 = A[gi][i] >> 8;
            e[0][i] = lop3_and_or(A[gi][i], 0x000F000Fu);
            e[1][i] = lop3_and_or(A[gi][i], 0x00F000F0u);
            e[2][i] = lop3_and_or(w8, 0x000F000Fu);
            e[3][i] = lop3_and_or(w8, 0x00F000F0u);
          }
          if (gi % Cfg::GPC == 0) {
            mma_16816_zc(dA, e[0][0], e[0][1], e[0][2], e[0][3], b0.x, b0.y);
            mma_16816_zc(dB, e[1][0], e[1][1], e[1][2], e[1][3], b0.z, b0.w);
          } else {
            mma_16816(dA, e[0][0], e[0][1], e[0][2], e[0][3], b0.x, b0.y);
            mma_16816(dB, e[1][0], e[1][1], e[1][2], e[1][3], b0.z, b0.w);
          }
          mma_16816(dA, e[2][0], e[2][1], e[2][2], e[2][3], b1.x, b1.y);
          mma_16816(dB, e[3][0], e[3][1], e[3][2], e[3][3], b1.z, b1.w);
          if (has_next && gi >= Cfg::GPS / 2) {
            // A[0..gi] are expanded: groups 2 (gi - GPS/2) and 2 (gi - GPS/2) + 1 are free
            if (gi == Cfg::GPS / 2 && !*abort_flag &&
                !mbar_wait(&wfull[wslot], wphase, p.status, kDevTimeoutFull))
              *abort_flag = 1;
            roll(2 * (gi - Cfg::GPS / 2));
            roll(2 * (gi - Cfg::GPS / 2) + 1);
          }
          if (gi % Cfg::GPC == Cfg::GPC - 1) fold(gi / Cfg::GPC);
        }
      } else {
        const uint8_t* stp = sring + sslot * Cfg::S_STAGE;
        const uint32_t svl[4] = {sv_lo.x, sv_lo.y, sv_lo.z, sv_lo.w}, svh[4] = {sv_hi.x, sv_hi.y, sv_hi.z, sv_hi.w};
        const uint32_t bvl[4] = {bv_lo.x, bv_lo.y, bv_lo.z, bv_lo.w}, bvh[4] = {bv_hi.x, bv_hi.y, bv_hi.z, bv_hi.w};
#pragma unroll
        for (int gi = 0; gi < 8; ++gi) {
          uint4 b0[NT], b1[NT];
#pragma unroll
          for (int tt = 0; tt < NT; ++tt) {
            const uint8_t* fb = stp + bf_off[tt] + gi * Cfg::BF_GROUP;
            b0[tt] = *reinterpret_cast<const uint4*>(fb);
            b1[tt] = *reinterpret_cast<const uint4*>(fb + Cfg::BF_GROUP / 2);
          }
          // expanded A registers: e[jj][i] for word i
          uint32_t e[4][4];
          if (BITS == 8) {
            // Byte codes: word d of a lane holds codes 4s4..4s4+3 of its
            // 16-byte chunk; prmt pairs bytes with 0x64 into the exact fp16
            // values 1024 + q.  MMA block q (k 16q..16q+15 of the group) is
            // chunk q of the group: the group's load q/2, words (0, 1) or
            // (2, 3) for the low and high row halves.
            const int ab = (gi & 1) * 2;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t lo = A[ab + q / 2][(q & 1) * 2], hi = A[ab + q / 2][(q & 1) * 2 + 1];
              e[q][0] = prmt(lo, 0x64646464u, 0x5140u);
              e[q][1] = prmt(hi, 0x64646464u, 0x5140u);
              e[q][2] = prmt(lo, 0x64646464u, 0x5342u);
              e[q][3] = prmt(hi, 0x64646464u, 0x5342u);
            }
            if (gi + 1 < 8) {
              const int nb = ((gi + 1) & 1) * 2;
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int li = 2 * (gi + 1) + j;
                ldmatrix_x4(wb_cur + (li / 4) * Cfg::W_BOX + lm_off[li % 4], A[nb + j][0], A[nb + j][1],
                            A[nb + j][2], A[nb + j][3]);
              }
              if (gi + 1 == 7) release_wslot();  // every load of the unit is issued
            }
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t w8 = A[gi][i] >> 8;
              e[0][i] = lop3_and_or(A[gi][i], 0x000F000Fu);
              e[1][i] = lop3_and_or(A[gi][i], 0x00F000F0u);
              e[2][i] = lop3_and_or(w8, 0x000F000Fu);
              e[3][i] = lop3_and_or(w8, 0x00F000F0u);
            }
          }
          if (has_next) {
            if (gi == 0 && !*abort_flag && !mbar_wait(&wfull[wslot], wphase, p.status, kDevTimeoutFull))
              *abort_flag = 1;
            ldmatrix_x4(wb_next + (gi / 4) * Cfg::W_BOX + lm_off[gi % 4], A[gi][0], A[gi][1], A[gi][2], A[gi][3]);
          }
          float dA[NT][4], dB[NT][4];
#pragma unroll
          for (int tt = 0; tt < NT; ++tt) {
            mma_16816_zc(dA[tt], e[0][0], e[0][1], e[0][2], e[0][3], b0[tt].x, b0[tt].y);
            mma_16816_zc(dB[tt], e[1][0], e[1][1], e[1][2], e[1][3], b0[tt].z, b0[tt].w);
            mma_16816(dA[tt], e[2][0], e[2][1], e[2][2], e[2][3], b1[tt].x, b1[tt].y);
            mma_16816(dB[tt], e[3][0], e[3][1], e[3][2], e[3][3], b1[tt].z, b1[tt].w);
          }
          // fold the group: y += s * (d - Z) + b * X
          const float s_r = (gi & 1) ? half_hi(svl[gi / 2]) : half_lo(svl[gi / 2]);
          const float s_r8 = (gi & 1) ? half_hi(svh[gi / 2]) : half_lo(svh[gi / 2]);
          const float b_r = (gi & 1) ? half_hi(bvl[gi / 2]) : half_lo(bvl[gi / 2]);
          const float b_r8 = (gi & 1) ? half_hi(bvh[gi / 2]) : half_lo(bvh[gi / 2]);
#pragma unroll
          for (int tt = 0; tt < NT; ++tt) {
            const float4 v =
                *reinterpret_cast<const float4*>(stp + xz_off + (gi * Cfg::XZ_COLS + tt * 8) * 8);  // X0, Z0, X1, Z1
            acc[tt][0] = fmaf(s_r, (dA[tt][0] + dB[tt][0]) - v.y, fmaf(b_r, v.x, acc[tt][0]));
            acc[tt][2] = fmaf(s_r8, (dA[tt][2] + dB[tt][2]) - v.y, fmaf(b_r8, v.x, acc[tt][2]));
            if (MT > 1) {  // a single token uses column 0 only
              acc[tt][1] = fmaf(s_r, (dA[tt][1] + dB[tt][1]) - v.w, fmaf(b_r, v.z, acc[tt][1]));
              acc[tt][3] = fmaf(s_r8, (dA[tt][3] + dB[tt][3]) - v.w, fmaf(b_r8, v.z, acc[tt][3]));
            }
          }
        }
      }
      if (has_next) {
        load_sb(wb_next);
        release_wslot();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[sslot]);

      const bool seg_end = (c == op.C - 1) || (j == nunits - 1);
      const int t_done = t;
      if (++sslot == SST) {
        sslot = 0;
        sphase ^= 1u;
      }
      if (++c == op.C) {
        c = 0;
        ++t;
      }
      if (!seg_end) continue;
      if constexpr (Cfg::COLS) {
        // a row's groups were folded in the lanes that hold the same tokens:
        // every one of them gets the sum
        if constexpr (Cfg::TPC == 1) {
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            acc[0][e] += __shfl_xor_sync(0xffffffffu, acc[0][e], 1);
            acc[0][e] += __shfl_xor_sync(0xffffffffu, acc[0][e], 2);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[0][e] += __shfl_xor_sync(0xffffffffu, acc[0][e], 2);
        }
      }
      const bool whole = (seg_begin == 0) && (c == 0);

      if (p.split > 1) {
        // Cluster split-K: this CTA's only segment.  Non-leaders store their
        // partial into the leader's shared memory and arrive on its barrier;
        // the leader adds them in rank order and writes y.
        uint32_t rank;
        asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
        const uint32_t recv = smem_u32(smem + Cfg::OFF_RECV);
        if (rank != 0) {
          {
            const uint32_t lrecv = recv + (rank - 1) * (Cfg::BN * Cfg::MPAD * 4);
            uint32_t rrecv;
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(rrecv) : "r"(lrecv));
#pragma unroll
            for (int tt = 0; tt < NT; ++tt)
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int rl = wrow + r + (Cfg::BN / 2) * hh;
                const uint32_t a = rrecv + (rl * Cfg::MPAD + tt * 8 + 2 * s4) * 4;
                asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(acc[tt][2 * hh]),
                             "f"(acc[tt][2 * hh + 1])
                             : "memory");
              }
          }
          __syncwarp();
          if (lane == 0) {
            uint32_t rbar;
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(rbar) : "r"(smem_u32(recv_bar)));
            asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(rbar) : "memory");
          }
        } else {
          if (!*abort_flag && !mbar_wait(recv_bar, 0, p.status, kDevTimeoutAccum)) *abort_flag = 1;
          asm volatile("fence.acq_rel.cluster;" ::: "memory");
          if (!*abort_flag) {
            for (int q = 1; q < p.split; ++q) {
              const uint32_t lrecv = recv + (q - 1) * (Cfg::BN * Cfg::MPAD * 4);
#pragma unroll
              for (int tt = 0; tt < NT; ++tt)
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                  const int rl = wrow + r + (Cfg::BN / 2) * hh;
                  float2 v;
                  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];"
                               : "=f"(v.x), "=f"(v.y)
                               : "r"(lrecv + (rl * Cfg::MPAD + tt * 8 + 2 * s4) * 4));
                  acc[tt][2 * hh] += v.x;
                  acc[tt][2 * hh + 1] += v.y;
                }
            }
            store_tile(op, t_done, acc);
          }
        }
      } else if (whole) {
        if (!*abort_flag) store_tile(op, t_done, acc);
      } else {
        // Split tile: publish this CTA's partial; the last contributor to
        // arrive adds the partials in CTA order.  A segment that is not this
        // CTA's final one does not wait for its arrival's result: thread 0
        // (consumer warp 0) fences and arrives while the other warps go on
        // consuming, and a tile found complete there is finished after the
        // final segment.
        const int slot_idx = (t_done == first_tile) ? 0 : 1;
        float* mine = p.part + ((size_t)blockIdx.x * 2 + slot_idx) * Cfg::PART;
        {
#pragma unroll
          for (int tt = 0; tt < NT; ++tt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int n = tt * 8 + 2 * s4 + (e & 1);
              const int rl = wrow + r + ((e & 2) ? Cfg::BN / 2 : 0);
              mine[rl * Cfg::MPAD + n] = acc[tt][e];
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(Cfg::CW * 32) : "memory");
        if (cw == 0 && lane == 0) {
          // One release fence for the whole CTA's partial (ordered before it by
          // the barrier), then the arrival; the last arrival acquires.
          const long long tu0 = (long long)t_done * op.C;
          const unsigned int ncontrib =
              (unsigned int)(cta_of_unit(tu0 + op.C - 1, op.U, op.G) - cta_of_unit(tu0, op.U, op.G) + 1);
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          const unsigned int old = atomicAdd(&p.counter[t_done], 1u);
          if (old == ncontrib - 1) {
            atomicExch(&p.counter[t_done], 0u);
            asm volatile("fence.acq_rel.gpu;" ::: "memory");
            fin_flag[slot_idx] = t_done + 1;  // finish tile t_done after the final segment
          }
        }
      }
      if (j == nunits - 1) {
        // Final segment: finish the split tiles this CTA completed.
        asm volatile("bar.sync 1, %0;" ::"r"(Cfg::CW * 32) : "memory");
#pragma unroll 1
        for (int q = 0; q < 2; ++q) {
          const int tf = fin_flag[q] - 1;
          if (tf < 0) continue;
          const long long tu0 = (long long)tf * op.C;
          const int i_first = cta_of_unit(tu0, op.U, op.G);
          const int i_last = cta_of_unit(tu0 + op.C - 1, op.U, op.G);
          float tot[NT][4];
#pragma unroll
          for (int tt = 0; tt < NT; ++tt)
#pragma unroll
            for (int e = 0; e < 4; ++e) tot[tt][e] = 0.f;
          for (int i = i_first; i <= i_last; ++i) {
            const int ft = (int)(unit_begin(i, op.U, op.G) / op.C);
            const float* src = p.part + ((size_t)i * 2 + (tf == ft ? 0 : 1)) * Cfg::PART;
#pragma unroll
            for (int tt = 0; tt < NT; ++tt)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int n = tt * 8 + 2 * s4 + (e & 1);
                const int rl = wrow + r + ((e & 2) ? Cfg::BN / 2 : 0);
                tot[tt][e] += __ldcg(src + rl * Cfg::MPAD + n);
              }
          }
          if (!*abort_flag) store_tile(op, tf, tot);
        }
      }
      // fin_flag and the partial slots are rewritten only after this barrier
      asm volatile("bar.sync 1, %0;" ::"r"(Cfg::CW * 32) : "memory");
#pragma unroll
      for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[tt][e] = 0.f;
      seg_begin = 0;
    }
    if (OPS_MAX > 1 && p.n_ops > 1) {
      // Matmul o is done here (y tiles, partials, finished split tiles):
      // count this CTA in the grid-wide tally the next matmul's x waits on.
      asm volatile("bar.sync 1, %0;" ::"r"(Cfg::CW * 32) : "memory");
      if (cw == 0 && lane == 0) {
        fin_flag[0] = 0;
        fin_flag[1] = 0;
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        atomicAdd(p.gbar + o, 1u);
      }
      asm volatile("bar.sync 1, %0;" ::"r"(Cfg::CW * 32) : "memory");
    }
  }
  if constexpr (XCHG) {
    // Row-parallel exchange.  A worker CTA (blockIdx < op.G) stored every
    // value it finished, with the call's epoch, into every rank's ll slot
    // as it wrote its tiles; it exits without waiting, so its SM is free for
    // the next kernel's weight stream.  The grid's last F CTAs are
    // finishers with no units: finisher f reads the rows of tiles
    // [f T / F, (f + 1) T / F) of every token from every rank's slot in this
    // rank's buffer,
    // waiting (bounded) on each word until it carries the epoch, and sums
    // them in rank order into y (every rank gets identical y).  Workers
    // never wait on finishers, so the grid completes whether or not the
    // finishers are resident from the start.
    const SkinnyOp& op = p.op[0];
    const unsigned int xe = *xepoch;
    if ((int)blockIdx.x >= op.G) {
      const int xpar = (int)(xe & 1u);
      const int F = (int)gridDim.x - op.G, f = (int)blockIdx.x - op.G;
      const int t0 = (int)((long long)f * op.T / F), t1 = (int)((long long)(f + 1) * op.T / F);
      const int R = (t1 - t0) * Cfg::BN;  // rows [t0 BN, t1 BN) of a token are contiguous
      const unsigned long long* slots = ar_ll_slot(p.ar, p.ar.rank, xpar, 0);
      if ((op.N & 1) == 0 && (reinterpret_cast<uintptr_t>(op.y) & (op.y_f32 ? 7u : 3u)) == 0) {
        // pairs of outputs (R and N even: a pair never straddles a token;
        // y aligned for the pair's store)
        for (int q = 2 * (cw * 32 + lane); q < p.M * R; q += 2 * Cfg::CW * 32) {
          const int n = q / R;
          const int row = t0 * Cfg::BN + q % R;
          if (row >= op.N) continue;
          const size_t idx = (size_t)n * op.N + row;
          float s0, s1;
          if (!ar_ll_sum2(p.ar, slots + idx, p.ar.n_ll, xe, &s0, &s1)) break;
          if (op.y_f32) {
            *reinterpret_cast<float2*>(reinterpret_cast<float*>(op.y) + idx) = make_float2(s0, s1);
          } else {
            *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(op.y) + idx) = __floats2half2_rn(s0, s1);
          }
        }
      } else {
        bool ok = true;
        for (int q = cw * 32 + lane; q < p.M * R && ok; q += Cfg::CW * 32) {
          const int n = q / R;
          const int row = t0 * Cfg::BN + q % R;
          if (row >= op.N) continue;
          const size_t idx = (size_t)n * op.N + row;
          float sum = 0.f;
          for (int rr = 0; rr < p.ar.P && ok; ++rr) {
            float v = 0.f;
            ok = ar_ll_load(p.ar, slots + (size_t)rr * p.ar.n_ll + idx, xe, &v);
            sum += v;
          }
          if (!ok) break;
          if (op.y_f32) reinterpret_cast<float*>(op.y)[idx] = sum;
          else reinterpret_cast<__half*>(op.y)[idx] = __float2half_rn(sum);
        }
      }
    }
    if (cw == 0 && lane == 0) ar_count_done(p.ar, xe);
  }
  if (p.amax) {
    // Greedy token: reduce the keys over the warp (lanes of one s4 share
    // tokens), then over the consumer warps through shared memory (the
    // cluster receive buffer is idle by now), then one atomicMax per token.
    unsigned long long* red = reinterpret_cast<unsigned long long*>(smem + Cfg::OFF_RECV);
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        unsigned long long v = best[tt][j];
#pragma unroll
        for (int o2 = 4; o2 < 32; o2 <<= 1) v = umax64(v, __shfl_xor_sync(0xffffffffu, v, o2));
        if (r == 0) red[cw * Cfg::MPAD + tt * 8 + 2 * s4 + j] = v;
      }
    asm volatile("bar.sync 1, %0;" ::"r"(Cfg::CW * 32) : "memory");
    const int tid = cw * 32 + lane;
    if (tid < p.M) {
      unsigned long long v = 0ull;
      for (int q = 0; q < Cfg::CW; ++q) v = umax64(v, red[q * Cfg::MPAD + tid]);
      if (!*abort_flag && v != 0ull) atomicMax(p.amax + tid, v);
    }
  }
}

// Scratch layout: the chain's grid-barrier word, the split-tile counters
// (zero between launches, whatever grid the previous launch used), then the
// partial slots, which need no initialisation.
constexpr size_t kGbarBytes = 256;
static_assert(kSkinnyChainMax * sizeof(unsigned int) <= kGbarBytes, "per-matmul tallies fit");

// One matmul's descriptor: tensor maps and schedule-independent sizes.
template <int MT, int BITS, bool WIDE>
bool make_op(const SkinnyArgs& a, SkinnyOp* op, std::string* err) {
  using Cfg = SkinnyCfg<MT, BITS, WIDE>;
  op->N = (int)a.N;
  op->K = (int)a.K;
  op->C = (int)((a.K + Cfg::CK - 1) / Cfg::CK);
  // a SwiGLU tile holds 64 output rows (64 gate + 64 up weight rows)
  const int tile_rows = a.swiglu ? Cfg::BN / 2 : Cfg::BN;
  op->T = (int)((a.N + tile_rows - 1) / tile_rows);
  op->U = (long long)op->T * op->C;
  op->gsh = a.group_size / kGroup;
  op->sb_tma = (a.K % Cfg::CK == 0 && op->gsh == 1) ? 1 : 0;
  op->y_f32 = a.y_f32 ? 1 : 0;
  op->swiglu = a.swiglu ? 1 : 0;
  op->y = a.y;
  op->scales = reinterpret_cast<const __half*>(a.scales);
  op->biases = reinterpret_cast<const __half*>(a.biases);
  op->scales2 = reinterpret_cast<const __half*>(a.swiglu ? a.scales2 : a.scales);
  op->biases2 = reinterpret_cast<const __half*>(a.swiglu ? a.biases2 : a.biases);
  if ((size_t)op->T > kMaxCounters) {
    *err = "too many row tiles for the skinny path's counter block";
    return false;
  }
  const uint64_t row_bytes = (uint64_t)a.K * BITS / 8;
  if (!encode_tmap_2d(&op->tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, row_bytes, (uint64_t)a.N, row_bytes, 128,
                      tile_rows, CU_TENSOR_MAP_SWIZZLE_128B, err))
    return false;
  if (a.swiglu) {
    if (!encode_tmap_2d(&op->tm_w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w2, row_bytes, (uint64_t)a.N, row_bytes, 128,
                        tile_rows, CU_TENSOR_MAP_SWIZZLE_128B, err))
      return false;
  } else {
    op->tm_w2 = op->tm_w;  // unused
  }
  {
    // x viewed as [K/64 groups][M tokens][64 halves]: one box = 8 groups x M tokens
    const uint64_t dims[3] = {(uint64_t)kGroup, (uint64_t)a.M, (uint64_t)(a.K / kGroup)};
    const uint64_t strides[2] = {(uint64_t)(a.x_ld ? a.x_ld : a.K) * 2, (uint64_t)kGroup * 2};
    const uint32_t box[3] = {(uint32_t)kGroup, (uint32_t)a.M, (uint32_t)Cfg::GPS};
    if (!encode_tmap_3d(&op->tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, err))
      return false;
  }
  op->tm_s = op->tm_b = op->tm_s2 = op->tm_b2 = op->tm_w;  // unused unless encoded below
  if (op->sb_tma) {
    const uint64_t G64 = (uint64_t)(a.K / kGroup);
    const void* srcs[4] = {a.scales, a.biases, a.scales2, a.biases2};
    CUtensorMap* maps[4] = {&op->tm_s, &op->tm_b, &op->tm_s2, &op->tm_b2};
    for (int i = 0; i < (a.swiglu ? 4 : 2); ++i)
      if (!encode_tmap_2d(maps[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, srcs[i], G64, (uint64_t)a.N, G64 * 2,
                          Cfg::GPS, tile_rows, CU_TENSOR_MAP_SWIZZLE_NONE, err))
        return false;
  }
  return true;
}

template <int MT, int OPS_MAX, int BITS, bool WIDE, bool XCHG>
cudaError_t set_smem_attr(int dev) {
  static thread_local int configured_dev = -1;
  // cudaFuncSetAttribute is per device; cheap enough to repeat on change.
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(qmm_skinny_kernel<MT, OPS_MAX, BITS, WIDE, XCHG>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SkinnyCfg<MT, BITS, WIDE>::SMEM);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  return cudaSuccess;
}

// Schedule of one matmul: with fewer row tiles than SMs, each tile gets
// `split` CTAs (a thread-block cluster reducing through distributed shared
// memory; one CTA per tile when split == 1).  Otherwise stream-K over all
// SMs.  With 16 tokens (clusters of at most 2) stream-K also takes the
// small-T shapes where it gives the busiest CTA fewer units: 5120 x 17408
// runs in 32.3 us instead of 43.2 (17 chunks per CTA in pairs, 10 units
// under stream-K).  With up to 8 tokens clusters of 3-4 stayed faster even
// where stream-K's busiest CTA has fewer units (5120 x 17408 at M=1: 17.0 us
// in clusters of 3, 19.0 us under stream-K).
struct SkinnyPlan {
  long long G;        // CTAs
  int split;          // CTAs per tile (1: stream-K, or one CTA per tile)
  long long busiest;  // units of the busiest CTA
};

template <int MT, int BITS, bool WIDE>
SkinnyPlan plan_cfg(const SkinnyArgs& a, int sm_count) {
  using Cfg = SkinnyCfg<MT, BITS, WIDE>;
  const long long tile_rows = a.swiglu ? Cfg::BN / 2 : Cfg::BN;
  const long long T = (a.N + tile_rows - 1) / tile_rows;
  const long long C = (a.K + Cfg::CK - 1) / Cfg::CK;
  const long long U = T * C;
  SkinnyPlan pl{sm_count, 1, 0};
  if (a.max_ctas > 0 && pl.G > a.max_ctas) pl.G = a.max_ctas;
  if (T <= pl.G) {
    long long split = pl.G / T;
    if (split > Cfg::SPLIT_MAX) split = Cfg::SPLIT_MAX;
    if (split > C) split = C;
    if (split < 1) split = 1;
    const long long cluster_span = (C + split - 1) / split;  // chunks of the busiest CTA
    const long long sk_span = (U + pl.G - 1) / pl.G;          // units of the busiest stream-K CTA
    if (MT < 16 || sk_span >= cluster_span) {
      pl.split = (int)split;
      pl.G = T * split;
    }
  }
  if (pl.split == 1 && T > pl.G) {
    // Whole tiles per CTA where that gives the busiest CTA at most 10% more
    // units: no split tiles, so no partial sums, counters or end-of-launch
    // fix-ups.  The fused SwiGLU gate|up (272 tiles, 2 on each of 136 CTAs)
    // went from 25.5 to 21.4 us at one token (10 units a CTA either way),
    // from 28.9 to 25.4 at four and from 45.9 to 43.3 at sixteen (20 units
    // against 19 under stream-K); the one-token 64-layer stack from 3.69 to
    // 3.47 ms.
    const long long tpc = (T + pl.G - 1) / pl.G;
    if (T % tpc == 0 && tpc * C * 10 <= (U + pl.G - 1) / pl.G * 11) pl.G = T / tpc;
  }
  if (pl.G > U) pl.G = U;
  pl.busiest = pl.split > 1 ? (C + pl.split - 1) / pl.split : (U + pl.G - 1) / pl.G;
  return pl;
}

template <int MT, int BITS, bool WIDE>
cudaError_t launch_cfg(const SkinnyArgs& a, const Scratch& scratch, cudaStream_t stream, bool pdl,
                       std::string* err) {
  using Cfg = SkinnyCfg<MT, BITS, WIDE>;
  int dev = 0;
  cudaGetDevice(&dev);
  const DeviceInfo& di = device_info(dev);
  const bool xchg = a.ar != nullptr;
  cudaError_t e = xchg ? set_smem_attr<MT, 1, BITS, WIDE, true>(dev) : set_smem_attr<MT, 1, BITS, WIDE, false>(dev);
  if (e != cudaSuccess) return e;
  SkinnyLaunch<1> p{};
  if (!make_op<MT, BITS, WIDE>(a, &p.op[0], err)) return cudaErrorInvalidValue;
  p.n_ops = 1;
  p.M = (int)a.M;
  const SkinnyOp& op = p.op[0];
  const SkinnyPlan pl = plan_cfg<MT, BITS, WIDE>(a, di.sm_count);
  p.split = pl.split;
  p.G = (int)pl.G;
  p.op[0].G = p.G;
  const size_t need = kGbarBytes + kCounterBytes + (size_t)p.G * 2 * Cfg::PART * sizeof(float);
  if (scratch.bytes < need || scratch.base == nullptr) {
    *err = "scratch too small for the skinny path";
    return cudaErrorInvalidValue;
  }
  uint8_t* base = reinterpret_cast<uint8_t*>(scratch.base);
  p.gbar = reinterpret_cast<unsigned int*>(base);
  p.counter = reinterpret_cast<unsigned int*>(base + kGbarBytes);
  p.part = reinterpret_cast<float*>(base + kGbarBytes + kCounterBytes);
  p.status = a.status;
  p.amax = a.amax;
  if (xchg) {
    if (!skinny_exchange_fits(a) || a.M * a.N > ar_ll_elems(a.ar->n_max) || a.ar->P < 1 ||
        a.ar->P > kArMaxRanks) {
      *err = "this shape cannot fuse the row-parallel exchange into the decode kernel";
      return cudaErrorInvalidValue;
    }
    p.ar = ar_params(*a.ar);
  }
  // Exchange finishers: about one CTA per 512 outputs (a pair of outputs
  // per consumer thread), at most the SMs the workers leave idle, whole
  // clusters under a cluster split.
  long long grid = p.G;
  if (xchg) {
    long long F = (a.M * a.N + 511) / 512;
    const long long idle = di.sm_count - p.G;
    if (F > idle) F = idle;
    if (F > op.T) F = op.T;
    if (F < 1) F = 1;
    F = (F + p.split - 1) / p.split * p.split;
    grid += F;
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int nattr = 0;
  if (pdl) {
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  if (p.split > 1) {
    attr[nattr].id = cudaLaunchAttributeClusterDimension;
    attr[nattr].val.clusterDim.x = (unsigned)p.split;
    attr[nattr].val.clusterDim.y = 1;
    attr[nattr].val.clusterDim.z = 1;
    ++nattr;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  return xchg ? cudaLaunchKernelEx(&cfg, qmm_skinny_kernel<MT, 1, BITS, WIDE, true>, p)
              : cudaLaunchKernelEx(&cfg, qmm_skinny_kernel<MT, 1, BITS, WIDE, false>, p);
}

// A chain of up to kSkinnyChainMax matmuls in one cooperative launch of one
// CTA per SM, stream-K for every matmul.
template <int MT>
cudaError_t launch_chain_cfg(const SkinnyArgs* ops, int n, const Scratch& scratch, cudaStream_t stream,
                             std::string* err) {
  using Cfg = SkinnyCfg<MT, 4, false>;  // chains take 4-bit codes in 8-group units
  int dev = 0;
  cudaGetDevice(&dev);
  const DeviceInfo& di = device_info(dev);
  cudaError_t e = set_smem_attr<MT, kSkinnyChainMax, 4, false, false>(dev);
  if (e != cudaSuccess) return e;
  static SkinnyLaunch<kSkinnyChainMax> p;  // large: build it outside the stack (copied at launch)
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  p = SkinnyLaunch<kSkinnyChainMax>{};
  for (int i = 0; i < n; ++i)
    if (!make_op<MT, 4, false>(ops[i], &p.op[i], err)) return cudaErrorInvalidValue;
  p.n_ops = n;
  p.M = (int)ops[0].M;
  p.G = di.sm_count;
  p.split = 1;
  for (int i = 0; i < n; ++i) p.op[i].G = p.op[i].U < p.G ? (int)p.op[i].U : p.G;
  const size_t need = kGbarBytes + kCounterBytes + (size_t)p.G * 2 * Cfg::PART * sizeof(float);
  if (scratch.bytes < need || scratch.base == nullptr) {
    *err = "scratch too small for the skinny path";
    return cudaErrorInvalidValue;
  }
  uint8_t* base = reinterpret_cast<uint8_t*>(scratch.base);
  p.gbar = reinterpret_cast<unsigned int*>(base);
  p.counter = reinterpret_cast<unsigned int*>(base + kGbarBytes);
  p.part = reinterpret_cast<float*>(base + kGbarBytes + kCounterBytes);
  p.status = ops[0].status;
  // The per-matmul tallies start at zero; stream order puts this after any
  // earlier launch that used the same scratch (this launch does not overlap
  // its predecessor).
  e = cudaMemsetAsync(p.gbar, 0, (size_t)n * sizeof(unsigned int), stream);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.G);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid-wide waits can complete
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qmm_skinny_kernel<MT, kSkinnyChainMax, 4, false, false>, p);
}

}  // namespace

size_t skinny_scratch_bytes(const SkinnyArgs& a, int device) {
  const DeviceInfo& di = device_info(device);
  const int mpad = a.M <= 8 ? 8 : 16;
  const int BN = 128;
  return kGbarBytes + kCounterBytes + (size_t)di.sm_count * 2 * BN * mpad * sizeof(float);
}

bool skinny_exchange_fits(const SkinnyArgs& a) {
  return a.M >= 1 && a.M <= 16 && !a.swiglu && !a.amax && a.y != nullptr;
}

size_t skinny_zeroed_bytes(const SkinnyArgs& a) {
  static_assert(SkinnyCfg<1>::BN == 128 && SkinnyCfg<8>::BN == 128 && SkinnyCfg<16>::BN == 128, "row tile");
  const int64_t tile_rows = a.swiglu ? 64 : 128;
  const size_t tiles = (size_t)((a.N + tile_rows - 1) / tile_rows);
  return kGbarBytes + (tiles < kMaxCounters ? tiles : kMaxCounters) * sizeof(unsigned int);
}

namespace {
// One token with 4-bit codes: 16-group units unless they leave the busiest
// CTA with more than 10% more k to stream than 8-group units (8192 x 5120: 3
// units of 1024 k per CTA in pairs against 5 of 512; there the wide units
// ran 11.3 us against 10.5), or lose the TMA path for scales and biases that
// 8-group units have (K a multiple of 512 but not of 1024, as the down shard
// at TP=2).  Where both give the same k the wide units were faster: 17408 x
// 5120 13.3 against 13.8 us, 5120 x 17408 15.4 against 16.4, lm_head
// (151936 x 5120, 1% more k) 76.2 against 86.2.
bool one_token_wide(const SkinnyArgs& a, int sm) {
  constexpr int CK8 = SkinnyCfg<1, 4, false>::CK, CK16 = SkinnyCfg<1, 4, true>::CK;
  const SkinnyPlan p8 = plan_cfg<1, 4, false>(a, sm), p16 = plan_cfg<1, 4, true>(a, sm);
  const long long k8 = p8.busiest * CK8, k16 = p16.busiest * CK16;
  const bool tma_sb8 = a.K % CK8 == 0 && a.group_size == kGroup, tma_sb16 = a.K % CK16 == 0 && a.group_size == kGroup;
  return k16 * 10 <= k8 * 11 && (tma_sb16 || !tma_sb8);
}

template <int MT, int BITS, bool WIDE>
SkinnySchedule schedule_of(const SkinnyArgs& a, int sm) {
  const SkinnyPlan pl = plan_cfg<MT, BITS, WIDE>(a, sm);
  SkinnySchedule sc;
  sc.tokens = MT;
  sc.unit_k = SkinnyCfg<MT, BITS, WIDE>::CK;
  sc.ctas = pl.G;
  sc.split = pl.split;
  sc.busiest_units = pl.busiest;
  return sc;
}
}  // namespace

SkinnySchedule skinny_schedule(const SkinnyArgs& a, int sm_count) {
  if (a.bits == 8) {
    if (a.M == 1) return schedule_of<1, 8, false>(a, sm_count);
    if (a.M <= 8) return schedule_of<8, 8, false>(a, sm_count);
    return schedule_of<16, 8, false>(a, sm_count);
  }
  if (a.M == 1)
    return one_token_wide(a, sm_count) ? schedule_of<1, 4, true>(a, sm_count) : schedule_of<1, 4, false>(a, sm_count);
  if (a.M <= 4) return schedule_of<4, 4, false>(a, sm_count);
  if (a.M <= 8) return schedule_of<8, 4, false>(a, sm_count);
  return schedule_of<16, 4, false>(a, sm_count);
}

cudaError_t launch_skinny(const SkinnyArgs& a, const Scratch& scratch, cudaStream_t stream, bool pdl,
                          std::string* err) {
  if (a.bits == 8) {
    if (a.M == 1) return launch_cfg<1, 8, false>(a, scratch, stream, pdl, err);
    if (a.M <= 8) return launch_cfg<8, 8, false>(a, scratch, stream, pdl, err);
    return launch_cfg<16, 8, false>(a, scratch, stream, pdl, err);
  }
  if (a.M == 1) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (one_token_wide(a, device_info(dev).sm_count)) return launch_cfg<1, 4, true>(a, scratch, stream, pdl, err);
    return launch_cfg<1, 4, false>(a, scratch, stream, pdl, err);
  }
  if (a.M <= 4) return launch_cfg<4, 4, false>(a, scratch, stream, pdl, err);
  if (a.M <= 8) return launch_cfg<8, 4, false>(a, scratch, stream, pdl, err);
  return launch_cfg<16, 4, false>(a, scratch, stream, pdl, err);
}

cudaError_t launch_skinny_chain(const SkinnyArgs* ops, int n, const Scratch& scratch, cudaStream_t stream,
                                std::string* err) {
  if (n < 1 || n > kSkinnyChainMax) {
    *err = "a chained launch takes 1 to " + std::to_string(kSkinnyChainMax) + " matmuls";
    return cudaErrorInvalidValue;
  }
  const int64_t M = ops[0].M;
  for (int i = 0; i < n; ++i)
    if (ops[i].bits != 4) {
      *err = "a chained launch takes 4-bit codes";
      return cudaErrorInvalidValue;
    }
  for (int i = 1; i < n; ++i)
    if (ops[i].M != M) {
      *err = "every matmul of a chain must have the same number of rows of x";
      return cudaErrorInvalidValue;
    }
  if (M == 1) return launch_chain_cfg<1>(ops, n, scratch, stream, err);
  if (M <= 8) return launch_chain_cfg<8>(ops, n, scratch, stream, err);
  return launch_chain_cfg<16>(ops, n, scratch, stream, err);
}

}  // namespace qw
