// qw_quant.cu -- affine dequantize / quantize kernels (4- or 8-bit codes,
// groups of 64 or 128) and the small elementwise epilogues of the
// linear-forward entry points.
//
// dequantize is bit-exact with the oracle under both roundings: every fp16
// product and sum goes through an explicitly rounded (.rn) f16x2 instruction.
// quantize is bit-exact with the oracle's quantizer: every fp32 step uses an
// explicitly rounded intrinsic so nothing is contracted into an fma.
#include <cuda_fp16.h>

#include "qw_internal.h"
#include "qw_ptx.cuh"

namespace qw {

namespace {

// One packed word of 8-bit codes (4 codes, k ascending from bit 0) of a group
// with scale pair s2 and bias pair b2: 4 fp16 weights as 2 words.
template <bool kRoundOnce>
__device__ __forceinline__ uint2 dequant_word8(uint32_t w, uint32_t s2, uint32_t b2) {
  uint2 o;
  // (q_even, q_odd) exact: prmt makes (1024 + q, 1024 + q'), minus 1024
  const uint32_t q01 = hsub2_rn(prmt(w, 0x64646464u, 0x5140u), 0x64006400u);
  const uint32_t q23 = hsub2_rn(prmt(w, 0x64646464u, 0x5342u), 0x64006400u);
  o.x = kRoundOnce ? hfma2_rn(q01, s2, b2) : hadd2_rn(hmul2_rn(q01, s2), b2);
  o.y = kRoundOnce ? hfma2_rn(q23, s2, b2) : hadd2_rn(hmul2_rn(q23, s2), b2);
  return o;
}

// One thread per packed word: 8 (4-bit) or 4 (8-bit) outputs per thread.
template <bool kRoundOnce, int BITS>
__global__ void dequantize_kernel(const uint32_t* __restrict__ w, const __half* __restrict__ scales,
                                  const __half* __restrict__ biases, void* __restrict__ out, int64_t N,
                                  int64_t words_per_row, int64_t groups, int words_per_group) {
  const int64_t total = N * words_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / words_per_row;
    const int64_t kw = i - n * words_per_row;
    const int64_t g = kw / words_per_group;
    const __half s = scales[n * groups + g];
    const __half b = biases[n * groups + g];
    const uint32_t s2 = (uint32_t)__half_as_ushort(s) * 0x10001u;
    const uint32_t b2 = (uint32_t)__half_as_ushort(b) * 0x10001u;
    if (BITS == 4) reinterpret_cast<uint4*>(out)[i] = dequant_word<kRoundOnce>(__ldg(w + i), s2, b2);
    else reinterpret_cast<uint2*>(out)[i] = dequant_word8<kRoundOnce>(__ldg(w + i), s2, b2);
  }
}

// One thread per group of GS weights (GS = 64 or 128, BITS = 4 or 8).  Two
// passes over the group's fp16 values (min/max, then codes), both from L1.
template <int BITS, int GS>
__global__ void quantize_kernel(const __half* __restrict__ w, uint32_t* __restrict__ wq, __half* __restrict__ scales,
                                __half* __restrict__ biases, int64_t ngroups) {
  constexpr int PF = 32 / BITS;                // codes per word
  constexpr float NBINS = (float)((1 << BITS) - 1);
  for (int64_t gidx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gidx < ngroups;
       gidx += (int64_t)gridDim.x * blockDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(w + gidx * GS);
    float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
#pragma unroll 4
    for (int i = 0; i < GS / 8; ++i) {
      const uint4 v = __ldg(src + i);
      const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float f = __half2float(h[j]);
        if (f < mn) mn = f;
        if (f > mx) mx = f;
      }
    }
    float scale = __fdiv_rn(__fsub_rn(mx, mn), NBINS);
    if (!(scale >= 1e-7f)) scale = 1e-7f;
    const __half sh = __float2half_rn(scale);
    const __half bh = __float2half_rn(mn);
    const float sf = __half2float(sh);
    const float bf = __half2float(bh);
    scales[gidx] = sh;
    biases[gidx] = bh;
    uint32_t* dst = wq + gidx * (GS / PF);
#pragma unroll 4
    for (int i = 0; i < GS / 8; ++i) {  // 8 values: one 4-bit word or two 8-bit words
      const uint4 v = __ldg(src + i);
      const __half* h = reinterpret_cast<const __half*>(&v);
      uint32_t word[8 / PF + (PF > 8 ? 1 : 0)] = {};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float r = rintf(__fdiv_rn(__fsub_rn(__half2float(h[j]), bf), sf));
        r = fminf(fmaxf(r, 0.0f), NBINS);
        word[j / PF] |= ((uint32_t)r) << (BITS * (j % PF));
      }
#pragma unroll
      for (int k = 0; k < 8 / PF; ++k) dst[i * (8 / PF) + k] = word[k];
    }
  }
}

// y[m][n] = fp16(fp16 y * global_scale) then fp16 add of linear_bias[n].
__global__ void affine_epilogue_kernel(__half* __restrict__ y, const __half* __restrict__ bias,
                                       const float* __restrict__ gscale, int64_t M, int64_t N) {
  const int64_t total = M * N;
  const float gs = gscale ? *gscale : 1.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    __half v = y[i];
    if (gscale) v = __float2half_rn(__fmul_rn(__half2float(v), gs));
    if (bias) v = __hadd_rn(v, bias[i % N]);
    y[i] = v;
  }
}

__global__ void f32_to_f16_kernel(const float* __restrict__ src, __half* __restrict__ dst, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(src[i]);
}

// y = silu(gate) * up on fp16 arrays, each op rounded to fp16 (the fused
// kernels' epilogue, for gate and up computed apart).
__global__ void swiglu_kernel(const __half* __restrict__ gate, const __half* __restrict__ up,
                              __half* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(swiglu_f16(__half2float(gate[i]), __half2float(up[i])));
}

int grid_for(int64_t work, int threads) {
  int64_t blocks = (work + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

}  // namespace

cudaError_t launch_dequantize(const uint32_t* w, const void* scales, const void* biases, void* out, int64_t N,
                              int64_t K, int group_size, int bits, int rounding, cudaStream_t stream) {
  if ((bits != 4 && bits != 8) || (group_size != 64 && group_size != 128)) return cudaErrorInvalidValue;
  const int64_t wpr = K * bits / 32;
  const int64_t total = N * wpr;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = grid_for(total, threads);
  const int wpg = group_size * bits / 32;
  const __half* sp = (const __half*)scales;
  const __half* bp = (const __half*)biases;
  const int64_t G = K / group_size;
  if (bits == 4) {
    if (rounding == 1) dequantize_kernel<true, 4><<<blocks, threads, 0, stream>>>(w, sp, bp, out, N, wpr, G, wpg);
    else dequantize_kernel<false, 4><<<blocks, threads, 0, stream>>>(w, sp, bp, out, N, wpr, G, wpg);
  } else {
    if (rounding == 1) dequantize_kernel<true, 8><<<blocks, threads, 0, stream>>>(w, sp, bp, out, N, wpr, G, wpg);
    else dequantize_kernel<false, 8><<<blocks, threads, 0, stream>>>(w, sp, bp, out, N, wpr, G, wpg);
  }
  return cudaGetLastError();
}

cudaError_t launch_quantize(const void* w, uint32_t* wq, void* scales, void* biases, int64_t N, int64_t K,
                            int group_size, int bits, cudaStream_t stream) {
  if ((bits != 4 && bits != 8) || (group_size != 64 && group_size != 128)) return cudaErrorInvalidValue;
  const int64_t ngroups = N * (K / group_size);
  if (ngroups == 0) return cudaSuccess;
  const int threads = 128;
  const int blocks = grid_for(ngroups, threads);
  const __half* wp = (const __half*)w;
  __half* sp = (__half*)scales;
  __half* bp = (__half*)biases;
  if (bits == 4 && group_size == 64) quantize_kernel<4, 64><<<blocks, threads, 0, stream>>>(wp, wq, sp, bp, ngroups);
  else if (bits == 4) quantize_kernel<4, 128><<<blocks, threads, 0, stream>>>(wp, wq, sp, bp, ngroups);
  else if (group_size == 64) quantize_kernel<8, 64><<<blocks, threads, 0, stream>>>(wp, wq, sp, bp, ngroups);
  else quantize_kernel<8, 128><<<blocks, threads, 0, stream>>>(wp, wq, sp, bp, ngroups);
  return cudaGetLastError();
}

cudaError_t launch_affine_epilogue(void* y, const void* linear_bias, const float* global_scale, int64_t M,
                                   int64_t N, cudaStream_t stream) {
  if (M * N == 0 || (!linear_bias && !global_scale)) return cudaSuccess;
  const int threads = 256;
  affine_epilogue_kernel<<<grid_for(M * N, threads), threads, 0, stream>>>(
      (__half*)y, (const __half*)linear_bias, global_scale, M, N);
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const void* gate, const void* up, void* y, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  swiglu_kernel<<<grid_for(n, threads), threads, 0, stream>>>((const __half*)gate, (const __half*)up, (__half*)y, n);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_f16(const float* src, void* dst, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  f32_to_f16_kernel<<<grid_for(n, threads), threads, 0, stream>>>(src, (__half*)dst, n);
  return cudaGetLastError();
}


// ------------------------------------------------------------ greedy token
namespace {

__global__ void argmax_finalize_kernel(const unsigned long long* keys, uint32_t* idx, int M) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m < M) idx[m] = 0xFFFFFFFFu - (uint32_t)(keys[m] & 0xFFFFFFFFull);
}

// One block per row; keys as in the skinny kernel's epilogue (order-preserving
// value above, complemented index below), reduced over the block.
// With `keys` set the block writes its row's best key instead of the index.
__global__ void argmax_rows_kernel(const __half* logits, int64_t N, uint32_t* idx, unsigned long long* keys) {
  const __half* row = logits + (size_t)blockIdx.x * N;
  unsigned long long best = 0ull;
  for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
    uint32_t b = __float_as_uint(__half2float(row[n]));
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    const unsigned long long k = ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
    best = v > best ? v : best;
  }
  __shared__ unsigned long long warp_best[32];
  if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long v = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v = warp_best[w] > v ? warp_best[w] : v;
    if (keys) keys[blockIdx.x] = v;
    else idx[blockIdx.x] = 0xFFFFFFFFu - (uint32_t)(v & 0xFFFFFFFFull);
  }
}

}  // namespace

cudaError_t launch_argmax_finalize(const unsigned long long* keys, uint32_t* idx, int64_t M, cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  argmax_finalize_kernel<<<(unsigned)((M + 127) / 128), 128, 0, stream>>>(keys, idx, (int)M);
  return cudaGetLastError();
}

cudaError_t launch_argmax_rows(const void* logits, int64_t M, int64_t N, uint32_t* idx, cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  argmax_rows_kernel<<<(unsigned)M, 512, 0, stream>>>(reinterpret_cast<const __half*>(logits), N, idx, nullptr);
  return cudaGetLastError();
}

cudaError_t launch_argmax_rows_keys(const void* logits, int64_t M, int64_t N, unsigned long long* keys,
                                    cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  argmax_rows_kernel<<<(unsigned)M, 512, 0, stream>>>(reinterpret_cast<const __half*>(logits), N, nullptr, keys);
  return cudaGetLastError();
}

}  // namespace qw
