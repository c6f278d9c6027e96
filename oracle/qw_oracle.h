/*
 * qw_oracle.h -- CPU restatement of the affine group-quantized matmul that
 * cr0sh/qw reaches through MLX `quantized_matmul`.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links or calls
 * this code; it is the checker used by tests/, __graft_entry__.smoke() and
 * the cpu_baseline / --impl reference legs of bench.py.
 *
 * Parity status: the reference pins no numeric values for this path (its
 * quantized-matmul tests are MLX-against-MLX differential tests) and its MLX
 * dependency cannot be built here, so these semantics are a restatement of
 * MLX's published affine scheme as the reference calls it:
 *   - operator shape   crates/mlxcel-core/cpp/mlx_cxx_bridge.h:872-883
 *                      ("y = x @ dequantize(w, scales, biases).T if transpose")
 *   - call sites       crates/mlxcel-core/cpp/mlx_cxx_bridge.cpp:1099-1133,
 *                      :2991-3017 (quantized_matmul), :3019-3069 (dequantize),
 *                      :6347-6393 (quantize)
 *   - packing rule     crates/mlxcel-core/src/layers.rs:1568-1570 and
 *                      :1846-1852 (packed_in * 32 == bits * groups * group_size)
 *   - packed dtype     crates/mlxcel-core/src/weights.rs:150-158 (U32 words)
 *   - defaults         crates/runtime/src/qwen3_5.rs:208-211 (group 64, 4 bits)
 * Third-party holder of the arithmetic: MLX (ml-explore/mlx) at commit
 * 7ca40033132dae444d45f7fc3daae57e24c13f6c (crates/mlx-cpp/CMakeLists.txt:83).
 *
 * Conventions fixed here (and matched bit-for-bit by the CUDA library):
 *   nibble order  element k of a row sits in word k/(32/bits) at bit
 *                 bits*(k % (32/bits)), lowest bits first;
 *   dequantize    QWO_ROUND_TWICE: t = fp16(s*q), w = fp16(t + b) -- fp16
 *                 multiply then fp16 add, each rounded to nearest-even, the
 *                 result of evaluating `scales * q + biases` as two fp16 ops;
 *                 QWO_ROUND_ONCE: w = fp16(s*q + b) rounded once;
 *   matmul        y[m][n] = fp16( sum_k x[m][k] * (s*q + b) ) with the
 *                 dequantized weight formed in fp32 and an fp32 accumulator
 *                 advanced in ascending k.
 */
#ifndef QW_ORACLE_H
#define QW_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { QWO_ROUND_TWICE = 0, QWO_ROUND_ONCE = 1 };

enum {
  QWO_OK = 0,
  QWO_EINVAL = 1,
  QWO_EUNSUPPORTED = 2
};

/* IEEE binary16 conversions (round to nearest, ties to even). */
uint16_t qwo_f32_to_f16(float f);
uint16_t qwo_f64_to_f16(double d);
float qwo_f16_to_f32(uint16_t h);
void qwo_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n);
void qwo_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n);

/* Affine quantizer over groups of `group_size` consecutive elements of each
 * row of w fp16 [N][K]:  s = max((max-min)/(2^bits-1), 1e-7) -> fp16,
 * b = fp16(min), q = clamp(rint((w - b) / s), 0, 2^bits-1).
 * wq: uint32 [N][K*bits/32], scales/biases: fp16 [N][K/group_size]. */
int qwo_quantize(const uint16_t* w, int64_t N, int64_t K, int group_size, int bits,
                 uint32_t* wq, uint16_t* scales, uint16_t* biases);

/* out fp16 [N][K] = dequantize(wq, scales, biases) under `rounding`. */
int qwo_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                   int64_t N, int64_t K, int group_size, int bits, int rounding,
                   uint16_t* out);

/* out f32 [N][K] = dequantize(wq, scales, biases) for float32 scales and
 * biases: ROUND_TWICE w = fp32(fp32(s*q) + b); ROUND_ONCE w = fmaf(s, q, b). */
int qwo_dequantize_f32(const uint32_t* wq, const float* scales, const float* biases, int64_t N, int64_t K,
                       int group_size, int bits, int rounding, float* out);

/* y fp16 [M][N] = x fp16 [M][K] . w^T for fp16 weights w [N][K]: products
 * and sums in fp32, ascending k (the matmul on weights formed in fp16). */
int qwo_matmul_f16w(const uint16_t* x, const uint16_t* w, int64_t M, int64_t N, int64_t K, uint16_t* y,
                    float* y32, int nthreads);

/* y fp16 [M][N] = x fp16 [M][K] . dequantize(w)^T (transpose = true form).
 * y32 (nullable) receives the fp32 accumulators before the final rounding.
 * nthreads <= 0 uses every OpenMP thread. */
int qwo_quantized_matmul(const uint16_t* x, const uint32_t* wq, const uint16_t* scales,
                         const uint16_t* biases, int64_t M, int64_t N, int64_t K,
                         int group_size, int bits, uint16_t* y, float* y32, int nthreads);

/* Threads the OpenMP runtime would use (1 when built without OpenMP). */
int qwo_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
