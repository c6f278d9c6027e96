/*
 * qw_qmm.h -- C ABI of the B200 affine group-quantized matmul library
 * (libqwqmm.so).  Drop-in for the quantized-linear operator surface that
 * cr0sh/qw's mlxcel-core exposes to its runtime crate: every entry point
 * below replaces one cxx bridge function, cited as
 *   crates/mlxcel-core/src/lib.rs:<line>             (Rust declaration)
 *   crates/mlxcel-core/cpp/mlx_cxx_bridge.cpp:<line> (C++ shim)
 *
 * Conventions
 *  - All tensors are device memory owned by the caller, described by
 *    qw_array (row-contiguous; leading dimensions of x / y are flattened, as
 *    MLX does).  Outputs are preallocated by the caller.
 *  - Every launch is stream-ordered on `stream` (a cudaStream_t; NULL = the
 *    legacy default stream).  Calls on distinct streams may run concurrently.
 *  - Errors are returned as qw_status codes and never abort; the message of
 *    the last failing call on this host thread is qw_last_error().  The
 *    reference has no error channel at this boundary (an MLX throw crosses the
 *    cxx bridge as std::terminate, crates/mlxcel-core/src/layers.rs:1255-1285),
 *    so the checks it performs at load time (layers.rs:1286-1318, :1409-1440,
 *    :1783-1868) are performed here on every call instead.
 *  - Supported quantization: mode "affine" with fp16 activations and
 *    scales/biases; bits 4 in groups of 64 (the Qwen 27B checkpoint,
 *    crates/runtime/src/qwen3_5.rs:208-211) and the per-tensor overrides'
 *    bits 4 or 8 in groups of 64 or 128 (qwen3_next.rs:39-74).  Other
 *    combinations MLX accepts return QW_EUNSUPPORTED.
 */
#ifndef QW_QMM_H
#define QW_QMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QW_ABI_VERSION 1

typedef enum qw_status {
  QW_OK = 0,
  QW_EINVAL = 1,       /* shapes, dtypes or parameters inconsistent */
  QW_EUNSUPPORTED = 2, /* valid for MLX, not implemented here (bits, group size, mode, dtype) */
  QW_ECUDA = 3,        /* a CUDA runtime call failed */
  QW_ETIMEOUT = 4,     /* a kernel gave up on a bounded wait (see qw_device_status) */
  QW_ENOMEM = 5        /* scratch allocation failed */
} qw_status;

typedef enum qw_dtype {
  QW_U32 = 1,
  QW_F16 = 2,
  QW_BF16 = 3,
  QW_F32 = 4
} qw_dtype;

/* A device array: the role of MlxArray (crates/mlxcel-core/cpp/mlx_cxx_bridge.h:16-22)
 * at this boundary.  strides are in elements; a stride array of all zeros is
 * read as row-contiguous. */
typedef struct qw_array {
  void* data;
  int32_t dtype; /* qw_dtype */
  int32_t ndim;  /* 1..4 */
  int64_t shape[4];
  int64_t strides[4];
} qw_array;

/* y = x @ dequantize(w, scales, biases).T  (transpose != 0)
 * x: f16 [..., K]; w: u32 [N, K*bits/32]; scales, biases: f16 [N, K/group_size];
 * y: f16 [..., N], or f32 [..., N] to receive the fp32 accumulators unrounded
 * (the row-parallel partial sums of a tensor-parallel shard).
 * transpose == 0 (y = x @ dequantize(w)) returns QW_EUNSUPPORTED.
 * Replaces: quantized_matmul, lib.rs:1134-1143, mlx_cxx_bridge.cpp:2991-3017. */
int qw_quantized_matmul(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases,
                        int transpose, int group_size, int bits, const char* mode, qw_array* y, void* stream);

/* One matmul of a chain: y = x @ dequantize(w, scales, biases).T. */
typedef struct qw_qmm_op {
  const qw_array* x;
  const qw_array* w;
  const qw_array* scales;
  const qw_array* biases;
  qw_array* y;
} qw_qmm_op;

/* Runs ops[0..n_ops) in order, as n_ops calls of qw_quantized_matmul
 * (transpose = true) would, where op i may read what earlier ops wrote (its x
 * may be an earlier y).  Every op is validated as qw_quantized_matmul
 * validates it, and all x must have the same number of rows M.  With
 * M <= 16 and 4-bit codes up to 24 matmuls share one cooperative launch of
 * one CTA per SM: a matmul's weights start streaming while the previous
 * matmul finishes, and a grid-wide count of finished CTAs orders the
 * dependent reads.  With larger M or 8-bit codes it issues one launch per op.
 * Measured slower than one qw_quantized_matmul call per linear on the
 * 64-layer decode stack (every chained matmul takes stream-K fix-ups and
 * the grid-wide wait puts its slowest CTA on the critical path); it helps
 * runs of short matmuls only (o-shaped 5120 x 6144: 13.4 us each in chains of
 * 8 against 17.7 us).  Bind qw_quantized_matmul for decode.
 * No counterpart in the reference: it fuses a sequence of the reference's
 * quantized_matmul calls (lib.rs:1134-1143) for decode loops whose
 * consecutive linears have nothing in between. */
int qw_quantized_matmul_chain(const qw_qmm_op* ops, int n_ops, int group_size, int bits, const char* mode,
                              void* stream);

/* Greedy token of a projection: idx[m] = argmax_n of the fp16 logits
 * (x @ dequantize(w, scales, biases).T)[m, n], the lowest n among equal
 * maxima, as uint32 [M]; logits (nullable) receives the fp16 logits.  With
 * M <= 16 the argmax is folded into the matmul's epilogue (one atomic per CTA
 * and token) and the logits need not be written; with larger M the logits
 * buffer is required and a row argmax follows the matmul.
 * Replaces: quantized_linear_forward (project_logits, crates/runtime/src/
 * qwen3_5.rs:1038-1044) followed by argmax_last_axis (lib.rs:2055,
 * mlx_cxx_bridge.cpp:4434-4436). */
int qw_quantized_matmul_argmax(const qw_array* x, const qw_array* w, const qw_array* scales,
                               const qw_array* biases, int group_size, int bits, const char* mode, qw_array* logits,
                               qw_array* idx, void* stream);

/* The k largest logits of each row and their indices: logits f16 [..., N]
 * (row-contiguous); idx u32 [..., k]; values f16 [..., k] (nullable), sorted
 * by value descending, lower index first among equal values (one of the
 * outcomes argpartition allows: the exact top-k set, ties at the k-th value
 * resolved toward lower indices).  Values compare by their fp16 bit pattern
 * made order-preserving (so -0 sorts below +0).  1 <= k < N, as the
 * reference's caller requires; k above 1024 returns QW_EUNSUPPORTED.
 * Replaces: argpartition(logits, -k, -1) + slice + take_along_axis in
 * top_k_candidate_logits (crates/runtime/src/qwen3_5_dflash.rs:1236-1266;
 * lib.rs:950, :876; mlx_cxx_bridge.cpp:2753, :2633). */
int qw_topk(const qw_array* logits, int k, qw_array* idx, qw_array* values, void* stream);

/* The LM-head projection followed by qw_topk: logits = x @ dequantize(w).T
 * (f16 [..., N]) into `logits`, or into a per-(device, stream) buffer the
 * library keeps when logits is null, then the top k of each row.
 * Replaces: project_logits (qwen3_5.rs:1038-1044) followed by
 * top_k_candidate_logits (qwen3_5_dflash.rs:1236-1266), the DFlash2
 * candidate step (qwen3_5_dflash.rs:1412). */
int qw_quantized_matmul_topk(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases,
                             int group_size, int bits, const char* mode, int k, qw_array* logits, qw_array* idx,
                             qw_array* values, void* stream);

/* SwiGLU input projections of a dense MLP, activation fused:
 *   y = silu(g) * u,  g = x @ dequantize(w_gate).T,  u = x @ dequantize(w_up).T,
 * evaluated as the reference does on fp16 arrays: g and u rounded to fp16,
 * then sigmoid(g), g * sigmoid(g) and the product with u each rounded to fp16.
 * Gate and up have the same shape [I, K*bits/32] and quantization; y is f16
 * (or f32) [..., I].  A checkpoint whose gate and up are stored as one
 * concatenated projection passes its two row halves as w_gate / w_up views.
 * One kernel per call: a row tile holds 64 gate rows and the same 64 up
 * rows, and only y is written.
 * Replaces: Mlp::forward_hidden (crates/runtime/src/qwen3_next.rs:463-487:
 * the gate and up quantized_matmul calls, or the fused projection and its two
 * slices) followed by compiled_swiglu_activation (lib.rs:627,
 * mlx_cxx_bridge.cpp:1205-1216, :1255-1265). */
int qw_quantized_matmul_swiglu(const qw_array* x, const qw_array* w_gate, const qw_array* scales_gate,
                               const qw_array* biases_gate, const qw_array* w_up, const qw_array* scales_up,
                               const qw_array* biases_up, int transpose, int group_size, int bits, const char* mode,
                               qw_array* y, void* stream);

/* y = silu(gate) * up elementwise on f16 arrays of one shape, rounded to
 * fp16 after each op as qw_quantized_matmul_swiglu's epilogue.
 * Replaces: compiled_swiglu_activation (lib.rs:627, mlx_cxx_bridge.cpp:1255-1265)
 * for gate and up computed apart (Mlp's Separate arm, qwen3_next.rs:465). */
int qw_swiglu_activation(const qw_array* gate, const qw_array* up, qw_array* y, void* stream);

/* Dense quantized SwiGLU MLP: y = (silu(x gate^T) * (x up^T)) @ dequantize(w_down).T,
 * the intermediate held in a per-(device, stream) buffer the library keeps.
 * All three projections share group_size, bits and mode.
 * Replaces: compiled_moe_expert_forward (lib.rs:1636-1652,
 * mlx_cxx_bridge.cpp:4203-4270) and Mlp::forward (qwen3_next.rs:458-461). */
int qw_swiglu_mlp(const qw_array* x, const qw_array* w_gate, const qw_array* scales_gate, const qw_array* biases_gate,
                  const qw_array* w_up, const qw_array* scales_up, const qw_array* biases_up, const qw_array* w_down,
                  const qw_array* scales_down, const qw_array* biases_down, int group_size, int bits,
                  const char* mode, qw_array* y, void* stream);

/* As qw_quantized_matmul for at most 16 rows of x, for callers that must not
 * have the library allocate device memory during the call (a runtime that
 * owns all of the GPU's memory in its own pool; a decode loop that cannot
 * absorb cudaFree's device-wide wait).  Allocates nothing: its scratch is a
 * fixed 4 MiB device array that every GPU loading the library holds until the
 * process exits.  The first call on a device resolves that array's address
 * (make it before any stream capture).  All calls on a device share the
 * array, so calls that overlap on the GPU race; calls on one stream are safe.
 * 4- or 8-bit codes in groups of 64 or 128.  More than 16 rows, or a shape
 * whose scratch exceeds the array, returns QW_EUNSUPPORTED.  A kernel
 * that gives up on a bounded wait leaves y incomplete and a code in the
 * array's status word, which qw_device_status reports (it allocates nothing).
 * No counterpart in the reference: MLX allocates through its own allocator. */
int qw_quantized_matmul_static_scratch(const qw_array* x, const qw_array* w, const qw_array* scales,
                                       const qw_array* biases, int transpose, int group_size, int bits,
                                       const char* mode, qw_array* y, void* stream);

/* ---------------------------------------------------------------- peer allreduce
 * Tensor parallelism's exchange step: the o and down projections are
 * row-parallel, each rank's matmul writes fp32 partial sums (y as float32),
 * and y = fp16(sum over ranks).  One process per GPU of one node; every rank
 * owns a buffer that all ranks map through CUDA IPC, and one kernel per call
 * stores the rank's partial into every rank's buffer over NVLink, flags it,
 * waits (bounded) for every rank's flag and sums in rank order, so every rank
 * gets bit-identical y.  Calls are stream-ordered and may be captured in a
 * CUDA graph; all ranks must make the same sequence of calls.  A rank whose
 * peers never arrive gives up after 2 s: its y is incomplete and
 * qw_device_status reports QW_ETIMEOUT.  No multicast or NVLS is used.
 * No counterpart in the reference, which runs on one device; it replaces the
 * ncclAllReduce(float32, sum) + fp16 cast of the tensor-parallel stack.
 *
 * Set-up: qw_allreduce_init on every rank (allocates and zeroes this rank's
 * buffer for up to max_elems floats per call, 64 KiB + 8 P max_elems +
 * 16 P min(max_elems, 2^21) bytes, and returns its IPC handle,
 * QW_IPC_HANDLE_BYTES bytes); exchange the handles (any host transport);
 * qw_allreduce_connect with all ranks' handles in rank order; then a
 * barrier across ranks before the first qw_allreduce_sum.  Peers store into
 * every rank's buffer, so qw_allreduce_destroy may run only once every
 * rank's calls have ended: each rank synchronizes its device, then a barrier
 * across ranks, then each rank destroys (destroy itself waits for this
 * device's work only).  Calls of a communicator run on its device. */
#define QW_IPC_HANDLE_BYTES 64
typedef struct qw_allreduce qw_allreduce;
int qw_allreduce_init(int world, int rank, int64_t max_elems, qw_allreduce** comm, unsigned char* handle);
int qw_allreduce_connect(qw_allreduce* comm, const unsigned char* handles);
/* y (f16 or f32, any shape) = sum over ranks of partial (f32, same element count). */
int qw_allreduce_sum(qw_allreduce* comm, const qw_array* partial, qw_array* y, void* stream);
int qw_allreduce_destroy(qw_allreduce* comm);

/* Row-parallel projection of a tensor-parallel layer (the o and down
 * projections), the matmul and the sum over ranks in one call: y (f16 or
 * f32 [M, N]) = sum over ranks r of x_r @ dequantize(w_r).T, where this rank
 * holds x_r [M, K_r] and w_r (scales, biases as in qw_quantized_matmul) [N,
 * K_r] of a K-split (the same N on every rank).  Every rank receives the
 * fp32 products summed in rank order and rounded once: bit for bit
 * qw_quantized_matmul into f32 then qw_allreduce_sum.  For M <= 16 and
 * M * N <= min(max_elems, 2^21) the exchange runs in the decode kernel: each
 * finished value goes to every rank as one 64-bit word tagged with the
 * call's epoch, and a few extra CTAs of the same launch wait for every
 * rank's words and sum them; one launch instead of two.  Otherwise the call
 * runs the matmul into the communicator's fp32 buffer and then the allreduce
 * kernel.  A collective call of the same sequence as qw_allreduce_sum (all
 * ranks, same order, same M and N); M * N <= max_elems.
 * Replaces: the o and down projections of a layer split over GPUs
 * (crates/runtime/src/qwen3_next.rs:142-160, 458-487 run them on one
 * device) followed by ncclAllReduce(float32, sum) and a cast. */
int qw_allreduce_matmul(qw_allreduce* comm, const qw_array* x, const qw_array* w, const qw_array* scales,
                        const qw_array* biases, int group_size, int bits, const char* mode, qw_array* y,
                        void* stream);

/* Greedy token of a vocabulary-sharded LM head under tensor parallelism:
 * this rank holds rows [index_base, index_base + N) of the head (w, scales,
 * biases as in qw_quantized_matmul_argmax) and every rank receives in idx
 * (uint32 [M]) the global argmax of each row of x over all ranks' logits,
 * the lowest global index among equal maxima, bit for bit what one GPU
 * holding the whole head returns.  Each rank reduces its own shard (folded
 * into the decode kernel's epilogue for M <= 16; logits required above),
 * then one kernel exchanges one 8-byte (value, index) key per row with every
 * rank over the communicator's buffers and takes the largest.  A collective
 * call of the same sequence as qw_allreduce_sum (all ranks, same order, same
 * M); 2 M <= max_elems.
 * Replaces: project_logits (crates/runtime/src/qwen3_5.rs:1038-1044) then
 * argmax_last_axis (lib.rs:2055) on a model split over GPUs, which the
 * single-device reference does not have. */
int qw_allreduce_argmax(qw_allreduce* comm, const qw_array* x, const qw_array* w, const qw_array* scales,
                        const qw_array* biases, int group_size, int bits, const char* mode, int64_t index_base,
                        qw_array* logits, qw_array* idx, void* stream);

/* y = x @ dequantize(w).T (+ linear_bias), linear_bias nullable f16 [N].
 * Replaces: quantized_linear_forward, lib.rs:591-601, mlx_cxx_bridge.cpp:1099-1133. */
int qw_quantized_linear_forward(const qw_array* x, const qw_array* w, const qw_array* scales,
                                const qw_array* biases, const qw_array* linear_bias, int group_size, int bits,
                                const char* mode, qw_array* y, void* stream);

/* y = fp16(fp16(x @ dequantize(w).T) * global_scale) (+ linear_bias).
 * global_scale nullable, f32 scalar in device memory.
 * Replaces: quantized_linear_forward_global_scale, lib.rs:604-615,
 * mlx_cxx_bridge.cpp:1135-1170. */
int qw_quantized_linear_forward_global_scale(const qw_array* x, const qw_array* w, const qw_array* scales,
                                             const qw_array* biases, const qw_array* global_scale,
                                             const qw_array* linear_bias, int group_size, int bits,
                                             const char* mode, qw_array* y, void* stream);

/* out f16 [N, K] = scales * q + biases, each product and sum rounded to fp16
 * (the fp16 op-by-op evaluation of MLX's CPU backend).
 * Replaces: dequantize, lib.rs:1152-1159, mlx_cxx_bridge.cpp:3019-3069. */
int qw_dequantize(const qw_array* w, const qw_array* scales, const qw_array* biases, int group_size, int bits,
                  const char* mode, qw_array* out, void* stream);

/* As qw_dequantize with an explicit rounding: 0 = two roundings (default
 * above), 1 = s*q + b rounded once (fused multiply-add in fp16). */
int qw_dequantize_rounding(const qw_array* w, const qw_array* scales, const qw_array* biases, int group_size,
                           int bits, const char* mode, int rounding, qw_array* out, void* stream);

/* Affine-quantize w f16 [N, K] into (wq u32, scales f16, biases f16):
 * s = max((max-min)/(2^bits-1), 1e-7) rounded to fp16, b = fp16(min),
 * q = clamp(rint((w - b) / s), 0, 2^bits-1) per group.
 * Replaces: quantize_weights{,_w,_scales,_biases}, lib.rs:2707-2742,
 * mlx_cxx_bridge.cpp:6347-6393. */
int qw_quantize(const qw_array* w, int group_size, int bits, const char* mode, qw_array* wq, qw_array* scales,
                qw_array* biases, void* stream);

/* Message of the last failing call on this host thread ("" if none). */
const char* qw_last_error(void);

/* Reads (and, if clear != 0, resets) the device-side status words that a
 * kernel sets when one of its bounded waits runs out (0 = none): the
 * library's own and the one in qw_quantized_matmul_static_scratch's array;
 * the first nonzero is returned.  Synchronises the device; allocates
 * nothing. */
int qw_device_status(int device, unsigned int* status, int clear);

/* The decode kernel's configuration and schedule for a matmul of m rows of x
 * (1..16) against an n x k weight (for a SwiGLU call, n gate rows), on a GPU
 * with sm_count SMs: the choice the matmul entry points make, computed on the
 * host without touching a device.  out (int64 [5]) receives the rows of x
 * the configuration takes (1, 4, 8 or 16), k per unit (512 or 1024), the
 * CTAs that take units, the CTAs per row tile under a cluster split (1:
 * stream-K or whole tiles per CTA) and the units of the busiest CTA.  For
 * tests and tuning; no counterpart in the reference. */
int qw_decode_schedule(int64_t m, int64_t n, int64_t k, int bits, int group_size, int swiglu, int sm_count,
                       int64_t* out);

/* QW_ABI_VERSION of the loaded library. */
int qw_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif
