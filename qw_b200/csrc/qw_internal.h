// qw_internal.h -- declarations shared by the C-ABI layer and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

struct qw_array;

namespace qw {

// Error reporting: the C-ABI stores a message in a thread-local string.
void set_error(const std::string& msg);
const char* last_error();

// TMA descriptor encoding through the driver entry point (no -lcuda).
bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                    uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle,
                    std::string* err);

bool encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[3],
                    const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle swizzle,
                    std::string* err);

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int max_smem_optin = 0;
};
const DeviceInfo& device_info(int device);

// Scratch memory for a launch: either the library's own per-device buffer or
// caller-supplied memory.  `bytes` is the capacity of `base`.
struct Scratch {
  void* base = nullptr;
  size_t bytes = 0;
};

// Skinny path (M <= 16): stream-K over (row tile, 512-wide k chunk) units.
struct ArComm;

struct SkinnyArgs {
  const void* x;         // fp16 [M][K], rows x_ld apart
  const uint32_t* w;     // [N][K/8]
  const void* scales;    // fp16 [N][K/64]
  const void* biases;    // fp16 [N][K/64]
  void* y;               // fp16 or fp32 [M][N]
  bool y_f32;
  int64_t M, N, K;
  int max_ctas;          // 0 = occupancy-derived
  unsigned int* status;  // device status word
  int64_t x_ld = 0;      // elements from one row of x to the next (0 = K)
  unsigned long long* amax = nullptr;  // greedy-token keys [M], zeroed by the caller (y may be null)
  int group_size = 64;   // 64 or 128
  int bits = 4;          // 4 or 8
  // SwiGLU (gate and up of an MLP, activation fused): w/scales/biases are the
  // gate projection's, w2/scales2/biases2 the up projection's, both [N] rows,
  // and y [M][N] = silu(x gate^T) * (x up^T).
  bool swiglu = false;
  const uint32_t* w2 = nullptr;
  const void* scales2 = nullptr;
  const void* biases2 = nullptr;
  // Row-parallel projection under tensor parallelism (M <= 16, not SwiGLU,
  // no greedy keys): y = the sum over the communicator's ranks of every
  // rank's x W^T, exchanged through the communicator's buffers in the
  // kernel's epilogue.  Null: y is this rank's product alone.
  const ArComm* ar = nullptr;
};
// The decode kernel's configuration and schedule for a matmul (the choice
// launch_skinny makes, computed without touching a device).
struct SkinnySchedule {
  int tokens;               // rows of x the configuration takes (1, 4, 8 or 16)
  int unit_k;               // k per unit (512 or 1024)
  long long ctas;           // CTAs that take units
  int split;                // CTAs per row tile under a cluster split (1: stream-K or whole tiles)
  long long busiest_units;  // units of the busiest CTA
};
SkinnySchedule skinny_schedule(const SkinnyArgs& a, int sm_count);
// Whether a skinny launch can fuse the row-parallel exchange for this shape
// (the communicator's ll slots must also hold M N values).
bool skinny_exchange_fits(const SkinnyArgs& a);
// Skinny-path scratch layout: split-tile counters (zero between launches) at
// the start, then the partial-sum slots.
constexpr size_t kSkinnyMaxCounters = 1u << 16;  // row tiles per launch
constexpr size_t kSkinnyCounterBytes = kSkinnyMaxCounters * sizeof(unsigned int);
// Scratch bytes the skinny path needs for a shape (0 when it runs unsplit).
size_t skinny_scratch_bytes(const SkinnyArgs& a, int device);
cudaError_t launch_skinny(const SkinnyArgs& a, const Scratch& scratch, cudaStream_t stream, bool pdl,
                          std::string* err);
// Matmuls of one chained skinny launch (bounded by the kernel parameter space).
constexpr int kSkinnyChainMax = 24;
// Up to kSkinnyChainMax matmuls with the same M <= 16, in order, each allowed
// to read any earlier one's y, in one cooperative launch.
cudaError_t launch_skinny_chain(const SkinnyArgs* ops, int n, const Scratch& scratch, cudaStream_t stream,
                                std::string* err);
// Bytes at the start of a skinny launch's scratch that must be zero when it
// starts (its grid-barrier word and split-tile counters).
size_t skinny_zeroed_bytes(const SkinnyArgs& a);
// The matmul entry points' argument checks (qw_api.cu), without touching the
// device; on QW_OK fills every field of `sa` but max_ctas and status, with M
// the rows of x (all of them, not limited to 16).
int check_qmm_call(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases,
                   int transpose, int group_size, int bits, const char* mode, qw_array* y, SkinnyArgs* sa);

// Prefill path (tcgen05, M >= 17).
struct PrefillArgs {
  const void* x;
  const uint32_t* w;
  const void* scales;
  const void* biases;
  void* y;
  bool y_f32;
  int64_t M, N, K;
  unsigned int* status;
  int64_t x_ld = 0;  // elements from one row of x to the next (0 = K)
  int bits = 4;          // 4 or 8
  int group_size = 64;   // 64 or 128
  // SwiGLU, as in SkinnyArgs: w/scales/biases the gate, w2/scales2/biases2 the up projection
  bool swiglu = false;
  const uint32_t* w2 = nullptr;
  const void* scales2 = nullptr;
  const void* biases2 = nullptr;
};
cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream, bool pdl, std::string* err);
bool prefill_available();

// Greedy token from the keys the skinny kernel left: idx[m] = the row.
cudaError_t launch_argmax_finalize(const unsigned long long* keys, uint32_t* idx, int64_t M, cudaStream_t stream);
// Greedy token of each row of fp16 logits [M][N] (lowest index among equal maxima).
cudaError_t launch_argmax_rows(const void* logits, int64_t M, int64_t N, uint32_t* idx, cudaStream_t stream);
// The same as keys: (order-preserving fp16 value << 32) | (2^32 - 1 - index).
cudaError_t launch_argmax_rows_keys(const void* logits, int64_t M, int64_t N, unsigned long long* keys,
                                    cudaStream_t stream);

// The k largest fp16 values of each of M rows of N (rows ld apart), sorted
// descending, lower index first among equal values; 1 <= k <= topk_max_k(), k < N.
int topk_max_k();
int64_t topk_max_n();
cudaError_t launch_topk_rows(const void* logits, int64_t ld, int64_t M, int64_t N, int k, uint32_t* idx,
                             void* values, cudaStream_t stream);

// One-shot allreduce of fp32 partials over NVLink peer memory (qw_allreduce.cu).
constexpr int kArMaxRanks = 8;
struct ArComm {
  void* peer_bufs[kArMaxRanks];  // every rank's shared buffer, mapped in this process
  unsigned int* counters;        // local: one epoch per chunk (allreduce_epoch_bytes())
  unsigned int* status;          // device status word
  int P = 0, rank = 0;
  int64_t n_max = 0;
};
size_t allreduce_buffer_bytes(int P, int64_t n_max);
// Outputs a fused row-parallel exchange can carry (the ll slots' length).
int64_t allreduce_ll_elems(int64_t n_max);
size_t allreduce_epoch_bytes();
// idx[m] = the global greedy token of row m over every rank's vocabulary
// shard: keys[m] is this rank's best (value, local index) key and its shard
// starts at row index_base; 2 M <= n_max.
cudaError_t launch_argmax_exchange(const ArComm& c, const unsigned long long* keys, int64_t index_base,
                                   uint32_t* idx, int64_t M, cudaStream_t stream);
// y[i] = sum over ranks of partial[i], rounded to fp16 (or kept fp32); n <= n_max.
cudaError_t launch_allreduce(const ArComm& c, const float* partial, void* out, bool out_f32, bool vec, int64_t n,
                             int sm_count, cudaStream_t stream);

// Status word of the static-scratch entry point's array on `device` (current
// and synchronized), cleared when `clear`; 0 when no such call ran there.
cudaError_t static_scratch_status(int device, unsigned int* v, bool clear);

// Quantize / dequantize kernels (affine, 4-bit, group 64 for now).
cudaError_t launch_dequantize(const uint32_t* w, const void* scales, const void* biases, void* out, int64_t N,
                              int64_t K, int group_size, int bits, int rounding, cudaStream_t stream);
cudaError_t launch_quantize(const void* w, uint32_t* wq, void* scales, void* biases, int64_t N, int64_t K,
                            int group_size, int bits, cudaStream_t stream);

// Elementwise epilogues used by the linear-forward entry points.
cudaError_t launch_affine_epilogue(void* y, const void* linear_bias, const float* global_scale, int64_t M,
                                   int64_t N, cudaStream_t stream);
cudaError_t launch_f32_to_f16(const float* src, void* dst, int64_t n, cudaStream_t stream);
// y = silu(gate) * up elementwise on n fp16 values.
cudaError_t launch_swiglu(const void* gate, const void* up, void* y, int64_t n, cudaStream_t stream);

}  // namespace qw
