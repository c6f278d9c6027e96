// qw_api.cu -- the C ABI (include/qw_qmm.h): argument validation mirroring
// the reference's load-time checks, dispatch to the kernels, per-stream
// scratch, TMA descriptor encoding and error reporting.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>
#include <algorithm>

#include "../../include/qw_qmm.h"
#include "qw_internal.h"

namespace qw {

// ------------------------------------------------------------------ errors
namespace {
thread_local std::string t_last_error;
}
void set_error(const std::string& msg) { t_last_error = msg; }
const char* last_error() { return t_last_error.c_str(); }

// ----------------------------------------------------------- device queries
const DeviceInfo& device_info(int device) {
  static std::mutex mu;
  static std::map<int, DeviceInfo> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  DeviceInfo d;
  d.device = device;
  cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  return cache.emplace(device, d).first->second;
}

// ------------------------------------------------------------ TMA encoding
namespace {
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Encoded descriptors by their arguments.  A descriptor is a function of its
// arguments only, and a decode loop encodes the same weight, scale and bias
// maps every step; the cache (per host thread, no locking) spares it those
// driver calls.
struct TmapKey {
  uint64_t base;
  uint64_t dims[3];
  uint64_t strides[2];
  uint32_t box[3];
  int32_t rank, dtype, swizzle, pad0, pad1;  // explicit padding: 80 bytes, no implicit holes
  bool operator==(const TmapKey& o) const { return std::memcmp(this, &o, sizeof(TmapKey)) == 0; }
};
static_assert(sizeof(TmapKey) == 80, "TmapKey has no implicit padding");
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    const unsigned char* b = reinterpret_cast<const unsigned char*>(&k);
    uint64_t h = 1469598103934665603ull;  // FNV-1a
    for (size_t i = 0; i < sizeof(TmapKey); ++i) h = (h ^ b[i]) * 1099511628211ull;
    return (size_t)h;
  }
};
constexpr size_t kTmapCacheMax = 4096;

bool encode_cached(int rank, CUtensorMapDataType dtype, const void* base, const cuuint64_t* dims,
                   const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swizzle, CUtensorMap* map,
                   CUresult* rc) {
  thread_local std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
  TmapKey k;
  std::memset(&k, 0, sizeof(k));
  k.base = reinterpret_cast<uint64_t>(base);
  for (int i = 0; i < rank; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
    if (i + 1 < rank) k.strides[i] = strides[i];
  }
  k.rank = rank;
  k.dtype = (int32_t)dtype;
  k.swizzle = (int32_t)swizzle;
  auto it = cache.find(k);
  if (it != cache.end()) {
    *map = it->second;
    *rc = CUDA_SUCCESS;
    return true;
  }
  auto fn = get_encode_fn();
  if (!fn) return false;
  const cuuint32_t estr[3] = {1, 1, 1};
  *rc = fn(map, dtype, rank, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (*rc == CUDA_SUCCESS) {
    if (cache.size() >= kTmapCacheMax) cache.clear();
    cache.emplace(k, *map);
  }
  return true;
}
}  // namespace

bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                    uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle,
                    std::string* err) {
  const cuuint64_t dims[2] = {dim0, dim1};
  const cuuint64_t strides[1] = {stride1_bytes};
  const cuuint32_t box[2] = {box0, box1};
  CUresult r = CUDA_SUCCESS;
  if (!encode_cached(2, dtype, base, dims, strides, box, swizzle, map, &r)) {
    *err = "cuTensorMapEncodeTiled is not available from the driver";
    return false;
  }
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ") for dims " + std::to_string(dim0) +
           "x" + std::to_string(dim1) + " stride " + std::to_string(stride1_bytes);
    return false;
  }
  return true;
}

bool encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[3],
                    const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle swizzle,
                    std::string* err) {
  const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  const cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
  const cuuint32_t b[3] = {box[0], box[1], box[2]};
  CUresult r = CUDA_SUCCESS;
  if (!encode_cached(3, dtype, base, d, st, b, swizzle, map, &r)) {
    *err = "cuTensorMapEncodeTiled is not available from the driver";
    return false;
  }
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled (3-D) failed (code " + std::to_string((int)r) + ")";
    return false;
  }
  return true;
}

// ------------------------------------------------- per-device resources
namespace {

struct DeviceRes {
  unsigned int* status = nullptr;
};

std::mutex g_res_mu;
std::map<int, DeviceRes> g_dev_res;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;

bool device_res(int device, DeviceRes** out, std::string* err) {
  std::lock_guard<std::mutex> lock(g_res_mu);
  auto it = g_dev_res.find(device);
  if (it == g_dev_res.end()) {
    DeviceRes r;
    if (cudaMalloc(&r.status, 256) != cudaSuccess || cudaMemset(r.status, 0, 256) != cudaSuccess) {
      *err = "could not allocate the device status word";
      return false;
    }
    it = g_dev_res.emplace(device, r).first;
  }
  *out = &it->second;
  return true;
}

// Scratch keyed by (device, stream): launches on one stream are ordered, so
// they can share it; launches on different streams never do.  Grows on
// demand; freshly allocated scratch is zeroed (the split-tile counters must
// start at zero and every kernel leaves them at zero).
bool scratch_for(int device, cudaStream_t stream, size_t bytes, Scratch* out, std::string* err) {
  std::lock_guard<std::mutex> lock(g_res_mu);
  Scratch& s = g_scratch[{device, stream}];
  if (s.bytes < bytes) {
    if (s.base) {
      cudaStreamSynchronize(stream);
      cudaFree(s.base);
      s = Scratch{};
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    void* p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) {
      cudaGetLastError();
      *err = "scratch allocation of " + std::to_string(want) + " bytes failed";
      return false;
    }
    if (cudaMemset(p, 0, want) != cudaSuccess) {
      cudaFree(p);
      *err = "scratch initialisation failed";
      return false;
    }
    s.base = p;
    s.bytes = want;
  }
  *out = s;
  return true;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("QW_DISABLE_PDL");
    return !(e && e[0] == '1');
  }();
  return on;
}

// ------------------------------------------------------------- validation
int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int64_t numel(const qw_array* a) {
  int64_t n = 1;
  for (int i = 0; i < a->ndim; ++i) n *= a->shape[i];
  return n;
}

bool contiguous(const qw_array* a) {
  bool all_zero = true;
  for (int i = 0; i < a->ndim; ++i) all_zero = all_zero && a->strides[i] == 0;
  if (all_zero) return true;
  int64_t expect = 1;
  for (int i = a->ndim - 1; i >= 0; --i) {
    if (a->shape[i] != 1 && a->strides[i] != expect) return false;
    expect *= a->shape[i];
  }
  return true;
}

const char* dtype_name(int d) {
  switch (d) {
    case QW_U32: return "uint32";
    case QW_F16: return "float16";
    case QW_BF16: return "bfloat16";
    case QW_F32: return "float32";
    default: return "unknown";
  }
}

int check_array(const qw_array* a, const char* what) {
  if (!a) return fail(QW_EINVAL, std::string(what) + " is null");
  if (a->ndim < 1 || a->ndim > 4) return fail(QW_EINVAL, std::string(what) + " must have 1 to 4 dimensions");
  for (int i = 0; i < a->ndim; ++i)
    if (a->shape[i] < 0) return fail(QW_EINVAL, std::string(what) + " has a negative dimension");
  if (!contiguous(a)) return fail(QW_EINVAL, std::string(what) + " must be row-contiguous");
  if (numel(a) > 0 && a->data == nullptr) return fail(QW_EINVAL, std::string(what) + " has a null data pointer");
  return QW_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// x: rows of K contiguous elements, one uniform step (*ld elements) from a
// row to the next, leading dimensions flattened (so a column slice of a
// wider matrix is accepted without a copy).  The step must keep every row
// 16-byte aligned (a TMA stride).
int check_x_rows(const qw_array* x, int64_t K, int64_t* ld) {
  if (!x) return fail(QW_EINVAL, "x is null");
  if (x->ndim < 1 || x->ndim > 4) return fail(QW_EINVAL, "x must have 1 to 4 dimensions");
  for (int i = 0; i < x->ndim; ++i)
    if (x->shape[i] < 0) return fail(QW_EINVAL, "x has a negative dimension");
  if (numel(x) > 0 && x->data == nullptr) return fail(QW_EINVAL, "x has a null data pointer");
  *ld = K;
  if (contiguous(x)) return QW_OK;
  const int last = x->ndim - 1;
  if (x->shape[last] != 1 && x->strides[last] != 1)
    return fail(QW_EINVAL, "x's last dimension must be contiguous");
  int64_t rows = 1;
  for (int i = 0; i < last; ++i) rows *= x->shape[i];
  if (rows <= 1) return QW_OK;
  // The leading dimensions must collapse into one row index: going outwards,
  // each stride equals the next inner one times that dimension's size.
  int64_t step = 0, inner = -1;
  for (int i = last - 1; i >= 0; --i) {
    if (x->shape[i] == 1) continue;
    if (inner < 0) {
      step = x->strides[i];
    } else if (x->strides[i] != inner) {
      return fail(QW_EINVAL, "x's leading dimensions must be contiguous over its rows");
    }
    inner = x->strides[i] * x->shape[i];
  }
  if (step < K) return fail(QW_EINVAL, "x's rows overlap (row stride below K)");
  if ((step * 2) % 16 != 0) return fail(QW_EINVAL, "x's row stride must be a multiple of 8 elements");
  *ld = step;
  return QW_OK;
}

// Mode / bits / group checks in the order of the reference's validators:
// mode allowlist (layers.rs:1367-1380), biases presence (layers.rs:1409-1440),
// bits and group bounds (layers.rs:1286-1318).
int check_quant_params(const char* mode, bool has_biases, int group_size, int bits) {
  if (!mode) return fail(QW_EINVAL, "mode is null");
  const bool affine = std::strcmp(mode, "affine") == 0;
  const bool blockfloat =
      std::strcmp(mode, "mxfp4") == 0 || std::strcmp(mode, "mxfp8") == 0 || std::strcmp(mode, "nvfp4") == 0;
  if (!affine && !blockfloat)
    return fail(QW_EINVAL, std::string("quantization mode \"") + mode +
                               "\" must be one of affine, mxfp4, mxfp8, nvfp4");
  if (affine && !has_biases) return fail(QW_EINVAL, "affine quantization requires biases");
  if (!affine && has_biases)
    return fail(QW_EINVAL, std::string("biases must be null for quantization mode \"") + mode + "\"");
  if (bits < 1 || bits > 32) return fail(QW_EINVAL, "bits must be between 1 and 32");
  if (group_size < 1 || group_size > (1 << 20)) return fail(QW_EINVAL, "group_size must be between 1 and 2^20");
  if (!affine) return fail(QW_EUNSUPPORTED, std::string("quantization mode \"") + mode + "\" is not supported");
  if ((bits != 4 && bits != 8) || (group_size != 64 && group_size != 128))
    return fail(QW_EUNSUPPORTED, "affine quantization is supported with bits 4 or 8 and group_size 64 or 128 (got bits=" +
                                     std::to_string(bits) + ", group_size=" + std::to_string(group_size) + ")");
  return QW_OK;
}

// Every supported configuration (4- or 8-bit codes in groups of 64 or 128)
// has the skinny decode kernel; chained launches take 4-bit codes.
bool skinny_config(int group_size, int bits) {
  return (bits == 4 || bits == 8) && (group_size == 64 || group_size == 128);
}
bool skinny_chain_config(int group_size, int bits) { return bits == 4 && skinny_config(group_size, bits); }

struct WeightDims {
  int64_t N, K, G;
};

// Packed-weight invariants (layers.rs:1568-1570, :1783-1868).
int check_weights(const qw_array* w, const qw_array* scales, const qw_array* biases, int group_size, int bits,
                  WeightDims* d) {
  int rc;
  if ((rc = check_array(w, "w")) || (rc = check_array(scales, "scales")) ||
      (biases && (rc = check_array(biases, "biases"))))
    return rc;
  if (w->dtype != QW_U32) return fail(QW_EINVAL, std::string("w must be uint32, got ") + dtype_name(w->dtype));
  if (w->ndim != 2) return fail(QW_EUNSUPPORTED, "w must be 2-D [N, K*bits/32]");
  if (scales->ndim != 2 || scales->shape[0] != w->shape[0])
    return fail(QW_EINVAL, "scales must be 2-D with the same row count as w");
  if (biases && (biases->ndim != scales->ndim || biases->shape[0] != scales->shape[0] ||
                 biases->shape[1] != scales->shape[1]))
    return fail(QW_EINVAL, "biases must have the same shape as scales");
  if (scales->dtype != QW_F16 || (biases && biases->dtype != QW_F16))
    return fail(QW_EUNSUPPORTED, std::string("scales/biases must be float16, got ") + dtype_name(scales->dtype));
  const int64_t packed_in = w->shape[1];
  const int64_t groups = scales->shape[1];
  if (packed_in * 32 != (int64_t)bits * groups * group_size)
    return fail(QW_EINVAL, "packed width " + std::to_string(packed_in) + " at " + std::to_string(bits) +
                               "-bit does not match " + std::to_string(groups) + " groups of " +
                               std::to_string(group_size));
  d->N = w->shape[0];
  d->K = packed_in * 32 / bits;
  d->G = groups;
  if (d->N > (int64_t)1 << 30 || d->K > (int64_t)1 << 28)
    return fail(QW_EUNSUPPORTED, "matrix dimensions beyond the supported range");
  if (!aligned(w->data, 16) || !aligned(scales->data, 16) || (biases && !aligned(biases->data, 16)))
    return fail(QW_EINVAL, "w, scales and biases must be 16-byte aligned");
  return QW_OK;
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int cuda_fail(cudaError_t e, const char* where) {
  return fail(QW_ECUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

// The up projection of a SwiGLU call (null for a plain matmul).
struct UpProj {
  const qw_array* w;
  const qw_array* scales;
  const qw_array* biases;
};

// Core of the matmul entry points.  y may be f16 or f32.  With `up`, w /
// scales / biases are the gate projection and y = silu(x gate^T) * (x up^T).
int run_qmm(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases, int transpose,
            int group_size, int bits, const char* mode, qw_array* y, void* stream_v, const UpProj* up = nullptr) {
  int rc;
  if ((rc = check_quant_params(mode, biases != nullptr, group_size, bits))) return rc;
  if (up && (rc = check_quant_params(mode, up->biases != nullptr, group_size, bits))) return rc;
  if (!transpose) return fail(QW_EUNSUPPORTED, "transpose=false is not supported");
  WeightDims d;
  if ((rc = check_weights(w, scales, biases, group_size, bits, &d))) return rc;
  if (up) {
    WeightDims du;
    if ((rc = check_weights(up->w, up->scales, up->biases, group_size, bits, &du))) return rc;
    if (du.N != d.N || du.K != d.K)
      return fail(QW_EINVAL, "gate and up projections must have the same shape (gate " + std::to_string(d.N) + "x" +
                                 std::to_string(d.K) + ", up " + std::to_string(du.N) + "x" + std::to_string(du.K) +
                                 ")");
  }
  int64_t x_ld = 0;
  if ((rc = check_x_rows(x, d.K, &x_ld)) || (rc = check_array(y, "y"))) return rc;
  if (x->dtype != QW_F16) return fail(QW_EUNSUPPORTED, std::string("x must be float16, got ") + dtype_name(x->dtype));
  if (x->shape[x->ndim - 1] != d.K)
    return fail(QW_EINVAL, "x's last dimension " + std::to_string(x->shape[x->ndim - 1]) +
                               " does not match the weights' input width " + std::to_string(d.K));
  const int64_t M = numel(x) / (d.K ? d.K : 1);
  if (y->dtype != QW_F16 && y->dtype != QW_F32)
    return fail(QW_EINVAL, std::string("y must be float16 or float32, got ") + dtype_name(y->dtype));
  if (y->shape[y->ndim - 1] != d.N || numel(y) != M * d.N)
    return fail(QW_EINVAL, "y must have shape [..., N] with the leading dimensions of x");
  if (M == 0 || d.N == 0) return QW_OK;
  if (!aligned(x->data, 16)) return fail(QW_EINVAL, "x must be 16-byte aligned");
  if (!aligned(y->data, y->dtype == QW_F32 ? 4 : 2)) return fail(QW_EINVAL, "y is misaligned");

  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DeviceRes* res = nullptr;
  std::string err;
  if (!device_res(dev, &res, &err)) return fail(QW_ENOMEM, err);
  cudaStream_t stream = as_stream(stream_v);
  const bool y32 = y->dtype == QW_F32;
  const size_t ysz = y32 ? 4 : 2;

  if ((M > 16 || !skinny_config(group_size, bits)) && prefill_available()) {
    PrefillArgs pa{x->data, (const uint32_t*)w->data, scales->data, biases->data, y->data, y32, M, d.N, d.K,
                   res->status};
    pa.x_ld = x_ld;
    pa.bits = bits;
    pa.group_size = group_size;
    if (up) {
      pa.swiglu = true;
      pa.w2 = (const uint32_t*)up->w->data;
      pa.scales2 = up->scales->data;
      pa.biases2 = up->biases->data;
    }
    ce = launch_prefill(pa, stream, pdl_enabled(), &err);
    if (ce != cudaSuccess) return err.empty() ? cuda_fail(ce, "prefill launch") : fail(QW_ECUDA, err);
    return QW_OK;
  }
  // Skinny path, 16 rows of x per launch.
  for (int64_t m0 = 0; m0 < M; m0 += 16) {
    const int64_t mb = (M - m0) < 16 ? (M - m0) : 16;
    SkinnyArgs sa{};
    sa.x = static_cast<const uint8_t*>(x->data) + m0 * x_ld * 2;
    sa.x_ld = x_ld;
    sa.w = (const uint32_t*)w->data;
    sa.scales = scales->data;
    sa.biases = biases->data;
    sa.y = static_cast<uint8_t*>(y->data) + m0 * d.N * ysz;
    sa.y_f32 = y32;
    sa.M = mb;
    sa.N = d.N;
    sa.K = d.K;
    sa.max_ctas = 0;
    sa.status = res->status;
    sa.group_size = group_size;
    sa.bits = bits;
    if (up) {
      sa.swiglu = true;
      sa.w2 = (const uint32_t*)up->w->data;
      sa.scales2 = up->scales->data;
      sa.biases2 = up->biases->data;
    }
    Scratch sc;
    if (!scratch_for(dev, stream, skinny_scratch_bytes(sa, dev), &sc, &err)) return fail(QW_ENOMEM, err);
    ce = launch_skinny(sa, sc, stream, pdl_enabled(), &err);
    if (ce != cudaSuccess) return err.empty() ? cuda_fail(ce, "skinny launch") : fail(QW_ECUDA, err);
  }
  return QW_OK;
}

// Per-(device, stream) device buffer for an intermediate activation (the
// MLP's silu(gate) * up), kept apart from the kernels' scratch.  Grows on
// demand like the scratch.
std::map<std::pair<int, cudaStream_t>, Scratch> g_act;

bool activation_for(int device, cudaStream_t stream, size_t bytes, void** out, std::string* err) {
  std::lock_guard<std::mutex> lock(g_res_mu);
  Scratch& s = g_act[{device, stream}];
  if (s.bytes < bytes) {
    if (s.base) {
      cudaStreamSynchronize(stream);
      cudaFree(s.base);
      s = Scratch{};
    }
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
      cudaGetLastError();
      *err = "activation buffer allocation of " + std::to_string(bytes) + " bytes failed";
      return false;
    }
    s.base = p;
    s.bytes = bytes;
  }
  *out = s.base;
  return true;
}

}  // namespace

int check_qmm_call(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases,
                   int transpose, int group_size, int bits, const char* mode, qw_array* y, SkinnyArgs* sa) {
  int rc;
  if ((rc = check_quant_params(mode, biases != nullptr, group_size, bits))) return rc;
  if (!transpose) return fail(QW_EUNSUPPORTED, "transpose=false is not supported");
  WeightDims d;
  if ((rc = check_weights(w, scales, biases, group_size, bits, &d))) return rc;
  int64_t x_ld = 0;
  if ((rc = check_x_rows(x, d.K, &x_ld)) || (rc = check_array(y, "y"))) return rc;
  if (x->dtype != QW_F16) return fail(QW_EUNSUPPORTED, std::string("x must be float16, got ") + dtype_name(x->dtype));
  if (x->shape[x->ndim - 1] != d.K)
    return fail(QW_EINVAL, "x's last dimension " + std::to_string(x->shape[x->ndim - 1]) +
                               " does not match the weights' input width " + std::to_string(d.K));
  const int64_t M = numel(x) / (d.K ? d.K : 1);
  if (y->dtype != QW_F16 && y->dtype != QW_F32)
    return fail(QW_EINVAL, std::string("y must be float16 or float32, got ") + dtype_name(y->dtype));
  if (y->shape[y->ndim - 1] != d.N || numel(y) != M * d.N)
    return fail(QW_EINVAL, "y must have shape [..., N] with the leading dimensions of x");
  *sa = SkinnyArgs{};
  sa->x = x->data;
  sa->w = (const uint32_t*)w->data;
  sa->scales = scales->data;
  sa->biases = biases->data;
  sa->y = y->data;
  sa->y_f32 = y->dtype == QW_F32;
  sa->M = M;
  sa->N = d.N;
  sa->K = d.K;
  sa->x_ld = x_ld;
  sa->group_size = group_size;
  sa->bits = bits;
  if (M == 0 || d.N == 0) return QW_OK;
  if (!aligned(x->data, 16)) return fail(QW_EINVAL, "x must be 16-byte aligned");
  if (!aligned(y->data, y->dtype == QW_F32 ? 4 : 2)) return fail(QW_EINVAL, "y is misaligned");
  return QW_OK;
}

}  // namespace qw

using namespace qw;

extern "C" {

int qw_quantized_matmul(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases,
                        int transpose, int group_size, int bits, const char* mode, qw_array* y, void* stream) {
  set_error("");
  return run_qmm(x, w, scales, biases, transpose, group_size, bits, mode, y, stream);
}

int qw_quantized_matmul_chain(const qw_qmm_op* ops, int n_ops, int group_size, int bits, const char* mode,
                              void* stream_v) {
  set_error("");
  if (n_ops < 0) return fail(QW_EINVAL, "n_ops must not be negative");
  if (n_ops > 0 && !ops) return fail(QW_EINVAL, "ops is null");
  if (n_ops == 0) return QW_OK;
  std::vector<SkinnyArgs> args((size_t)n_ops);
  int rc;
  for (int i = 0; i < n_ops; ++i) {
    const qw_qmm_op& o = ops[i];
    if ((rc = check_qmm_call(o.x, o.w, o.scales, o.biases, 1, group_size, bits, mode, o.y, &args[i]))) {
      set_error("op " + std::to_string(i) + ": " + last_error());
      return rc;
    }
    if (args[i].M != args[0].M)
      return fail(QW_EINVAL, "op " + std::to_string(i) + " has " + std::to_string(args[i].M) +
                                 " rows of x, op 0 has " + std::to_string(args[0].M));
  }
  const int64_t M = args[0].M;
  if (M > 16 || args[0].M == 0 || !skinny_chain_config(group_size, bits)) {
    // Prefill-sized (or empty) chains: one launch per matmul, in order.
    for (int i = 0; i < n_ops; ++i) {
      const qw_qmm_op& o = ops[i];
      if ((rc = run_qmm(o.x, o.w, o.scales, o.biases, 1, group_size, bits, mode, o.y, stream_v))) return rc;
    }
    return QW_OK;
  }
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DeviceRes* res = nullptr;
  std::string err;
  if (!device_res(dev, &res, &err)) return fail(QW_ENOMEM, err);
  cudaStream_t stream = as_stream(stream_v);
  size_t need = 0;
  for (auto& a : args) {
    a.status = res->status;
    a.max_ctas = 0;
    const size_t b = skinny_scratch_bytes(a, dev);
    need = b > need ? b : need;
  }
  Scratch sc;
  if (!scratch_for(dev, stream, need, &sc, &err)) return fail(QW_ENOMEM, err);
  // Matmuls with no rows of y (N == 0) have nothing to compute.
  std::vector<SkinnyArgs> live;
  live.reserve(args.size());
  for (auto& a : args)
    if (a.N > 0) live.push_back(a);
  for (size_t i0 = 0; i0 < live.size(); i0 += kSkinnyChainMax) {
    const int n = (int)std::min(live.size() - i0, (size_t)kSkinnyChainMax);
    ce = launch_skinny_chain(live.data() + i0, n, sc, stream, &err);
    if (ce != cudaSuccess) return err.empty() ? cuda_fail(ce, "chained skinny launch") : fail(QW_ECUDA, err);
  }
  return QW_OK;
}

namespace {

// Checks of a greedy-token call (qw_quantized_matmul_argmax and
// qw_allreduce_argmax); on QW_OK fills the weight shape, the rows M of x and
// x's row step.
int check_argmax_call(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases,
                      int group_size, int bits, const char* mode, const qw_array* logits, const qw_array* idx,
                      WeightDims* d, int64_t* M_out, int64_t* x_ld) {
  int rc;
  if ((rc = check_quant_params(mode, biases != nullptr, group_size, bits))) return rc;
  if ((rc = check_weights(w, scales, biases, group_size, bits, d))) return rc;
  if ((rc = check_x_rows(x, d->K, x_ld)) || (rc = check_array(idx, "idx"))) return rc;
  if (logits && (rc = check_array(logits, "logits"))) return rc;
  if (x->dtype != QW_F16) return fail(QW_EUNSUPPORTED, std::string("x must be float16, got ") + dtype_name(x->dtype));
  if (x->shape[x->ndim - 1] != d->K)
    return fail(QW_EINVAL, "x's last dimension " + std::to_string(x->shape[x->ndim - 1]) +
                               " does not match the weights' input width " + std::to_string(d->K));
  const int64_t M = numel(x) / (d->K ? d->K : 1);
  if (idx->dtype != QW_U32 || numel(idx) != M)
    return fail(QW_EINVAL, "idx must be uint32 with one element per row of x");
  if (logits && (logits->dtype != QW_F16 || logits->shape[logits->ndim - 1] != d->N || numel(logits) != M * d->N))
    return fail(QW_EINVAL, "logits must be float16 [..., N] with the leading dimensions of x");
  if (M > 0 && d->N == 0) return fail(QW_EINVAL, "argmax over an empty row (N == 0)");
  if (M > 0 && (!aligned(x->data, 16) || !aligned(idx->data, 4) || (logits && !aligned(logits->data, 2))))
    return fail(QW_EINVAL, "x must be 16-byte aligned, idx 4-byte aligned");
  if (M > 16 || !skinny_config(group_size, bits))
    if (!logits) return fail(QW_EINVAL, "a logits buffer is required when x has more than 16 rows");
  *M_out = M;
  return QW_OK;
}

// keys[m] = (order-preserving fp16 logit << 32) | (2^32 - 1 - row) of the best
// row of each of the M rows of x: folded into the decode kernel's epilogue for
// up to 16 rows (logits written only if given), else the matmul into logits
// and a row reduction.
int argmax_keys(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases,
                int group_size, int bits, const char* mode, qw_array* logits, const WeightDims& d, int64_t M,
                int64_t x_ld, unsigned long long* keys, void* stream_v) {
  cudaStream_t stream = as_stream(stream_v);
  cudaError_t ce;
  int rc;
  if (M > 16 || !skinny_config(group_size, bits)) {
    if ((rc = run_qmm(x, w, scales, biases, 1, group_size, bits, mode, logits, stream_v))) return rc;
    ce = launch_argmax_rows_keys(logits->data, M, d.N, keys, stream);
    return ce == cudaSuccess ? QW_OK : cuda_fail(ce, "argmax launch");
  }
  int dev = 0;
  ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DeviceRes* res = nullptr;
  std::string err;
  if (!device_res(dev, &res, &err)) return fail(QW_ENOMEM, err);
  SkinnyArgs sa{};
  sa.x = x->data;
  sa.w = (const uint32_t*)w->data;
  sa.scales = scales->data;
  sa.biases = biases->data;
  sa.y = logits ? logits->data : nullptr;
  sa.y_f32 = false;
  sa.M = M;
  sa.N = d.N;
  sa.K = d.K;
  sa.max_ctas = 0;
  sa.status = res->status;
  sa.x_ld = x_ld;
  sa.group_size = group_size;
  sa.bits = bits;
  Scratch sc;
  if (!scratch_for(dev, stream, skinny_scratch_bytes(sa, dev), &sc, &err)) return fail(QW_ENOMEM, err);
  ce = cudaMemsetAsync(keys, 0, (size_t)M * sizeof(unsigned long long), stream);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaMemsetAsync");
  sa.amax = keys;
  ce = launch_skinny(sa, sc, stream, pdl_enabled(), &err);
  if (ce != cudaSuccess) return err.empty() ? cuda_fail(ce, "skinny launch") : fail(QW_ECUDA, err);
  return QW_OK;
}

}  // namespace

int qw_quantized_matmul_argmax(const qw_array* x, const qw_array* w, const qw_array* scales,
                               const qw_array* biases, int group_size, int bits, const char* mode, qw_array* logits,
                               qw_array* idx, void* stream_v) {
  set_error("");
  WeightDims d;
  int64_t M = 0, x_ld = 0;
  int rc = check_argmax_call(x, w, scales, biases, group_size, bits, mode, logits, idx, &d, &M, &x_ld);
  if (rc != QW_OK) return rc;
  if (M == 0) return QW_OK;
  cudaStream_t stream = as_stream(stream_v);
  cudaError_t ce;
  if (M > 16 || !skinny_config(group_size, bits)) {
    if ((rc = run_qmm(x, w, scales, biases, 1, group_size, bits, mode, logits, stream_v))) return rc;
    ce = launch_argmax_rows(logits->data, M, d.N, (uint32_t*)idx->data, stream);
    return ce == cudaSuccess ? QW_OK : cuda_fail(ce, "argmax launch");
  }
  int dev = 0;
  ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  std::string err;
  Scratch sc;
  SkinnyArgs probe{};
  probe.M = M;
  probe.N = d.N;
  probe.K = d.K;
  if (!scratch_for(dev, stream, skinny_scratch_bytes(probe, dev), &sc, &err)) return fail(QW_ENOMEM, err);
  // keys in the first 256 bytes of the scratch (the chains' tallies use the first 96)
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(sc.base) + 128);
  if ((rc = argmax_keys(x, w, scales, biases, group_size, bits, mode, logits, d, M, x_ld, keys, stream_v)))
    return rc;
  ce = launch_argmax_finalize(keys, (uint32_t*)idx->data, M, stream);
  return ce == cudaSuccess ? QW_OK : cuda_fail(ce, "argmax launch");
}

int qw_quantized_matmul_swiglu(const qw_array* x, const qw_array* w_gate, const qw_array* scales_gate,
                               const qw_array* biases_gate, const qw_array* w_up, const qw_array* scales_up,
                               const qw_array* biases_up, int transpose, int group_size, int bits, const char* mode,
                               qw_array* y, void* stream) {
  set_error("");
  const UpProj up{w_up, scales_up, biases_up};
  return run_qmm(x, w_gate, scales_gate, biases_gate, transpose, group_size, bits, mode, y, stream, &up);
}

int qw_swiglu_activation(const qw_array* gate, const qw_array* up, qw_array* y, void* stream) {
  set_error("");
  int rc;
  if ((rc = check_array(gate, "gate")) || (rc = check_array(up, "up")) || (rc = check_array(y, "y"))) return rc;
  if (gate->dtype != QW_F16 || up->dtype != QW_F16 || y->dtype != QW_F16)
    return fail(QW_EUNSUPPORTED, "gate, up and y must be float16");
  const int64_t n = numel(gate);
  if (numel(up) != n || numel(y) != n || gate->ndim != up->ndim || gate->ndim != y->ndim)
    return fail(QW_EINVAL, "gate, up and y must have the same shape");
  for (int i = 0; i < gate->ndim; ++i)
    if (gate->shape[i] != up->shape[i] || gate->shape[i] != y->shape[i])
      return fail(QW_EINVAL, "gate, up and y must have the same shape");
  const cudaError_t ce = launch_swiglu(gate->data, up->data, y->data, n, as_stream(stream));
  return ce == cudaSuccess ? QW_OK : cuda_fail(ce, "swiglu launch");
}

int qw_swiglu_mlp(const qw_array* x, const qw_array* w_gate, const qw_array* scales_gate, const qw_array* biases_gate,
                  const qw_array* w_up, const qw_array* scales_up, const qw_array* biases_up, const qw_array* w_down,
                  const qw_array* scales_down, const qw_array* biases_down, int group_size, int bits,
                  const char* mode, qw_array* y, void* stream_v) {
  set_error("");
  int rc;
  if ((rc = check_array(w_gate, "w_gate"))) return rc;
  if (w_gate->ndim != 2) return fail(QW_EUNSUPPORTED, "w_gate must be 2-D [N, K*bits/32]");
  if (!x) return fail(QW_EINVAL, "x is null");
  if (x->ndim < 1 || x->ndim > 4) return fail(QW_EINVAL, "x must have 1 to 4 dimensions");
  const int64_t inter = w_gate->shape[0];
  const int64_t K = x->ndim ? x->shape[x->ndim - 1] : 0;
  const int64_t M = K ? numel(x) / K : 0;
  // h = silu(x gate^T) * (x up^T), [M, inter] fp16, in this stream's activation buffer
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  void* hbuf = nullptr;
  std::string err;
  const size_t hbytes = (size_t)(M * inter) * 2;
  if (hbytes && !activation_for(dev, as_stream(stream_v), hbytes, &hbuf, &err)) return fail(QW_ENOMEM, err);
  qw_array h{};
  h.data = hbuf;
  h.dtype = QW_F16;
  h.ndim = 2;
  h.shape[0] = M;
  h.shape[1] = inter;
  h.strides[0] = inter;
  h.strides[1] = 1;
  const UpProj up{w_up, scales_up, biases_up};
  if ((rc = run_qmm(x, w_gate, scales_gate, biases_gate, 1, group_size, bits, mode, &h, stream_v, &up))) return rc;
  return run_qmm(&h, w_down, scales_down, biases_down, 1, group_size, bits, mode, y, stream_v);
}

// Checks shared by the top-k entry points: logits f16 [..., N] contiguous,
// idx u32 and values f16 (nullable) [..., k] with the same leading dims.
static int check_topk(const qw_array* logits, int64_t N, int k, const qw_array* idx, const qw_array* values,
                      int64_t* M) {
  int rc;
  if ((rc = check_array(idx, "idx")) || (values && (rc = check_array(values, "values")))) return rc;
  if (k < 1 || (int64_t)k >= N)
    return fail(QW_EINVAL, "k=" + std::to_string(k) + " must be in 1.." + std::to_string(N - 1) +
                               " for rows of " + std::to_string(N) + " logits");
  if (k > topk_max_k())
    return fail(QW_EUNSUPPORTED, "k=" + std::to_string(k) + " is above the supported " +
                                     std::to_string(topk_max_k()));
  if (N > topk_max_n())
    return fail(QW_EUNSUPPORTED, "rows of " + std::to_string(N) + " logits are above the supported " +
                                     std::to_string(topk_max_n()));
  *M = numel(logits) / N;
  if (idx->dtype != QW_U32 || idx->shape[idx->ndim - 1] != k || numel(idx) != *M * k)
    return fail(QW_EINVAL, "idx must be uint32 [..., k] with the leading dimensions of the logits");
  if (values && (values->dtype != QW_F16 || values->shape[values->ndim - 1] != k || numel(values) != *M * k))
    return fail(QW_EINVAL, "values must be float16 [..., k] with the leading dimensions of the logits");
  if (!aligned(idx->data, 4) || (values && !aligned(values->data, 2)))
    return fail(QW_EINVAL, "idx or values misaligned");
  return QW_OK;
}

int qw_topk(const qw_array* logits, int k, qw_array* idx, qw_array* values, void* stream) {
  set_error("");
  int rc;
  if ((rc = check_array(logits, "logits"))) return rc;
  if (logits->dtype != QW_F16) return fail(QW_EUNSUPPORTED, "logits must be float16");
  const int64_t N = logits->shape[logits->ndim - 1];
  int64_t M = 0;
  if ((rc = check_topk(logits, N, k, idx, values, &M))) return rc;
  const cudaError_t ce =
      launch_topk_rows(logits->data, N, M, N, k, (uint32_t*)idx->data, values ? values->data : nullptr,
                       as_stream(stream));
  return ce == cudaSuccess ? QW_OK : cuda_fail(ce, "top-k launch");
}

int qw_quantized_matmul_topk(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases,
                             int group_size, int bits, const char* mode, int k, qw_array* logits, qw_array* idx,
                             qw_array* values, void* stream_v) {
  set_error("");
  int rc;
  if ((rc = check_array(w, "w"))) return rc;
  if (w->ndim != 2) return fail(QW_EUNSUPPORTED, "w must be 2-D [N, K*bits/32]");
  if (!x) return fail(QW_EINVAL, "x is null");
  if (x->ndim < 1 || x->ndim > 4) return fail(QW_EINVAL, "x must have 1 to 4 dimensions");
  const int64_t N = w->shape[0];
  const int64_t K = x->shape[x->ndim - 1];
  const int64_t M = K ? numel(x) / K : 0;
  qw_array lg{};
  if (logits) {
    lg = *logits;
  } else {
    // logits in this stream's activation buffer
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
    std::string err;
    void* buf = nullptr;
    const size_t bytes = (size_t)(M * N) * 2;
    if (bytes && !activation_for(dev, as_stream(stream_v), bytes, &buf, &err)) return fail(QW_ENOMEM, err);
    lg.data = buf;
    lg.dtype = QW_F16;
    lg.ndim = 2;
    lg.shape[0] = M;
    lg.shape[1] = N;
    lg.strides[0] = N;
    lg.strides[1] = 1;
  }
  if (lg.dtype != QW_F16) return fail(QW_EINVAL, "logits must be float16");
  int64_t Mk = 0;
  if ((rc = check_topk(&lg, N, k, idx, values, &Mk))) return rc;
  if ((rc = run_qmm(x, w, scales, biases, 1, group_size, bits, mode, &lg, stream_v))) return rc;
  if (M == 0) return QW_OK;
  const cudaError_t ce = launch_topk_rows(lg.data, N, M, N, k, (uint32_t*)idx->data,
                                          values ? values->data : nullptr, as_stream(stream_v));
  return ce == cudaSuccess ? QW_OK : cuda_fail(ce, "top-k launch");
}

// ------------------------------------------------------ peer allreduce
struct qw_allreduce {
  ArComm comm;
  int device = -1;
  void* own = nullptr;                 // this rank's shared buffer (cudaMalloc)
  bool opened[kArMaxRanks] = {};       // peer buffers mapped through IPC
  int sm_count = 0;
  unsigned long long* keys = nullptr;  // greedy-token keys of this rank's shard, n_max / 2 rows
  float* partial = nullptr;            // this rank's fp32 product where the exchange is not fused, n_max
};

int qw_allreduce_init(int world, int rank, int64_t max_elems, qw_allreduce** out, unsigned char* handle) {
  set_error("");
  if (!out || !handle) return fail(QW_EINVAL, "out and handle must not be null");
  *out = nullptr;
  if (world < 1 || world > kArMaxRanks) return fail(QW_EUNSUPPORTED, "world size must be 1 to 8");
  if (rank < 0 || rank >= world) return fail(QW_EINVAL, "rank out of range");
  if (max_elems < 1 || max_elems > ((int64_t)1 << 28)) return fail(QW_EINVAL, "max_elems must be 1 to 2^28");
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DeviceRes* res = nullptr;
  std::string err;
  if (!device_res(dev, &res, &err)) return fail(QW_ENOMEM, err);
  auto* c = new qw_allreduce();
  c->device = dev;
  c->sm_count = device_info(dev).sm_count;
  c->comm.P = world;
  c->comm.rank = rank;
  c->comm.n_max = (max_elems + 3) / 4 * 4;  // keeps every slot 16-byte aligned
  c->comm.status = res->status;
  const size_t bytes = allreduce_buffer_bytes(world, c->comm.n_max);
  if ((ce = cudaMalloc(&c->own, bytes)) != cudaSuccess || (ce = cudaMemset(c->own, 0, bytes)) != cudaSuccess ||
      (ce = cudaMalloc(reinterpret_cast<void**>(&c->comm.counters), allreduce_epoch_bytes())) != cudaSuccess ||
      (ce = cudaMemset(c->comm.counters, 0, allreduce_epoch_bytes())) != cudaSuccess ||
      (ce = cudaMalloc(reinterpret_cast<void**>(&c->keys), (size_t)(c->comm.n_max / 2 + 1) * 8)) != cudaSuccess ||
      (ce = cudaMalloc(reinterpret_cast<void**>(&c->partial), (size_t)c->comm.n_max * sizeof(float))) != cudaSuccess) {
    cudaGetLastError();
    qw_allreduce_destroy(c);
    return cuda_fail(ce, "allreduce buffer allocation");
  }
  c->comm.peer_bufs[rank] = c->own;
  cudaIpcMemHandle_t h;
  if ((ce = cudaIpcGetMemHandle(&h, c->own)) != cudaSuccess) {
    qw_allreduce_destroy(c);
    return cuda_fail(ce, "cudaIpcGetMemHandle");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == QW_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof h);
  *out = c;
  return QW_OK;
}

int qw_allreduce_connect(qw_allreduce* c, const unsigned char* handles) {
  set_error("");
  if (!c || !handles) return fail(QW_EINVAL, "comm and handles must not be null");
  for (int r = 0; r < c->comm.P; ++r) {
    if (r == c->comm.rank || c->opened[r]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles + (size_t)r * QW_IPC_HANDLE_BYTES, sizeof h);
    void* p = nullptr;
    const cudaError_t ce = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (ce != cudaSuccess) return cuda_fail(ce, ("cudaIpcOpenMemHandle of rank " + std::to_string(r)).c_str());
    c->comm.peer_bufs[r] = p;
    c->opened[r] = true;
  }
  return QW_OK;
}

}  // extern "C"

namespace {
// A communicator call runs on the communicator's device, once every rank's
// buffer is mapped.
int check_comm_ready(const qw_allreduce* c) {
  if (!c) return fail(QW_EINVAL, "comm is null");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != c->device)
    return fail(QW_EINVAL, "the current device is not the communicator's (device " + std::to_string(c->device) + ")");
  for (int r = 0; r < c->comm.P; ++r)
    if (!c->comm.peer_bufs[r]) return fail(QW_EINVAL, "rank " + std::to_string(r) + " is not connected");
  return QW_OK;
}
}  // namespace

extern "C" {

int qw_allreduce_sum(qw_allreduce* c, const qw_array* partial, qw_array* y, void* stream) {
  set_error("");
  int rc;
  if ((rc = check_comm_ready(c))) return rc;
  if ((rc = check_array(partial, "partial")) || (rc = check_array(y, "y"))) return rc;
  if (partial->dtype != QW_F32) return fail(QW_EINVAL, "partial must be float32");
  if (y->dtype != QW_F16 && y->dtype != QW_F32) return fail(QW_EINVAL, "y must be float16 or float32");
  const int64_t n = numel(partial);
  if (numel(y) != n) return fail(QW_EINVAL, "y must have as many elements as partial");
  if (n > c->comm.n_max)
    return fail(QW_EINVAL, std::to_string(n) + " elements exceed the communicator's " +
                               std::to_string(c->comm.n_max));
  const bool y32 = y->dtype == QW_F32;
  const bool vec = n % 4 == 0 && aligned(partial->data, 16) && aligned(y->data, y32 ? 16 : 8);
  const cudaError_t ce = launch_allreduce(c->comm, static_cast<const float*>(partial->data), y->data, y32, vec, n,
                                          c->sm_count, as_stream(stream));
  return ce == cudaSuccess ? QW_OK : cuda_fail(ce, "allreduce launch");
}

int qw_allreduce_matmul(qw_allreduce* c, const qw_array* x, const qw_array* w, const qw_array* scales,
                        const qw_array* biases, int group_size, int bits, const char* mode, qw_array* y,
                        void* stream) {
  set_error("");
  int rc;
  if ((rc = check_comm_ready(c))) return rc;
  SkinnyArgs sa;
  if ((rc = check_qmm_call(x, w, scales, biases, 1, group_size, bits, mode, y, &sa))) return rc;
  const int64_t n = sa.M * sa.N;
  if (n > c->comm.n_max)
    return fail(QW_EINVAL, std::to_string(n) + " output elements exceed the communicator's " +
                               std::to_string(c->comm.n_max));
  if (n == 0) return QW_OK;  // nothing is launched, on every rank alike
  cudaStream_t st = as_stream(stream);
  sa.ar = &c->comm;
  if (skinny_config(group_size, bits) && skinny_exchange_fits(sa) && n <= allreduce_ll_elems(c->comm.n_max)) {
    DeviceRes* res = nullptr;
    std::string err;
    if (!device_res(c->device, &res, &err)) return fail(QW_ENOMEM, err);
    sa.status = res->status;
    Scratch sc;
    if (!scratch_for(c->device, st, skinny_scratch_bytes(sa, c->device), &sc, &err)) return fail(QW_ENOMEM, err);
    const cudaError_t ce = launch_skinny(sa, sc, st, pdl_enabled(), &err);
    if (ce != cudaSuccess) return err.empty() ? cuda_fail(ce, "skinny launch") : fail(QW_ECUDA, err);
    return QW_OK;
  }
  // Larger shapes: this rank's fp32 product, then the allreduce kernel.
  qw_array part{};
  part.data = c->partial;
  part.dtype = QW_F32;
  part.ndim = 2;
  part.shape[0] = sa.M;
  part.shape[1] = sa.N;
  if ((rc = run_qmm(x, w, scales, biases, 1, group_size, bits, mode, &part, stream))) return rc;
  const bool y32 = y->dtype == QW_F32;
  const bool vec = n % 4 == 0 && aligned(y->data, y32 ? 16 : 8);
  const cudaError_t ce = launch_allreduce(c->comm, c->partial, y->data, y32, vec, n, c->sm_count, st);
  return ce == cudaSuccess ? QW_OK : cuda_fail(ce, "allreduce launch");
}

int qw_allreduce_argmax(qw_allreduce* c, const qw_array* x, const qw_array* w, const qw_array* scales,
                        const qw_array* biases, int group_size, int bits, const char* mode, int64_t index_base,
                        qw_array* logits, qw_array* idx, void* stream) {
  set_error("");
  int rc;
  if ((rc = check_comm_ready(c))) return rc;
  WeightDims d;
  int64_t M = 0, x_ld = 0;
  if ((rc = check_argmax_call(x, w, scales, biases, group_size, bits, mode, logits, idx, &d, &M, &x_ld))) return rc;
  if (index_base < 0 || index_base + d.N > (int64_t)0xFFFFFFFF)
    return fail(QW_EINVAL, "the shard's rows [index_base, index_base + N) must lie below 2^32 - 1");
  if (2 * M > c->comm.n_max)
    return fail(QW_EINVAL, std::to_string(M) + " rows exceed the communicator's " +
                               std::to_string(c->comm.n_max / 2) + " (max_elems / 2)");
  if (M == 0) return QW_OK;  // nothing is launched, on every rank alike
  if ((rc = argmax_keys(x, w, scales, biases, group_size, bits, mode, logits, d, M, x_ld, c->keys, stream)))
    return rc;
  const cudaError_t ce = launch_argmax_exchange(c->comm, c->keys, index_base, (uint32_t*)idx->data, M,
                                                as_stream(stream));
  return ce == cudaSuccess ? QW_OK : cuda_fail(ce, "argmax exchange launch");
}

int qw_allreduce_destroy(qw_allreduce* c) {
  set_error("");
  if (!c) return QW_OK;
  // this rank's calls end before its buffers go (the peers' calls are the
  // caller's to wait for: a barrier across ranks)
  int prev = 0;
  cudaGetDevice(&prev);
  if (c->device >= 0 && cudaSetDevice(c->device) == cudaSuccess) cudaDeviceSynchronize();
  for (int r = 0; r < kArMaxRanks; ++r)
    if (c->opened[r]) cudaIpcCloseMemHandle(c->comm.peer_bufs[r]);
  if (c->own) cudaFree(c->own);
  if (c->comm.counters) cudaFree(c->comm.counters);
  if (c->keys) cudaFree(c->keys);
  if (c->partial) cudaFree(c->partial);
  cudaGetLastError();
  cudaSetDevice(prev);
  delete c;
  return QW_OK;
}

static int linear_common(const qw_array* x, const qw_array* w, const qw_array* scales, const qw_array* biases,
                         const qw_array* global_scale, const qw_array* linear_bias, int group_size, int bits,
                         const char* mode, qw_array* y, void* stream) {
  set_error("");
  int rc;
  if (y && y->dtype != QW_F16) return fail(QW_EINVAL, "linear forward output must be float16");
  if (global_scale) {
    if ((rc = check_array(global_scale, "global_scale"))) return rc;
    if (global_scale->dtype != QW_F32 || numel(global_scale) != 1)
      return fail(QW_EINVAL, "global_scale must be a float32 scalar");
  }
  if (linear_bias) {
    if ((rc = check_array(linear_bias, "linear_bias"))) return rc;
    if (linear_bias->dtype != QW_F16 || numel(linear_bias) != w->shape[0])
      return fail(QW_EINVAL, "linear_bias must be float16 with N elements");
  }
  if ((rc = run_qmm(x, w, scales, biases, 1, group_size, bits, mode, y, stream))) return rc;
  const int64_t N = w->shape[0];
  const int64_t M = N ? numel(y) / N : 0;
  cudaError_t ce = launch_affine_epilogue(y->data, linear_bias ? linear_bias->data : nullptr,
                                          global_scale ? (const float*)global_scale->data : nullptr, M, N,
                                          as_stream(stream));
  if (ce != cudaSuccess) return cuda_fail(ce, "epilogue launch");
  return QW_OK;
}

int qw_quantized_linear_forward(const qw_array* x, const qw_array* w, const qw_array* scales,
                                const qw_array* biases, const qw_array* linear_bias, int group_size, int bits,
                                const char* mode, qw_array* y, void* stream) {
  return linear_common(x, w, scales, biases, nullptr, linear_bias, group_size, bits, mode, y, stream);
}

int qw_quantized_linear_forward_global_scale(const qw_array* x, const qw_array* w, const qw_array* scales,
                                             const qw_array* biases, const qw_array* global_scale,
                                             const qw_array* linear_bias, int group_size, int bits,
                                             const char* mode, qw_array* y, void* stream) {
  return linear_common(x, w, scales, biases, global_scale, linear_bias, group_size, bits, mode, y, stream);
}

int qw_dequantize_rounding(const qw_array* w, const qw_array* scales, const qw_array* biases, int group_size,
                           int bits, const char* mode, int rounding, qw_array* out, void* stream) {
  set_error("");
  int rc;
  if ((rc = check_quant_params(mode, biases != nullptr, group_size, bits))) return rc;
  if (rounding != 0 && rounding != 1) return fail(QW_EINVAL, "rounding must be 0 or 1");
  WeightDims d;
  if ((rc = check_weights(w, scales, biases, group_size, bits, &d))) return rc;
  if ((rc = check_array(out, "out"))) return rc;
  if (out->dtype != QW_F16 || out->ndim != 2 || out->shape[0] != d.N || out->shape[1] != d.K)
    return fail(QW_EINVAL, "out must be float16 [N, K]");
  if (!aligned(out->data, 16)) return fail(QW_EINVAL, "out must be 16-byte aligned");
  cudaError_t ce = launch_dequantize((const uint32_t*)w->data, scales->data, biases->data, out->data, d.N, d.K,
                                     group_size, bits, rounding, as_stream(stream));
  if (ce != cudaSuccess) return cuda_fail(ce, "dequantize launch");
  return QW_OK;
}

int qw_dequantize(const qw_array* w, const qw_array* scales, const qw_array* biases, int group_size, int bits,
                  const char* mode, qw_array* out, void* stream) {
  return qw_dequantize_rounding(w, scales, biases, group_size, bits, mode, 0, out, stream);
}

int qw_quantize(const qw_array* w, int group_size, int bits, const char* mode, qw_array* wq, qw_array* scales,
                qw_array* biases, void* stream) {
  set_error("");
  int rc;
  if ((rc = check_quant_params(mode, biases != nullptr, group_size, bits))) return rc;
  if ((rc = check_array(w, "w")) || (rc = check_array(wq, "wq")) || (rc = check_array(scales, "scales")) ||
      (rc = check_array(biases, "biases")))
    return rc;
  if (w->dtype != QW_F16 || w->ndim != 2) return fail(QW_EUNSUPPORTED, "w must be float16 [N, K]");
  const int64_t N = w->shape[0], K = w->shape[1];
  if (K % group_size != 0) return fail(QW_EINVAL, "K must be a multiple of group_size");
  if (wq->dtype != QW_U32 || wq->ndim != 2 || wq->shape[0] != N || wq->shape[1] != K * bits / 32)
    return fail(QW_EINVAL, "wq must be uint32 [N, K*bits/32]");
  if (scales->dtype != QW_F16 || scales->ndim != 2 || scales->shape[0] != N || scales->shape[1] != K / group_size ||
      biases->dtype != QW_F16 || biases->ndim != 2 || biases->shape[0] != N || biases->shape[1] != K / group_size)
    return fail(QW_EINVAL, "scales and biases must be float16 [N, K/group_size]");
  if (!aligned(w->data, 16) || !aligned(wq->data, 16))
    return fail(QW_EINVAL, "w and wq must be 16-byte aligned");
  cudaError_t ce = launch_quantize(w->data, (uint32_t*)wq->data, scales->data, biases->data, N, K, group_size,
                                   bits, as_stream(stream));
  if (ce != cudaSuccess) return cuda_fail(ce, "quantize launch");
  return QW_OK;
}

const char* qw_last_error(void) { return qw::last_error(); }

int qw_device_status(int device, unsigned int* status, int clear) {
  set_error("");
  if (!status) return fail(QW_EINVAL, "status is null");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t ce = cudaSetDevice(device);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaSetDevice");
  // No allocation here: a device whose status word was never created ran no
  // kernel that could set it, and the static-scratch array exists already.
  unsigned int* lib_status = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_res_mu);
    auto it = g_dev_res.find(device);
    if (it != g_dev_res.end()) lib_status = it->second.status;
  }
  ce = cudaDeviceSynchronize();
  unsigned int v = 0, vs = 0;
  if (ce == cudaSuccess && lib_status) ce = cudaMemcpy(&v, lib_status, sizeof v, cudaMemcpyDeviceToHost);
  if (ce == cudaSuccess && clear && v != 0) {
    ce = cudaMemset(lib_status, 0, sizeof v);
    // A kernel that gave up may have left split-tile counters raised.
    std::lock_guard<std::mutex> lock(g_res_mu);
    for (auto& kv : g_scratch)
      if (kv.first.first == device && kv.second.base) cudaMemset(kv.second.base, 0, kv.second.bytes);
  }
  if (ce == cudaSuccess) ce = static_scratch_status(device, &vs, clear != 0);
  cudaSetDevice(prev);
  if (ce != cudaSuccess) return cuda_fail(ce, "reading the device status");
  if (v == 0) v = vs;
  *status = v;
  return v ? QW_ETIMEOUT : QW_OK;
}

int qw_decode_schedule(int64_t m, int64_t n, int64_t k, int bits, int group_size, int swiglu, int sm_count,
                       int64_t* out) {
  set_error("");
  if (!out) return fail(QW_EINVAL, "out is null");
  if (m < 1 || m > 16) return fail(QW_EINVAL, "the decode kernel takes 1 to 16 rows of x");
  if (!skinny_config(group_size, bits))
    return fail(QW_EUNSUPPORTED, "the decode kernel takes bits 4 or 8 in groups of 64 or 128");
  if (n < 1 || k < 1 || k % group_size != 0 || n > ((int64_t)1 << 30) || k > ((int64_t)1 << 28))
    return fail(QW_EINVAL, "n and k must be positive, k a multiple of group_size");
  if (sm_count < 1) return fail(QW_EINVAL, "sm_count must be positive");
  SkinnyArgs a{};
  a.M = m;
  a.N = n;
  a.K = k;
  a.bits = bits;
  a.group_size = group_size;
  a.swiglu = swiglu != 0;
  const SkinnySchedule sc = skinny_schedule(a, sm_count);
  out[0] = sc.tokens;
  out[1] = sc.unit_k;
  out[2] = sc.ctas;
  out[3] = sc.split;
  out[4] = sc.busiest_units;
  return QW_OK;
}

int qw_abi_version(void) { return QW_ABI_VERSION; }

}  // extern "C"
