// qw_static_scratch.cu -- qw_quantized_matmul_static_scratch: the skinny
// quantized matmul (at most 16 rows of x per call) with its scratch taken
// from a fixed array in device memory instead of memory the library
// allocates.
//
// Who needs it.  qw_quantized_matmul allocates, on first use, a status word
// per device and a scratch buffer per (device, stream), and grows the buffer
// (cudaFree + cudaMalloc) when a larger shape needs more.  Some callers cannot
// have that happen inside a matmul call:
//  - a runtime that reserves all of the GPU's memory up front for its own pool
//    (weights, KV cache, activations), so that a library's cudaMalloc fails or
//    pushes the pool out of memory at an arbitrary point of serving;
//  - a decode loop with a latency budget per token: cudaFree waits for the
//    whole device to go idle, and a first call on a new stream would pay for
//    an allocation in the middle of the loop.
// This entry point calls no cudaMalloc, cudaFree or other allocating routine.
// The caller still passes every input and output; the only memory the path
// needs besides those is the array below, which exists once per device from
// the moment the library's code is loaded on that device until the process
// exits.
//
// Set-up.  A device array's name in host code is only a handle the runtime
// uses to look the array up, not an address a kernel can use.  The first call
// on a device (with that device current, as it is for the call) resolves the
// array's device address with cudaGetSymbolAddress, once, and caches it; that
// first call also loads the module holding the array on that device.  Make the
// first call on each device before any stream capture begins.
//
// Sharing.  Every call on a device uses the same array, and the array keeps
// whatever the previous call left in it.  Each call clears the part that must
// start at zero (the split-tile counters of its shape) on its own stream
// before its kernel runs; the partial sums need no clearing (every launch
// writes them before it reads them).  Two calls whose work overlaps on the GPU
// -- on different streams without an ordering between them, or from several
// host threads -- race on the array and may return wrong results.  Calls on
// one stream are ordered and safe.
//
// Limits: 4- or 8-bit weights in groups of 64 or 128 (the skinny kernel), 16 rows of x per
// call (its tile), and the scratch that the shape needs on this device at
// most kStaticScratchBytes minus the status word (a 256-byte header, the
// split-tile counters, 4 bytes per 128 output rows up to 256 KiB, plus two
// partial-sum slots of 128 x 16 floats per SM).  On a 148-SM B200 a call needs
// at most 2.6 MiB.  Other requests return QW_EUNSUPPORTED with a message.
//
// Errors: like qw_quantized_matmul's.  A kernel that gives up on one of its
// bounded waits records the cause in a status word at the start of this
// array; qw_device_status reads it (and clears it on request) together with
// the library's own status word, without allocating.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/qw_qmm.h"
#include "qw_internal.h"

namespace qw {

constexpr size_t kStaticScratchBytes = 4u << 20;  // 4 MiB on every device that loads the library
constexpr size_t kStaticStatusBytes = 256;        // status word, padded to keep the counters aligned
constexpr int64_t kStaticMaxRows = 16;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices];  // device address of g_static_scratch per device, once resolved

int static_fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

// Device address of the array on `device`, which must be the current device.
bool static_scratch_address(int device, void** out, std::string* err) {
  if (device < 0 || device >= kMaxDevices) {
    *err = "device ordinal " + std::to_string(device) + " is beyond the " + std::to_string(kMaxDevices) +
           " devices this entry point tracks";
    return false;
  }
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_ptr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *err = std::string("cudaGetSymbolAddress of the static scratch failed: ") + cudaGetErrorString(e);
      return false;
    }
    g_static_ptr[device] = p;
  }
  *out = g_static_ptr[device];
  return true;
}

}  // namespace

// The static array's status word on `device` (0 if no static-scratch call has
// run there), cleared when `clear`; allocates nothing.  The caller has made
// `device` current and synchronized it.
cudaError_t static_scratch_status(int device, unsigned int* v, bool clear) {
  *v = 0;
  void* p = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (device >= 0 && device < kMaxDevices) p = g_static_ptr[device];
  }
  if (p == nullptr) return cudaSuccess;  // never resolved: no call ran on this device
  cudaError_t ce = cudaMemcpy(v, p, sizeof *v, cudaMemcpyDeviceToHost);
  if (ce == cudaSuccess && clear && *v != 0) ce = cudaMemset(p, 0, sizeof *v);
  return ce;
}

}  // namespace qw

using namespace qw;

extern "C" int qw_quantized_matmul_static_scratch(const qw_array* x, const qw_array* w, const qw_array* scales,
                                                  const qw_array* biases, int transpose, int group_size, int bits,
                                                  const char* mode, qw_array* y, void* stream_v) {
  set_error("");
  SkinnyArgs sa{};
  int rc = check_qmm_call(x, w, scales, biases, transpose, group_size, bits, mode, y, &sa);
  if (rc != QW_OK) return rc;
  if (sa.M == 0 || sa.N == 0) return QW_OK;
  if ((bits != 4 && bits != 8) || (group_size != 64 && group_size != 128))
    return static_fail(QW_EUNSUPPORTED,
                       "qw_quantized_matmul_static_scratch takes 4- or 8-bit weights in groups of 64 or 128");
  if (sa.M > kStaticMaxRows)
    return static_fail(QW_EUNSUPPORTED, "qw_quantized_matmul_static_scratch takes at most " +
                                            std::to_string(kStaticMaxRows) + " rows of x per call, got " +
                                            std::to_string(sa.M));
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return static_fail(QW_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(ce));
  std::string err;
  void* base = nullptr;
  if (!static_scratch_address(dev, &base, &err)) return static_fail(QW_ECUDA, err);

  const size_t capacity = kStaticScratchBytes - kStaticStatusBytes;
  const size_t need = skinny_scratch_bytes(sa, dev);
  if (need > capacity)
    return static_fail(QW_EUNSUPPORTED, "this shape needs " + std::to_string(need) +
                                            " bytes of scratch on this device; the static scratch holds " +
                                            std::to_string(capacity));
  uint8_t* scratch = static_cast<uint8_t*>(base) + kStaticStatusBytes;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_v);
  ce = cudaMemsetAsync(scratch, 0, skinny_zeroed_bytes(sa), stream);
  if (ce != cudaSuccess) return static_fail(QW_ECUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(ce));

  sa.max_ctas = 0;
  sa.status = static_cast<unsigned int*>(base);
  ce = launch_skinny(sa, Scratch{scratch, capacity}, stream, /*pdl=*/false, &err);
  if (ce != cudaSuccess)
    return static_fail(QW_ECUDA, err.empty() ? std::string("skinny launch: ") + cudaGetErrorString(ce) : err);
  return QW_OK;
}
