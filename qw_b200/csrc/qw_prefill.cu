// qw_prefill.cu -- prefill (M >= 17) affine 4-bit quantized matmul on the
// 5th-generation tensor cores.  Placeholder until the tcgen05 kernel lands:
// reports itself unavailable so the dispatcher uses the skinny path.
#include "qw_internal.h"

namespace qw {

bool prefill_available() { return false; }

cudaError_t launch_prefill(const PrefillArgs&, cudaStream_t, bool, std::string* err) {
  *err = "prefill kernel not built";
  return cudaErrorNotSupported;
}

}  // namespace qw
