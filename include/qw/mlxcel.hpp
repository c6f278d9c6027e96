// qw/mlxcel.hpp -- C++ host mirror of mlxcel-core's quantized-linear operator
// surface, over libqwqmm.so's C ABI (include/qw_qmm.h).
//
// The names, argument order and meaning follow the cxx bridge functions of
// crates/mlxcel-core/src/lib.rs and the types of crates/mlxcel-core/src/
// layers.rs that the runtime crate calls (QuantizedWeight, UnifiedLinear) and
// of crates/runtime/src/qwen3_next.rs (Mlp), so a C++ runtime, or a test
// written like the reference's ffi_tests.rs, reads the same.  Differences:
//   - device arrays (qw::Array, owning a cudaMalloc buffer or viewing one) in
//     place of MlxArray, and an explicit cudaStream_t (default: the legacy
//     stream) in place of MLX's thread-local stream;
//   - a qw::Error exception (status code + message) where the bridge aborts
//     the process on an MLX exception (layers.rs:1255-1285);
//   - fp16 activations only, as the library computes.
// Header-only; link libqwqmm.so and the CUDA runtime.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "../qw_qmm.h"

namespace qw {

class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

inline void check(int rc) {
  if (rc != QW_OK) throw Error(rc, std::string("qw status ") + std::to_string(rc) + ": " + qw_last_error());
}
inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(QW_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

enum class DType : int32_t { U32 = QW_U32, F16 = QW_F16, BF16 = QW_BF16, F32 = QW_F32 };

inline size_t dtype_size(DType d) { return d == DType::F16 || d == DType::BF16 ? 2 : 4; }

// A row-contiguous device array, owning its buffer or viewing another's: the
// role MlxArray plays at this boundary (mlx_cxx_bridge.h:16-22).
class Array {
 public:
  Array() = default;

  static Array empty(std::vector<int64_t> shape, DType dt) {
    Array a;
    a.shape_ = std::move(shape);
    a.dt_ = dt;
    const size_t bytes = a.nbytes();
    void* p = nullptr;
    if (bytes) check_cuda(cudaMalloc(&p, bytes), "cudaMalloc");
    a.buf_ = std::shared_ptr<void>(p, [](void* q) {
      if (q) cudaFree(q);
    });
    a.ptr_ = p;
    return a;
  }

  static Array from_host(const void* data, std::vector<int64_t> shape, DType dt, cudaStream_t s = nullptr) {
    Array a = empty(std::move(shape), dt);
    if (a.nbytes()) {
      check_cuda(cudaMemcpyAsync(a.ptr_, data, a.nbytes(), cudaMemcpyHostToDevice, s), "cudaMemcpyAsync");
      check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    }
    return a;
  }

  template <class T>
  std::vector<T> to_host(cudaStream_t s = nullptr) const {
    std::vector<T> out(nbytes() / sizeof(T));
    if (nbytes()) {
      check_cuda(cudaMemcpyAsync(out.data(), ptr_, nbytes(), cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync");
      check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    }
    return out;
  }

  // Rows [r0, r1) of the leading dimension, as a view.
  Array rows(int64_t r0, int64_t r1) const {
    if (shape_.empty() || r0 < 0 || r1 > shape_[0] || r0 > r1) throw Error(QW_EINVAL, "row range out of bounds");
    Array v = *this;
    v.shape_[0] = r1 - r0;
    v.ptr_ = static_cast<uint8_t*>(ptr_) + (size_t)r0 * (nbytes() / (size_t)(shape_[0] ? shape_[0] : 1));
    return v;
  }

  Array reshape(std::vector<int64_t> shape) const {
    Array v = *this;
    v.shape_ = std::move(shape);
    if (v.numel() != numel()) throw Error(QW_EINVAL, "reshape changes the element count");
    return v;
  }

  const std::vector<int64_t>& shape() const { return shape_; }
  DType dtype() const { return dt_; }
  void* data() const { return ptr_; }
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : shape_) n *= d;
    return n;
  }
  size_t nbytes() const { return (size_t)numel() * dtype_size(dt_); }

  // The C ABI's descriptor (all-zero strides: row-contiguous).
  qw_array desc() const {
    qw_array d;
    std::memset(&d, 0, sizeof d);
    d.data = ptr_;
    d.dtype = (int32_t)dt_;
    d.ndim = (int32_t)shape_.size();
    for (size_t i = 0; i < shape_.size() && i < 4; ++i) d.shape[i] = shape_[i];
    return d;
  }

 private:
  std::shared_ptr<void> buf_;
  void* ptr_ = nullptr;
  std::vector<int64_t> shape_;
  DType dt_ = DType::F16;
};

namespace detail {
inline std::vector<int64_t> with_last(const std::vector<int64_t>& s, int64_t last) {
  std::vector<int64_t> out = s;
  if (out.empty()) out.push_back(last);
  else out.back() = last;
  return out;
}
// A descriptor for an optional array (null when absent).
struct OptDesc {
  qw_array d;
  const qw_array* p;
  explicit OptDesc(const Array* a) : d(a ? a->desc() : qw_array{}), p(a ? &d : nullptr) {}
};
}  // namespace detail

// quantized_matmul (lib.rs:1134-1143): y = x @ dequantize(w, scales, biases).T
inline Array quantized_matmul(const Array& x, const Array& w, const Array& scales, const Array* biases,
                              bool transpose, int group_size, int bits, const std::string& mode,
                              cudaStream_t s = nullptr) {
  Array y = Array::empty(detail::with_last(x.shape(), w.shape().empty() ? 0 : w.shape()[0]), DType::F16);
  const qw_array xd = x.desc(), wd = w.desc(), sd = scales.desc();
  const detail::OptDesc bd(biases);
  qw_array yd = y.desc();
  check(qw_quantized_matmul(&xd, &wd, &sd, bd.p, transpose ? 1 : 0, group_size, bits, mode.c_str(), &yd, s));
  return y;
}

// quantized_linear_forward (lib.rs:591-601): the quantized arm of a linear layer
inline Array quantized_linear_forward(const Array& x, const Array& w, const Array& scales, const Array* biases,
                                      const Array* linear_bias, int group_size, int bits, const std::string& mode,
                                      cudaStream_t s = nullptr) {
  Array y = Array::empty(detail::with_last(x.shape(), w.shape()[0]), DType::F16);
  const qw_array xd = x.desc(), wd = w.desc(), sd = scales.desc();
  const detail::OptDesc bd(biases), lb(linear_bias);
  qw_array yd = y.desc();
  check(qw_quantized_linear_forward(&xd, &wd, &sd, bd.p, lb.p, group_size, bits, mode.c_str(), &yd, s));
  return y;
}

// quantized_linear_forward_global_scale (lib.rs:604-615)
inline Array quantized_linear_forward_global_scale(const Array& x, const Array& w, const Array& scales,
                                                   const Array* biases, const Array* global_scale,
                                                   const Array* linear_bias, int group_size, int bits,
                                                   const std::string& mode, cudaStream_t s = nullptr) {
  Array y = Array::empty(detail::with_last(x.shape(), w.shape()[0]), DType::F16);
  const qw_array xd = x.desc(), wd = w.desc(), sd = scales.desc();
  const detail::OptDesc bd(biases), gs(global_scale), lb(linear_bias);
  qw_array yd = y.desc();
  check(qw_quantized_linear_forward_global_scale(&xd, &wd, &sd, bd.p, gs.p, lb.p, group_size, bits, mode.c_str(),
                                                 &yd, s));
  return y;
}

// dequantize (lib.rs:1152-1159): fp16 [N, K]
inline Array dequantize(const Array& w, const Array& scales, const Array* biases, int group_size, int bits,
                        const std::string& mode, cudaStream_t s = nullptr) {
  const int64_t K = w.shape().back() * 32 / bits;
  Array out = Array::empty({w.shape()[0], K}, DType::F16);
  const qw_array wd = w.desc(), sd = scales.desc();
  const detail::OptDesc bd(biases);
  qw_array od = out.desc();
  check(qw_dequantize(&wd, &sd, bd.p, group_size, bits, mode.c_str(), &od, s));
  return out;
}

// quantize_weights{_w,_scales,_biases} (mlx_cxx_bridge.cpp:6347-6393): (w, scales, biases)
inline std::tuple<Array, Array, Array> quantize_weights(const Array& w, int group_size, int bits,
                                                        const std::string& mode = "affine",
                                                        cudaStream_t s = nullptr) {
  const int64_t N = w.shape()[0], K = w.shape().back();
  Array wq = Array::empty({N, K * bits / 32}, DType::U32);
  Array sc = Array::empty({N, K / group_size}, DType::F16);
  Array bi = Array::empty({N, K / group_size}, DType::F16);
  const qw_array wd = w.desc();
  qw_array qd = wq.desc(), sd = sc.desc(), bd = bi.desc();
  check(qw_quantize(&wd, group_size, bits, mode.c_str(), &qd, &sd, &bd, s));
  return {wq, sc, bi};
}

// compiled_swiglu_activation (lib.rs:627): silu(gate) * x
inline Array compiled_swiglu_activation(const Array& gate, const Array& x, cudaStream_t s = nullptr) {
  Array y = Array::empty(gate.shape(), DType::F16);
  const qw_array gd = gate.desc(), xd = x.desc();
  qw_array yd = y.desc();
  check(qw_swiglu_activation(&gd, &xd, &yd, s));
  return y;
}

// compiled_moe_expert_forward (lib.rs:1636-1652): down(silu(gate(x)) * up(x))
inline Array compiled_moe_expert_forward(const Array& x, const Array& gate_proj, const Array& gate_scales,
                                         const Array* gate_biases, const Array& up_proj, const Array& up_scales,
                                         const Array* up_biases, const Array& down_proj,
                                         const Array& down_scales, const Array* down_biases, int group_size,
                                         int bits, const std::string& mode, cudaStream_t s = nullptr) {
  Array y = Array::empty(detail::with_last(x.shape(), down_proj.shape()[0]), DType::F16);
  const qw_array xd = x.desc(), gw = gate_proj.desc(), gs = gate_scales.desc(), uw = up_proj.desc(),
                 us = up_scales.desc(), dw = down_proj.desc(), ds = down_scales.desc();
  const detail::OptDesc gb(gate_biases), ub(up_biases), db(down_biases);
  qw_array yd = y.desc();
  check(qw_swiglu_mlp(&xd, &gw, &gs, gb.p, &uw, &us, ub.p, &dw, &ds, db.p, group_size, bits, mode.c_str(), &yd, s));
  return y;
}

// top_k_candidate_logits (qwen3_5_dflash.rs:1236-1266): (ids u32 [..., k], values f16 [..., k])
inline std::pair<Array, Array> top_k_candidate_logits(const Array& logits, int k, cudaStream_t s = nullptr) {
  Array idx = Array::empty(detail::with_last(logits.shape(), k), DType::U32);
  Array val = Array::empty(detail::with_last(logits.shape(), k), DType::F16);
  const qw_array ld = logits.desc();
  qw_array id = idx.desc(), vd = val.desc();
  check(qw_topk(&ld, k, &id, &vd, s));
  return {idx, val};
}

// QuantizedWeight (layers.rs:35-174)
struct QuantizedWeight {
  Array weight;  // u32 [N, K*bits/32]
  Array scales;  // f16 [N, K/group_size]
  std::optional<Array> biases;
  int group_size = 64;
  int bits = 4;
  std::string mode = "affine";
  std::optional<Array> global_scale;  // f32 scalar

  // QuantizedWeight::new: affine, with biases
  QuantizedWeight(Array w, Array s, Array b, int gs, int nbits)
      : weight(std::move(w)), scales(std::move(s)), biases(std::move(b)), group_size(gs), bits(nbits) {}

  const Array* biases_ptr() const { return biases ? &*biases : nullptr; }
  int64_t out_features() const { return weight.shape()[0]; }
  int64_t in_features() const { return weight.shape().back() * 32 / bits; }
};

// The quantized arm of UnifiedLinear (layers.rs:2023-2093)
class UnifiedLinear {
 public:
  UnifiedLinear(QuantizedWeight w, std::optional<Array> bias) : w_(std::move(w)), bias_(std::move(bias)) {}

  const QuantizedWeight* quantized_weight() const { return &w_; }

  Array forward(const Array& x, cudaStream_t s = nullptr) const {
    const Array* lb = bias_ ? &*bias_ : nullptr;
    if (w_.global_scale)
      return quantized_linear_forward_global_scale(x, w_.weight, w_.scales, w_.biases_ptr(), &*w_.global_scale, lb,
                                                   w_.group_size, w_.bits, w_.mode, s);
    return quantized_linear_forward(x, w_.weight, w_.scales, w_.biases_ptr(), lb, w_.group_size, w_.bits, w_.mode,
                                    s);
  }

 private:
  QuantizedWeight w_;
  std::optional<Array> bias_;
};

// Mlp (qwen3_next.rs:449-487): gate and up run as one fused SwiGLU kernel.
class Mlp {
 public:
  Mlp(UnifiedLinear gate, UnifiedLinear up, UnifiedLinear down)
      : gate_(std::move(gate)), up_(std::move(up)), down_(std::move(down)) {}

  Array forward_hidden(const Array& x, cudaStream_t s = nullptr) const {
    const QuantizedWeight& g = *gate_.quantized_weight();
    const QuantizedWeight& u = *up_.quantized_weight();
    Array h = Array::empty(detail::with_last(x.shape(), g.out_features()), DType::F16);
    const qw_array xd = x.desc(), gw = g.weight.desc(), gs = g.scales.desc(), uw = u.weight.desc(),
                   us = u.scales.desc();
    const detail::OptDesc gb(g.biases_ptr()), ub(u.biases_ptr());
    qw_array hd = h.desc();
    check(qw_quantized_matmul_swiglu(&xd, &gw, &gs, gb.p, &uw, &us, ub.p, 1, g.group_size, g.bits, g.mode.c_str(),
                                     &hd, s));
    return h;
  }

  Array forward(const Array& x, cudaStream_t s = nullptr) const { return down_.forward(forward_hidden(x, s), s); }

 private:
  UnifiedLinear gate_, up_, down_;
};

}  // namespace qw
