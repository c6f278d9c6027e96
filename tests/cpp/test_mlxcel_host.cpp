// C++ tests of the host mirror (include/qw/mlxcel.hpp) over libqwqmm.so, in
// the style of the reference's crates/mlxcel-core/src/ffi_tests.rs: the
// fused entry points against their op-at-a-time compositions, the
// QuantizedWeight accessors, dequantize's commutation with row slices, the
// load-time validation as exceptions, and the matmul against the CPU oracle
// (oracle/qw_oracle.h, linked as test infrastructure).  Needs a GPU; run by
// tests/test_cpp_host.py.  Prints one line per test and exits non-zero on
// the first failure.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <string>
#include <vector>

#include "../../include/qw/mlxcel.hpp"
#include "../../oracle/qw_oracle.h"

namespace {

int g_failed = 0;

#define EXPECT(cond)                                                          \
  do {                                                                        \
    if (!(cond)) {                                                            \
      std::fprintf(stderr, "  %s:%d: expected %s\n", __FILE__, __LINE__, #cond); \
      throw std::runtime_error("expectation failed");                         \
    }                                                                         \
  } while (0)

void run(const char* name, const std::function<void()>& fn) {
  try {
    fn();
    std::printf("PASS %s\n", name);
  } catch (const std::exception& e) {
    std::printf("FAIL %s: %s\n", name, e.what());
    ++g_failed;
  }
}

// splitmix64 + Box-Muller: seeded N(0, sigma) fp16 data
struct Rng {
  uint64_t s;
  explicit Rng(uint64_t seed) : s(seed) {}
  uint64_t next() {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  double uniform() { return ((next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
  double normal() { return std::sqrt(-2.0 * std::log(uniform())) * std::cos(6.283185307179586 * uniform()); }
};

std::vector<uint16_t> normal_f16(size_t n, double sigma, uint64_t seed) {
  Rng r(seed);
  std::vector<uint16_t> v(n);
  for (auto& h : v) h = qwo_f32_to_f16((float)(r.normal() * sigma));
  return v;
}

struct HostQuant {
  std::vector<uint32_t> wq;
  std::vector<uint16_t> s, b;
};

// random_quantized_weight (ffi_tests.rs:2086-2107): N(0, 0.02) weights quantized
HostQuant random_quantized_weight(int64_t N, int64_t K, uint64_t seed, int gs = 64, int bits = 4) {
  const std::vector<uint16_t> w = normal_f16((size_t)(N * K), 0.02, seed);
  HostQuant q;
  q.wq.resize((size_t)(N * K * bits / 32));
  q.s.resize((size_t)(N * K / gs));
  q.b.resize((size_t)(N * K / gs));
  if (qwo_quantize(w.data(), N, K, gs, bits, q.wq.data(), q.s.data(), q.b.data()) != QWO_OK)
    throw std::runtime_error("oracle quantize failed");
  return q;
}

struct DevQuant {
  qw::Array w, s, b;
};
DevQuant upload(const HostQuant& q, int64_t N, int64_t K, int gs = 64, int bits = 4) {
  return {qw::Array::from_host(q.wq.data(), {N, K * bits / 32}, qw::DType::U32),
          qw::Array::from_host(q.s.data(), {N, K / gs}, qw::DType::F16),
          qw::Array::from_host(q.b.data(), {N, K / gs}, qw::DType::F16)};
}

// max |y - y_ref| / rms(y_ref)
double rel_err(const std::vector<uint16_t>& y, const std::vector<float>& ref) {
  double ss = 0, mx = 0;
  for (size_t i = 0; i < ref.size(); ++i) {
    ss += (double)ref[i] * ref[i];
    mx = std::fmax(mx, std::fabs((double)qwo_f16_to_f32(y[i]) - ref[i]));
  }
  const double rms = std::sqrt(ss / (double)(ref.size() ? ref.size() : 1));
  return rms > 0 ? mx / rms : mx;
}

}  // namespace

int main() {
  constexpr double kTol = 1e-2;  // max |y - y_ref| <= 1e-2 rms(y_ref)

  // ffi_tests.rs:2983-3004
  run("test_unified_linear_quantized_weight_accessor", [] {
    const HostQuant q = random_quantized_weight(2, 64, 1);
    DevQuant d = upload(q, 2, 64);
    qw::UnifiedLinear linear(qw::QuantizedWeight(d.w, d.s, d.b, 64, 4), std::nullopt);
    const qw::QuantizedWeight* w = linear.quantized_weight();
    EXPECT(w != nullptr);
    EXPECT(w->group_size == 64 && w->bits == 4 && w->mode == "affine");
    EXPECT(w->biases.has_value());
    EXPECT(w->in_features() == 64 && w->out_features() == 2);
  });

  run("quantized_matmul_matches_cpu_oracle", [&] {
    const int64_t N = 1000, K = 2048;
    const HostQuant q = random_quantized_weight(N, K, 2);
    DevQuant d = upload(q, N, K);
    for (int64_t M : {1, 5, 16, 40}) {
      const std::vector<uint16_t> x = normal_f16((size_t)(M * K), 1.0, 100 + M);
      std::vector<uint16_t> yr((size_t)(M * N));
      std::vector<float> y32((size_t)(M * N));
      EXPECT(qwo_quantized_matmul(x.data(), q.wq.data(), q.s.data(), q.b.data(), M, N, K, 64, 4, yr.data(),
                                  y32.data(), 0) == QWO_OK);
      qw::Array xd = qw::Array::from_host(x.data(), {M, K}, qw::DType::F16);
      qw::Array y = qw::quantized_matmul(xd, d.w, d.s, &d.b, true, 64, 4, "affine");
      EXPECT(y.shape() == std::vector<int64_t>({M, N}));
      EXPECT(rel_err(y.to_host<uint16_t>(), y32) <= kTol);
    }
  });

  run("quantize_weights_matches_cpu_oracle_bit_for_bit", [] {
    const int64_t N = 96, K = 512;
    const std::vector<uint16_t> w = normal_f16((size_t)(N * K), 0.02, 3);
    HostQuant q;
    q.wq.resize((size_t)(N * K / 8));
    q.s.resize((size_t)(N * K / 64));
    q.b.resize((size_t)(N * K / 64));
    EXPECT(qwo_quantize(w.data(), N, K, 64, 4, q.wq.data(), q.s.data(), q.b.data()) == QWO_OK);
    auto [wq, s, b] = qw::quantize_weights(qw::Array::from_host(w.data(), {N, K}, qw::DType::F16), 64, 4);
    EXPECT(wq.to_host<uint32_t>() == q.wq);
    EXPECT(s.to_host<uint16_t>() == q.s);
    EXPECT(b.to_host<uint16_t>() == q.b);
  });

  // ffi_tests.rs:3792-3850, restated on row slices of the device arrays
  run("dequantize_commutes_with_output_axis_slice", [] {
    const int64_t N = 192, K = 512;
    const HostQuant q = random_quantized_weight(N, K, 4);
    DevQuant d = upload(q, N, K);
    const std::vector<uint16_t> full = qw::dequantize(d.w, d.s, &d.b, 64, 4, "affine").to_host<uint16_t>();
    qw::Array bs = d.b.rows(64, 160);
    const std::vector<uint16_t> part =
        qw::dequantize(d.w.rows(64, 160), d.s.rows(64, 160), &bs, 64, 4, "affine").to_host<uint16_t>();
    EXPECT(std::vector<uint16_t>(full.begin() + 64 * K, full.begin() + 160 * K) == part);
    std::vector<uint16_t> ref((size_t)(N * K));
    EXPECT(qwo_dequantize(q.wq.data(), q.s.data(), q.b.data(), N, K, 64, 4, QWO_ROUND_TWICE, ref.data()) ==
           QWO_OK);
    EXPECT(full == ref);
  });

  // ffi_tests.rs:2321-2370 (affine here: the library runs affine codes only)
  run("quantized_linear_forward_global_scale_matches_manual_path", [] {
    const int64_t N = 96, K = 128, M = 3;
    const HostQuant q = random_quantized_weight(N, K, 5);
    DevQuant d = upload(q, N, K);
    const float gsv = 1.23f;
    qw::Array gs = qw::Array::from_host(&gsv, {1}, qw::DType::F32);
    const std::vector<uint16_t> lbh = normal_f16((size_t)N, 1.0, 6);
    qw::Array lb = qw::Array::from_host(lbh.data(), {N}, qw::DType::F16);
    const std::vector<uint16_t> xh = normal_f16((size_t)(M * K), 1.0, 7);
    qw::Array x = qw::Array::from_host(xh.data(), {1, M, K}, qw::DType::F16);
    const std::vector<uint16_t> fused =
        qw::quantized_linear_forward_global_scale(x, d.w, d.s, &d.b, &gs, &lb, 64, 4, "affine").to_host<uint16_t>();
    const std::vector<uint16_t> mm =
        qw::quantized_linear_forward(x, d.w, d.s, &d.b, nullptr, 64, 4, "affine").to_host<uint16_t>();
    // reference: astype(multiply(mm, global_scale), fp16) + linear_bias, op by op in fp16
    for (size_t i = 0; i < mm.size(); ++i) {
      const uint16_t scaled = qwo_f32_to_f16(qwo_f16_to_f32(mm[i]) * gsv);
      const uint16_t ref = qwo_f32_to_f16(qwo_f16_to_f32(scaled) + qwo_f16_to_f32(lbh[i % N]));
      EXPECT(fused[i] == ref);
    }
  });

  // compiled_moe_expert_forward (mlx_cxx_bridge.cpp:4238-4283) against its
  // op-at-a-time fallback: gate, up, silu(gate) * up, down
  run("compiled_moe_expert_forward_matches_op_at_a_time", [&] {
    const int64_t H = 128, I = 256;
    const HostQuant gq = random_quantized_weight(I, H, 8), uq = random_quantized_weight(I, H, 9),
                    dq = random_quantized_weight(H, I, 10);
    DevQuant g = upload(gq, I, H), u = upload(uq, I, H), dn = upload(dq, H, I);
    for (int64_t M : {1, 40}) {
      const std::vector<uint16_t> xh = normal_f16((size_t)(M * H), 1.0, 11 + M);
      qw::Array x = qw::Array::from_host(xh.data(), {1, M, H}, qw::DType::F16);
      qw::Array fused =
          qw::compiled_moe_expert_forward(x, g.w, g.s, &g.b, u.w, u.s, &u.b, dn.w, dn.s, &dn.b, 64, 4, "affine");
      qw::Array gate = qw::quantized_matmul(x, g.w, g.s, &g.b, true, 64, 4, "affine");
      qw::Array up = qw::quantized_matmul(x, u.w, u.s, &u.b, true, 64, 4, "affine");
      qw::Array act = qw::compiled_swiglu_activation(gate, up);
      qw::Array down = qw::quantized_matmul(act, dn.w, dn.s, &dn.b, true, 64, 4, "affine");
      EXPECT(fused.shape() == down.shape());
      const std::vector<uint16_t> a = fused.to_host<uint16_t>(), b = down.to_host<uint16_t>();
      std::vector<float> ref(b.size());
      for (size_t i = 0; i < b.size(); ++i) ref[i] = qwo_f16_to_f32(b[i]);
      EXPECT(rel_err(a, ref) <= kTol);
      // the Mlp wrapper runs the same fused path
      qw::Mlp mlp(qw::UnifiedLinear(qw::QuantizedWeight(g.w, g.s, g.b, 64, 4), std::nullopt),
                  qw::UnifiedLinear(qw::QuantizedWeight(u.w, u.s, u.b, 64, 4), std::nullopt),
                  qw::UnifiedLinear(qw::QuantizedWeight(dn.w, dn.s, dn.b, 64, 4), std::nullopt));
      EXPECT(mlp.forward(x).to_host<uint16_t>() == a);
    }
  });

  // qwen3_5_dflash.rs:3884-3938: four peaks over a flat floor; k bounds
  run("candidate_top_k_peaks_and_bounds", [] {
    const int64_t n = 80922;
    std::vector<uint16_t> lg((size_t)n, qwo_f32_to_f16(-1000.f));
    const int64_t ids[4] = {0, 80000, 80001, 80921};
    const float vals[4] = {40.f, 50.f, 60.f, 70.f};
    for (int i = 0; i < 4; ++i) lg[(size_t)ids[i]] = qwo_f32_to_f16(vals[i]);
    auto [idx, val] = qw::top_k_candidate_logits(qw::Array::from_host(lg.data(), {1, 1, n}, qw::DType::F16), 4);
    const std::vector<uint32_t> ih = idx.to_host<uint32_t>();
    const std::vector<uint16_t> vh = val.to_host<uint16_t>();
    EXPECT(ih == std::vector<uint32_t>({80921, 80001, 80000, 0}));
    EXPECT(qwo_f16_to_f32(vh[0]) == 70.f && qwo_f16_to_f32(vh[3]) == 40.f);
    std::vector<uint16_t> z(4, 0);
    qw::Array zd = qw::Array::from_host(z.data(), {1, 1, 4}, qw::DType::F16);
    for (int bad : {0, 4, 5}) {
      bool threw = false;
      try {
        qw::top_k_candidate_logits(zd, bad);
      } catch (const qw::Error& e) {
        threw = e.code() == QW_EINVAL;
      }
      EXPECT(threw);
    }
    qw::top_k_candidate_logits(zd, 1);
  });

  // the load-time validators (layers.rs:1286-1318, :1568-1570) as exceptions
  run("invalid_calls_throw_with_status", [] {
    const HostQuant q = random_quantized_weight(64, 128, 12);
    DevQuant d = upload(q, 64, 128);
    const std::vector<uint16_t> xh = normal_f16(128, 1.0, 13);
    qw::Array x = qw::Array::from_host(xh.data(), {1, 128}, qw::DType::F16);
    auto code_of = [&](const std::function<void()>& f) {
      try {
        f();
      } catch (const qw::Error& e) {
        return e.code();
      }
      return 0;
    };
    EXPECT(code_of([&] { qw::quantized_matmul(x, d.w, d.s, &d.b, true, 64, 8, "affine"); }) == QW_EINVAL);
    EXPECT(code_of([&] { qw::quantized_matmul(x, d.w, d.s, &d.b, true, 32, 4, "affine"); }) == QW_EUNSUPPORTED);
    EXPECT(code_of([&] { qw::quantized_matmul(x, d.w, d.s, nullptr, true, 64, 4, "affine"); }) == QW_EINVAL);
    EXPECT(code_of([&] { qw::quantized_matmul(x, d.w, d.s, &d.b, false, 64, 4, "affine"); }) ==
           QW_EUNSUPPORTED);
  });

  std::printf(g_failed ? "FAILED %d\n" : "ALL PASSED\n", g_failed);
  return g_failed ? 1 : 0;
}
