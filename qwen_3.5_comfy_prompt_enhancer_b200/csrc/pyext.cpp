// Python binding of the qlin C ABI for torch tensors (module `_qlin_ext`).
//
// The Python entry points (kernels/gemm.py, kernels/w4.py, kernels/norm.py)
// hand their tensors to these functions, which make the checks the
// reference's call sites rely on (dtype, rank, contiguity, shapes, one CUDA
// device for every tensor) and call the extern "C" functions of libqlin.so
// on torch's current stream of that device.  Doing this in C++ instead of
// Python + ctypes keeps the host cost of one call to a few microseconds.
//
// Checks raise ValueError / TypeError (pybind11 translates
// py::value_error / py::type_error); a failing C-ABI call returns its
// qlin_status, which the Python caller turns into QlinError.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/utils/pybind.h>

#include <optional>
#include <string>

#include "qlin.h"

namespace py = pybind11;
using at::Tensor;
using OptT = std::optional<Tensor>;

namespace {

constexpr int64_t kGroup = 64;

const char* dtype_name(c10::ScalarType t) {
  switch (t) {
    case c10::ScalarType::Char: return "torch.int8";
    case c10::ScalarType::Byte: return "torch.uint8";
    case c10::ScalarType::Float: return "torch.float32";
    case c10::ScalarType::BFloat16: return "torch.bfloat16";
    default: return c10::toString(t);
  }
}

// Python's repr of a shape tuple: (4, 2048) or (128,).
std::string shape(const Tensor& t) {
  std::string s = "(";
  for (int64_t i = 0; i < t.dim(); ++i) {
    if (i) s += ", ";
    s += std::to_string(t.size(i));
  }
  if (t.dim() == 1) s += ",";
  return s + ")";
}

std::string dims(int64_t a, int64_t b) { return "[" + std::to_string(a) + ", " + std::to_string(b) + "]"; }

// Every tensor of one call lives on the device of its first operand.
struct Call {
  c10::DeviceIndex dev = -1;

  void need(const Tensor& t, const char* name, c10::ScalarType dt, int64_t rank, bool contiguous = true) {
    if (!t.is_cuda())
      throw py::value_error(std::string(name) + " must be a CUDA tensor (no CPU path), got " + t.device().str());
    if (dev < 0) dev = t.get_device();
    else if (t.get_device() != dev)
      throw py::value_error(std::string(name) + " is on cuda:" + std::to_string(t.get_device()) +
                            ", the other operands on cuda:" + std::to_string(dev));
    if (t.scalar_type() != dt)
      throw py::type_error(std::string(name) + " must be " + dtype_name(dt) + ", got " + dtype_name(t.scalar_type()));
    if (t.dim() != rank)
      throw py::value_error(std::string(name) + " must be " + std::to_string(rank) + "-D, got shape " + shape(t));
    if (contiguous && !t.is_contiguous()) throw py::value_error(std::string(name) + " must be contiguous");
  }

  // 2-D tensor whose rows may be strided but whose elements are contiguous.
  void need_rows(const Tensor& t, const char* name, c10::ScalarType dt) {
    need(t, name, dt, 2, false);
    if (t.size(1) > 1 && t.stride(1) != 1)
      throw py::value_error(std::string(name) + " must have unit stride along its last dimension");
  }

  // int8 activations + per-64 fp32 scales; returns (M, K).
  std::pair<int64_t, int64_t> acts(const Tensor& a_q, const Tensor& a_s) {
    need(a_q, "a_q", at::kChar, 2);
    need(a_s, "a_s", at::kFloat, 2);
    const int64_t M = a_q.size(0), K = a_q.size(1);
    if (a_s.size(0) != M || a_s.size(1) * kGroup != K)
      throw py::value_error("a_s must be [M, K/64] = " + dims(M, K / kGroup) + ", got " + shape(a_s));
    return {M, K};
  }

  // W8 weight [K, N] int8 + [N] fp32 column scales; returns N.
  int64_t w8(const Tensor& b, const Tensor& b_s, int64_t K, const std::string& name) {
    need(b, name.c_str(), at::kChar, 2);
    need(b_s, (name + "_s").c_str(), at::kFloat, 1);
    if (b.size(0) != K)
      throw py::value_error(name + " must be [K=" + std::to_string(K) + ", N], got " + shape(b));
    if (b_s.size(0) != b.size(1))
      throw py::value_error(name + " scales must have N=" + std::to_string(b.size(1)) + " entries, got " +
                            std::to_string(b_s.size(0)));
    return b.size(1);
  }

  // W4 weight [K/2, N] uint8 + [K/WGRP, N] bf16 scales (+ uint8 zeros);
  // returns (N, WGRP).
  std::pair<int64_t, int64_t> w4(const Tensor& b, const Tensor& b_s, const OptT& b_z, int64_t K,
                                 const std::string& name) {
    need(b, name.c_str(), at::kByte, 2);
    need(b_s, (name + "_s").c_str(), at::kBFloat16, 2);
    if (b.size(0) * 2 != K)
      throw py::value_error(name + " must be [K//2=" + std::to_string(K / 2) + ", N], got " + shape(b));
    const int64_t N = b.size(1);
    if (b_s.size(1) != N || b_s.size(0) == 0 || K % b_s.size(0) != 0)
      throw py::value_error(name + " scales must be [K//WGRP, " + std::to_string(N) + "], got " + shape(b_s));
    if (b_z) {
      need(*b_z, (name + "_z").c_str(), at::kByte, 2);
      if (b_z->sizes() != b_s.sizes())
        throw py::value_error(name + " zeros must match scales " + shape(b_s) + ", got " + shape(*b_z));
    }
    return {N, K / b_s.size(0)};
  }

  void out_mn(const Tensor& t, const char* name, int64_t M, int64_t N) {
    if (t.size(0) != M || t.size(1) != N)
      throw py::value_error(std::string(name) + " must be " + dims(M, N) + ", got " + shape(t));
  }

  void quant_out(const Tensor& out_q, const Tensor& out_s, int64_t M, int64_t N) {
    need(out_q, "out_q", at::kChar, 2);
    need(out_s, "out_s", at::kFloat, 2);
    if (out_q.size(0) != M || out_q.size(1) != N || out_s.size(0) != M || out_s.size(1) != N / kGroup)
      throw py::value_error("out_q/out_s must be " + dims(M, N) + " / " + dims(M, N / kGroup));
  }

  // Runs `f(stream)` with the call's device current.
  template <class F>
  int launch(F&& f) {
    c10::cuda::CUDAGuard guard(dev);
    return f(static_cast<void*>(c10::cuda::getCurrentCUDAStream(dev).stream()));
  }
};

template <class T>
const T* cptr(const Tensor& t) {
  return static_cast<const T*>(t.data_ptr());
}
template <class T>
const T* cptr(const OptT& t) {
  return t ? static_cast<const T*>(t->data_ptr()) : nullptr;
}

// ---------------------------------------------------------------- kernels/gemm.py
int gemm_i8(const Tensor& a_q, const Tensor& a_s, const Tensor& b, const Tensor& b_s, const Tensor& out,
            const OptT& residual) {
  Call c;
  const auto [M, K] = c.acts(a_q, a_s);
  const int64_t N = c.w8(b, b_s, K, "b");
  c.need_rows(out, "out", at::kBFloat16);
  c.out_mn(out, "out", M, N);
  if (residual) {
    c.need_rows(*residual, "residual", at::kBFloat16);
    c.out_mn(*residual, "residual", M, N);
  }
  return c.launch([&](void* st) {
    return qlin_gemm_i8(cptr<int8_t>(a_q), cptr<float>(a_s), M, K, cptr<int8_t>(b), cptr<float>(b_s), N,
                        out.data_ptr(), out.stride(0), cptr<void>(residual), residual ? residual->stride(0) : 0, st);
  });
}

int mlp_gate_up(const Tensor& a_q, const Tensor& a_s, const Tensor& wg, const Tensor& sg, const Tensor& wu,
                const Tensor& su, const Tensor& out) {
  Call c;
  const auto [M, K] = c.acts(a_q, a_s);
  const int64_t N = c.w8(wg, sg, K, "wg");
  if (c.w8(wu, su, K, "wu") != N) throw py::value_error("gate and up weights must have the same N");
  c.need(out, "out", at::kBFloat16, 2);
  c.out_mn(out, "out", M, N);
  return c.launch([&](void* st) {
    return qlin_mlp_gate_up(cptr<int8_t>(a_q), cptr<float>(a_s), M, K, cptr<int8_t>(wg), cptr<float>(sg),
                            cptr<int8_t>(wu), cptr<float>(su), N, out.data_ptr(), out.stride(0), st);
  });
}

int mlp_gate_up_quant(const Tensor& a_q, const Tensor& a_s, const Tensor& wg, const Tensor& sg, const Tensor& wu,
                      const Tensor& su, const Tensor& out_q, const Tensor& out_s) {
  Call c;
  const auto [M, K] = c.acts(a_q, a_s);
  const int64_t N = c.w8(wg, sg, K, "wg");
  if (c.w8(wu, su, K, "wu") != N) throw py::value_error("gate and up weights must have the same N");
  c.quant_out(out_q, out_s, M, N);
  return c.launch([&](void* st) {
    return qlin_mlp_gate_up_quant(cptr<int8_t>(a_q), cptr<float>(a_s), M, K, cptr<int8_t>(wg), cptr<float>(sg),
                                  cptr<int8_t>(wu), cptr<float>(su), N, static_cast<int8_t*>(out_q.data_ptr()),
                                  static_cast<float*>(out_s.data_ptr()), st);
  });
}

int proj3(const Tensor& a_q, const Tensor& a_s, const OptT& w1, const OptT& s1, const OptT& w2, const OptT& s2,
          const OptT& w3, const OptT& s3, const Tensor& out) {
  Call c;
  const auto [M, K] = c.acts(a_q, a_s);
  const OptT* w[3] = {&w1, &w2, &w3};
  const OptT* s[3] = {&s1, &s2, &s3};
  int64_t n[3] = {0, 0, 0};
  for (int i = 0; i < 3; ++i) {
    if (!*w[i]) continue;
    const std::string name = "w" + std::to_string(i + 1);
    if (!*s[i]) throw py::value_error(name + " has no scales");
    n[i] = c.w8(**w[i], **s[i], K, name);
  }
  const int64_t NT = n[0] + n[1] + n[2];
  c.need_rows(out, "out", at::kBFloat16);
  if (out.size(0) != M || out.size(1) < NT)
    throw py::value_error("out must be [" + std::to_string(M) + ", >=" + std::to_string(NT) + "], got " + shape(out));
  return c.launch([&](void* st) {
    return qlin_proj3(cptr<int8_t>(a_q), cptr<float>(a_s), M, K, cptr<int8_t>(w1), cptr<float>(s1), n[0],
                      cptr<int8_t>(w2), cptr<float>(s2), n[1], cptr<int8_t>(w3), cptr<float>(s3), n[2],
                      out.data_ptr(), out.stride(0), st);
  });
}

// ---------------------------------------------------------------- kernels/w4.py
int gemm_w4(const Tensor& a_q, const Tensor& a_s, const Tensor& b, const Tensor& b_s, const Tensor& out,
            const OptT& residual, const OptT& b_z) {
  Call c;
  const auto [M, K] = c.acts(a_q, a_s);
  const auto [N, wgrp] = c.w4(b, b_s, b_z, K, "b");
  c.need_rows(out, "out", at::kBFloat16);
  c.out_mn(out, "out", M, N);
  if (residual) {
    c.need_rows(*residual, "residual", at::kBFloat16);
    c.out_mn(*residual, "residual", M, N);
  }
  return c.launch([&](void* st) {
    return qlin_gemm_w4(cptr<int8_t>(a_q), cptr<float>(a_s), M, K, cptr<uint8_t>(b), cptr<void>(b_s),
                        cptr<uint8_t>(b_z), N, wgrp, out.data_ptr(), out.stride(0), cptr<void>(residual),
                        residual ? residual->stride(0) : 0, st);
  });
}

int proj3_w4(const Tensor& a_q, const Tensor& a_s, const OptT& w1, const OptT& s1, const OptT& w2, const OptT& s2,
             const OptT& w3, const OptT& s3, const Tensor& out, const OptT& z1, const OptT& z2, const OptT& z3) {
  Call c;
  const auto [M, K] = c.acts(a_q, a_s);
  const OptT* w[3] = {&w1, &w2, &w3};
  const OptT* s[3] = {&s1, &s2, &s3};
  const OptT* z[3] = {&z1, &z2, &z3};
  int64_t n[3] = {0, 0, 0};
  int64_t wgrp = 0;
  for (int i = 0; i < 3; ++i) {
    if (!*w[i]) continue;
    const std::string name = "w" + std::to_string(i + 1);
    if (!*s[i]) throw py::value_error(name + " has no scales");
    const auto [ni, wg] = c.w4(**w[i], **s[i], *z[i], K, name);
    if (wgrp == 0) wgrp = wg;
    else if (wg != wgrp) throw py::value_error("all proj3_w4 segments must share one weight group size");
    n[i] = ni;
  }
  const int64_t NT = n[0] + n[1] + n[2];
  c.need_rows(out, "out", at::kBFloat16);
  if (out.size(0) != M || out.size(1) < NT)
    throw py::value_error("out must be [" + std::to_string(M) + ", >=" + std::to_string(NT) + "], got " + shape(out));
  // a missing segment contributes no columns: its pointers stay null
  auto wp = [&](int i) { return *w[i] ? cptr<uint8_t>(*w[i]) : nullptr; };
  auto sp = [&](int i) { return *w[i] ? cptr<void>(*s[i]) : nullptr; };
  auto zp = [&](int i) { return *w[i] ? cptr<uint8_t>(*z[i]) : nullptr; };
  return c.launch([&](void* st) {
    return qlin_proj3_w4(cptr<int8_t>(a_q), cptr<float>(a_s), M, K, wp(0), sp(0), zp(0), n[0], wp(1), sp(1), zp(1),
                         n[1], wp(2), sp(2), zp(2), n[2], wgrp ? wgrp : 64, out.data_ptr(), out.stride(0), st);
  });
}

int mlp_gate_up_quant_w4(const Tensor& a_q, const Tensor& a_s, const Tensor& wg, const Tensor& sg, const Tensor& wu,
                         const Tensor& su, const Tensor& out_q, const Tensor& out_s, const OptT& zg,
                         const OptT& zu) {
  Call c;
  const auto [M, K] = c.acts(a_q, a_s);
  const auto [N, wgrp] = c.w4(wg, sg, zg, K, "wg");
  const auto [Nu, wgrp_u] = c.w4(wu, su, zu, K, "wu");
  if (Nu != N || wgrp_u != wgrp) throw py::value_error("gate and up weights must have the same N and group size");
  c.quant_out(out_q, out_s, M, N);
  return c.launch([&](void* st) {
    return qlin_mlp_gate_up_quant_w4(cptr<int8_t>(a_q), cptr<float>(a_s), M, K, cptr<uint8_t>(wg), cptr<void>(sg),
                                     cptr<uint8_t>(zg), cptr<uint8_t>(wu), cptr<void>(su), cptr<uint8_t>(zu), N,
                                     wgrp, static_cast<int8_t*>(out_q.data_ptr()),
                                     static_cast<float*>(out_s.data_ptr()), st);
  });
}

// ---------------------------------------------------------------- kernels/norm.py
int quant_row(const Tensor& x, const Tensor& q, const Tensor& s) {
  Call c;
  c.need_rows(x, "x", at::kBFloat16);
  c.need(q, "q", at::kChar, 2);
  c.need(s, "s", at::kFloat, 2);
  const int64_t M = q.size(0), K = q.size(1);
  if (x.size(0) != M || x.size(1) != K || s.size(0) != M || s.size(1) != K / kGroup)
    throw py::value_error("shapes must be x [M,K], q [M,K], s [M,K/64]; got " + shape(x) + ", " + shape(q) + ", " +
                          shape(s));
  return c.launch([&](void* st) {
    return qlin_quant_row(x.data_ptr(), x.stride(0), M, K, static_cast<int8_t*>(q.data_ptr()),
                          static_cast<float*>(s.data_ptr()), st);
  });
}

int rmsnorm_quant(const Tensor& x, const Tensor& w, const Tensor& q, const Tensor& s, double eps, bool one_plus) {
  Call c;
  c.need_rows(x, "x", at::kBFloat16);
  c.need(q, "q", at::kChar, 2);
  c.need(s, "s", at::kFloat, 2);
  c.need(w, "w", at::kBFloat16, 1);
  const int64_t M = q.size(0), K = q.size(1);
  if (x.size(0) != M || x.size(1) != K || s.size(0) != M || s.size(1) != K / kGroup || w.size(0) != K)
    throw py::value_error("shapes must be x [M,K], w [K], q [M,K], s [M,K/64]; got " + shape(x) + ", " + shape(w) +
                          ", " + shape(q) + ", " + shape(s));
  return c.launch([&](void* st) {
    return qlin_rmsnorm_quant(x.data_ptr(), x.stride(0), w.data_ptr(), M, K, static_cast<float>(eps),
                              one_plus ? 1 : 0, static_cast<int8_t*>(q.data_ptr()),
                              static_cast<float*>(s.data_ptr()), st);
  });
}

// v [T, N] contiguous, z [T, >= N] (rows strided), w [HD]; q/s or out.
int norm_gated(const Tensor& v, const Tensor& z, const Tensor& w, const OptT& q, const OptT& s, const OptT& out,
               double eps) {
  Call c;
  c.need(v, "v", at::kBFloat16, 2);
  c.need_rows(z, "z", at::kBFloat16);
  c.need(w, "w", at::kBFloat16, 1);
  const int64_t T = v.size(0), N = v.size(1), HD = w.size(0);
  if (z.size(0) != T || z.size(1) < N)
    throw py::value_error("z must be [" + std::to_string(T) + ", >=" + std::to_string(N) + "], got " + shape(z));
  if (HD == 0 || N % HD != 0) throw py::value_error("w must have head_dim entries dividing N, got " + shape(w));
  if (out) {
    c.need(*out, "out", at::kBFloat16, 2);
    c.out_mn(*out, "out", T, N);
    return c.launch([&](void* st) {
      return qlin_norm_gated(v.data_ptr(), z.data_ptr(), z.stride(0), w.data_ptr(), T, N, HD, static_cast<float>(eps),
                             out->data_ptr(), st);
    });
  }
  c.need(*q, "q", at::kChar, 2);
  c.need(*s, "s", at::kFloat, 2);
  if (q->size(0) != T || q->size(1) != N || s->size(0) != T || s->size(1) != N / kGroup)
    throw py::value_error("q/s must be " + dims(T, N) + " / " + dims(T, N / kGroup));
  return c.launch([&](void* st) {
    return qlin_norm_gated_quant(v.data_ptr(), z.data_ptr(), z.stride(0), w.data_ptr(), T, N, HD,
                                 static_cast<float>(eps), static_cast<int8_t*>(q->data_ptr()),
                                 static_cast<float*>(s->data_ptr()), st);
  });
}

int gate_mul_quant(const Tensor& a, const Tensor& g, const Tensor& q, const Tensor& s, int64_t hd) {
  Call c;
  c.need(a, "a", at::kBFloat16, 2);
  c.need_rows(g, "g", at::kBFloat16);
  c.need(q, "q", at::kChar, 2);
  c.need(s, "s", at::kFloat, 2);
  const int64_t M = a.size(0), N = a.size(1);
  if (g.size(0) != M || g.size(1) < 2 * N)
    throw py::value_error("g must be [" + std::to_string(M) + ", >=" + std::to_string(2 * N) + "], got " + shape(g));
  if (q.size(0) != M || q.size(1) != N || s.size(0) != M || s.size(1) != N / kGroup)
    throw py::value_error("q/s must be " + dims(M, N) + " / " + dims(M, N / kGroup));
  return c.launch([&](void* st) {
    return qlin_gate_mul_quant(a.data_ptr(), g.data_ptr(), g.stride(0), M, N, hd, static_cast<int8_t*>(q.data_ptr()),
                               static_cast<float*>(s.data_ptr()), st);
  });
}

int silu_mul_quant(const Tensor& g, const Tensor& u, const Tensor& q, const Tensor& s) {
  Call c;
  c.need(q, "q", at::kChar, 2);
  c.need(s, "s", at::kFloat, 2);
  c.need(g, "g", at::kBFloat16, 2);
  c.need(u, "u", at::kBFloat16, 2);
  const int64_t M = q.size(0), N = q.size(1);
  c.out_mn(g, "g", M, N);
  c.out_mn(u, "u", M, N);
  if (s.size(0) != M || s.size(1) != N / kGroup) throw py::value_error("s must be " + dims(M, N / kGroup));
  return c.launch([&](void* st) {
    return qlin_silu_mul_quant(g.data_ptr(), u.data_ptr(), M, N, static_cast<int8_t*>(q.data_ptr()),
                               static_cast<float*>(s.data_ptr()), st);
  });
}

int gate_proj(const Tensor& a_q, const Tensor& a_s, const Tensor& wb, const Tensor& wa, const Tensor& beta,
              const Tensor& gate, const Tensor& dt_bias, const Tensor& a_log) {
  Call c;
  const auto [M, K] = c.acts(a_q, a_s);
  c.need(wb, "wb", at::kBFloat16, 2);
  c.need(wa, "wa", at::kBFloat16, 2);
  c.need(beta, "beta", at::kFloat, 2);
  c.need(gate, "gate", at::kFloat, 2);
  c.need(dt_bias, "dt_bias", at::kBFloat16, 1);
  c.need(a_log, "a_log", at::kBFloat16, 1);
  const int64_t NB = wb.size(0);
  if (wb.size(1) != K || wa.size(0) != NB || wa.size(1) != K)
    throw py::value_error("wb/wa must be [NB, K=" + std::to_string(K) + "], got " + shape(wb) + ", " + shape(wa));
  c.out_mn(beta, "beta", M, NB);
  c.out_mn(gate, "gate", M, NB);
  if (dt_bias.size(0) != NB || a_log.size(0) != NB) throw py::value_error("dt_bias / a_log must have NB entries");
  return c.launch([&](void* st) {
    return qlin_gate_proj(cptr<int8_t>(a_q), cptr<float>(a_s), M, K, wb.data_ptr(), wa.data_ptr(), NB,
                          dt_bias.data_ptr(), a_log.data_ptr(), static_cast<float*>(beta.data_ptr()),
                          static_cast<float*>(gate.data_ptr()), st);
  });
}

// ---------------------------------------------------------------- kernels/attention.py, kernels/linear_attn.py
// Tensors of the decode neighbours may be 1-D rows (the reference's batch-1
// calls pass ws.q[0], ws.mixed[0], ...): these checks look at dtype,
// device, contiguity of the last dimension and element counts.
void need_any(Call& c, const Tensor& t, const char* name, c10::ScalarType dt) {
  c.need(t, name, dt, t.dim(), false);
  if (t.dim() == 0 || t.stride(t.dim() - 1) != 1)
    throw py::value_error(std::string(name) + " must have unit stride along its last dimension");
}

const int32_t* pos_ptr(Call& c, const OptT& pos_dev) {
  if (!pos_dev) return nullptr;
  c.need(*pos_dev, "pos (device)", at::kInt, pos_dev->dim());
  if (pos_dev->numel() != 1) throw py::value_error("a device-side position is a one-element int32 tensor");
  return static_cast<const int32_t*>(pos_dev->data_ptr());
}

int qk_norm_rope(const Tensor& proj, const Tensor& qn, const Tensor& kn, const Tensor& invf, const Tensor& qout,
                 const Tensor& kvc, const OptT& kvs, int64_t pos0, const OptT& pos_dev, double eps, bool kv_int8,
                 bool batch, int64_t kv_stride, int64_t kvs_stride) {
  Call c;
  c.need_rows(proj, "proj", at::kBFloat16);
  c.need(qn, "qn", at::kBFloat16, 1);
  c.need(kn, "kn", at::kBFloat16, 1);
  c.need(invf, "invf", at::kFloat, 1);
  c.need(qout, "qout", at::kBFloat16, 2);
  c.need(kvc, "kvc", kv_int8 ? at::kChar : at::kBFloat16, 2);
  if (kv_int8) {
    if (!kvs) throw py::value_error("kv_int8=True requires the kvs scales tensor");
    c.need(*kvs, "kvs", at::kFloat, 2);
  }
  const int64_t T = proj.size(0), HD = qn.size(0);
  if (kn.size(0) != HD || HD == 0) throw py::value_error("qn and kn must both have head_dim entries");
  const int64_t NQ = qout.size(1) / HD, NKV = kvc.size(1) / (2 * HD), RD = 2 * invf.size(0);
  if (qout.size(0) != T || qout.size(1) != NQ * HD) throw py::value_error("qout must be [T, nq * head_dim]");
  const int32_t* pd = pos_ptr(c, pos_dev);
  return c.launch([&](void* st) {
    return qlin_qk_norm_rope(proj.data_ptr(), proj.stride(0), qn.data_ptr(), kn.data_ptr(),
                             static_cast<const float*>(invf.data_ptr()), RD, qout.data_ptr(), kvc.data_ptr(),
                             kv_int8 ? static_cast<float*>(kvs->data_ptr()) : nullptr, T, NQ, NKV, HD, pos0, pd,
                             static_cast<float>(eps), kv_int8 ? 1 : 0, batch ? 1 : 0, kv_stride, kvs_stride, st);
  });
}

int attn_decode(const Tensor& q, const Tensor& kvc, const Tensor& out, int64_t pos, const OptT& pos_dev,
                int64_t max_pos, const OptT& kvs, bool kv_int8, int64_t batch, int64_t nq, int64_t nkv, int64_t hd) {
  Call c;
  need_any(c, q, "q", at::kBFloat16);
  need_any(c, out, "out", at::kBFloat16);
  c.need(kvc, "kvc", kv_int8 ? at::kChar : at::kBFloat16, kvc.dim());
  if (kv_int8) {
    if (!kvs) throw py::value_error("kv_int8=True requires the kvs scales tensor");
    c.need(*kvs, "kvs", at::kFloat, kvs->dim());
  }
  if (q.numel() != batch * nq * hd || out.numel() != batch * nq * hd || !q.is_contiguous() || !out.is_contiguous())
    throw py::value_error("q and out must be contiguous with batch * nq * hd elements");
  const int64_t kv_stride = batch > 1 ? kvc.numel() / batch : 0;
  const int64_t kvs_stride = (batch > 1 && kvs) ? kvs->numel() / batch : 0;
  const int32_t* pd = pos_ptr(c, pos_dev);
  return c.launch([&](void* st) {
    return qlin_attn_decode(q.data_ptr(), kvc.data_ptr(), kvs ? static_cast<const float*>(kvs->data_ptr()) : nullptr,
                            out.data_ptr(), pos, pd, max_pos, batch, nq, nkv, hd, kv_int8 ? 1 : 0, kv_stride,
                            kvs_stride, st);
  });
}

int delta_decode(const Tensor& qkv, const Tensor& g, const Tensor& beta, const Tensor& state, const Tensor& out,
                 int64_t batch) {
  Call c;
  need_any(c, qkv, "qkv", at::kBFloat16);
  c.need(g, "g", at::kFloat, g.dim());
  c.need(beta, "beta", at::kFloat, beta.dim());
  c.need(state, "state", at::kFloat, state.dim());
  need_any(c, out, "out", at::kBFloat16);
  if (state.dim() < 2) throw py::value_error("state must be [batch*nh, dk, dv]");
  const int64_t dv = state.size(state.dim() - 1), dk = state.size(state.dim() - 2);
  const int64_t nh = g.numel() / batch;
  if (g.numel() != batch * nh || beta.numel() != batch * nh || state.numel() != batch * nh * dk * dv)
    throw py::value_error("g / beta must hold batch * nh values and state batch * nh * dk * dv");
  if (out.numel() != batch * nh * dv || !out.is_contiguous()) throw py::value_error("out must hold batch * nh * dv");
  const int64_t ldq = qkv.dim() >= 2 ? qkv.stride(0) : 0;
  if (qkv.dim() == 1 && batch != 1) throw py::value_error("a 1-D qkv row serves batch 1 only");
  return c.launch([&](void* st) {
    return qlin_delta_decode(qkv.data_ptr(), ldq, static_cast<const float*>(g.data_ptr()),
                             static_cast<const float*>(beta.data_ptr()), static_cast<float*>(state.data_ptr()),
                             out.data_ptr(), batch, nh, dk, dv, st);
  });
}

int conv_silu(const Tensor& x, const Tensor& w, const Tensor& state, const Tensor& y, int64_t T, bool batch) {
  Call c;
  c.need_rows(x, "x", at::kBFloat16);
  c.need(w, "w", at::kBFloat16, 2);
  c.need(state, "state", at::kBFloat16, 2);
  c.need(y, "y", at::kBFloat16, 2);
  const int64_t C = x.size(1);
  if (w.size(0) != C || state.size(1) != C || y.size(1) != C || y.size(0) < T || x.size(0) < T)
    throw py::value_error("conv_silu: x [T, C], w [C, ks], state [rows, C], y [T, C] required");
  if (state.size(0) < (batch ? 3 * T : 3)) throw py::value_error("conv_silu: state has too few rows");
  return c.launch([&](void* st) {
    return qlin_conv_silu(x.data_ptr(), x.stride(0), w.data_ptr(), w.size(1), state.data_ptr(), y.data_ptr(), T, C,
                          batch ? 1 : 0, st);
  });
}

int conv_state_update(const Tensor& x, const Tensor& state, int64_t T, int64_t batch) {
  Call c;
  c.need_rows(x, "x", at::kBFloat16);
  c.need(state, "state", at::kBFloat16, 2);
  const int64_t C = x.size(1);
  if (state.size(1) != C || x.size(0) < T || state.size(0) < 3 * batch)
    throw py::value_error("conv_state_update: x [T, C], state [3 * batch, C] required");
  return c.launch([&](void* st) {
    return qlin_conv_state_update(x.data_ptr(), x.stride(0), state.data_ptr(), T, C, 4, batch, st);
  });
}

int conv_silu_update(const Tensor& x, const Tensor& w, const Tensor& state, const Tensor& y, int64_t batch) {
  Call c;
  c.need_rows(x, "x", at::kBFloat16);
  c.need(w, "w", at::kBFloat16, 2);
  c.need(state, "state", at::kBFloat16, 2);
  c.need(y, "y", at::kBFloat16, 2);
  const int64_t C = x.size(1);
  if (w.size(0) != C || state.size(1) != C || y.size(1) != C || y.size(0) < batch || x.size(0) < batch ||
      state.size(0) < 3 * batch)
    throw py::value_error("conv_silu_update: x [B, C], w [C, ks], state [3B, C], y [B, C] required");
  return c.launch([&](void* st) {
    return qlin_conv_silu_update(x.data_ptr(), x.stride(0), w.data_ptr(), w.size(1), state.data_ptr(), y.data_ptr(),
                                 batch, C, st);
  });
}

int attn_prefill(const Tensor& q, const Tensor& kvc, const Tensor& out, int64_t T, int64_t pos0, const OptT& kvs,
                 bool kv_int8, int64_t nq, int64_t nkv, int64_t hd) {
  Call c;
  c.need(q, "q", at::kBFloat16, 2);
  c.need(out, "out", at::kBFloat16, 2);
  c.need(kvc, "kvc", kv_int8 ? at::kChar : at::kBFloat16, 2);
  if (kv_int8) {
    if (!kvs) throw py::value_error("kv_int8=True requires the kvs scales tensor");
    c.need(*kvs, "kvs", at::kFloat, 2);
  }
  if (q.size(0) < T || q.size(1) != nq * hd || out.size(0) < T || out.size(1) != nq * hd)
    throw py::value_error("q and out must be [>= T, nq * hd]");
  if (kvc.size(1) != 2 * nkv * hd || kvc.size(0) < pos0 + T)
    throw py::value_error("kvc must be [>= pos0 + T, 2 * nkv * hd]");
  return c.launch([&](void* st) {
    return qlin_attn_prefill(q.data_ptr(), kvc.data_ptr(), kv_int8 ? static_cast<const float*>(kvs->data_ptr()) : nullptr,
                             out.data_ptr(), T, pos0, nq, nkv, hd, kv_int8 ? 1 : 0, st);
  });
}

int delta_prefill(const Tensor& qkv, const Tensor& g, const Tensor& beta, const Tensor& state, const Tensor& out,
                  int64_t T) {
  Call c;
  c.need_rows(qkv, "qkv", at::kBFloat16);
  c.need(g, "g", at::kFloat, 2);
  c.need(beta, "beta", at::kFloat, 2);
  c.need(state, "state", at::kFloat, 3);
  c.need(out, "out", at::kBFloat16, 2);
  const int64_t nh = state.size(0), dk = state.size(1), dv = state.size(2);
  if (g.size(0) < T || g.size(1) != nh || beta.size(0) < T || beta.size(1) != nh)
    throw py::value_error("g / beta must be [>= T, nh]");
  if (out.size(0) < T || out.size(1) != nh * dv || qkv.size(0) < T || qkv.size(1) < (2 * dk + dv) * nh)
    throw py::value_error("qkv must be [>= T, (2 dk + dv) nh] and out [>= T, nh dv]");
  return c.launch([&](void* st) {
    return qlin_delta_prefill(qkv.data_ptr(), qkv.stride(0), static_cast<const float*>(g.data_ptr()),
                              static_cast<const float*>(beta.data_ptr()), static_cast<float*>(state.data_ptr()),
                              out.data_ptr(), T, nh, dk, dv, st);
  });
}

}  // namespace

PYBIND11_MODULE(_qlin_ext, m) {
  m.doc() = "torch-tensor binding of the qlin C ABI (checks + launch on the current stream)";
  m.def("gemm_i8", &gemm_i8);
  m.def("mlp_gate_up", &mlp_gate_up);
  m.def("mlp_gate_up_quant", &mlp_gate_up_quant);
  m.def("proj3", &proj3);
  m.def("gemm_w4", &gemm_w4);
  m.def("proj3_w4", &proj3_w4);
  m.def("mlp_gate_up_quant_w4", &mlp_gate_up_quant_w4);
  m.def("quant_row", &quant_row);
  m.def("rmsnorm_quant", &rmsnorm_quant);
  m.def("norm_gated", &norm_gated);
  m.def("gate_mul_quant", &gate_mul_quant);
  m.def("silu_mul_quant", &silu_mul_quant);
  m.def("gate_proj", &gate_proj);
  m.def("qk_norm_rope", &qk_norm_rope);
  m.def("attn_decode", &attn_decode);
  m.def("delta_decode", &delta_decode);
  m.def("conv_silu", &conv_silu);
  m.def("conv_state_update", &conv_state_update);
  m.def("conv_silu_update", &conv_silu_update);
  m.def("attn_prefill", &attn_prefill);
  m.def("delta_prefill", &delta_prefill);
}
