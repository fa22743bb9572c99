// GELU epilogue math: GELU(x) = x * Phi(x) with Phi the standard normal CDF
// (the exact-erf GELU of torch.nn.functional.gelu), to fp32 accuracy
// (max relative error 7.5e-6 on [-8, 8] and absolute error below 1e-6
// everywhere, see gelu_fit.py).
//
// With u = |x|:  erfc(u/sqrt2) = 2^(Q(u) - u^2 * log2(e)/2), where
// Q(u) = log2(erfcx(u/sqrt2)) and erfcx(z) = exp(z^2) erfc(z).  Q is smooth
// and slowly varying, so a degree-10 polynomial (a Chebyshev least-squares
// fit on [0, 8], converted to monomials by gelu_fit.py) evaluates it with
// ten fused multiply-adds; one ex2 finishes erfc.  Phi = 1 - erfc/2 for
// x >= 0 and erfc/2 for x < 0.  Past u = 8, erfc(u/sqrt2) < 1.3e-15, so u is
// clamped inside Q only.
//
// Pairs of values are evaluated with the packed fp32x2 FMA of sm_100, which
// halves the issue slots of the polynomial.
#pragma once

#include "common.cuh"

namespace cti {

namespace gelu_detail {
// Q(u) = sum_k C_k u^k (gelu_fit.py, degree 10, Chebyshev fit on [0, 8]).
constexpr float C0 = 8.310687917401083e-06f, C1 = -1.1512506008148193f,
                C2 = 0.26276615262031555f, C3 = -0.05365163832902908f,
                C4 = 0.008176298812031746f, C5 = -0.0007422473281621933f,
                C6 = -4.1401798966944625e-07f, C7 = 1.0348962860007305e-05f,
                C8 = -1.3962661569166812e-06f, C9 = 8.502458825887516e-08f,
                C10 = -2.080758010336581e-09f;
constexpr float kU0 = 8.0f;
constexpr float kNegHalfLog2e = -0.72134752044448170368f;  // -log2(e)/2
}  // namespace gelu_detail

CTI_DEVICE uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

CTI_DEVICE void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

CTI_DEVICE uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

CTI_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

CTI_DEVICE float gelu_finish(float x, float q) {
  const float h = 0.5f * ex2_approx(q);
  const float phi = x >= 0.0f ? 1.0f - h : h;
  return x * phi;
}

// GELU of two values.
CTI_DEVICE void gelu2(float x0, float x1, float& g0, float& g1) {
  using namespace gelu_detail;
  const float u0 = fabsf(x0), u1 = fabsf(x1);
  const uint64_t uc = f2_pack(fminf(u0, kU0), fminf(u1, kU0));
  uint64_t acc = f2_pack(C10, C10);
  acc = f2_fma(acc, uc, f2_pack(C9, C9));
  acc = f2_fma(acc, uc, f2_pack(C8, C8));
  acc = f2_fma(acc, uc, f2_pack(C7, C7));
  acc = f2_fma(acc, uc, f2_pack(C6, C6));
  acc = f2_fma(acc, uc, f2_pack(C5, C5));
  acc = f2_fma(acc, uc, f2_pack(C4, C4));
  acc = f2_fma(acc, uc, f2_pack(C3, C3));
  acc = f2_fma(acc, uc, f2_pack(C2, C2));
  acc = f2_fma(acc, uc, f2_pack(C1, C1));
  acc = f2_fma(acc, uc, f2_pack(C0, C0));
  const uint64_t u = f2_pack(u0, u1);
  const uint64_t uu = f2_fma(u, u, f2_pack(0.0f, 0.0f));
  const uint64_t q = f2_fma(uu, f2_pack(kNegHalfLog2e, kNegHalfLog2e), acc);
  float q0, q1;
  f2_unpack(q, q0, q1);
  g0 = gelu_finish(x0, q0);
  g1 = gelu_finish(x1, q1);
}

CTI_DEVICE float gelu1(float x) {
  float g0, g1;
  gelu2(x, 0.0f, g0, g1);
  return g0;
}

// Epilogue activation of a pair (CTI_ACT_*).
CTI_DEVICE void act2(int act, float& a, float& b) {
  if (act == CTI_ACT_GELU) {
    gelu2(a, b, a, b);
  } else if (act == CTI_ACT_RELU) {
    a = fmaxf(a, 0.0f);
    b = fmaxf(b, 0.0f);
  }
}

}  // namespace cti
