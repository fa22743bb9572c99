// GELU epilogue math: GELU(x) = x * Phi(x) with Phi the standard normal CDF
// (the exact-erf GELU of torch.nn.functional.gelu), to near fp32 accuracy
// (relative error below 1.6e-5 on [-4.5, 4.5], 5e-6 on [-3, 3], absolute
// error below 7.2e-7 everywhere; gelu_fit.py prints both).
//
// With u = |x|:  erfc(u/sqrt2) = 2^(Q(u) - u^2 * log2(e)/2), where
// Q(u) = log2(erfcx(u/sqrt2)) and erfcx(z) = exp(z^2) erfc(z).  Q is smooth
// and slowly varying, so a degree-6 polynomial (a Chebyshev least-squares
// fit on [0, 4.5], converted to monomials by gelu_fit.py) evaluates it with
// six fused multiply-adds; one ex2 finishes erfc; then
// GELU(x) = max(x, 0) - |x| * erfc(|x|/sqrt2)/2.  Past u = 4.5,
// erfc(u/sqrt2) < 6.8e-6 and u is clamped inside Q only (the exact -u^2
// term keeps the decay).
//
// Pairs of values are evaluated with the packed fp32x2 FMA of sm_100, which
// halves the issue slots of the polynomial.
#pragma once

#include "common.cuh"

namespace cti {

namespace gelu_detail {
// Q(u) = sum_k C_k u^k (gelu_fit.py, degree 6, Chebyshev fit on [0, 4.5]).
constexpr float C0 = -6.183180630614515e-06f, C1 = -1.1510794162750244f,
                C2 = 0.26230019330978394f, C3 = -0.05317788943648338f,
                C4 = 0.008000310510396957f, C5 = -0.000760704861022532f,
                C6 = 3.341770207043737e-05f;
constexpr float kU0 = 4.5f;
constexpr float kNegHalfLog2e = -0.72134752044448170368f;  // -log2(e)/2
}  // namespace gelu_detail

CTI_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// In-place GELU of N values (N even), ordered so that the N/2 packed Horner
// chains interleave: every step issues N/2 independent f32x2 FMAs.  Uses
//   GELU(x) = max(x, 0) - |x| * erfc(|x|/sqrt2)/2,
// which is exact on both sides (no 1 - Phi cancellation for x << 0); the
// factor 1/2 is folded into the constant term (log2(1/2) = -1).
// Infinite inputs give NaN.
template <int N>
CTI_DEVICE void gelu_n(float (&v)[N]) {
  using namespace gelu_detail;
  constexpr int P = N / 2;
  uint64_t uc[P], acc[P];
#pragma unroll
  for (int p = 0; p < P; ++p) {
    uc[p] = f2_pack(fminf(fabsf(v[2 * p]), kU0), fminf(fabsf(v[2 * p + 1]), kU0));
    acc[p] = f2_pack(C6, C6);
  }
  const float coef[6] = {C5, C4, C3, C2, C1, C0 - 1.0f};
#pragma unroll
  for (int k = 0; k < 6; ++k) {
    const uint64_t ck = f2_pack(coef[k], coef[k]);
#pragma unroll
    for (int p = 0; p < P; ++p) acc[p] = f2_fma(acc[p], uc[p], ck);
  }
  const uint64_t neg_half_log2e = f2_pack(kNegHalfLog2e, kNegHalfLog2e);
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const uint64_t x = f2_pack(v[2 * p], v[2 * p + 1]);
    const uint64_t q = f2_fma(f2_mul(x, x), neg_half_log2e, acc[p]);
    float q0, q1;
    f2_unpack(q, q0, q1);
    const float h0 = ex2_approx(q0), h1 = ex2_approx(q1);  // erfc(|x|/sqrt2)/2
    v[2 * p] = fmaf(-fabsf(v[2 * p]), h0, fmaxf(v[2 * p], 0.0f));
    v[2 * p + 1] = fmaf(-fabsf(v[2 * p + 1]), h1, fmaxf(v[2 * p + 1], 0.0f));
  }
}

// GELU of two values.
CTI_DEVICE void gelu2(float x0, float x1, float& g0, float& g1) {
  float v[2] = {x0, x1};
  gelu_n<2>(v);
  g0 = v[0];
  g1 = v[1];
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

// Epilogue activation of N values.
template <int N>
CTI_DEVICE void act_n(int act, float (&v)[N]) {
  if (act == CTI_ACT_GELU) {
    gelu_n<N>(v);
  } else if (act == CTI_ACT_RELU) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = fmaxf(v[i], 0.0f);
  }
}

}  // namespace cti
