// GELU epilogue math: GELU(x) = x * Phi(x) with Phi the standard normal CDF
// (the exact-erf GELU of torch.nn.functional.gelu), to near fp32 accuracy
// (relative error below 9.2e-6 on [-4.5, 4.5], absolute error below 5.3e-7
// everywhere; gelu_fit.py prints both).
//
// With u = |x| and h(u) = erfc(u/sqrt2)/2:  GELU(x) = max(x, 0) - u * h(u),
// exact on both sides (no 1 - Phi cancellation for x << 0), and
// h(u) = 2^P(u) with P(u) = log2(erfc(u/sqrt2)/2) smooth - its -u^2 decay is
// itself a polynomial term - so a degree-7 polynomial (a Chebyshev
// least-squares fit on [0, 6], converted to monomials by gelu_fit.py)
// evaluates it with seven fused multiply-adds, and one ex2 finishes h.
// u is not clamped: past 6 the polynomial keeps falling (its largest value
// for u > 6 is P(6) = -29.9, so h <= 9.9e-10 there, and it goes to 0), which
// saves one min per value over clamping u to the fit range.
//
// Pairs of values are evaluated with the packed fp32x2 FMA of sm_100, which
// halves the issue slots of the polynomial.
#pragma once

#include "common.cuh"

namespace cti {

namespace gelu_detail {
// P(u) = sum_k C_k u^k (gelu_fit.py, degree 7, Chebyshev fit on [0, 6]).
constexpr float C0 = -0.9999869465827942f, C1 = -1.1513246297836304f,
                C2 = -0.4582974314689636f, C3 = -0.0541183240711689f,
                C4 = 0.008582375012338161f, C5 = -0.0009488713694736362f,
                C6 = 6.386057066265494e-05f, C7 = -1.9449223600531695e-06f;
}  // namespace gelu_detail

// In-place GELU of N values (N even), ordered so that the N/2 packed Horner
// chains interleave: every step issues N/2 independent f32x2 FMAs.
// Infinite inputs give NaN.
template <int N>
CTI_DEVICE void gelu_n(float (&v)[N]) {
  using namespace gelu_detail;
  constexpr int P = N / 2;
  uint64_t uc[P], acc[P];
#pragma unroll
  for (int p = 0; p < P; ++p) {
    uc[p] = f2_pack(fabsf(v[2 * p]), fabsf(v[2 * p + 1]));
    acc[p] = f2_pack(C7, C7);
  }
  const float coef[7] = {C6, C5, C4, C3, C2, C1, C0};
#pragma unroll
  for (int k = 0; k < 7; ++k) {
    const uint64_t ck = f2_pack(coef[k], coef[k]);
#pragma unroll
    for (int p = 0; p < P; ++p) acc[p] = f2_fma(acc[p], uc[p], ck);
  }
#pragma unroll
  for (int p = 0; p < P; ++p) {
    float q0, q1;
    f2_unpack(acc[p], q0, q1);
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
