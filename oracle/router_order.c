/*
 * Order-matched CPU restatement of the Top-2 router.  TEST ONLY.
 *
 * Same arithmetic as TopKGate.forward (baseline/infer.py:298-309) -
 * logits = x . w_g^T + b, top-2, softmax scores - but with the summation
 * order of the sm_100a kernel made explicit so expert indices can be
 * compared bit for bit: every logit is the sum of two fused-multiply-add
 * chains, one over the even d = 0, 2, 4, ... and one over the odd
 * d = 1, 3, 5, ..., each in increasing order starting from 0.0f; then
 * logit = (even + odd) + bias, two more roundings.  (The kernel runs the
 * two chains as the two lanes of one packed fp32x2 FMA.)  D is even.
 * Top-2 scans experts in order with strict '>' (the lower id wins a tie,
 * as in fused_top2_gate_kernel, online_best/infer.py:1710-1757).
 * renorm=1 -> gates p1/(p1+p2), p2/(p1+p2); renorm=0 -> raw softmax p1, p2.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, sizeof(f));
  return f;
}

void router_order_ref(const uint16_t* x, const float* wg, const float* bg, int64_t T, int D,
                      int E, int renorm, int32_t* idx2, float* gate2, float* logits_out) {
  float l[1024];
  for (int64_t t = 0; t < T; ++t) {
    const uint16_t* xr = x + t * D;
    for (int e = 0; e < E; ++e) {
      const float* w = wg + (int64_t)e * D;
      float even = 0.0f, odd = 0.0f;
      for (int d = 0; d < D; d += 2) {
        even = fmaf(bf16_to_f32(xr[d]), w[d], even);
        odd = fmaf(bf16_to_f32(xr[d + 1]), w[d + 1], odd);
      }
      l[e] = (even + odd) + bg[e];
      if (logits_out) logits_out[t * E + e] = l[e];
    }
    float b1 = l[0], b2 = 0.0f;
    int i1 = 0, i2 = -1;
    for (int e = 1; e < E; ++e) {
      if (l[e] > b1) {
        b2 = b1;
        i2 = i1;
        b1 = l[e];
        i1 = e;
      } else if (i2 < 0 || l[e] > b2) {
        b2 = l[e];
        i2 = e;
      }
    }
    float g1, g2;
    if (renorm) {
      const float r = expf(b2 - b1);
      const float inv = 1.0f / (1.0f + r);
      g1 = inv;
      g2 = r * inv;
    } else {
      float s = 0.0f;
      for (int e = 0; e < E; ++e) s += expf(l[e] - b1);
      g1 = 1.0f / s;
      g2 = expf(b2 - b1) / s;
    }
    idx2[2 * t] = i1;
    idx2[2 * t + 1] = i2;
    gate2[2 * t] = g1;
    gate2[2 * t + 1] = g2;
  }
}
