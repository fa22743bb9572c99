/*
 * Order-matched CPU restatement of the Top-2 router.  TEST ONLY.
 *
 * Same arithmetic as TopKGate.forward (baseline/infer.py:298-309) -
 * logits = x . w_g^T + b, top-2, softmax scores - but with the summation
 * order of the sm_100a kernel made explicit so expert indices can be
 * compared bit for bit: the d-range is cut into S contiguous parts (S from
 * router_split below, the rule the kernel documents), each part is one
 * fused-multiply-add chain over its d in increasing order starting from
 * 0.0f, the parts are combined as ((p0+p1)+(p2+p3)) / (p0+p1) / p0, and
 * the bias is added in a separate rounding.
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

int router_split(int D, int E) {
  const int max_split = E <= 64 ? 2 : 1;
  for (int s = max_split; s > 1; s >>= 1)
    if (D % (8 * s) == 0) return s;
  return 1;
}

void router_order_ref(const uint16_t* x, const float* wg, const float* bg, int64_t T, int D,
                      int E, int renorm, int32_t* idx2, float* gate2, float* logits_out) {
  float l[1024];
  const int S = router_split(D, E);
  const int dq = D / S;
  for (int64_t t = 0; t < T; ++t) {
    const uint16_t* xr = x + t * D;
    for (int e = 0; e < E; ++e) {
      const float* w = wg + (int64_t)e * D;
      float p[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int s = 0; s < S; ++s)
        for (int d = s * dq; d < (s + 1) * dq; ++d) p[s] = fmaf(bf16_to_f32(xr[d]), w[d], p[s]);
      float acc;
      if (S == 4)
        acc = (p[0] + p[1]) + (p[2] + p[3]);
      else if (S == 2)
        acc = p[0] + p[1];
      else
        acc = p[0];
      l[e] = acc + bg[e];
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
