// Stage 1: fp32 Top-2 router over bf16 activations.
//
// Restates TopKGate.forward (baseline/infer.py:298-309: logits = w_g(x),
// softmax, topk(2)) and the fused_top2_gate_kernel of online_best/infer.py:
// 1624-1778 (strict '>' scan, lower expert id wins a tie) for any E <= 128,
// with fp32 weights.  One thread owns one token; its E logits live in
// registers as E independent fused-multiply-add chains over d = 0..D-1 (the
// order the CPU restatement in oracle/router_order.c reproduces bit for bit).
// Activations and router weights are staged through shared memory in
// 32-wide d-slices: x is converted to fp32 and transposed so that the 32
// lanes of a warp read 32 consecutive words, and the weight slice is stored
// d-major so every lane reads the same float4 (a broadcast).
//
// The block also produces the dispatch metadata: for each of its 128 tokens
// the rank of each route among the block's earlier routes to the same expert
// (token order, k=0 before k=1), and the block's per-expert histogram.
#include "common.cuh"

namespace cti {
namespace {

constexpr int kTok = CTI_ROUTER_BLOCK_TOKENS;  // tokens (= threads) per block
constexpr int kDs = 32;                        // d-slice staged per step

template <int EMAX>
__global__ void __launch_bounds__(kTok) router_kernel(const __nv_bfloat16* __restrict__ x,
                                                     const float* __restrict__ wg,
                                                     const float* __restrict__ bg, int64_t T,
                                                     int D, int E, int renorm,
                                                     int32_t* __restrict__ idx2,
                                                     float* __restrict__ gate2,
                                                     int32_t* __restrict__ route_rank,
                                                     int32_t* __restrict__ block_hist,
                                                     int32_t* status) {
  __shared__ float xs[kDs][kTok + 1];
  __shared__ __align__(16) float ws[kDs][EMAX];
  __shared__ int cnt[EMAX];

  const int tid = threadIdx.x;
  const int64_t t0 = (int64_t)blockIdx.x * kTok;
  const int64_t t = t0 + tid;
  const bool valid = t < T;

  float acc[EMAX];
#pragma unroll
  for (int e = 0; e < EMAX; ++e) acc[e] = 0.0f;

  for (int d0 = 0; d0 < D; d0 += kDs) {
    // Stage x[t0:t0+128, d0:d0+32] as fp32, transposed.  512 chunks of 8
    // bf16 (16 bytes): chunk c covers token c/4, d-offset (c%4)*8.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = tid + i * kTok;
      const int tok = c >> 2;
      const int part = (c & 3) * 8;
      float v[8];
      if (t0 + tok < T) {
        const uint4 raw = *reinterpret_cast<const uint4*>(x + (t0 + tok) * D + d0 + part);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          v[2 * j] = f.x;
          v[2 * j + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) xs[part + j][tok] = v[j];
    }
    // Stage wg[:, d0:d0+32] d-major; experts >= E read as zero.
    for (int i = tid; i < kDs * EMAX; i += kTok) {
      const int e = i / kDs;
      const int dd = i % kDs;
      ws[dd][e] = (e < E) ? wg[(int64_t)e * D + d0 + dd] : 0.0f;
    }
    __syncthreads();
#pragma unroll 4
    for (int dd = 0; dd < kDs; ++dd) {
      const float xv = xs[dd][tid];
      const float4* w4 = reinterpret_cast<const float4*>(&ws[dd][0]);
#pragma unroll
      for (int q = 0; q < EMAX / 4; ++q) {
        const float4 w = w4[q];
        acc[4 * q + 0] = fmaf(xv, w.x, acc[4 * q + 0]);
        acc[4 * q + 1] = fmaf(xv, w.y, acc[4 * q + 1]);
        acc[4 * q + 2] = fmaf(xv, w.z, acc[4 * q + 2]);
        acc[4 * q + 3] = fmaf(xv, w.w, acc[4 * q + 3]);
      }
    }
    __syncthreads();
  }

  // logits, then top-2 by a strict '>' scan in expert order (lower id wins).
  float best1 = 0.0f, best2 = 0.0f;
  int i1 = 0, i2 = -1;
#pragma unroll
  for (int e = 0; e < EMAX; ++e) {
    if (e < E) {
      const float l = acc[e] + bg[e];
      acc[e] = l;
      if (e == 0) {
        best1 = l;
        i1 = 0;
      } else if (l > best1) {
        best2 = best1;
        i2 = i1;
        best1 = l;
        i1 = e;
      } else if (i2 < 0 || l > best2) {
        best2 = l;
        i2 = e;
      }
    }
  }

  float g1, g2;
  if (renorm) {
    // p1/(p1+p2) and p2/(p1+p2): the softmax denominator cancels.
    const float r = expf(best2 - best1);
    const float inv = 1.0f / (1.0f + r);
    g1 = inv;
    g2 = r * inv;
  } else {
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < EMAX; ++e)
      if (e < E) s += expf(acc[e] - best1);
    g1 = 1.0f / s;
    g2 = expf(best2 - best1) / s;
  }

  // Block-level ranks and histogram.  Warps run one after the other so the
  // ranks follow token order; inside a warp, routes are grouped by expert
  // with ballots (one round per distinct expert present in the warp).
  for (int e = tid; e < EMAX; e += kTok) cnt[e] = 0;
  __syncthreads();
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const unsigned lt = (1u << lane) - 1u;
  int rank0 = 0, rank1 = 0;
  for (int w = 0; w < kTok / 32; ++w) {
    if (warp == w) {
      bool done0 = !valid, done1 = !valid;
      while (true) {
        const unsigned p0 = __ballot_sync(0xffffffffu, !done0);
        const unsigned p1 = __ballot_sync(0xffffffffu, !done1);
        if ((p0 | p1) == 0u) break;
        const int e = p0 ? __shfl_sync(0xffffffffu, i1, __ffs(p0) - 1)
                         : __shfl_sync(0xffffffffu, i2, __ffs(p1) - 1);
        const unsigned b0 = __ballot_sync(0xffffffffu, valid && i1 == e);
        const unsigned b1 = __ballot_sync(0xffffffffu, valid && i2 == e);
        const int base = cnt[e];
        const int before = base + __popc(b0 & lt) + __popc(b1 & lt);
        if (!done0 && i1 == e) {
          rank0 = before;
          done0 = true;
        }
        if (!done1 && i2 == e) {
          rank1 = before;
          done1 = true;
        }
        __syncwarp();
        if (lane == 0) cnt[e] = base + __popc(b0) + __popc(b1);
        __syncwarp();
      }
    }
    __syncthreads();
  }

  if (valid) {
    reinterpret_cast<int2*>(idx2)[t] = make_int2(i1, i2);
    reinterpret_cast<float2*>(gate2)[t] = make_float2(g1, g2);
    reinterpret_cast<int2*>(route_rank)[t] = make_int2(rank0, rank1);
  }
  for (int e = tid; e < E; e += kTok) block_hist[(int64_t)blockIdx.x * E + e] = cnt[e];
  (void)status;
}

template <int EMAX>
cudaError_t launch_router(const __nv_bfloat16* x, const float* wg, const float* bg, int64_t T,
                          int D, int E, int renorm, int32_t* idx2, float* gate2, int32_t* rank,
                          int32_t* hist, int32_t* status, cudaStream_t s) {
  const int64_t blocks = (T + kTok - 1) / kTok;
  router_kernel<EMAX><<<(unsigned)blocks, kTok, 0, s>>>(x, wg, bg, T, D, E, renorm, idx2, gate2,
                                                        rank, hist, status);
  return cudaGetLastError();
}

}  // namespace
}  // namespace cti

extern "C" int cti_moe_router(const void* x_bf16, const float* wg, const float* bg, int64_t T,
                              int D, int E, int renorm, int32_t* idx2, float* gate2,
                              int32_t* route_rank, int32_t* block_hist, int32_t* status,
                              void* stream) {
  using namespace cti;
  if (T < 0 || D <= 0 || E < 2 || E > CTI_MAX_EXPERTS) return CTI_ERR_INVALID_ARG;
  if (D % kDs != 0) return CTI_ERR_UNSUPPORTED;
  if (T == 0) return CTI_OK;
  if (!x_bf16 || !wg || !bg || !idx2 || !gate2 || !route_rank || !block_hist)
    return CTI_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) != 0 || (reinterpret_cast<uintptr_t>(idx2) & 7) ||
      (reinterpret_cast<uintptr_t>(gate2) & 7) || (reinterpret_cast<uintptr_t>(route_rank) & 7))
    return CTI_ERR_INVALID_ARG;
  const auto* x = static_cast<const __nv_bfloat16*>(x_bf16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  if (E <= 8)
    err = launch_router<8>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist,
                           status, s);
  else if (E <= 16)
    err = launch_router<16>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist,
                            status, s);
  else if (E <= 32)
    err = launch_router<32>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist,
                            status, s);
  else if (E <= 64)
    err = launch_router<64>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist,
                            status, s);
  else
    err = launch_router<128>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist,
                             status, s);
  return err == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}
