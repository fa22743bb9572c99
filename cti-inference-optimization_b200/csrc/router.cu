// Stage 1: fp32 Top-2 router over bf16 activations.
//
// Restates TopKGate.forward (baseline/infer.py:298-309: logits = w_g(x),
// softmax, topk(2)) and the fused_top2_gate_kernel of online_best/infer.py:
// 1624-1778 (strict '>' scan, lower expert id wins a tie) for any E <= 128,
// with fp32 weights.
//
// Summation order (reproduced bit for bit by oracle/router_order.c): every
// logit is one fused-multiply-add chain over d = 0..D-1 in increasing order,
// starting from 0, and the bias is added after it.
//
// The logits of a 128-token block are a [128 x D] x [D x E] fp32 product,
// computed as a register-tiled SGEMM: each thread owns a 4-token x 4-expert
// tile (16 independent chains) and, per d, reads one float4 of activations
// and one float4 of weights from shared memory - two conflict-free loads per
// 16 FMAs, so the kernel is bound by the FMA pipe rather than by shared
// memory.  Activations and router weights are staged 32 d at a time
// (activations converted to fp32, both d-major), and the global loads of the
// next step are in flight while the current step's FMAs run.
//
// The block also produces the dispatch metadata: for each of its 128 tokens
// the rank of each route among the block's earlier routes to the same expert
// (token order, k=0 before k=1), and the block's per-expert histogram.
#include "common.cuh"

namespace cti {
namespace {

constexpr int kTok = CTI_ROUTER_BLOCK_TOKENS;  // 128 tokens per block
constexpr int kDC = 32;                        // d-values staged per step

template <int EMAX>
struct RouterSmem {
  static constexpr int kStage = kDC * kTok + kDC * EMAX;
  static constexpr int kLogits = kTok * (EMAX + 1);
  static constexpr int kFloats = kStage > kLogits ? kStage : kLogits;
  static constexpr size_t kBytes = (size_t)kFloats * 4 + (size_t)(1 + kTok / 32) * EMAX * 4;
};

template <int EMAX>
constexpr int router_threads() {
  return 8 * EMAX < kTok ? kTok : 8 * EMAX;
}

template <int EMAX>
__global__ void __launch_bounds__(router_threads<EMAX>()) router_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ wg,
    const float* __restrict__ bg, int64_t T, int D, int E, int renorm,
    int32_t* __restrict__ idx2, float* __restrict__ gate2, int32_t* __restrict__ route_rank,
    int32_t* __restrict__ block_hist) {
  constexpr int EG = EMAX / 4;       // expert groups of 4
  constexpr int NG = 32 * EG;        // GEMM threads: 32 token groups x EG expert groups
  constexpr int NT = NG < kTok ? kTok : NG;  // at least one thread per token
  // Dynamic shared memory: xs[kDC][kTok] and ws[kDC][EMAX] while the
  // logits are accumulated, then reused as lg[kTok][EMAX + 1]; then cnt[EMAX]
  // (block counts) and the per-warp counts [kTok/32][EMAX].
  extern __shared__ __align__(16) float smem_f[];
  float (*xs)[kTok] = reinterpret_cast<float (*)[kTok]>(smem_f);
  float (*ws)[EMAX] = reinterpret_cast<float (*)[EMAX]>(smem_f + kDC * kTok);
  float (*lg)[EMAX + 1] = reinterpret_cast<float (*)[EMAX + 1]>(smem_f);
  int* cnt = reinterpret_cast<int*>(smem_f + RouterSmem<EMAX>::kFloats);

  const int tid = threadIdx.x;
  const int eg = tid % EG;   // experts 4*eg .. 4*eg+3
  const int tg = tid / EG;   // tokens  4*tg .. 4*tg+3
  const bool gemm = tid < NG;
  const int64_t t0 = (int64_t)blockIdx.x * kTok;

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  // x chunks are prefetched into registers one step ahead: chunk c of a
  // d-step is token c % 128, 8-wide d-part c / 128 (consecutive lanes store
  // consecutive tokens in shared memory).
  constexpr int kXChunks = kTok * (kDC / 8);                   // 512 per step
  constexpr int kXPerThread = (kXChunks + NT - 1) / NT;
  constexpr int kWChunks = EMAX * (kDC / 4);                   // float4s of wg per step
  constexpr int kWPerThread = (kWChunks + NT - 1) / NT;
  uint4 xpre[kXPerThread];
  float4 wpre[kWPerThread];
  auto load_step = [&](int d0) {
    const int dc = min(kDC, D - d0);
#pragma unroll
    for (int q = 0; q < kXPerThread; ++q) {
      const int c = tid + q * NT;
      const int tok = c % kTok;
      const int part = c / kTok;
      xpre[q] = (c < kXChunks && part * 8 < dc && t0 + tok < T)
                    ? __ldg(reinterpret_cast<const uint4*>(x + (t0 + tok) * D + d0) + part)
                    : make_uint4(0, 0, 0, 0);
    }
    // wg[e][d0 + 4*j .. +3] for chunk c = e * (kDC/4) + j (coalesced along d).
#pragma unroll
    for (int q = 0; q < kWPerThread; ++q) {
      const int c = tid + q * NT;
      const int e = c / (kDC / 4);
      const int j = c % (kDC / 4);
      wpre[q] = (c < kWChunks && e < E && 4 * j < dc)
                    ? __ldg(reinterpret_cast<const float4*>(wg + (int64_t)e * D + d0) + j)
                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  };
  load_step(0);
  for (int d0 = 0; d0 < D; d0 += kDC) {
    const int dc = min(kDC, D - d0);  // a multiple of 8
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kXPerThread; ++q) {
      const int c = tid + q * NT;
      if (c < kXChunks) {
        const int tok = c % kTok;
        const int part = c / kTok;
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&xpre[q]);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 f = __bfloat1622float2(h[u]);
          xs[part * 8 + 2 * u][tok] = f.x;
          xs[part * 8 + 2 * u + 1][tok] = f.y;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kWPerThread; ++q) {
      const int c = tid + q * NT;
      if (c < kWChunks) {
        const int e = c / (kDC / 4);
        const int j = c % (kDC / 4);
        ws[4 * j + 0][e] = wpre[q].x;
        ws[4 * j + 1][e] = wpre[q].y;
        ws[4 * j + 2][e] = wpre[q].z;
        ws[4 * j + 3][e] = wpre[q].w;
      }
    }
    __syncthreads();
    if (d0 + kDC < D) load_step(d0 + kDC);  // in flight during this step's FMAs
    if (gemm) {
      float4 xv = *reinterpret_cast<const float4*>(&xs[0][4 * tg]);
      float4 wv = *reinterpret_cast<const float4*>(&ws[0][4 * eg]);
#pragma unroll 8
      for (int dd = 0; dd < dc; ++dd) {
        // Operands of step dd+1 are loaded before the FMAs of step dd.
        const int nd = dd + 1 < dc ? dd + 1 : dd;
        const float4 xn = *reinterpret_cast<const float4*>(&xs[nd][4 * tg]);
        const float4 wn = *reinterpret_cast<const float4*>(&ws[nd][4 * eg]);
        const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
        const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
        xv = xn;
        wv = wn;
      }
    }
  }
  __syncthreads();  // xs/ws are about to be overwritten by lg
  if (gemm) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) lg[4 * tg + i][4 * eg + j] = acc[i][j];
  }
  __syncthreads();

  // One thread per token: logits, top-2 by a strict '>' scan in expert order
  // (lower id wins), gates.
  const bool has_tok = tid < kTok;
  const int64_t t = t0 + tid;
  const bool valid = has_tok && t < T;
  int i1 = 0, i2 = -1;
  float g1 = 0.0f, g2 = 0.0f;
  if (has_tok) {
    float best1 = 0.0f, best2 = 0.0f;
    for (int e = 0; e < E; ++e) {
      const float l = lg[tid][e] + bg[e];
      lg[tid][e] = l;
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
    if (renorm) {
      // p1/(p1+p2) and p2/(p1+p2): the softmax denominator cancels.
      const float r = expf(best2 - best1);
      const float inv = 1.0f / (1.0f + r);
      g1 = inv;
      g2 = r * inv;
    } else {
      float sum = 0.0f;
      for (int e = 0; e < E; ++e) sum += expf(lg[tid][e] - best1);
      g1 = 1.0f / sum;
      g2 = expf(best2 - best1) / sum;
    }
  }

  // Block-level ranks and histogram.  Every warp ranks its 32 tokens' routes
  // at once (routes grouped by expert with ballots, one round per distinct
  // expert; k=0 before k=1 within a token) and records its own per-expert
  // counts; then an exclusive prefix over the warps per expert turns the
  // in-warp ranks into in-block ranks in token order.
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const unsigned lt = (1u << lane) - 1u;
  int* wcnt = cnt + EMAX;  // [kTok / 32][EMAX] per-warp counts
  for (int i = tid; i < (kTok / 32) * EMAX; i += NT) wcnt[i] = 0;
  __syncthreads();
  int rank0 = 0, rank1 = 0;
  if (warp < kTok / 32) {
    bool done0 = !valid, done1 = !valid;
    while (true) {
      const unsigned p0 = __ballot_sync(0xffffffffu, !done0);
      const unsigned p1 = __ballot_sync(0xffffffffu, !done1);
      if ((p0 | p1) == 0u) break;
      const int e = p0 ? __shfl_sync(0xffffffffu, i1, __ffs(p0) - 1)
                       : __shfl_sync(0xffffffffu, i2, __ffs(p1) - 1);
      const unsigned b0 = __ballot_sync(0xffffffffu, valid && i1 == e);
      const unsigned b1 = __ballot_sync(0xffffffffu, valid && i2 == e);
      const int before = __popc(b0 & lt) + __popc(b1 & lt);
      if (!done0 && i1 == e) {
        rank0 = before;
        done0 = true;
      }
      if (!done1 && i2 == e) {
        rank1 = before;
        done1 = true;
      }
      if (lane == 0) wcnt[warp * EMAX + e] = __popc(b0) + __popc(b1);
    }
  }
  __syncthreads();
  // Exclusive prefix over warps, per expert; cnt[e] = block total.
  for (int e = tid; e < EMAX; e += NT) {
    int run = 0;
#pragma unroll
    for (int w = 0; w < kTok / 32; ++w) {
      const int v = wcnt[w * EMAX + e];
      wcnt[w * EMAX + e] = run;
      run += v;
    }
    cnt[e] = run;
  }
  __syncthreads();
  if (valid) {
    rank0 += wcnt[warp * EMAX + i1];
    rank1 += wcnt[warp * EMAX + i2];
  }

  if (valid) {
    reinterpret_cast<int2*>(idx2)[t] = make_int2(i1, i2);
    reinterpret_cast<float2*>(gate2)[t] = make_float2(g1, g2);
    reinterpret_cast<int2*>(route_rank)[t] = make_int2(rank0, rank1);
  }
  for (int e = tid; e < E; e += NT) block_hist[(int64_t)blockIdx.x * E + e] = cnt[e];
}

template <int EMAX>
cudaError_t launch_router(const __nv_bfloat16* x, const float* wg, const float* bg, int64_t T,
                          int D, int E, int renorm, int32_t* idx2, float* gate2, int32_t* rank,
                          int32_t* hist, cudaStream_t s) {
  const int64_t blocks = (T + kTok - 1) / kTok;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(router_kernel<EMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)RouterSmem<EMAX>::kBytes) != cudaSuccess)
      return cudaErrorInvalidValue;
    attr_set = true;
  }
  router_kernel<EMAX><<<(unsigned)blocks, router_threads<EMAX>(), RouterSmem<EMAX>::kBytes, s>>>(x, wg, bg, T, D, E, renorm, idx2,
                                                            gate2, rank, hist);
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
  if (D % 8 != 0) return CTI_ERR_UNSUPPORTED;
  if (T == 0) return CTI_OK;
  if (!x_bf16 || !wg || !bg || !idx2 || !gate2 || !route_rank || !block_hist)
    return CTI_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) != 0 || (reinterpret_cast<uintptr_t>(wg) & 15) ||
      (reinterpret_cast<uintptr_t>(idx2) & 7) ||
      (reinterpret_cast<uintptr_t>(gate2) & 7) || (reinterpret_cast<uintptr_t>(route_rank) & 7))
    return CTI_ERR_INVALID_ARG;
  const auto* x = static_cast<const __nv_bfloat16*>(x_bf16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  (void)status;
  if (E <= 8)
    err = launch_router<8>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist, s);
  else if (E <= 16)
    err = launch_router<16>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist, s);
  else if (E <= 32)
    err = launch_router<32>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist, s);
  else if (E <= 64)
    err = launch_router<64>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist, s);
  else
    err = launch_router<128>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist, s);
  return err == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}
