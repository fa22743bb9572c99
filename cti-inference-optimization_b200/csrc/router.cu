// Stage 1: fp32 Top-2 router over bf16 activations.
//
// Restates TopKGate.forward (baseline/infer.py:298-309: logits = w_g(x),
// softmax, topk(2)) and the fused_top2_gate_kernel of online_best/infer.py:
// 1624-1778 (strict '>' scan, lower expert id wins a tie) for any E <= 128,
// with fp32 weights.
//
// Summation order (reproduced bit for bit by oracle/router_order.c): the
// d-range is cut into S contiguous parts (S = cti_moe_router_split(D, E));
// part s is one fused-multiply-add chain over its d in increasing order,
// starting from 0; the parts are combined as ((p0 + p1) + (p2 + p3)) for
// S = 4, (p0 + p1) for S = 2; then the bias is added.  The kernel uses
// S <= 2 (S = 2 when E <= 64 and D % 16 == 0).
//
// Work split: S adjacent lanes share one token, each owning one part, so a
// block of 256 tokens runs 256*S/TPT threads (TPT tokens per lane group).
// A lane streams its part of the token rows straight from HBM into
// registers, 16 bytes at a time with the next load in flight; the router
// weights are staged once per d-slab in shared memory, part-interleaved and
// padded so the S parts read different banks while the lanes of one part
// read the same address (a broadcast).  The S partial logits are combined
// with two xor-shuffles, which leaves every lane of the group with the same
// bits.
//
// The block also produces the dispatch metadata: for each of its 256 tokens
// the rank of each route among the block's earlier routes to the same expert
// (token order, k=0 before k=1), and the block's per-expert histogram.
#include "common.cuh"

namespace cti {
namespace {

constexpr int kTok = CTI_ROUTER_BLOCK_TOKENS;  // tokens per block
constexpr int kWsFloats = 6144;                // 24 KB of staged router weights

int router_split(int D, int E) {
  const int max_split = E <= 64 ? 2 : 1;
  for (int s = max_split; s > 1; s >>= 1)
    if (D % (8 * s) == 0) return s;
  return 1;
}

template <int EMAX, int TPT, int S>
__global__ void __launch_bounds__(kTok * S / TPT) router_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ wg,
    const float* __restrict__ bg, int64_t T, int D, int E, int renorm,
    int32_t* __restrict__ idx2, float* __restrict__ gate2, int32_t* __restrict__ route_rank,
    int32_t* __restrict__ block_hist) {
  constexpr int NT = kTok * S / TPT;           // threads per block
  constexpr int GROUPS = kTok / TPT;           // token slots per j-group
  constexpr int EP = EMAX + (S > 1 ? 4 : 0);   // padded expert row
  constexpr int DSL = kWsFloats / (S * EP) / 8 * 8;  // d-slab per part
  static_assert(DSL % 8 == 0, "slab must hold whole 16-byte loads");
  __shared__ __align__(16) float ws[DSL][S][EP];
  __shared__ int cnt[EMAX];

  const int tid = threadIdx.x;
  const int part = tid % S;
  const int slot = tid / S;
  const int dq = D / S;  // d-values per part (a multiple of 8)
  const int64_t t0 = (int64_t)blockIdx.x * kTok;
  int64_t tok[TPT];
  bool valid[TPT];
  const uint4* xr[TPT];
#pragma unroll
  for (int j = 0; j < TPT; ++j) {
    tok[j] = t0 + j * GROUPS + slot;
    valid[j] = tok[j] < T;
    xr[j] = reinterpret_cast<const uint4*>(x + (valid[j] ? tok[j] : 0) * D + part * dq);
  }

  float acc[TPT][EMAX];
#pragma unroll
  for (int j = 0; j < TPT; ++j)
#pragma unroll
    for (int e = 0; e < EMAX; ++e) acc[j][e] = 0.0f;

  for (int d0 = 0; d0 < dq; d0 += DSL) {
    const int ds = min(DSL, dq - d0);
    __syncthreads();
    // ws[dd][p][e] = wg[e][p*dq + d0 + dd]; consecutive threads read
    // consecutive d of one expert row (coalesced).
    for (int i = tid; i < EMAX * S * ds; i += NT) {
      const int e = i / (S * ds);
      const int rem = i - e * (S * ds);
      const int p = rem / ds;
      const int dd = rem - p * ds;
      ws[dd][p][e] = (e < E) ? wg[(int64_t)e * D + p * dq + d0 + dd] : 0.0f;
    }
    __syncthreads();
    uint4 cur[TPT];
#pragma unroll
    for (int j = 0; j < TPT; ++j) cur[j] = valid[j] ? __ldg(xr[j] + d0 / 8) : make_uint4(0, 0, 0, 0);
    for (int dd = 0; dd < ds; dd += 8) {
      uint4 nxt[TPT];
      const bool more = dd + 8 < ds;
#pragma unroll
      for (int j = 0; j < TPT; ++j)
        nxt[j] = (valid[j] && more) ? __ldg(xr[j] + (d0 + dd + 8) / 8) : make_uint4(0, 0, 0, 0);
      float xv[TPT][8];
#pragma unroll
      for (int j = 0; j < TPT; ++j) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&cur[j]);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 f = __bfloat1622float2(h[u]);
          xv[j][2 * u] = f.x;
          xv[j][2 * u + 1] = f.y;
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4* w4 = reinterpret_cast<const float4*>(&ws[dd + u][part][0]);
#pragma unroll
        for (int q = 0; q < EMAX / 4; ++q) {
          const float4 w = w4[q];
#pragma unroll
          for (int j = 0; j < TPT; ++j) {
            acc[j][4 * q + 0] = fmaf(xv[j][u], w.x, acc[j][4 * q + 0]);
            acc[j][4 * q + 1] = fmaf(xv[j][u], w.y, acc[j][4 * q + 1]);
            acc[j][4 * q + 2] = fmaf(xv[j][u], w.z, acc[j][4 * q + 2]);
            acc[j][4 * q + 3] = fmaf(xv[j][u], w.w, acc[j][4 * q + 3]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < TPT; ++j) cur[j] = nxt[j];
    }
  }

  // Combine the parts: ((p0 + p1) + (p2 + p3)); addition is commutative, so
  // every lane of the group ends with the same value.
#pragma unroll
  for (int off = 1; off < S; off <<= 1)
#pragma unroll
    for (int j = 0; j < TPT; ++j)
#pragma unroll
      for (int e = 0; e < EMAX; ++e) acc[j][e] += __shfl_xor_sync(0xffffffffu, acc[j][e], off);

  // Logits, then top-2 by a strict '>' scan in expert order (lower id wins).
  int i1[TPT], i2[TPT];
  float g1[TPT], g2[TPT];
#pragma unroll
  for (int j = 0; j < TPT; ++j) {
    float best1 = 0.0f, best2 = 0.0f;
    int a1 = 0, a2 = -1;
#pragma unroll
    for (int e = 0; e < EMAX; ++e) {
      if (e < E) {
        const float l = acc[j][e] + bg[e];
        acc[j][e] = l;
        if (e == 0) {
          best1 = l;
          a1 = 0;
        } else if (l > best1) {
          best2 = best1;
          a2 = a1;
          best1 = l;
          a1 = e;
        } else if (a2 < 0 || l > best2) {
          best2 = l;
          a2 = e;
        }
      }
    }
    if (renorm) {
      // p1/(p1+p2) and p2/(p1+p2): the softmax denominator cancels.
      const float r = expf(best2 - best1);
      const float inv = 1.0f / (1.0f + r);
      g1[j] = inv;
      g2[j] = r * inv;
    } else {
      float sum = 0.0f;
#pragma unroll
      for (int e = 0; e < EMAX; ++e)
        if (e < E) sum += expf(acc[j][e] - best1);
      g1[j] = 1.0f / sum;
      g2[j] = expf(best2 - best1) / sum;
    }
    i1[j] = a1;
    i2[j] = a2;
  }

  // Block-level ranks and histogram.  Token groups j, then warps, run one
  // after the other so the ranks follow token order (within a warp, lane
  // groups are in token order); inside a warp, routes are grouped by expert
  // with ballots (one round per distinct expert).  Only part 0 of each lane
  // group takes part.
  for (int e = tid; e < EMAX; e += NT) cnt[e] = 0;
  __syncthreads();
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const unsigned lt = (1u << lane) - 1u;
  int rank0[TPT], rank1[TPT];
#pragma unroll
  for (int j = 0; j < TPT; ++j) {
    rank0[j] = rank1[j] = 0;
    const bool mine = valid[j] && part == 0;
    for (int w = 0; w < NT / 32; ++w) {
      if (warp == w) {
        bool done0 = !mine, done1 = !mine;
        while (true) {
          const unsigned p0 = __ballot_sync(0xffffffffu, !done0);
          const unsigned p1 = __ballot_sync(0xffffffffu, !done1);
          if ((p0 | p1) == 0u) break;
          const int e = p0 ? __shfl_sync(0xffffffffu, i1[j], __ffs(p0) - 1)
                           : __shfl_sync(0xffffffffu, i2[j], __ffs(p1) - 1);
          const unsigned b0 = __ballot_sync(0xffffffffu, mine && i1[j] == e);
          const unsigned b1 = __ballot_sync(0xffffffffu, mine && i2[j] == e);
          const int base = cnt[e];
          const int before = base + __popc(b0 & lt) + __popc(b1 & lt);
          if (!done0 && i1[j] == e) {
            rank0[j] = before;
            done0 = true;
          }
          if (!done1 && i2[j] == e) {
            rank1[j] = before;
            done1 = true;
          }
          __syncwarp();
          if (lane == 0) cnt[e] = base + __popc(b0) + __popc(b1);
          __syncwarp();
        }
      }
      __syncthreads();
    }
  }

  if (part == 0) {
#pragma unroll
    for (int j = 0; j < TPT; ++j) {
      if (valid[j]) {
        reinterpret_cast<int2*>(idx2)[tok[j]] = make_int2(i1[j], i2[j]);
        reinterpret_cast<float2*>(gate2)[tok[j]] = make_float2(g1[j], g2[j]);
        reinterpret_cast<int2*>(route_rank)[tok[j]] = make_int2(rank0[j], rank1[j]);
      }
    }
  }
  for (int e = tid; e < E; e += NT) block_hist[(int64_t)blockIdx.x * E + e] = cnt[e];
}

template <int EMAX, int TPT, int S>
cudaError_t launch_router(const __nv_bfloat16* x, const float* wg, const float* bg, int64_t T,
                          int D, int E, int renorm, int32_t* idx2, float* gate2, int32_t* rank,
                          int32_t* hist, cudaStream_t s) {
  const int64_t blocks = (T + kTok - 1) / kTok;
  static bool attr_set = false;
  if (!attr_set) {
    // Two blocks per SM need more than the default shared-memory carveout.
    cudaFuncSetAttribute(router_kernel<EMAX, TPT, S>,
                         cudaFuncAttributePreferredSharedMemoryCarveout,
                         (int)cudaSharedmemCarveoutMaxShared);
    attr_set = true;
  }
  router_kernel<EMAX, TPT, S><<<(unsigned)blocks, kTok * S / TPT, 0, s>>>(
      x, wg, bg, T, D, E, renorm, idx2, gate2, rank, hist);
  return cudaGetLastError();
}

}  // namespace
}  // namespace cti

extern "C" int cti_moe_router_split(int D, int E) {
  if (D <= 0 || E < 1) return 0;
  return cti::router_split(D, E);
}

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
  if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) != 0 || (reinterpret_cast<uintptr_t>(idx2) & 7) ||
      (reinterpret_cast<uintptr_t>(gate2) & 7) || (reinterpret_cast<uintptr_t>(route_rank) & 7))
    return CTI_ERR_INVALID_ARG;
  const auto* x = static_cast<const __nv_bfloat16*>(x_bf16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  (void)status;
  const int sp = router_split(D, E);
  if (E <= 8)
    err = sp == 2 ? launch_router<8, 1, 2>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank,
                                           block_hist, s)
                  : launch_router<8, 1, 1>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank,
                                           block_hist, s);
  else if (E <= 16)
    err = sp == 2 ? launch_router<16, 1, 2>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank,
                                            block_hist, s)
                  : launch_router<16, 1, 1>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank,
                                            block_hist, s);
  else if (E <= 32)
    err = sp == 2 ? launch_router<32, 1, 2>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank,
                                            block_hist, s)
                  : launch_router<32, 1, 1>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank,
                                            block_hist, s);
  else if (E <= 64)
    err = sp == 2 ? launch_router<64, 1, 2>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank,
                                            block_hist, s)
                  : launch_router<64, 1, 1>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank,
                                            block_hist, s);
  else
    err = launch_router<128, 1, 1>(x, wg, bg, T, D, E, renorm, idx2, gate2, route_rank,
                                   block_hist, s);
  return err == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}
