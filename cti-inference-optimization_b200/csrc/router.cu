// Stage 1: fp32 Top-2 router over bf16 activations.
//
// Restates TopKGate.forward (baseline/infer.py:298-309: logits = w_g(x),
// softmax, topk(2)) and the fused_top2_gate_kernel of online_best/infer.py:
// 1624-1778 (strict '>' scan, lower expert id wins a tie) for any E <= 128,
// with fp32 weights.
//
// Summation order (reproduced bit for bit by oracle/router_order.c): every
// logit is the sum of two fused-multiply-add chains, one over the even d
// and one over the odd d, each in increasing d starting from 0; then
// logit = (even + odd) + bias.  The two chains are the two lanes of one
// packed fma.rn.f32x2: the pair (x[d], x[d+1]) of a token row times the pair
// (w[d], w[d+1]) of an expert row, both adjacent in memory, so one issue
// does two FMAs with no data rearranged.
//
// The logits of a 128-token block are a [128 x D] x [D x E] fp32 product,
// computed as a register-tiled SGEMM: each thread owns TPT tokens x 4
// experts (tokens tg + TG*i, experts eg + EG*j), each an accumulator pair,
// so the token rows and expert rows a warp reads at once are consecutive
// rows, which the 16-byte row padding spreads over the banks.  Activations
// (bf16, [token][d]) and router weights (fp32, [expert][d]) stream through a
// kStages-deep ring of shared-memory stages, kDC d-values each, filled with
// cp.async straight from global memory: coalesced row segments, no register
// staging, and kStages-1 steps of loads in flight while a step is
// multiplied.  Per 8 d-values a thread reads TPT x 16 bytes of activations
// and 4 x 32 bytes of weights for TPT x 4 x 4 packed FMAs.
//
// The block also produces the dispatch metadata: for each of its 128 tokens
// the rank of each route among the block's earlier routes to the same expert
// (token order, k=0 before k=1), and the block's per-expert histogram.
#include "common.cuh"

namespace cti {
namespace {

constexpr int kTok = CTI_ROUTER_BLOCK_TOKENS;  // 128 tokens per block
constexpr int kDC = 32;                        // d-values per stage
constexpr int kStages = 4;
constexpr int kXPitch = kDC * 2 + 16;          // bytes per token row of a stage (padded)
constexpr int kWPitch = kDC * 4 + 16;          // bytes per expert row of a stage (padded)

template <int EMAX>
struct RouterSmem {
  static constexpr size_t kXStage = (size_t)kTok * kXPitch;
  static constexpr size_t kWStage = (size_t)EMAX * kWPitch;
  static constexpr size_t kRing = kStages * (kXStage + kWStage);
  static constexpr size_t kLogits = (size_t)kTok * (EMAX + 1) * 4;
  static constexpr size_t kMain = kRing > kLogits ? kRing : kLogits;
  static constexpr size_t kBytes = kMain + (size_t)(1 + kTok / 32) * EMAX * 4;
};

// Thread tile: TPT tokens x 4 experts.  EG expert groups of 4, TG token
// groups, NT = TG * EG threads (at least one thread per token of the block).
template <int EMAX>
struct RouterTile {
  static constexpr int EG = EMAX / 4;
  static constexpr int TPT = EMAX <= 8 ? 2 : (EMAX <= 32 ? 4 : 8);
  static constexpr int TG = kTok / TPT;
  static constexpr int NT = TG * EG;
  static_assert(NT >= kTok && NT <= 512, "router block size");
};

template <int EMAX>
constexpr int router_threads() {
  return RouterTile<EMAX>::NT;
}

// 16-byte global -> shared copy; src_bytes = 0 fills the destination with zeros.
CTI_DEVICE void cp_async16(void* smem_dst, const void* gmem_src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src), "r"(src_bytes)
               : "memory");
}
CTI_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CTI_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int EMAX>
__global__ void __launch_bounds__(router_threads<EMAX>()) router_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ wg,
    const float* __restrict__ bg, int64_t T, int D, int E, int renorm,
    int32_t* __restrict__ idx2, float* __restrict__ gate2, int32_t* __restrict__ route_rank,
    int32_t* __restrict__ block_hist) {
  // The dispatch scan may be scheduled now; it waits for this grid to
  // complete before it reads the histograms.
  grid_dependents_launch();
  using SM = RouterSmem<EMAX>;
  using TL = RouterTile<EMAX>;
  constexpr int EG = TL::EG;
  constexpr int TG = TL::TG;
  constexpr int TPT = TL::TPT;
  constexpr int NT = TL::NT;
  // Dynamic shared memory: the stage ring while the logits are accumulated,
  // then reused as lg[kTok][EMAX + 1]; then cnt[EMAX] (block counts) and the
  // per-warp counts [kTok/32][EMAX].
  extern __shared__ __align__(16) uint8_t smem_b[];
  float (*lg)[EMAX + 1] = reinterpret_cast<float (*)[EMAX + 1]>(smem_b);
  int* cnt = reinterpret_cast<int*>(smem_b + SM::kMain);

  const int tid = threadIdx.x;
  const int eg = tid % EG;   // experts eg + EG*j, j = 0..3
  const int tg = tid / EG;   // tokens  tg + TG*i, i = 0..TPT-1
  const int64_t t0 = (int64_t)blockIdx.x * kTok;

  uint64_t acc[TPT][4];  // (even-d chain, odd-d chain) per token and expert
#pragma unroll
  for (int i = 0; i < TPT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0ull;  // both lanes +0.0f

  // Stage s of the ring: x part [kTok][kXPitch] bytes, then w part
  // [EMAX][kWPitch] bytes.  Step k covers d in [k*kDC, k*kDC + kDC).
  auto x_stage = [&](int s) { return smem_b + (size_t)s * (SM::kXStage + SM::kWStage); };
  auto w_stage = [&](int s) { return x_stage(s) + SM::kXStage; };
  const int nsteps = (D + kDC - 1) / kDC;
  auto issue = [&](int k) {
    const int d0 = k * kDC;
    const int dc = min(kDC, D - d0);  // a multiple of 8
    uint8_t* xs = x_stage(k % kStages);
    uint8_t* ws = w_stage(k % kStages);
    constexpr int kXParts = kDC / 8;   // 16-byte parts per token row
    for (int c = tid; c < kTok * kXParts; c += NT) {
      const int tok = c / kXParts;
      const int part = c % kXParts;
      const bool ok = t0 + tok < T && part * 8 < dc;
      const __nv_bfloat16* src = ok ? x + (t0 + tok) * D + d0 + part * 8 : x;
      cp_async16(xs + tok * kXPitch + part * 16, src, ok ? 16 : 0);
    }
    constexpr int kWParts = kDC / 4;
    for (int c = tid; c < EMAX * kWParts; c += NT) {
      const int e = c / kWParts;
      const int part = c % kWParts;
      const bool ok = e < E && part * 4 < dc;
      const float* src = ok ? wg + (int64_t)e * D + d0 + part * 4 : wg;
      cp_async16(ws + e * kWPitch + part * 16, src, ok ? 16 : 0);
    }
  };
#pragma unroll
  for (int k = 0; k < kStages - 1; ++k) {
    if (k < nsteps) issue(k);
    cp_async_commit();
  }
  for (int k = 0; k < nsteps; ++k) {
    cp_async_wait<kStages - 2>();
    __syncthreads();  // step k has landed for all threads; step k-1's slot is free
    if (k + kStages - 1 < nsteps) issue(k + kStages - 1);
    cp_async_commit();
    {
      const int dc = min(kDC, D - k * kDC);
      const uint8_t* xs = x_stage(k % kStages) + tg * kXPitch;
      const uint8_t* ws = w_stage(k % kStages) + eg * kWPitch;
      // Two steps in flight give the next step's loads cover; at EMAX 128
      // (512 threads, 128 registers each) one step keeps the tile in registers.
#pragma unroll(EMAX >= 128 ? 1 : 2)
      for (int d8 = 0; d8 < dc / 8; ++d8) {
        uint64_t xp[TPT][4], wp[4][4];  // (d + 2q, d + 2q + 1) pairs, q = 0..3
#pragma unroll
        for (int i = 0; i < TPT; ++i) {
          const uint4 raw = *reinterpret_cast<const uint4*>(xs + i * TG * kXPitch + d8 * 16);
          const uint32_t w32[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int q = 0; q < 4; ++q)
            xp[i][q] = f2_pack(__uint_as_float(w32[q] << 16),
                               __uint_as_float(w32[q] & 0xffff0000u));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4* wr = reinterpret_cast<const float4*>(ws + j * EG * kWPitch + d8 * 32);
          const float4 a = wr[0], b = wr[1];
          wp[j][0] = f2_pack(a.x, a.y);
          wp[j][1] = f2_pack(a.z, a.w);
          wp[j][2] = f2_pack(b.x, b.y);
          wp[j][3] = f2_pack(b.z, b.w);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int i = 0; i < TPT; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = f2_fma(xp[i][q], wp[j][q], acc[i][j]);
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // xs/ws are about to be overwritten by lg
#pragma unroll
  for (int i = 0; i < TPT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float even, odd;
      f2_unpack(acc[i][j], even, odd);
      lg[tg + TG * i][eg + EG * j] = even + odd;
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
  static uint64_t configured = 0;
  if (ensure_smem_limit(router_kernel<EMAX>, (int)RouterSmem<EMAX>::kBytes, configured) !=
      cudaSuccess)
    return cudaErrorInvalidValue;
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
