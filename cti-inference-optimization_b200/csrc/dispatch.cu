// Stage 2 (dispatch) and stage 4 (combine).
//
// Dispatch restates the reference's per-expert grouping of routes
// (baseline/infer.py:336-346: for each expert, `mask.nonzero()` in token
// order, then `x_flat[token_idx]`; online_best/infer.py:1205-1290 count /
// prefix / pack kernels) as a deterministic counting sort:
//   1. dispatch_scan_kernel: one CTA turns the router's per-block expert
//      histograms into expert offsets[E+1] and per-block base offsets (an
//      exclusive prefix over blocks, then over experts, with warp-shuffle
//      scans).
//   2. dispatch_scatter_kernel: per block of 32 tokens, one thread per token
//      computes the sorted position of its two routes (block base + in-block
//      rank from the router), then the block copies the 32 rows to both
//      positions with 16-byte vector loads/stores.
// Routes of one expert come out in token order, exactly the order of the
// reference's `nonzero()`.
//
// Combine restates `out_flat[token_idx] += expert_out * weight`
// (baseline/infer.py:350-353) and moe_top2_reduce_kernel
// (online_best/infer.py:1603-1621): per block of 32 tokens, the token's two
// expert-output rows are weighted by the gates in fp32 and written as one
// bf16 row, 16 bytes per load and store.
#include "common.cuh"

namespace cti {
namespace {

constexpr int kScanThreads = 1024;
constexpr int kScanCache = 16;  // block counts a thread keeps in registers between the passes

CTI_DEVICE int warp_inclusive_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  return v;
}

// hist: [nblk, E] per-block expert counts; rewritten in place into
// per-block base positions.  offsets: [E+1].  Thread (e, c) owns expert e
// over one contiguous chunk of blocks; chunk sums are scanned per expert by
// one warp each (32 chunks per shuffle round), expert totals by warp 0, and
// each thread then writes its chunk's running bases.  Chunks of up to 16
// blocks (nblk <= 16 * 1024 / E) stay in registers between the two passes.
__global__ void __launch_bounds__(kScanThreads) dispatch_scan_kernel(int32_t* __restrict__ hist,
                                                                    int64_t nblk, int E,
                                                                    int32_t* __restrict__ offsets) {
  __shared__ int32_t part[kScanThreads];
  __shared__ int32_t total[CTI_MAX_EXPERTS];
  __shared__ int32_t base[CTI_MAX_EXPERTS + 1];
  grid_dependents_launch();
  grid_dependency_wait();  // hist comes from the router
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int chunks = kScanThreads / E;  // block-chunks per expert
  const int64_t per = (nblk + chunks - 1) / chunks;
  const int e = tid % E;
  const int c = tid / E;
  const bool active = c < chunks;
  const int64_t b_lo = active ? c * per : 0;
  const int64_t b_hi = active ? min(nblk, b_lo + per) : 0;
  const bool cached = per <= kScanCache;

  int32_t cache[kScanCache];
  int32_t sum = 0;
  if (cached) {
#pragma unroll
    for (int i = 0; i < kScanCache; ++i) {
      const int64_t b = b_lo + i;
      cache[i] = b < b_hi ? hist[b * E + e] : 0;
    }
#pragma unroll
    for (int i = 0; i < kScanCache; ++i) sum += cache[i];
  } else {
    for (int64_t b = b_lo; b < b_hi; ++b) sum += hist[b * E + e];
  }
  part[tid] = sum;
  __syncthreads();
  // Exclusive prefix over the chunks of each expert.
  for (int ee = warp; ee < E; ee += kScanThreads / 32) {
    int carry = 0;
    for (int c0 = 0; c0 < chunks; c0 += 32) {
      const int cc = c0 + lane;
      const int v = cc < chunks ? part[cc * E + ee] : 0;
      const int incl = warp_inclusive_scan(v, lane);
      if (cc < chunks) part[cc * E + ee] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) total[ee] = carry;
  }
  __syncthreads();
  // Exclusive prefix over the experts.
  if (warp == 0) {
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int ee = e0 + lane;
      const int v = ee < E ? total[ee] : 0;
      const int incl = warp_inclusive_scan(v, lane);
      if (ee < E) base[ee] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) base[E] = carry;
  }
  __syncthreads();
  if (tid <= E) offsets[tid] = base[tid];
  if (active) {
    int32_t run = base[e] + part[tid];
    if (cached) {
#pragma unroll
      for (int i = 0; i < kScanCache; ++i) {
        const int64_t b = b_lo + i;
        if (b < b_hi) {
          hist[b * E + e] = run;
          run += cache[i];
        }
      }
    } else {
      for (int64_t b = b_lo; b < b_hi; ++b) {
        const int32_t v = hist[b * E + e];
        hist[b * E + e] = run;
        run += v;
      }
    }
  }
}

constexpr int kRowsPerBlock = 32;  // tokens per block in scatter / combine

// Block of 256 threads per 32 tokens.  Phase 1: one thread per token reads
// its expert ids, in-block ranks and block bases and computes the two sorted
// positions.  Phase 2: the block copies the 32 rows as 16-byte chunks, every
// thread with several independent loads in flight.  D % 8 == 0.
__global__ void __launch_bounds__(256) dispatch_scatter_kernel(
    const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ idx2,
    const int32_t* __restrict__ route_rank, const int32_t* __restrict__ block_base, int64_t T,
    int D, int E, int32_t* __restrict__ perm_inv, int32_t* __restrict__ sorted_token,
    __nv_bfloat16* __restrict__ xperm, int32_t* status) {
  __shared__ int2 pos_s[kRowsPerBlock];
  grid_dependents_launch();
  grid_dependency_wait();  // routes from the router, block bases from the scan
  const int64_t t0 = (int64_t)blockIdx.x * kRowsPerBlock;
  const int64_t R = 2 * T;
  if (threadIdx.x < kRowsPerBlock) {
    const int64_t t = t0 + threadIdx.x;
    int2 p = make_int2(-1, -1);
    if (t < T) {
      const int2 e = reinterpret_cast<const int2*>(idx2)[t];
      const int2 rk = reinterpret_cast<const int2*>(route_rank)[t];
      const int64_t blk = t / CTI_ROUTER_BLOCK_TOKENS;
      if (e.x < 0 || e.x >= E || e.y < 0 || e.y >= E) {
        raise_status(status, CTI_ERR_BOUNDS, (int32_t)t);
      } else {
        const int64_t p0 = (int64_t)block_base[blk * E + e.x] + rk.x;
        const int64_t p1 = (int64_t)block_base[blk * E + e.y] + rk.y;
        if (p0 < 0 || p0 >= R || p1 < 0 || p1 >= R) {
          raise_status(status, CTI_ERR_BOUNDS, (int32_t)t);
        } else {
          p = make_int2((int)p0, (int)p1);
          sorted_token[p0] = (int32_t)t;
          sorted_token[p1] = (int32_t)t;
        }
      }
      // A token that failed a check gets (-1, -1): the combine then skips
      // it instead of reading whatever an earlier call left in perm_inv.
      reinterpret_cast<int2*>(perm_inv)[t] = p;
    }
    pos_s[threadIdx.x] = p;
  }
  __syncthreads();
  if (xperm == nullptr) return;
  const int nchunk = D / 8;
  for (int c = threadIdx.x; c < kRowsPerBlock * nchunk; c += blockDim.x) {
    const int r = c / nchunk;
    const int ch = c - r * nchunk;
    const int2 p = pos_s[r];
    if (p.x < 0) continue;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + (t0 + r) * D) + ch);
    reinterpret_cast<uint4*>(xperm + (int64_t)p.x * D)[ch] = v;
    reinterpret_cast<uint4*>(xperm + (int64_t)p.y * D)[ch] = v;
  }
}

// Same shape: phase 1 loads each token's two sorted positions and gates,
// phase 2 combines the two expert rows chunk by chunk in fp32.
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ Y,
                                                     int64_t Y_rows,
                                                     const int32_t* __restrict__ perm_inv,
                                                     const float* __restrict__ gate2, int64_t T,
                                                     int D, __nv_bfloat16* __restrict__ out,
                                                     int32_t* status) {
  __shared__ int2 pos_s[kRowsPerBlock];
  __shared__ float2 gate_s[kRowsPerBlock];
  grid_dependency_wait();  // Y from the expert FFN
  const int64_t t0 = (int64_t)blockIdx.x * kRowsPerBlock;
  if (threadIdx.x < kRowsPerBlock) {
    const int64_t t = t0 + threadIdx.x;
    int2 p = make_int2(-1, -1);
    float2 g = make_float2(0.0f, 0.0f);
    if (t < T) {
      p = reinterpret_cast<const int2*>(perm_inv)[t];
      g = reinterpret_cast<const float2*>(gate2)[t];
      if (p.x < 0 || p.x >= Y_rows || p.y < 0 || p.y >= Y_rows) {
        raise_status(status, CTI_ERR_BOUNDS, (int32_t)t);
        p = make_int2(-1, -1);
      }
    }
    pos_s[threadIdx.x] = p;
    gate_s[threadIdx.x] = g;
  }
  __syncthreads();
  const int nchunk = D / 8;
  for (int c = threadIdx.x; c < kRowsPerBlock * nchunk; c += blockDim.x) {
    const int r = c / nchunk;
    const int ch = c - r * nchunk;
    const int2 p = pos_s[r];
    if (p.x < 0) continue;
    const float2 g = gate_s[r];
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(Y + (int64_t)p.x * D) + ch);
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(Y + (int64_t)p.y * D) + ch);
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fa = __bfloat1622float2(ha[j]);
      const float2 fb = __bfloat1622float2(hb[j]);
      ow[j] = pack_bf16x2(fmaf(g.y, fb.x, g.x * fa.x), fmaf(g.y, fb.y, g.x * fa.y));
    }
    reinterpret_cast<uint4*>(out + (t0 + r) * D)[ch] = o;
  }
}

inline bool misaligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0;
}

}  // namespace
}  // namespace cti

extern "C" size_t cti_moe_dispatch_workspace_bytes(int64_t T, int E) {
  if (T <= 0 || E <= 0) return 0;
  const int64_t nblk = (T + CTI_ROUTER_BLOCK_TOKENS - 1) / CTI_ROUTER_BLOCK_TOKENS;
  return (size_t)nblk * (size_t)E * sizeof(int32_t);
}

extern "C" int cti_moe_dispatch(const void* x_bf16, const int32_t* idx2, const int32_t* route_rank,
                                int32_t* block_hist, int64_t T, int D, int E, int32_t* offsets,
                                int32_t* perm_inv, int32_t* sorted_token, void* xperm_bf16,
                                int32_t* status, void* stream) {
  using namespace cti;
  if (T < 0 || D <= 0 || E < 2 || E > CTI_MAX_EXPERTS) return CTI_ERR_INVALID_ARG;
  if (D % 8 != 0) return CTI_ERR_UNSUPPORTED;
  if (2 * T > INT32_MAX) return CTI_ERR_UNSUPPORTED;
  if (!offsets) return CTI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 0) {
    // No routes: every expert segment is empty.
    return cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (E + 1), s) == cudaSuccess
               ? CTI_OK
               : CTI_ERR_CUDA;
  }
  if (!idx2 || !route_rank || !block_hist || !perm_inv || !sorted_token)
    return CTI_ERR_INVALID_ARG;
  if (xperm_bf16 && (!x_bf16 || misaligned(x_bf16, 16) || misaligned(xperm_bf16, 16)))
    return CTI_ERR_INVALID_ARG;
  if (misaligned(idx2, 8) || misaligned(route_rank, 8) || misaligned(perm_inv, 8))
    return CTI_ERR_INVALID_ARG;
  const int64_t nblk = (T + CTI_ROUTER_BLOCK_TOKENS - 1) / CTI_ROUTER_BLOCK_TOKENS;
  if (launch_dependent(dispatch_scan_kernel, dim3(1), dim3(kScanThreads), 0, s, block_hist, nblk,
                       E, offsets) != cudaSuccess)
    return CTI_ERR_CUDA;
  const int64_t blocks = (T + kRowsPerBlock - 1) / kRowsPerBlock;
  return launch_dependent(dispatch_scatter_kernel, dim3((unsigned)blocks), dim3(256), 0, s,
                          static_cast<const __nv_bfloat16*>(x_bf16), idx2, route_rank,
                          block_hist, T, D, E, perm_inv, sorted_token,
                          static_cast<__nv_bfloat16*>(xperm_bf16), status) == cudaSuccess
             ? CTI_OK
             : CTI_ERR_CUDA;
}

extern "C" int cti_moe_combine(const void* Y_bf16, int64_t Y_rows, const int32_t* perm_inv,
                               const float* gate2, int64_t T, int D, void* out_bf16,
                               int32_t* status, void* stream) {
  using namespace cti;
  if (T < 0 || D <= 0 || Y_rows < 0) return CTI_ERR_INVALID_ARG;
  if (D % 8 != 0) return CTI_ERR_UNSUPPORTED;
  if (T == 0) return CTI_OK;
  if (!Y_bf16 || !perm_inv || !gate2 || !out_bf16) return CTI_ERR_INVALID_ARG;
  if (misaligned(Y_bf16, 16) || misaligned(out_bf16, 16) || misaligned(perm_inv, 8) ||
      misaligned(gate2, 8))
    return CTI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t blocks = (T + kRowsPerBlock - 1) / kRowsPerBlock;
  return launch_dependent(combine_kernel, dim3((unsigned)blocks), dim3(256), 0, s,
                          static_cast<const __nv_bfloat16*>(Y_bf16), Y_rows, perm_inv, gate2, T,
                          D, static_cast<__nv_bfloat16*>(out_bf16), status) == cudaSuccess
             ? CTI_OK
             : CTI_ERR_CUDA;
}
