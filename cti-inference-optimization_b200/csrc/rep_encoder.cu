// The RepEncoder in one kernel: embedding-bag pooling of the F features,
// LayerNorm over the F * 64 pooled columns and the Linear to d_model,
//
//   x[t]  = concat_f  sum_{id in bag(t, f)} table[base_f + clamp(id)]      (fp32 sums, bf16)
//   y[t]  = W . LN(x[t]) + b,   LN(x) = (x - mean) * rstd * gamma + beta
//
// (baseline/infer.py:253-265 RepEncoder.forward; online_best/infer.py:793-827
// pooling, :829-858 LayerNorm, :1061-1085 the three launches this replaces),
// without the [T, F * 64] pooled tensor ever leaving the SM.  The LayerNorm is
// folded into the GEMM:
//
//   y[t, n] = rstd_t * (sum_k Wg[n, k] x[t, k] - mean_t * r1[n]) + c[n],
//   Wg = W * gamma (bf16), r1[n] = sum_k Wg[n, k], c = W beta + b,
//
// so the tensor cores multiply the raw pooled row (rounded to bf16, as the
// pooled tensor of the unfused path is) while its mean and variance are
// summed alongside.  mean and variance come from the bf16 values in fp32 as
// sum(x) and sum(x^2) (one pass).
//
// Persistent over 128-token tiles; the K dimension of the GEMM is walked one
// feature (64 columns) at a time, so each pooled feature chunk is consumed as
// soon as it is complete.  Per CTA (1024 threads, one CTA per SM):
//   warp 0      TMA producer: the Wg slab of each feature ([N x 64] bf16,
//               128-byte swizzle) into a 3-deep ring (Wg stays in L2).
//   warp 1      TMEM owner and MMA issuer: acc[tile % 2] (N fp32 columns)
//               += A_f Wg_f^T, M 128, N = d_model, K 64 (four MMAs).
//   warps 2-5   epilogue, one TMEM lane quadrant each, thread = row.
//   warps 6-31  pooling: 104 groups of 8 lanes walk the CTA's bags (tile,
//               feature, row) as one flat stream, a group every 104th bag;
//               each lane owns 8 of the row's 64 columns and sums the bag in
//               order in fp32 exactly as cti_embbag_sum does (ids UNROLL at
//               a time, their rows loaded before any is added), then writes
//               the bf16 row slice into the feature's A chunk ([128 x 64],
//               128-byte swizzle, 4-deep ring) and adds the slice's sum and
//               sum of squares into the tile's row statistics.  The stride
//               (104) is below the chunk size (128), so every pooling warp
//               touches every chunk and arrives on it exactly once.
// Every wait is a bounded mbarrier wait; a wait that runs out records its
// site in the status word and the roles unwind.
#include "common.cuh"
#include "tmap.cuh"

namespace cti {
namespace {

constexpr int kRB = 128;            // tokens per tile
constexpr int kDim = 64;            // embedding width (columns per feature)
constexpr int kRThreads = 1024;
constexpr int kPoolWarp0 = 6;
constexpr int kPoolWarps = 32 - kPoolWarp0;
constexpr int kGroups = kPoolWarps * 4;  // 8-lane groups
constexpr int kAStages = 4;
constexpr int kWStages = 3;
constexpr int kMaxN = 256;
constexpr int kPoolUnroll = 4;
constexpr uint32_t kAChunk = kRB * kDim * 2;     // 16 KB
constexpr uint32_t kWSlab = kMaxN * kDim * 2;    // 32 KB
constexpr size_t kRSmem = 1024 + kAStages * (size_t)kAChunk + kWStages * (size_t)kWSlab +
                          2 * kRB * sizeof(float2) + 512;
static_assert(kRSmem <= 232448, "shared memory per CTA");
static_assert(kGroups < kRB && kGroups % 4 == 0, "every pooling warp meets every chunk");

CTI_DEVICE void add8(float* acc, const uint4& raw) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]);
    acc[2 * j] += f.x;
    acc[2 * j + 1] += f.y;
  }
}

__global__ void __launch_bounds__(kRThreads, 1)
    rep_encoder_kernel(const __grid_constant__ CUtensorMap tmW,
                       const int64_t* __restrict__ values, int64_t n_values,
                       const int64_t* __restrict__ row_offsets,
                       const int64_t* __restrict__ val_offsets,
                       const int64_t* __restrict__ table_row_base,
                       const int64_t* __restrict__ vocab, const __half* __restrict__ table,
                       int64_t table_rows, int64_t B, int F, int N,
                       const float* __restrict__ r1, const float* __restrict__ cvec, float eps,
                       __nv_bfloat16* __restrict__ out, int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;                                  // [kAStages] A chunks
  uint8_t* sW = sA + kAStages * (size_t)kAChunk;        // [kWStages] Wg slabs
  float2* stats = reinterpret_cast<float2*>(sW + kWStages * (size_t)kWSlab);  // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(stats + 2 * kRB);
  uint64_t* a_full = bars;                    // [kAStages] chunk written (pool warps)
  uint64_t* a_empty = a_full + kAStages;      // [kAStages] chunk's MMAs done
  uint64_t* w_full = a_empty + kAStages;      // [kWStages]
  uint64_t* w_empty = w_full + kWStages;      // [kWStages]
  uint64_t* acc_full = w_empty + kWStages;    // [2] tile's MMAs done
  uint64_t* acc_empty = acc_full + 2;         // [2] epilogue read it (4 warps)
  uint64_t* st_full = acc_empty + 2;          // [2] tile's statistics complete (pool warps)
  uint64_t* st_empty = st_full + 2;           // [2] statistics read and cleared (4 warps)
  uint64_t* drain = st_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  static_assert((2 * kAStages + 2 * kWStages + 9) * 8 + 8 <= 512, "barrier area");

  const int warp = warp_id();
  const int lane = lane_id();
  const int64_t ntiles = (B + kRB - 1) / kRB;
  const int64_t my_tiles =
      (int64_t)blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t nchunks = my_tiles * F;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], kPoolWarps);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
      mbar_init(&st_full[i], kPoolWarps);
      mbar_init(&st_empty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < 2 * kRB; i += blockDim.x) stats[i] = make_float2(0.0f, 0.0f);
  if (threadIdx.x == 32) prefetch_tensormap(&tmW);
  grid_dependency_wait();
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * (uint32_t)N);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- Wg producer ----------------
    if (lane == 0) {
      const uint32_t slab = (uint32_t)N * kDim * 2;
      int64_t c = 0;
      for (; c < nchunks; ++c) {
        const int s = (int)(c % kWStages);
        if (!mbar_wait(&w_empty[s], (uint32_t)((c / kWStages) & 1) ^ 1u, status, 0x701,
                       abort_flag))
          break;
        mbar_arrive_expect_tx(&w_full[s], slab);
        tma_load_2d(sW + (size_t)s * kWSlab, &tmW, &w_full[s], (int)(c % F) * kDim, 0);
      }
      for (int q = 1; q <= kWStages; ++q)
        if (c - q >= 0)
          mbar_wait(&w_full[(c - q) % kWStages], (uint32_t)(((c - q) / kWStages) & 1), status,
                    0x702, nullptr);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kRB, (uint32_t)N);
      bool any = false;
      for (int64_t c = 0; c < nchunks; ++c) {
        const int64_t ti = c / F;
        const int f = (int)(c % F);
        const int ab = (int)(ti & 1);
        const int s = (int)(c % kAStages);
        const int ws = (int)(c % kWStages);
        if (f == 0 && !mbar_wait(&acc_empty[ab], (uint32_t)((ti >> 1) & 1) ^ 1u, status, 0x703,
                                 abort_flag))
          break;
        if (!mbar_wait(&a_full[s], (uint32_t)((c / kAStages) & 1), status, 0x704, abort_flag) ||
            !mbar_wait(&w_full[ws], (uint32_t)((c / kWStages) & 1), status, 0x705, abort_flag))
          break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + (size_t)s * kAChunk);
        const uint32_t w0 = smem_u32(sW + (size_t)ws * kWSlab);
#pragma unroll
        for (int kk = 0; kk < kDim / 16; ++kk)
          umma_bf16(tmem_base + (uint32_t)(ab * N), smem_desc_sw128(a0 + kk * 32),
                    smem_desc_sw128(w0 + kk * 32), idesc, (f | kk) != 0 ? 1u : 0u);
        umma_commit(&a_empty[s]);
        umma_commit(&w_empty[ws]);
        if (f == F - 1) umma_commit(&acc_full[ab]);
        any = true;
      }
      if (any) {
        umma_commit(drain);
        mbar_wait(drain, 0, status, 0x706, nullptr);
      }
    }
  } else if (warp < kPoolWarp0) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const float inv_k = 1.0f / (float)(F * kDim);
    for (int64_t ti = 0; ti < my_tiles; ++ti) {
      const int ab = (int)(ti & 1);
      if (!mbar_wait(&st_full[ab], (uint32_t)((ti >> 1) & 1), status, 0x707, abort_flag) ||
          !mbar_wait(&acc_full[ab], (uint32_t)((ti >> 1) & 1), status, 0x708, abort_flag))
        break;
      tc_fence_after();
      const float2 sm = stats[ab * kRB + r];
      const float mean = sm.x * inv_k;
      const float var = fmaxf(sm.y * inv_k - mean * mean, 0.0f);
      const float rstd = rsqrtf(var + eps);
      const float shift = -mean * rstd;
      const int64_t row = (blockIdx.x + ti * gridDim.x) * kRB + r;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * N);
      for (int n0 = 0; n0 < N; n0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32_sync(taddr + (uint32_t)n0, v);
        if (row < B) {
          uint4* dst = reinterpret_cast<uint4*>(out + row * N + n0);
#pragma unroll
          for (int g8 = 0; g8 < 4; ++g8) {
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int n = n0 + 8 * g8 + e;
              y[e] = fmaf(rstd, __uint_as_float(v[8 * g8 + e]), fmaf(shift, __ldg(r1 + n), __ldg(cvec + n)));
            }
            uint4 w;
            w.x = pack_bf16x2(y[0], y[1]);
            w.y = pack_bf16x2(y[2], y[3]);
            w.z = pack_bf16x2(y[4], y[5]);
            w.w = pack_bf16x2(y[6], y[7]);
            dst[g8] = w;
          }
        }
      }
      stats[ab * kRB + r] = make_float2(0.0f, 0.0f);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc_empty[ab]);
        mbar_arrive(&st_empty[ab]);
      }
    }
  } else {
    // ---------------- pooling ----------------
    const int sub = lane & 7;
    const int G = (warp - kPoolWarp0) * 4 + (lane >> 3);
    const int64_t nbags = nchunks * kRB;
    int64_t cur_chunk = -1;
    bool ok = true;
    for (int64_t k = G; ok; k += kGroups) {
      // The warp's four groups hold 4 consecutive bags of one chunk.
      const int64_t c = k < nbags ? k / kRB : nchunks;
      if (c != cur_chunk) {
        if (cur_chunk >= 0) {
          // Leaving chunk cur_chunk: its rows from this warp are written.
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&a_full[cur_chunk % kAStages]);
            if (cur_chunk % F == F - 1 || c == nchunks) mbar_arrive(&st_full[(cur_chunk / F) & 1]);
          }
        }
        if (c == nchunks) break;
        const int64_t ti = c / F;
        ok = mbar_wait(&a_empty[c % kAStages], (uint32_t)((c / kAStages) & 1) ^ 1u, status,
                       0x709, abort_flag);
        if (ok && c % F == 0)
          ok = mbar_wait(&st_empty[ti & 1], (uint32_t)((ti >> 1) & 1) ^ 1u, status, 0x70a,
                         abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        cur_chunk = c;
      }
      const int64_t ti = c / F;
      const int f = (int)(c % F);
      const int r = (int)(k % kRB);
      const int64_t b = (blockIdx.x + ti * gridDim.x) * kRB + r;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
      if (b < B) {
        const int64_t* roff = row_offsets + (int64_t)f * (B + 1);
        const int64_t start = roff[b];
        const int64_t end = roff[b + 1];
        const int64_t vbase = val_offsets[f];
        const int64_t rbase = table_row_base[f];
        const int64_t vmax = vocab[f] - 1;
        const bool valid = start <= end && start >= 0 && vbase >= 0 && vbase + end <= n_values &&
                           vmax >= 0 && rbase >= 0 && rbase + vmax < table_rows;
        if (!valid) {
          if (sub == 0) raise_status(status, CTI_ERR_BOUNDS, (int32_t)(b * F + f));
        } else {
          const int64_t* vals = values + vbase;
          int64_t i = start;
          for (; i + kPoolUnroll <= end; i += kPoolUnroll) {
            uint4 raw[kPoolUnroll];
#pragma unroll
            for (int u = 0; u < kPoolUnroll; ++u) {
              int64_t id = __ldg(vals + i + u);
              id = id < 0 ? 0 : (id > vmax ? vmax : id);
              raw[u] = __ldg(reinterpret_cast<const uint4*>(table + (rbase + id) * kDim) + sub);
            }
#pragma unroll
            for (int u = 0; u < kPoolUnroll; ++u) add8(acc, raw[u]);
          }
          for (; i < end; ++i) {
            int64_t id = __ldg(vals + i);
            id = id < 0 ? 0 : (id > vmax ? vmax : id);
            add8(acc, __ldg(reinterpret_cast<const uint4*>(table + (rbase + id) * kDim) + sub));
          }
        }
      }
      // bf16 slice into the swizzled chunk row; its sums into the row stats.
      uint4 w;
      w.x = pack_bf16x2(acc[0], acc[1]);
      w.y = pack_bf16x2(acc[2], acc[3]);
      w.z = pack_bf16x2(acc[4], acc[5]);
      w.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(sA + (size_t)(c % kAStages) * kAChunk + r * 128 +
                                ((sub ^ (r & 7)) << 4)) = w;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
      float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 p = __bfloat1622float2(h[j]);
        s1 += p.x + p.y;
        s2 = fmaf(p.x, p.x, fmaf(p.y, p.y, s2));
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      }
      if (sub == 0 && b < B) {
        atomicAdd(&stats[(ti & 1) * kRB + r].x, s1);
        atomicAdd(&stats[(ti & 1) * kRB + r].y, s2);
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * (uint32_t)N);
  }
}

}  // namespace
}  // namespace cti

extern "C" int cti_rep_encoder_fused(const int64_t* values, int64_t n_values,
                                     const int64_t* row_offsets, const int64_t* val_offsets,
                                     const int64_t* table_row_base, const int64_t* vocab,
                                     const void* table_f16, int64_t table_rows, int64_t B, int F,
                                     int dim, const void* wg_bf16, const float* r1,
                                     const float* c, int N, float eps, void* out_bf16,
                                     int32_t* status, void* stream) {
  using namespace cti;
  if (B < 0 || F <= 0 || n_values < 0 || table_rows < 0 || !(eps >= 0.0f))
    return CTI_ERR_INVALID_ARG;
  if (dim != kDim || (N != 128 && N != 256)) return CTI_ERR_UNSUPPORTED;
  if ((int64_t)F * kDim > 65535) return CTI_ERR_UNSUPPORTED;
  if (B == 0) return CTI_OK;
  if (!row_offsets || !val_offsets || !table_row_base || !vocab || !table_f16 || !wg_bf16 ||
      !r1 || !c || !out_bf16 || (n_values > 0 && !values))
    return CTI_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(table_f16) | reinterpret_cast<uintptr_t>(out_bf16)) & 15)
    return CTI_ERR_INVALID_ARG;
  CUtensorMap tmW;
  if (!make_tmap_bf16_2d(&tmW, wg_bf16, (uint64_t)N, (uint64_t)F * kDim, (uint64_t)F * kDim,
                         (uint32_t)N, kDim))
    return CTI_ERR_INVALID_ARG;
  static uint64_t configured = 0;
  if (ensure_smem_limit(rep_encoder_kernel, (int)kRSmem, configured) != cudaSuccess)
    return CTI_ERR_CUDA;
  const int sms = device_sm_count();
  if (sms <= 0) return CTI_ERR_CUDA;
  const int64_t ntiles = (B + kRB - 1) / kRB;
  const int grid = (int)(ntiles < sms ? ntiles : sms);
  return launch_dependent(rep_encoder_kernel, dim3(grid), dim3(kRThreads), kRSmem,
                          static_cast<cudaStream_t>(stream), tmW, values, n_values, row_offsets,
                          val_offsets, table_row_base, vocab,
                          static_cast<const __half*>(table_f16), table_rows, B, F, N, r1, c, eps,
                          static_cast<__nv_bfloat16*>(out_bf16), status) == cudaSuccess
             ? CTI_OK
             : CTI_ERR_CUDA;
}
