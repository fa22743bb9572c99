// The CTR head in one kernel: the configuration's MLP head (d_model -> Hd ->
// 1 with ReLU) followed by the clamp and sigmoid of the reference head,
//
//   logits[t] = clamp(w2 . relu(W1 h[t] + b1) + b2, -limit, limit)
//   probs[t]  = sigmoid(logits[t]),
//
// replacing final_linear_clamp_kernel (online_best/infer.py:861-887; launched
// at :2529-2567: row dot + bias, clamp to +-15, optional sigmoid) and the
// separate Linear / ReLU / Linear / clamp / sigmoid launches of the MLP head.
// The [T, Hd] hidden activation never leaves the SM.
//
// Persistent over 128-row tiles of h:
//   warp 0     TMA producer: the tile's D/64 K slabs ([128 x 64] bf16,
//              128-byte swizzle) into a 2-deep ring of whole tiles; W1
//              ([Hd x D]) once per CTA, resident for the whole kernel;
//   warp 1     TMEM owner and MMA issuer: acc[b] (Hd fp32 columns) =
//              h tile @ W1^T, M = 128, N = Hd, two accumulators so the MMA of
//              the next tile overlaps the epilogue of this one;
//   warps 2-5  epilogue, one per TMEM lane quadrant, thread = row: + b1,
//              ReLU and the dot with w2 in fp32, + b2, clamp, sigmoid.
// HBM-bound: reads T x D x 2 bytes, writes 8 bytes per row.
#include "common.cuh"
#include "tmap.cuh"

namespace cti {
namespace {

constexpr int kHBM = 128;
constexpr int kHBK = 64;
constexpr int kHMaxD = 256;
constexpr int kHMaxHd = 128;
constexpr int kHThreads = 192;
constexpr size_t kHSlab = (size_t)kHBM * kHBK * 2;                  // 16 KB
constexpr size_t kHTile = (kHMaxD / kHBK) * kHSlab;                  // 64 KB
constexpr size_t kHW1 = (size_t)kHMaxHd * kHMaxD * 2;                // 64 KB
constexpr size_t kHSmem = 1024 + 2 * kHTile + kHW1 + (size_t)2 * kHMaxHd * 4 + 256;
static_assert(kHSmem <= 232448, "shared memory per CTA");

__global__ void __launch_bounds__(kHThreads, 1)
    ctr_head_kernel(const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmW1,
                    int64_t T, int D, int Hd, const float* __restrict__ b1,
                    const float* __restrict__ w2, const float* __restrict__ b2, float limit,
                    float* __restrict__ logits, float* __restrict__ probs, int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;                 // [2] h tiles
  uint8_t* sw1 = tiles + 2 * kHTile;     // W1, D/64 slabs of [Hd x 64]
  float* b1s = reinterpret_cast<float*>(sw1 + kHW1);
  float* w2s = b1s + kHMaxHd;
  uint64_t* bars = reinterpret_cast<uint64_t*>(w2s + kHMaxHd);
  uint64_t* hfull = bars;        // [2] h tile landed
  uint64_t* hempty = bars + 2;   // [2] MMAs done reading it
  uint64_t* w1full = bars + 4;
  uint64_t* afull = bars + 5;    // [2] accumulator ready
  uint64_t* aempty = bars + 7;   // [2] epilogue done reading it
  uint64_t* drain = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int nk = D / kHBK;
  const int64_t ntiles = (T + kHBM - 1) / kHBM;
  const uint32_t tmem_cols = Hd <= 64 ? 128u : 256u;  // two accumulators, a power of two

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&hfull[i], 1);
      mbar_init(&hempty[i], 1);
      mbar_init(&afull[i], 1);
      mbar_init(&aempty[i], 4);
    }
    mbar_init(w1full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&tmH);
    prefetch_tensormap(&tmW1);
  }
  for (int i = threadIdx.x; i < Hd; i += blockDim.x) {
    b1s[i] = b1[i];
    w2s[i] = w2[i];
  }
  grid_dependency_wait();  // h comes from the kernels before this one
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(w1full, (uint32_t)(nk * Hd * kHBK * 2));
      for (int kb = 0; kb < nk; ++kb)
        tma_load_2d(sw1 + (size_t)kb * Hd * kHBK * 2, &tmW1, w1full, kb * kHBK, 0);
      int it = 0, issued = 0;
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int b = it & 1;
        if (!mbar_wait(&hempty[b], (uint32_t)((it >> 1) & 1) ^ 1u, status, 0x501, abort_flag))
          break;
        mbar_arrive_expect_tx(&hfull[b], (uint32_t)(nk * kHSlab));
        for (int kb = 0; kb < nk; ++kb)
          tma_load_2d(tiles + b * kHTile + kb * kHSlab, &tmH, &hfull[b], kb * kHBK,
                      (int32_t)(t * kHBM));
        ++issued;
      }
      // Let the loads in flight land before the CTA can exit.
      mbar_wait(w1full, 0, status, 0x502, nullptr);
      for (int i = 1; i <= 2; ++i)
        if (issued - i >= 0)
          mbar_wait(&hfull[(issued - i) & 1], (uint32_t)(((issued - i) >> 1) & 1), status, 0x502,
                    nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kHBM, (uint32_t)Hd);
      bool any = false;
      if (mbar_wait(w1full, 0, status, 0x503, abort_flag)) {
        int it = 0;
        for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
          const int b = it & 1;
          const uint32_t ph = (uint32_t)((it >> 1) & 1);
          if (!mbar_wait(&aempty[b], ph ^ 1u, status, 0x504, abort_flag)) break;
          if (!mbar_wait(&hfull[b], ph, status, 0x505, abort_flag)) break;
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(b * (tmem_cols / 2));
          const uint32_t a0 = smem_u32(tiles + b * kHTile);
          const uint32_t w0 = smem_u32(sw1);
          for (int kb = 0; kb < nk; ++kb)
#pragma unroll
            for (int kk = 0; kk < kHBK / 16; ++kk)
              umma_bf16(d, smem_desc_sw128(a0 + kb * kHSlab + kk * 32),
                        smem_desc_sw128(w0 + kb * Hd * kHBK * 2 + kk * 32), idesc,
                        (kb | kk) != 0 ? 1u : 0u);
          umma_commit(&hempty[b]);
          umma_commit(&afull[b]);
          any = true;
        }
      }
      if (any) {
        umma_commit(drain);
        mbar_wait(drain, 0, status, 0x506, nullptr);
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const float bias2 = *b2;
    int it = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int b = it & 1;
      if (!mbar_wait(&afull[b], (uint32_t)((it >> 1) & 1), status, 0x507, abort_flag)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * (tmem_cols / 2));
      float acc = 0.0f;
      for (int c0 = 0; c0 < Hd; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + (uint32_t)c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          acc = fmaf(fmaxf(__uint_as_float(v[i]) + b1s[c0 + i], 0.0f), w2s[c0 + i], acc);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&aempty[b]);
      const int64_t row = t * kHBM + r;
      if (row < T) {
        const float lg = fminf(fmaxf(acc + bias2, -limit), limit);
        if (logits) logits[row] = lg;
        if (probs) probs[row] = 1.0f / (1.0f + expf(-lg));
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

}  // namespace
}  // namespace cti

extern "C" int cti_ctr_head(const void* h_bf16, const void* W1_bf16, const float* b1,
                            const float* w2, const float* b2, int64_t T, int D, int Hd,
                            float limit, float* logits, float* probs, int32_t* status,
                            void* stream) {
  using namespace cti;
  if (T < 0 || D <= 0 || Hd <= 0 || !(limit > 0.0f)) return CTI_ERR_INVALID_ARG;
  if (D % kHBK != 0 || D > kHMaxD || Hd % 32 != 0 || Hd > kHMaxHd) return CTI_ERR_UNSUPPORTED;
  if (T == 0) return CTI_OK;
  if (!h_bf16 || !W1_bf16 || !b1 || !w2 || !b2 || (!logits && !probs)) return CTI_ERR_INVALID_ARG;
  CUtensorMap tmH, tmW1;
  if (!make_tmap_bf16_2d(&tmH, h_bf16, (uint64_t)T, (uint64_t)D, (uint64_t)D, kHBM, kHBK) ||
      !make_tmap_bf16_2d(&tmW1, W1_bf16, (uint64_t)Hd, (uint64_t)D, (uint64_t)D, (uint32_t)Hd,
                         kHBK))
    return CTI_ERR_INVALID_ARG;
  static uint64_t configured = 0;
  if (ensure_smem_limit(ctr_head_kernel, (int)kHSmem, configured) != cudaSuccess)
    return CTI_ERR_CUDA;
  const int sms = device_sm_count();
  if (sms <= 0) return CTI_ERR_CUDA;
  const int64_t ntiles = (T + kHBM - 1) / kHBM;
  const int grid = (int)(ntiles < sms ? ntiles : sms);
  return launch_dependent(ctr_head_kernel, dim3(grid), dim3(kHThreads), kHSmem,
                          static_cast<cudaStream_t>(stream), tmH, tmW1, T, D, Hd, b1, w2, b2,
                          limit, logits, probs, status) == cudaSuccess
             ? CTI_OK
             : CTI_ERR_CUDA;
}
