// Stage 3: grouped expert GEMM on the sm_100a tensor cores (tcgen05 + TMEM).
//
//   C[rows of group g, :] = act(A[rows, :K] @ W[g % Gw]^T + bias[g % Gw])
//
// This replaces the reference's sparse fc1/fc2 Triton GEMMs
// (online_best/infer.py:1293-1600: BLOCK_M=32 mma.sync tiles, one program
// per (m-tile, n-tile, expert) with empty tiles exiting early) by one
// persistent, warp-specialised kernel per GEMM:
//
//   warp 0      TMA producer: 128x64 A tiles and BNx64 weight tiles, 128-byte
//               swizzled, into a STAGES-deep shared-memory ring (mbarrier
//               full/empty pairs, transaction-count completion).
//   warp 1      allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN,
//               K=16, bf16 -> fp32) into one of two TMEM accumulators and
//               commits each ring slot back to the producer.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (thread = row),
//               + bias, activation, bf16 pack, row stores; frees the
//               accumulator so the MMA of the next tile overlaps this one.
//
// Tiles are enumerated from the device-side group offsets (no host sync):
// each CTA builds the per-group m-tile prefix in shared memory and walks
// tiles blockIdx.x, blockIdx.x + gridDim.x, ...  A tile may run past the end
// of its group; TMA zero-fills rows past the end of A, and the epilogue
// stores only the group's own rows.
#include "common.cuh"
#include "gelu.cuh"
#include "sched.cuh"
#include "tmap.cuh"

namespace cti {
namespace {

template <int BN>
struct GG {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + GroupSched::smem_bytes() + 256;
};

template <int BN>
__global__ void __launch_bounds__(192, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const int32_t* __restrict__ group_offsets, int G, int Gw,
                        int64_t rows_total, int N, int K, const float* __restrict__ bias, int act,
                        __nv_bfloat16* __restrict__ C, int32_t* status) {
  using P = GG<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;
  uint8_t* sched_mem = ring + P::STAGES * P::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sched_mem + GroupSched::smem_bytes());
  uint64_t* full = bars;
  uint64_t* empty = bars + P::STAGES;
  uint64_t* tfull = bars + 2 * P::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < P::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  GroupSched sched;
  sched.init(sched_mem, group_offsets, G, rows_total, P::BM, N / BN, status);
  if (warp == 1) {
    tmem_alloc(tmem_slot, P::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = sched.total_tiles();
  const int kblocks = K / P::BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const TileCoord tc = sched.decode(t);
        const int wrow = (tc.g % Gw) * N + tc.n_idx * BN;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, status, 0x101, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = ring + stage * P::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], P::STAGE_BYTES);
          tma_load_2d(sa, &tmA, &full[stage], kb * P::BK, tc.row0);
          tma_load_2d(sa + P::A_BYTES, &tmB, &full[stage], kb * P::BK, wrow);
          ++issued;
          if (++stage == P::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
      // Let every load this thread issued land before the CTA can exit.
      for (int i = 1; i <= P::STAGES && i <= issued; ++i) {
        const int64_t n = issued - i;
        mbar_wait(&full[n % P::STAGES], (uint32_t)((n / P::STAGES) & 1), status, 0x102, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(P::BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool any = false;
      for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t aph = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(&tempty[acc], aph ^ 1u, status, 0x103, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, 0x104, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(ring + stage * P::STAGE_BYTES);
          const uint32_t b = a + P::A_BYTES;
#pragma unroll
          for (int k = 0; k < P::BK / 16; ++k) {
            umma_bf16(d_tmem, smem_desc_sw128(a + k * 32), smem_desc_sw128(b + k * 32), idesc,
                      (kb | k) != 0 ? 1u : 0u);
          }
          any = true;
          umma_commit(&empty[stage]);
          if (++stage == P::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (any) {
        umma_commit(drain);
        mbar_wait(drain, 0, status, 0x105, nullptr);
      }
    }
  } else {
    const int q = warp & 3;  // the TMEM lane quadrant this warp may read
    const int r = q * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      const TileCoord tc = sched.decode(t);
      const int acc = it & 1;
      const uint32_t aph = (uint32_t)(it >> 1) & 1u;
      if (!mbar_wait(&tfull[acc], aph, status, 0x106, abort_flag)) break;
      tc_fence_after();
      const int gw = tc.g % Gw;
      const float* bptr = bias ? bias + (int64_t)gw * N + tc.n_idx * BN : nullptr;
      __nv_bfloat16* crow = C + ((int64_t)tc.row0 + r) * N + tc.n_idx * BN;
      const bool live = r < tc.rows;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32),
                           v);
        tmem_ld_wait();
        if (live) {
          float bv[32];
          if (bptr) {
            const float4* b4 = reinterpret_cast<const float4*>(bptr + c * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 bb = __ldg(b4 + j);
              bv[4 * j] = bb.x;
              bv[4 * j + 1] = bb.y;
              bv[4 * j + 2] = bb.z;
              bv[4 * j + 3] = bb.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) bv[j] = 0.0f;
          }
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float lo = __uint_as_float(v[2 * j]) + bv[2 * j];
            float hi = __uint_as_float(v[2 * j + 1]) + bv[2 * j + 1];
            act2(act, lo, hi);
            packed[j] = pack_bf16x2(lo, hi);
          }
          uint4* dst = reinterpret_cast<uint4*>(crow + c * 32);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2],
                                packed[4 * j + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, P::TMEM_COLS);
  }
}

template <int BN>
int launch_grouped_gemm(const void* A, const void* W, const float* bias, const int32_t* offs,
                        int G, int Gw, int64_t rows_total, int N, int K, int act, void* C,
                        int32_t* status, cudaStream_t s) {
  using P = GG<BN>;
  CUtensorMap tmA, tmB;
  if (!make_tmap_bf16_2d(&tmA, A, (uint64_t)rows_total, (uint64_t)K, (uint64_t)K, P::BM, P::BK))
    return CTI_ERR_INVALID_ARG;
  if (!make_tmap_bf16_2d(&tmB, W, (uint64_t)Gw * N, (uint64_t)K, (uint64_t)K, BN, P::BK))
    return CTI_ERR_INVALID_ARG;
  static uint64_t configured = 0;
  if (ensure_smem_limit(grouped_gemm_kernel<BN>, (int)P::SMEM, configured) != cudaSuccess)
    return CTI_ERR_CUDA;
  const int sms = device_sm_count();
  if (sms <= 0) return CTI_ERR_CUDA;
  const int64_t max_tiles = ((rows_total + P::BM - 1) / P::BM + G) * (N / BN);
  const int grid = (int)(max_tiles < sms ? max_tiles : sms);
  grouped_gemm_kernel<BN><<<grid, 192, P::SMEM, s>>>(tmA, tmB, offs, G, Gw, rows_total, N, K,
                                                     bias, act,
                                                     static_cast<__nv_bfloat16*>(C), status);
  return cudaGetLastError() == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}

}  // namespace
}  // namespace cti

extern "C" int cti_moe_grouped_gemm(const void* A_bf16, const void* W_bf16, const float* bias,
                                    const int32_t* group_offsets, int G, int Gw,
                                    int64_t rows_total, int N, int K, int act, void* C_bf16,
                                    int32_t* status, void* stream) {
  using namespace cti;
  if (G < 1 || G > GroupSched::kMaxGroups || Gw < 1 || rows_total < 0 || N <= 0 || K <= 0)
    return CTI_ERR_INVALID_ARG;
  if (act < CTI_ACT_NONE || act > CTI_ACT_GELU) return CTI_ERR_INVALID_ARG;
  if (N % 128 != 0 || K % 64 != 0) return CTI_ERR_UNSUPPORTED;
  if (rows_total >= ((int64_t)1 << 31) - 256) return CTI_ERR_UNSUPPORTED;
  if (!W_bf16 || !group_offsets || !C_bf16) return CTI_ERR_INVALID_ARG;
  if (rows_total == 0) return CTI_OK;
  if (!A_bf16) return CTI_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(C_bf16) & 15) || (bias && (reinterpret_cast<uintptr_t>(bias) & 15)))
    return CTI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (N % 256 == 0)
    return launch_grouped_gemm<256>(A_bf16, W_bf16, bias, group_offsets, G, Gw, rows_total, N, K,
                                    act, C_bf16, status, s);
  return launch_grouped_gemm<128>(A_bf16, W_bf16, bias, group_offsets, G, Gw, rows_total, N, K,
                                  act, C_bf16, status, s);
}
