// Stage 3, fused: the whole expert FFN of a 128-row tile in one CTA,
//
//   Y[rows] = act(Xp[rows] @ W1[e]^T + b1[e]) @ W2[e]^T + b2[e],
//
// with the [128, d_ff] hidden activation never leaving the SM.  The
// reference writes that hidden tensor to HBM between its fc1 and fc2 Triton
// GEMMs (packed_hidden, E*T*F elements; online_best/infer.py:2028-2034,
// :2128-2167); at d_model 256 / d_ff 1024 that round trip alone costs about
// as much HBM time as the GEMMs' tensor time.
//
// Per tile (128 token rows of one expert), d_ff is processed in 128-wide
// chunks c:
//   GEMM1(c): acc1[c%2] (TMEM, 128 cols) = X[128, D] @ W1[e][c*128:+128, :]^T
//   epilogue: acc1 -> +b1 -> GELU -> bf16 -> H (shared memory, laid out
//             exactly as a TMA 128-byte-swizzled K-major tile)
//   GEMM2(c): acc2 (TMEM, D cols) += H @ W2[e][:, c*128:+128]^T
// The MMA thread issues GEMM2(c) only after GEMM1(c+2), so the tensor core
// works on other chunks while the epilogue warps run the GELU of chunk c.
// After the last chunk, acc2 + b2 is written to Y as bf16.
//
// Roles (576 threads): warp 0 TMA producer (X tile once per tile; W1/W2
// slabs through a ring of 32 KB stages), warp 1 TMEM owner and MMA issuer
// (tcgen05.mma M=128, K=16, bf16 -> fp32; N=128 for GEMM1, N=D for GEMM2),
// warps 2-17 epilogue
// (four warps per TMEM lane quadrant, each owning 32 of a chunk's 128
// columns and a quarter of the output columns; the expert's biases are
// staged in shared memory once per expert change).
//
// TMEM: acc2 in columns [0, D), acc1 buffers at 256 and 384 (512 allocated).
// Shared memory (D=256): X 64 KB + H 32 KB + ring 3x32 KB + biases 5 KB +
// scheduler 2 KB.  One H buffer suffices with the two-chunk lag: the
// epilogue writes H(c) after GEMM2(c-1) has read H(c-1), still well before
// GEMM2(c) is due.  d_ff <= 1024 (one expert's b1 in shared memory).
#include "common.cuh"
#include "gelu.cuh"
#include "sched.cuh"
#include "tmap.cuh"

namespace cti {
namespace {

constexpr int kBM = 128;
constexpr int kFC = 128;           // d_ff chunk
constexpr int kBK = 64;            // bf16 elements per 128-byte swizzled row
constexpr int kSlab = kBM * kBK * 2;  // 16 KB: one 128x64 bf16 tile
// Weight ring stages of 32 KB: each wait on a stage covers 8 MMAs (GEMM1,
// N=128) or 4 MMAs of N=256 (GEMM2), enough tensor work to hide the cost of
// the wait and fence on the issuing thread.
constexpr int kStage = 2 * kSlab;
constexpr int kEpiWarps = 16;
constexpr int kMaxF = 1024;  // b1 of one expert staged in shared memory
using Sched = GroupSchedT<256>;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kThreads = 64 + kEpiThreads;
constexpr uint32_t kAcc1Col = 256;
// GEMM2 of chunk c is issued after GEMM1 of chunk c+kLag: between the end of
// GEMM1(c) and the start of GEMM2(c) the tensor core has 2*kLag GEMMs of other
// chunks to run, which is the time the epilogue has for the GELU of chunk c.
constexpr int kLag = 2;

template <int D>
struct FF {
  static constexpr int XK = D / kBK;          // X k-slabs
  static constexpr int G1S = XK / 2;          // ring stages of W1 per chunk (2 k-slabs each)
  static constexpr int KPS2 = kStage / (D * kBK * 2);  // W2 k-slabs [D x 64] per stage
  static constexpr int G2S = 2 / KPS2;        // ring stages of W2 per chunk
  static constexpr int STAGES = D == 256 ? 3 : 4;
  static constexpr size_t X_BYTES = (size_t)XK * kSlab;
  static constexpr size_t H_BYTES = (size_t)2 * kSlab;  // one 128x128 hidden chunk
  static constexpr size_t RING_BYTES = (size_t)STAGES * kStage;
  static constexpr size_t BIAS_BYTES = (size_t)(kMaxF + D) * 4;
  static constexpr size_t SMEM =
      1024 + X_BYTES + H_BYTES + RING_BYTES + BIAS_BYTES + Sched::smem_bytes() + 256;
};

// Writes 32 consecutive bf16 columns (four 16-byte chunks, starting at
// chunk j0 of the row) of row r into a 128x64 K-major slab with the
// 128-byte swizzle (chunk j of row r lives at chunk position j ^ (r % 8)),
// the layout TMA produces and UMMA reads.
CTI_DEVICE void store_row32_swizzled(uint8_t* slab, int r, int j0, const uint32_t (&w)[16]) {
  uint8_t* row = slab + r * 128;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int pos = (j0 + j) ^ (r & 7);
    *reinterpret_cast<uint4*>(row + pos * 16) =
        make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  }
}

// One arrival per warp: the lanes' prior writes are ordered before lane 0's
// (release) arrive by the warp barrier.  Barriers signalled this way count
// warps, not threads.
CTI_DEVICE void warp_arrive(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fused_ffn_kernel(const __grid_constant__ CUtensorMap tmX,
                     const __grid_constant__ CUtensorMap tmW1,
                     const __grid_constant__ CUtensorMap tmW2,
                     const int32_t* __restrict__ group_offsets, int G, int Gw, int64_t rows_total,
                     int F, const float* __restrict__ b1, const float* __restrict__ b2, int act,
                     __nv_bfloat16* __restrict__ Y, int32_t* status) {
  using P = FF<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sx = smem;
  uint8_t* sh = sx + P::X_BYTES;
  uint8_t* ring = sh + P::H_BYTES;
  float* b1s = reinterpret_cast<float*>(ring + P::RING_BYTES);
  float* b2s = b1s + kMaxF;
  uint8_t* sched_mem = reinterpret_cast<uint8_t*>(b2s + D);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sched_mem + Sched::smem_bytes());
  uint64_t* full = bars;
  uint64_t* empty = full + P::STAGES;
  uint64_t* x_full = empty + P::STAGES;
  uint64_t* x_empty = x_full + 1;
  uint64_t* a1_full = x_empty + 1;  // [2]
  uint64_t* a1_empty = a1_full + 2;  // [2]
  uint64_t* h_full = a1_empty + 2;
  uint64_t* h_empty = h_full + 1;
  uint64_t* a2_full = h_empty + 1;
  uint64_t* a2_empty = a2_full + 1;
  uint64_t* drain = a2_empty + 1;
  uint64_t* bfree = drain + 1;   // epilogue threads done with the staged biases
  uint64_t* bready = bfree + 1;  // new biases staged
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int nch = F / kFC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(x_full, 1);
    mbar_init(x_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a1_full[i], 1);
      mbar_init(&a1_empty[i], kEpiWarps);
    }
    mbar_init(h_full, kEpiWarps);
    mbar_init(h_empty, 1);
    mbar_init(a2_full, 1);
    mbar_init(a2_empty, kEpiWarps);
    mbar_init(drain, 1);
    mbar_init(bfree, kEpiWarps);
    mbar_init(bready, kEpiWarps);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&tmX);
    prefetch_tensormap(&tmW1);
    prefetch_tensormap(&tmW2);
  }
  Sched sched;
  sched.init(sched_mem, group_offsets, G, rows_total, kBM, 1, status);
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = sched.total_tiles();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0, x_issued = 0;
      int it = 0;
      bool ok = true;
      // Claims the next ring stage (bounded wait) and arms it for kStage bytes.
      auto acquire = [&]() -> uint8_t* {
        if (!mbar_wait(&empty[stage], phase ^ 1u, status, 0x201, abort_flag)) return nullptr;
        mbar_arrive_expect_tx(&full[stage], kStage);
        return ring + stage * kStage;
      };
      auto advance = [&]() {
        ++issued;
        if (++stage == P::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        const TileCoord tc = sched.decode(t);
        const int gw = tc.g % Gw;
        if (!mbar_wait(x_empty, (uint32_t)(it & 1) ^ 1u, status, 0x202, abort_flag)) break;
        mbar_arrive_expect_tx(x_full, (uint32_t)P::X_BYTES);
        for (int kb = 0; kb < P::XK; ++kb)
          tma_load_2d(sx + kb * kSlab, &tmX, x_full, kb * kBK, tc.row0);
        ++x_issued;
        for (int s = 0; s < nch + kLag && ok; ++s) {
          if (s < nch) {  // W1 rows [s*128, +128), two 64-wide k-slabs per stage
            for (int j = 0; j < P::G1S && ok; ++j) {
              uint8_t* buf = acquire();
              if (!buf) {
                ok = false;
                break;
              }
              for (int h = 0; h < 2; ++h)
                tma_load_2d(buf + h * kSlab, &tmW1, &full[stage], (2 * j + h) * kBK,
                            gw * F + s * kFC);
              advance();
            }
          }
          if (s >= kLag && ok) {  // W2 [D rows, 64 k] slabs of chunk s-kLag
            const int c = s - kLag;
            for (int j = 0; j < P::G2S && ok; ++j) {
              uint8_t* buf = acquire();
              if (!buf) {
                ok = false;
                break;
              }
              for (int h = 0; h < P::KPS2; ++h)
                tma_load_2d(buf + h * (D * kBK * 2), &tmW2, &full[stage],
                            c * kFC + (j * P::KPS2 + h) * kBK, gw * D);
              advance();
            }
          }
        }
      }
      // Let every load this thread issued land before the CTA can exit.
      for (int i = 1; i <= P::STAGES && i <= issued; ++i) {
        const int64_t n = issued - i;
        mbar_wait(&full[n % P::STAGES], (uint32_t)((n / P::STAGES) & 1), status, 0x203, nullptr);
      }
      (void)kSlab;
      if (x_issued > 0) mbar_wait(x_full, (uint32_t)((x_issued - 1) & 1), status, 0x204, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc1 = idesc_bf16_f32(kBM, 128);  // GEMM1: N = d_ff chunk
      const uint32_t idesc2 = idesc_bf16_f32(kBM, D);    // GEMM2: N = d_model
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool any = false, ok = true;
      const uint32_t x_addr = smem_u32(sx);
      const uint32_t h_addr = smem_u32(sh);
      const uint32_t ring_addr = smem_u32(ring);
      auto advance = [&]() {
        if (++stage == P::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        if (!mbar_wait(x_full, (uint32_t)(it & 1), status, 0x205, abort_flag)) break;
        tc_fence_after();
        for (int s = 0; s < nch + kLag && ok; ++s) {
          if (s < nch) {  // GEMM1(s)
            const int64_t gc = (int64_t)it * nch + s;
            const int b = (int)(gc & 1);
            const uint32_t k = (uint32_t)(gc >> 1);
            if (!mbar_wait(&a1_empty[b], (k & 1u) ^ 1u, status, 0x206, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + kAcc1Col + (uint32_t)b * 128u;
            for (int j = 0; j < P::G1S; ++j) {
              if (!mbar_wait(&full[stage], phase, status, 0x207, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t b0 = ring_addr + stage * kStage;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int kb = 2 * j + h;
                const uint32_t a0 = x_addr + kb * kSlab;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                  umma_bf16(d, smem_desc_sw128(a0 + kk * 32),
                            smem_desc_sw128(b0 + h * kSlab + kk * 32), idesc1,
                            (kb | kk) != 0 ? 1u : 0u);
              }
              any = true;
              umma_commit(&empty[stage]);
              advance();
            }
            if (!ok) break;
            umma_commit(&a1_full[b]);
            if (s == nch - 1) umma_commit(x_empty);
          }
          if (s >= kLag) {  // GEMM2(s-kLag), N = D in one instruction
            const int c = s - kLag;
            const int64_t gc = (int64_t)it * nch + c;
            if (c == 0) {
              if (!mbar_wait(a2_empty, (uint32_t)(it & 1) ^ 1u, status, 0x208, abort_flag)) {
                ok = false;
                break;
              }
            }
            if (!mbar_wait(h_full, (uint32_t)(gc & 1), status, 0x209, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            for (int j = 0; j < P::G2S; ++j) {
              if (!mbar_wait(&full[stage], phase, status, 0x20a, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t b0 = ring_addr + stage * kStage;
#pragma unroll
              for (int h = 0; h < P::KPS2; ++h) {
                const int kb = j * P::KPS2 + h;
                const uint32_t a0 = h_addr + kb * kSlab;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                  umma_bf16(tmem_base, smem_desc_sw128(a0 + kk * 32),
                            smem_desc_sw128(b0 + h * (D * kBK * 2) + kk * 32), idesc2,
                            (c | kb | kk) != 0 ? 1u : 0u);
              }
              umma_commit(&empty[stage]);
              advance();
            }
            if (!ok) break;
            umma_commit(h_empty);
            if (c == nch - 1) umma_commit(a2_full);
          }
        }
      }
      if (any) {
        umma_commit(drain);
        mbar_wait(drain, 0, status, 0x20b, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // 16 warps: four per TMEM lane quadrant q; warp group `sub` owns chunk
    // columns [sub*32, sub*32+32) and output columns [sub*D/4, (sub+1)*D/4).
    const int ew = warp - 2;           // 0..15
    const int q = warp & 3;            // TMEM lane quadrant of this warp
    const int sub = ew >> 2;           // 0..3
    const int r = q * 32 + lane;       // tile row owned by this thread
    const int etid = ew * 32 + lane;   // 0..511
    constexpr int kOutCols = D / 4;
    int it = 0;
    int staged_gw = -1;
    uint32_t n_staged = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
      const TileCoord tc = sched.decode(t);
      const int gw = tc.g % Gw;
      if (gw != staged_gw) {  // the same decision in every epilogue thread
        if (n_staged > 0) {   // everyone is done with the previous expert's biases
          warp_arrive(bfree, lane);
          if (!mbar_wait(bfree, (n_staged - 1) & 1u, status, 0x20f, abort_flag)) break;
        }
        for (int i = etid; i < F; i += kEpiThreads) b1s[i] = b1[(int64_t)gw * F + i];
        for (int i = etid; i < D; i += kEpiThreads) b2s[i] = b2[(int64_t)gw * D + i];
        warp_arrive(bready, lane);
        if (!mbar_wait(bready, n_staged & 1u, status, 0x210, abort_flag)) break;
        ++n_staged;
        staged_gw = gw;
      }
      for (int c = 0; c < nch; ++c) {
        const int64_t gc = (int64_t)it * nch + c;
        const int b = (int)(gc & 1);
        const uint32_t k = (uint32_t)(gc >> 1);
        if (!mbar_wait(&a1_full[b], k & 1u, status, 0x20c, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + kAcc1Col + (uint32_t)b * 128u +
                               (uint32_t)sub * 32u,
                           v);
        tmem_ld_wait();
        tc_fence_before();
        warp_arrive(&a1_empty[b], lane);

        const float* bc = b1s + c * kFC + sub * 32;
        uint32_t w[16];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float a[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) a[i] = __uint_as_float(v[16 * h + i]) + bc[16 * h + i];
          act_n<16>(act, a);
#pragma unroll
          for (int i = 0; i < 8; ++i) w[8 * h + i] = pack_bf16x2(a[2 * i], a[2 * i + 1]);
        }
        if (!mbar_wait(h_empty, (uint32_t)(gc & 1) ^ 1u, status, 0x20d, abort_flag)) {
          ok = false;
          break;
        }
        store_row32_swizzled(sh + (size_t)(sub >> 1) * kSlab, r, (sub & 1) * 4, w);
        fence_proxy_async_smem();
        warp_arrive(h_full, lane);
      }
      if (!ok) break;

      // Output: acc2 + b2 -> bf16 rows of Y.
      if (!mbar_wait(a2_full, (uint32_t)(it & 1), status, 0x20e, abort_flag)) break;
      tc_fence_after();
      uint32_t o[kOutCols];
      const uint32_t taddr2 = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)sub * kOutCols;
#pragma unroll
      for (int j = 0; j < kOutCols / 32; ++j) {
        uint32_t tmp[32];
        tmem_ld_32x32b_x32(taddr2 + 32 * j, tmp);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[32 * j + i] = tmp[i];
      }
      tmem_ld_wait();
      tc_fence_before();
      warp_arrive(a2_empty, lane);
      if (r < tc.rows) {
        const float* bo = b2s + sub * kOutCols;
        uint4* dst = reinterpret_cast<uint4*>(Y + ((int64_t)tc.row0 + r) * D + sub * kOutCols);
#pragma unroll
        for (int j = 0; j < kOutCols / 8; ++j) {
          uint4 pk;
          pk.x = pack_bf16x2(__uint_as_float(o[8 * j]) + bo[8 * j],
                             __uint_as_float(o[8 * j + 1]) + bo[8 * j + 1]);
          pk.y = pack_bf16x2(__uint_as_float(o[8 * j + 2]) + bo[8 * j + 2],
                             __uint_as_float(o[8 * j + 3]) + bo[8 * j + 3]);
          pk.z = pack_bf16x2(__uint_as_float(o[8 * j + 4]) + bo[8 * j + 4],
                             __uint_as_float(o[8 * j + 5]) + bo[8 * j + 5]);
          pk.w = pack_bf16x2(__uint_as_float(o[8 * j + 6]) + bo[8 * j + 6],
                             __uint_as_float(o[8 * j + 7]) + bo[8 * j + 7]);
          dst[j] = pk;
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int D>
int launch_fused(const void* Xp, const void* W1, const float* b1, const void* W2, const float* b2,
                 const int32_t* offs, int G, int Gw, int64_t rows_total, int F, int act, void* Y,
                 int32_t* status, cudaStream_t s) {
  using P = FF<D>;
  CUtensorMap tmX, tmW1, tmW2;
  if (!make_tmap_bf16_2d(&tmX, Xp, (uint64_t)rows_total, D, D, kBM, kBK) ||
      !make_tmap_bf16_2d(&tmW1, W1, (uint64_t)Gw * F, D, D, 128, kBK) ||
      !make_tmap_bf16_2d(&tmW2, W2, (uint64_t)Gw * D, (uint64_t)F, (uint64_t)F, D, kBK))
    return CTI_ERR_INVALID_ARG;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(fused_ffn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)P::SMEM) != cudaSuccess)
      return CTI_ERR_CUDA;
    attr_set = true;
  }
  const int sms = device_sm_count();
  if (sms <= 0) return CTI_ERR_CUDA;
  const int64_t max_tiles = (rows_total + kBM - 1) / kBM + G;
  const int grid = (int)(max_tiles < sms ? max_tiles : sms);
  fused_ffn_kernel<D><<<grid, kThreads, P::SMEM, s>>>(tmX, tmW1, tmW2, offs, G, Gw, rows_total, F,
                                                       b1, b2, act,
                                                       static_cast<__nv_bfloat16*>(Y), status);
  return cudaGetLastError() == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}

}  // namespace
}  // namespace cti

extern "C" int cti_moe_expert_ffn_fused(const void* Xp_bf16, const void* W1_bf16, const float* b1,
                                        const void* W2_bf16, const float* b2,
                                        const int32_t* group_offsets, int G, int Gw,
                                        int64_t rows_total, int D, int F, int act, void* Y_bf16,
                                        int32_t* status, void* stream) {
  using namespace cti;
  if (G < 1 || Gw < 1 || rows_total < 0 || F <= 0) return CTI_ERR_INVALID_ARG;
  if (act < CTI_ACT_NONE || act > CTI_ACT_GELU) return CTI_ERR_INVALID_ARG;
  if ((D != 128 && D != 256) || F % kFC != 0 || F > kMaxF || G > Sched::kMaxGroups)
    return CTI_ERR_UNSUPPORTED;
  if (rows_total >= ((int64_t)1 << 31) - 256) return CTI_ERR_UNSUPPORTED;
  if (!W1_bf16 || !W2_bf16 || !b1 || !b2 || !group_offsets || !Y_bf16) return CTI_ERR_INVALID_ARG;
  if (rows_total == 0) return CTI_OK;
  if (!Xp_bf16) return CTI_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(Y_bf16) & 15) || (reinterpret_cast<uintptr_t>(b1) & 15) ||
      (reinterpret_cast<uintptr_t>(b2) & 15))
    return CTI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 256)
    return launch_fused<256>(Xp_bf16, W1_bf16, b1, W2_bf16, b2, group_offsets, G, Gw, rows_total,
                             F, act, Y_bf16, status, s);
  return launch_fused<128>(Xp_bf16, W1_bf16, b1, W2_bf16, b2, group_offsets, G, Gw, rows_total, F,
                           act, Y_bf16, status, s);
}
