// Stage 3, fused, on CTA pairs: the expert FFN of a 256-row tile on two SMs,
//
//   Y[rows] = act(Xp[rows] @ W1[e]^T + b1[e]) @ W2[e]^T + b2[e],
//
// with one tcgen05.mma.cta_group::2 instruction stream for both SMs of a
// thread-block cluster of two.  The same schedule as fused_ffn.cu (d_ff in
// 128-wide chunks c; GEMM1(c) -> acc1 in TMEM; bias + GELU -> bf16 H(c)
// written back into TMEM; GEMM2(c) reads A = H(c) from TMEM and accumulates
// acc2 = Y in TMEM; GEMM2(c) issued after GEMM1(c+1)), but on pairs:
//
//   * each CTA holds its own 128 rows of the tile (X in shared memory; acc1,
//     H and acc2 in its TMEM), and HALF of every weight chunk: rows
//     [64r, 64r + 64) of the W1 chunk and rows [128r, 128r + 128) of the W2
//     chunk, r = its rank in the pair.  One M = 256 MMA reads A from both
//     CTAs and B from both halves, so each SM streams half as many weight
//     bytes per FLOP as the one-CTA kernel, and the shared-memory operand
//     reads of GEMM1 drop from 128 to 96 bytes per clock at full tensor rate;
//   * the freed shared memory double-buffers both weight rings (two
//     whole-chunk slots each), so the next chunk's weights load while the
//     current one is multiplied;
//   * the even CTA (leader) issues every MMA.  Barriers it waits on live in
//     its shared memory: the peer's TMA loads complete on them
//     (cp.async.bulk.tensor ... .cta_group::2) and the peer's epilogue warps
//     arrive on them through shared::cluster addresses.  MMA completions
//     that both CTAs wait for are committed twice, once to each CTA's copy
//     of the barrier.
//
// Roles per CTA (576 threads): warp 0 TMA producer (its X rows and its
// weight halves), warp 1 TMEM allocation for the pair and, in the leader,
// the MMA issuer, warps 2-17 epilogue (its 128 rows of acc1/H and acc2).
// TMEM per CTA: acc2 in columns [0, 256), acc1 buffers at 256 and 384.
// Shared memory per CTA: X 64 KB + W1 ring 2 x 32 KB + W2 ring 2 x 32 KB +
// biases 5 KB + scheduler 2 KB.  d_model 256, d_ff a multiple of 128 up to
// 1024.
//
// Every wait is bounded (common.cuh); a CTA that gives up sets its abort
// flag, its roles unwind, the peer's waits run out in turn, and both CTAs
// meet at the final cluster barrier before freeing TMEM.
#include "common.cuh"
#include "gelu.cuh"
#include "sched.cuh"
#include "tmap.cuh"

namespace cti {
namespace {

constexpr int kPD = 256;               // d_model
constexpr int kPBM = 128;              // rows per CTA; a pair tile has 256
constexpr int kPFC = 128;              // d_ff chunk
constexpr int kPBK = 64;               // bf16 per 128-byte swizzled row
constexpr int kPXK = kPD / kPBK;       // 4 X k-slabs
constexpr int kPEpiWarps = 16;
constexpr int kPThreads = 64 + kPEpiWarps * 32;
constexpr int kPMaxF = 1024;
constexpr int kPNSlot = 2;
constexpr uint32_t kPAcc1Col = 256;
using PSched = GroupSchedT<256>;

constexpr size_t kPXSlab = (size_t)kPBM * kPBK * 2;          // 16 KB: [128 x 64]
constexpr size_t kPXBytes = kPXK * kPXSlab;                   // 64 KB
constexpr size_t kPW1Slab = (size_t)(kPFC / 2) * kPBK * 2;    // 8 KB: [64 x 64]
constexpr size_t kPW1Slot = kPXK * kPW1Slab;                  // 32 KB: half a W1 chunk
constexpr size_t kPW2Slab = (size_t)(kPD / 2) * kPBK * 2;     // 16 KB: [128 x 64]
constexpr size_t kPW2Slot = 2 * kPW2Slab;                     // 32 KB: half a W2 chunk
constexpr size_t kPBias = (size_t)(kPMaxF + kPD) * 4;
constexpr size_t kPSmem = 1024 + kPXBytes + kPNSlot * (kPW1Slot + kPW2Slot) + kPBias +
                          PSched::smem_bytes() + 512;
static_assert(kPSmem <= 232448, "shared memory per CTA");

CTI_DEVICE void pair_warp_arrive_local(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

CTI_DEVICE void pair_warp_arrive_remote(uint32_t cluster_bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive_cluster(cluster_bar);
}

// Commits the completion of every pair MMA issued so far to the barrier at
// the same offset in both CTAs.
CTI_DEVICE void commit_both(uint64_t* bar) {
  umma_commit_pair(mapa_shared(bar, 0));
  umma_commit_pair(mapa_shared(bar, 1));
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    fused_ffn_pair_kernel(const __grid_constant__ CUtensorMap tmX,
                          const __grid_constant__ CUtensorMap tmW1,
                          const __grid_constant__ CUtensorMap tmW2,
                          const int32_t* __restrict__ group_offsets, int G, int Gw,
                          int64_t rows_total, int F, const float* __restrict__ b1,
                          const float* __restrict__ b2, int act,
                          __nv_bfloat16* __restrict__ Y, int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sx = smem;
  uint8_t* ring1 = sx + kPXBytes;                       // W1 halves
  uint8_t* ring2 = ring1 + kPNSlot * kPW1Slot;          // W2 halves
  float* b1s = reinterpret_cast<float*>(ring2 + kPNSlot * kPW2Slot);
  float* b2s = b1s + kPMaxF;
  uint8_t* sched_mem = reinterpret_cast<uint8_t*>(b2s + kPD);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sched_mem + PSched::smem_bytes());
  // Waited on by the leader's MMA thread (arrivals and bytes from both CTAs):
  uint64_t* full1 = bars;            // [2] W1 halves of both CTAs landed
  uint64_t* full2 = full1 + 2;       // [2] W2 halves landed
  uint64_t* x_full = full2 + 2;      // X rows of both CTAs landed
  uint64_t* h_full = x_full + 1;     // [2][2] half h of H(c) written by both epilogues
  uint64_t* a2_empty = h_full + 4;   // both epilogues have read acc2
  uint64_t* drain = a2_empty + 1;
  // Waited on in each CTA (committed by the leader to both copies):
  uint64_t* empty1 = drain + 1;      // [2] a W1 slot may be refilled
  uint64_t* empty2 = empty1 + 2;     // [2]
  uint64_t* x_empty = empty2 + 2;
  uint64_t* a1_full = x_empty + 1;   // [2] GEMM1(c) done
  uint64_t* a2_full = a1_full + 2;   // GEMM2 of the tile's last chunk done
  // Local to the epilogue of each CTA:
  uint64_t* bfree = a2_full + 1;
  uint64_t* bready = bfree + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_cta_rank();
  const bool leader = rank == 0;
  const int nch = F / kPFC;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPNSlot; ++s) {
      mbar_init(&full1[s], 1);
      mbar_init(&full2[s], 1);
      mbar_init(&empty1[s], 1);
      mbar_init(&empty2[s], 1);
    }
    mbar_init(x_full, 1);
    mbar_init(x_empty, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&h_full[i], 2 * kPEpiWarps);
    mbar_init(a2_empty, 2 * kPEpiWarps);
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&a1_full[i], 1);
    mbar_init(a2_full, 1);
    mbar_init(bfree, kPEpiWarps);
    mbar_init(bready, kPEpiWarps);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&tmX);
    prefetch_tensormap(&tmW1);
    prefetch_tensormap(&tmW2);
  }
  grid_dependents_launch();
  grid_dependency_wait();  // offsets and rows come from the dispatch kernels
  PSched sched;
  sched.init(sched_mem, group_offsets, G, rows_total, 2 * kPBM, 1, status);
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Both CTAs' barriers are initialised and the pair's TMEM is allocated
  // before either CTA signals the other.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = sched.total_tiles();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t full1_c[2] = {mapa_shared(&full1[0], 0), mapa_shared(&full1[1], 0)};
      const uint32_t full2_c[2] = {mapa_shared(&full2[0], 0), mapa_shared(&full2[1], 0)};
      const uint32_t x_full_c = mapa_shared(x_full, 0);
      int n1 = 0, n2 = 0, x_issued = 0;
      int it = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs, ++it) {
        const TileCoord tc = sched.decode(t);
        const int gw = tc.g % Gw;
        const int my_row0 = tc.row0 + (int)rank * kPBM;
        if (!mbar_wait_cluster(x_empty, (uint32_t)(it & 1) ^ 1u, status, 0x302, abort_flag)) break;
        if (leader) mbar_arrive_expect_tx(x_full, (uint32_t)(2 * kPXBytes));
        for (int kb = 0; kb < kPXK; ++kb)
          tma_load_2d_pair(sx + kb * kPXSlab, &tmX, x_full_c, kb * kPBK, my_row0);
        ++x_issued;
        if (t + npairs < total) {  // the next tile's rows into L2
          const TileCoord nx = sched.decode(t + npairs);
          for (int kb = 0; kb < kPXK; ++kb)
            tma_prefetch_l2_2d(&tmX, kb * kPBK, nx.row0 + (int)rank * kPBM);
        }
        for (int s = 0; s <= nch && ok; ++s) {
          if (s < nch) {  // this CTA's half of W1 chunk s
            const int slot = n1 & 1;
            if (!mbar_wait_cluster(&empty1[slot], (uint32_t)((n1 >> 1) & 1) ^ 1u, status, 0x301,
                                   abort_flag)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(&full1[slot], (uint32_t)(2 * kPW1Slot));
            uint8_t* buf = ring1 + slot * kPW1Slot;
            for (int kb = 0; kb < kPXK; ++kb)
              tma_load_2d_pair(buf + kb * kPW1Slab, &tmW1, full1_c[slot], kb * kPBK,
                               gw * F + s * kPFC + (int)rank * (kPFC / 2));
            ++n1;
          }
          if (s >= 1) {  // this CTA's half of W2 chunk s-1: output rows [128r, +128)
            const int c = s - 1;
            const int slot = n2 & 1;
            if (!mbar_wait_cluster(&empty2[slot], (uint32_t)((n2 >> 1) & 1) ^ 1u, status, 0x303,
                                   abort_flag)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(&full2[slot], (uint32_t)(2 * kPW2Slot));
            uint8_t* buf = ring2 + slot * kPW2Slot;
            for (int h = 0; h < 2; ++h)
              tma_load_2d_pair(buf + h * kPW2Slab, &tmW2, full2_c[slot], c * kPFC + h * kPBK,
                               gw * kPD + (int)rank * (kPD / 2));
            ++n2;
          }
        }
      }
      // The leader's full barriers count both CTAs' bytes: once their last
      // armed phases complete, no load of either CTA is in flight.
      if (leader) {
        for (int i = 1; i <= kPNSlot; ++i) {
          if (n1 - i >= 0)
            mbar_wait_cluster(&full1[(n1 - i) & 1], (uint32_t)(((n1 - i) >> 1) & 1), status,
                              0x304, nullptr);
          if (n2 - i >= 0)
            mbar_wait_cluster(&full2[(n2 - i) & 1], (uint32_t)(((n2 - i) >> 1) & 1), status,
                              0x304, nullptr);
        }
        if (x_issued > 0)
          mbar_wait_cluster(x_full, (uint32_t)((x_issued - 1) & 1), status, 0x304, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (leader && lane == 0) {
      const uint32_t idesc1 = idesc_bf16_f32(2 * kPBM, kPFC);  // GEMM1: M 256, N 128
      const uint32_t idesc2 = idesc_bf16_f32(2 * kPBM, kPD);   // GEMM2: M 256, N 256
      int n1 = 0, n2 = 0;
      int it = 0;
      bool any = false, ok = true;
      const uint32_t x_addr = smem_u32(sx);
      const uint32_t ring1_addr = smem_u32(ring1);
      const uint32_t ring2_addr = smem_u32(ring2);
      for (int t = pair; t < total && ok; t += npairs, ++it) {
        if (!mbar_wait_cluster(x_full, (uint32_t)(it & 1), status, 0x305, abort_flag)) break;
        tc_fence_after();
        for (int s = 0; s <= nch && ok; ++s) {
          if (s < nch) {  // GEMM1(s) into acc1[(it*nch + s) % 2]
            const int b = (it * nch + s) & 1;
            const uint32_t d = tmem_base + kPAcc1Col + (uint32_t)b * 128u;
            const int slot = n1 & 1;
            if (!mbar_wait_cluster(&full1[slot], (uint32_t)((n1 >> 1) & 1), status, 0x307,
                                   abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t b0 = ring1_addr + (uint32_t)(slot * kPW1Slot);
#pragma unroll
            for (int kb = 0; kb < kPXK; ++kb) {
#pragma unroll
              for (int kk = 0; kk < kPBK / 16; ++kk)
                umma_bf16_pair(d, smem_desc_sw128(x_addr + kb * kPXSlab + kk * 32),
                               smem_desc_sw128(b0 + kb * kPW1Slab + kk * 32), idesc1,
                               (kb | kk) != 0 ? 1u : 0u);
            }
            commit_both(&empty1[slot]);
            commit_both(&a1_full[b]);
            if (s == nch - 1) commit_both(x_empty);
            any = true;
            ++n1;
          }
          if (s >= 1) {  // GEMM2(s-1): acc2 += H(s-1) @ W2 chunk, A from TMEM
            const int c = s - 1;
            const int gc = it * nch + c;
            const int b = gc & 1;
            const uint32_t k = (uint32_t)(gc >> 1);
            if (c == 0 &&
                !mbar_wait_cluster(a2_empty, (uint32_t)(it & 1) ^ 1u, status, 0x308, abort_flag)) {
              ok = false;
              break;
            }
            const int slot = n2 & 1;
            if (!mbar_wait_cluster(&full2[slot], (uint32_t)((n2 >> 1) & 1), status, 0x30a,
                                   abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t h_tmem = tmem_base + kPAcc1Col + (uint32_t)b * 128u;
            const uint32_t b0 = ring2_addr + (uint32_t)(slot * kPW2Slot);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (!mbar_wait_cluster(&h_full[2 * b + h], k & 1u, status, 0x309, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < kPBK / 16; ++kk)
                umma_bf16_ts_pair(tmem_base, h_tmem + (uint32_t)(h * 64 + kk * 16),
                                  smem_desc_sw128(b0 + (uint32_t)(h * kPW2Slab) + kk * 32),
                                  idesc2, (c | h | kk) != 0 ? 1u : 0u);
            }
            if (!ok) break;
            commit_both(&empty2[slot]);
            if (c == nch - 1) commit_both(a2_full);
            ++n2;
          }
        }
      }
      if (any) {
        umma_commit_pair(mapa_shared(drain, 0));
        mbar_wait_cluster(drain, 0, status, 0x30b, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // 16 warps: four per TMEM lane quadrant q; warp group `sub` owns chunk
    // columns [sub*16, +16) of each 64-column half and output columns
    // [sub*64, +64).  H(c) half h goes into the first 8 of the thread's 16
    // columns of that half, so GEMM2's K step kk of half h reads 8
    // contiguous columns at 64h + 16kk (the layout of fused_ffn.cu).
    const int ew = warp - 2;
    const int q = warp & 3;
    const int sub = ew >> 2;
    const int r = q * 32 + lane;
    const int etid = ew * 32 + lane;
    constexpr int kOutCols = kPD / 4;
    const uint32_t h_full_c[4] = {mapa_shared(&h_full[0], 0), mapa_shared(&h_full[1], 0),
                                  mapa_shared(&h_full[2], 0), mapa_shared(&h_full[3], 0)};
    const uint32_t a2_empty_c = mapa_shared(a2_empty, 0);
    int it = 0;
    int staged_gw = -1;
    uint32_t n_staged = 0;
    bool ok = true;
    for (int t = pair; t < total && ok; t += npairs, ++it) {
      const TileCoord tc = sched.decode(t);
      const int gw = tc.g % Gw;
      const int my_row0 = tc.row0 + (int)rank * kPBM;
      const int my_rows = tc.rows - (int)rank * kPBM;  // may be <= 0 in the last tile
      if (gw != staged_gw) {
        if (n_staged > 0) {
          pair_warp_arrive_local(bfree, lane);
          if (!mbar_wait(bfree, (n_staged - 1) & 1u, status, 0x30f, abort_flag)) break;
        }
        for (int i = etid; i < F; i += kPEpiWarps * 32) b1s[i] = b1[(int64_t)gw * F + i];
        for (int i = etid; i < kPD; i += kPEpiWarps * 32) b2s[i] = b2[(int64_t)gw * kPD + i];
        pair_warp_arrive_local(bready, lane);
        if (!mbar_wait(bready, n_staged & 1u, status, 0x310, abort_flag)) break;
        ++n_staged;
        staged_gw = gw;
      }
      for (int c = 0; c < nch; ++c) {
        const int gc = it * nch + c;
        const int b = gc & 1;
        const uint32_t k = (uint32_t)(gc >> 1);
        if (!mbar_wait_cluster(&a1_full[b], k & 1u, status, 0x30c, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + kPAcc1Col +
                               (uint32_t)b * 128u + (uint32_t)sub * 16u;
        uint32_t v[2][16];
        tmem_ld_32x32b_x16(tbase, v[0]);
        tmem_ld_32x32b_x16(tbase + 64u, v[1]);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float4* bc = reinterpret_cast<const float4*>(b1s + c * kPFC + h * 64 + sub * 16);
          float a[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 bb = bc[i];
            a[4 * i + 0] = __uint_as_float(v[h][4 * i + 0]) + bb.x;
            a[4 * i + 1] = __uint_as_float(v[h][4 * i + 1]) + bb.y;
            a[4 * i + 2] = __uint_as_float(v[h][4 * i + 2]) + bb.z;
            a[4 * i + 3] = __uint_as_float(v[h][4 * i + 3]) + bb.w;
          }
          act_n<16>(act, a);
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = pack_bf16x2(a[2 * i], a[2 * i + 1]);
          tmem_st_32x32b_x8(tbase + (uint32_t)(h * 64), w);
          tmem_st_wait();
          tc_fence_before();
          pair_warp_arrive_remote(h_full_c[2 * b + h], lane);
        }
      }
      if (!ok) break;

      // Output: acc2 + b2 -> bf16 rows of Y (this CTA's rows of the tile).
      if (!mbar_wait_cluster(a2_full, (uint32_t)(it & 1), status, 0x30e, abort_flag)) break;
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
      pair_warp_arrive_remote(a2_empty_c, lane);
      if (r < my_rows) {
        const float* bo = b2s + sub * kOutCols;
        uint4* dst = reinterpret_cast<uint4*>(Y + ((int64_t)my_row0 + r) * kPD + sub * kOutCols);
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

  // Neither CTA leaves (or frees the pair's TMEM) while the other may still
  // signal its barriers or read its tensor memory.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

}  // namespace

// The pair kernel for d_model 256 (the host checks the shape).
int launch_fused_pair(const void* Xp, const void* W1, const float* b1, const void* W2,
                      const float* b2, const int32_t* offs, int G, int Gw, int64_t rows_total,
                      int F, int act, void* Y, int32_t* status, cudaStream_t s) {
  CUtensorMap tmX, tmW1, tmW2;
  if (!make_tmap_bf16_2d(&tmX, Xp, (uint64_t)rows_total, kPD, kPD, kPBM, kPBK) ||
      !make_tmap_bf16_2d(&tmW1, W1, (uint64_t)Gw * F, kPD, kPD, kPFC / 2, kPBK) ||
      !make_tmap_bf16_2d(&tmW2, W2, (uint64_t)Gw * kPD, (uint64_t)F, (uint64_t)F, kPD / 2, kPBK))
    return CTI_ERR_INVALID_ARG;
  static uint64_t configured = 0;
  if (ensure_smem_limit(fused_ffn_pair_kernel, (int)kPSmem, configured) != cudaSuccess)
    return CTI_ERR_CUDA;
  const int sms = device_sm_count();
  if (sms < 2) return CTI_ERR_CUDA;
  const int64_t max_tiles = (rows_total + 2 * kPBM - 1) / (2 * kPBM) + G;
  const int64_t pairs = max_tiles < sms / 2 ? max_tiles : sms / 2;
  return launch_dependent(fused_ffn_pair_kernel, dim3((unsigned)(2 * pairs)), dim3(kPThreads),
                          kPSmem, s, tmX, tmW1, tmW2, offs, G, Gw, rows_total, F, b1, b2, act,
                          static_cast<__nv_bfloat16*>(Y), status) == cudaSuccess
             ? CTI_OK
             : CTI_ERR_CUDA;
}

}  // namespace cti

extern "C" int cti_moe_expert_ffn_fused_pair(const void* Xp_bf16, const void* W1_bf16,
                                             const float* b1, const void* W2_bf16,
                                             const float* b2, const int32_t* group_offsets, int G,
                                             int Gw, int64_t rows_total, int D, int F, int act,
                                             void* Y_bf16, int32_t* status, void* stream) {
  using namespace cti;
  if (G < 1 || Gw < 1 || rows_total < 0 || F <= 0) return CTI_ERR_INVALID_ARG;
  if (act < CTI_ACT_NONE || act > CTI_ACT_GELU) return CTI_ERR_INVALID_ARG;
  if (D != kPD || F % kPFC != 0 || F > kPMaxF || G > PSched::kMaxGroups)
    return CTI_ERR_UNSUPPORTED;
  if (rows_total >= ((int64_t)1 << 31) - 512) return CTI_ERR_UNSUPPORTED;
  if (!W1_bf16 || !W2_bf16 || !b1 || !b2 || !group_offsets || !Y_bf16) return CTI_ERR_INVALID_ARG;
  if (rows_total == 0) return CTI_OK;
  if (!Xp_bf16) return CTI_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(Y_bf16) & 15) || (reinterpret_cast<uintptr_t>(b1) & 15) ||
      (reinterpret_cast<uintptr_t>(b2) & 15))
    return CTI_ERR_INVALID_ARG;
  return launch_fused_pair(Xp_bf16, W1_bf16, b1, W2_bf16, b2, group_offsets, G, Gw, rows_total, F,
                           act, Y_bf16, status, static_cast<cudaStream_t>(stream));
}
