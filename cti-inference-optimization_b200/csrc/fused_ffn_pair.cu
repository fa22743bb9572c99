// Stage 3, fused, on CTA pairs: the expert FFN of a 256-row tile on two SMs,
//
//   Y[rows] = act(Xp[rows] @ W1[e]^T + b1[e]) @ W2[e]^T + b2[e],
//
// issued as one tcgen05.mma.cta_group::2 stream for both SMs of a
// thread-block cluster of two.  Every MMA is M = 256 (128 rows per SM) x
// N = 256 x K = 16: each instruction gives each SM 128 cycles of tensor work.
//
// Per tile, d_ff is processed in 256-wide chunks c:
//   GEMM1(c): acc1 (TMEM, 256 fp32 columns) = X[256, D] @ W1[e][c*256:+256, :]^T
//   epilogue: acc1 -> registers (acc1 is free again at once) -> +b1 -> GELU
//             -> bf16 H(c) in shared memory, one 64-wide K slab at a time
//   GEMM2(c): acc2 (TMEM, D = 256 columns) += H(c) @ W2[e][:, c*256:+256]^T,
//             slab by slab as the epilogue finishes each
// The MMA thread issues GEMM1(c+1) as soon as the epilogue has drained
// acc1, then GEMM2(c): the tensor core runs GEMM1(c+1) while the epilogue
// turns chunk c into H(c).  After the last chunk, acc2 + b2 goes to Y.
//
// The pair: each CTA holds its own 128 rows (X and H in its shared memory,
// acc1 / acc2 in its TMEM) and HALF of every weight K-slab ([128 x 64]: the
// W1 rows [c*256 + 128r, +128) or the W2 output rows [128r, +128) of the
// chunk, r = its rank), so each SM streams half the weight bytes per FLOP of
// a one-SM tile.  W1 and W2 slabs stream through two rings of their own
// (4 and 2 slabs), each filled by a producer warp: GEMM2's slabs wait in
// their ring until the epilogue has written the matching H slab, and with
// one ring for both they held the slots GEMM1(c+1)'s slabs needed.  The
// even CTA (leader) issues every MMA; the barriers it waits on live in its
// shared memory - the peer's TMA loads complete on them (.cta_group::2), and
// the peer's epilogue arrivals reach them through one forwarding thread of
// the peer (a cluster-scope arrival per completed phase, warp 1 lane 0); MMA
// completions that both CTAs wait for are committed twice, once to each
// CTA's copy of the barrier.
//
// Roles per CTA (608 threads): warp 0 TMA producer of X and W1, warp 1 TMEM
// allocation for the pair and the MMA issuer (leader) or the forwarding
// thread (peer), warp 2 TMA producer of
// W2, warps 3-18 epilogue.  Epilogue warp (lane quadrant q, group s) owns
// rows 32q..32q+31 and, of every 64-wide K slab, columns [16s, 16s + 16).
// Biases are read through the read-only cache, one slab ahead.  The output
// rows go out transposed inside groups of four lanes, so that each 32-byte
// store of a warp writes four whole 128-byte row segments.
// TMEM per CTA: acc2 columns [0, 256), acc1 [256, 512).
// Shared memory per CTA: barriers and scheduler first, then (1024-aligned)
// X 64 KB + H 64 KB + W1 ring 64 KB + W2 ring 32 KB.  d_model 256; d_ff a
// multiple of 256 up to 1024.
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
constexpr int kPFC = 256;              // d_ff chunk
constexpr int kPBK = 64;               // bf16 per 128-byte swizzled row
constexpr int kPSlabs = kPD / kPBK;    // 4 K slabs of X, of a W1 chunk, of a W2 chunk, of H
constexpr int kPEpiWarps = 16;
constexpr int kPEpi0 = 3;              // first epilogue warp
constexpr int kPThreads = 32 * kPEpi0 + kPEpiWarps * 32;
constexpr int kPMaxF = 1024;
constexpr int kW1Ring = 4;             // W1 K slabs in flight
constexpr int kW2Ring = 2;             // W2 K slabs in flight
constexpr uint32_t kPAcc1Col = 256;
using PSched = GroupSchedT<128>;

constexpr size_t kPSlab = (size_t)kPBM * kPBK * 2;            // 16 KB: [128 x 64] bf16
constexpr size_t kPXBytes = kPSlabs * kPSlab;                  // 64 KB
constexpr size_t kPHBytes = kPSlabs * kPSlab;                  // 64 KB
constexpr size_t kPW1Bytes = kW1Ring * kPSlab;                 // 64 KB
constexpr size_t kPW2Bytes = kW2Ring * kPSlab;                 // 32 KB
constexpr size_t kPBarBytes = 512;
constexpr size_t kPSmall = kPBarBytes + PSched::smem_bytes();  // ahead of the aligned part
constexpr size_t kPSmem = kPSmall + 1023 + kPXBytes + kPHBytes + kPW1Bytes + kPW2Bytes;
static_assert(kPSmem <= 232448, "shared memory per CTA");

CTI_DEVICE void pair_warp_arrive_local(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// Commits the completion of every pair MMA issued so far to the barrier at
// the same offset in both CTAs.
CTI_DEVICE void commit_both(uint64_t* bar) {
  umma_commit_pair(mapa_shared(bar, 0));
  umma_commit_pair(mapa_shared(bar, 1));
}

// 16-byte store into a 128-byte-swizzled K-major slab: row r, chunk j.
CTI_DEVICE void st_swizzled16(uint8_t* slab, int r, int j, uint4 v) {
  *reinterpret_cast<uint4*>(slab + r * 128 + ((j ^ (r & 7)) << 4)) = v;
}

// This thread's 16 b1 values of one K slab.
CTI_DEVICE void load_bias16(float4 (&b)[4], const float* p) {
#pragma unroll
  for (int i = 0; i < 4; ++i) b[i] = __ldg(reinterpret_cast<const float4*>(p) + i);
}

// One weight K slab of this CTA's half into ring slot n % slots, once the
// MMAs reading the slot's previous contents have completed.  The leader's
// full barrier counts the bytes of both CTAs.
CTI_DEVICE bool load_pair_slab(uint8_t* ring, uint64_t* full, uint64_t* empty,
                               const uint32_t* full_c, int slots, int& n, const CUtensorMap* map,
                               int k0, int row0, bool leader, int32_t* status, int where,
                               volatile int* abort_flag) {
  const int slot = n % slots;
  if (!mbar_wait_cluster(&empty[slot], (uint32_t)((n / slots) & 1) ^ 1u, status, where,
                         abort_flag))
    return false;
  if (leader) mbar_arrive_expect_tx(&full[slot], (uint32_t)(2 * kPSlab));
  tma_load_2d_pair(ring + slot * kPSlab, map, full_c[slot], k0, row0);
  ++n;
  return true;
}

// The leader waits for the last armed phase of each slot of a ring (both
// CTAs' bytes), so that no load of either CTA is still in flight.
CTI_DEVICE void drain_ring(uint64_t* full, int slots, int n, int32_t* status, int where) {
  for (int i = 1; i <= slots; ++i)
    if (n - i >= 0)
      mbar_wait_cluster(&full[(n - i) % slots], (uint32_t)(((n - i) / slots) & 1), status, where,
                        nullptr);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    fused_ffn_pair_kernel(const __grid_constant__ CUtensorMap tmX,
                          const __grid_constant__ CUtensorMap tmW1,
                          const __grid_constant__ CUtensorMap tmW2,
                          const int32_t* __restrict__ group_offsets, int G, int Gw,
                          int64_t rows_total, int F, const float* __restrict__ b1,
                          const float* __restrict__ b2, int act,
                          __nv_bfloat16* __restrict__ Y, int32_t* status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint8_t* sched_mem = smem_raw + kPBarBytes;
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw + kPSmall) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sx = smem;
  uint8_t* sh = sx + kPXBytes;          // H(c): 4 K slabs [128 x 64]
  uint8_t* ring1 = sh + kPHBytes;       // W1 K slabs
  uint8_t* ring2 = ring1 + kPW1Bytes;   // W2 K slabs
  // Waited on by the leader's MMA thread (arrivals and bytes from both CTAs):
  uint64_t* full1 = bars;                 // [kW1Ring] W1 slab of both CTAs landed
  uint64_t* full2 = full1 + kW1Ring;      // [kW2Ring] W2 slab of both CTAs landed
  uint64_t* x_full = full2 + kW2Ring;     // X rows of both CTAs landed
  uint64_t* acc1_free = x_full + 1;       // both epilogues have drained acc1
  uint64_t* h_full = acc1_free + 1;       // [4] H slab written by both epilogues
  uint64_t* a2_empty = h_full + kPSlabs;  // both epilogues have read acc2
  uint64_t* drain = a2_empty + 1;
  // The peer's epilogue arrives on these local copies; its forwarding thread
  // passes each completed phase on to the leader with one cluster arrival.
  uint64_t* acc1_fwd = drain + 1;
  uint64_t* h_fwd = acc1_fwd + 1;         // [4]
  uint64_t* a2_fwd = h_fwd + kPSlabs;
  // Waited on in each CTA (committed by the leader to both copies):
  uint64_t* empty1 = a2_fwd + 1;          // [kW1Ring] W1 slot may be refilled
  uint64_t* empty2 = empty1 + kW1Ring;    // [kW2Ring] W2 slot may be refilled
  uint64_t* x_empty = empty2 + kW2Ring;
  uint64_t* a1_full = x_empty + 1;        // GEMM1(c) done
  uint64_t* h_empty = a1_full + 1;        // [4] GEMM2 has read H slab kb
  uint64_t* a2_full = h_empty + kPSlabs;  // GEMM2 of the tile's last chunk done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a2_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_cta_rank();
  const bool leader = rank == 0;
  const int nch = F / kPFC;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kW1Ring; ++s) {
      mbar_init(&full1[s], 1);
      mbar_init(&empty1[s], 1);
    }
    for (int s = 0; s < kW2Ring; ++s) {
      mbar_init(&full2[s], 1);
      mbar_init(&empty2[s], 1);
    }
    mbar_init(x_full, 1);
    mbar_init(x_empty, 1);
    // Leader: its own epilogue warps plus the peer's forwarding thread.
    mbar_init(acc1_free, kPEpiWarps + 1);
    mbar_init(acc1_fwd, kPEpiWarps);
    for (int i = 0; i < kPSlabs; ++i) {
      mbar_init(&h_full[i], kPEpiWarps + 1);
      mbar_init(&h_fwd[i], kPEpiWarps);
      mbar_init(&h_empty[i], 1);
    }
    mbar_init(a2_empty, kPEpiWarps + 1);
    mbar_init(a2_fwd, kPEpiWarps);
    mbar_init(drain, 1);
    mbar_init(a1_full, 1);
    mbar_init(a2_full, 1);
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
    // ------------------------------------------------------ X / W1 producer
    if (lane == 0) {
      uint32_t full_c[kW1Ring];
      for (int s = 0; s < kW1Ring; ++s) full_c[s] = mapa_shared(&full1[s], 0);
      const uint32_t x_full_c = mapa_shared(x_full, 0);
      int n = 0, x_issued = 0;  // W1 slabs issued, X tiles issued
      int it = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs, ++it) {
        const TileCoord tc = sched.decode(t);
        const int gw = tc.g % Gw;
        const int my_row0 = tc.row0 + (int)rank * kPBM;
        if (!mbar_wait_cluster(x_empty, (uint32_t)(it & 1) ^ 1u, status, 0x402, abort_flag)) break;
        if (leader) mbar_arrive_expect_tx(x_full, (uint32_t)(2 * kPXBytes));
        for (int kb = 0; kb < kPSlabs; ++kb)
          tma_load_2d_pair(sx + kb * kPSlab, &tmX, x_full_c, kb * kPBK, my_row0);
        ++x_issued;
        if (t + npairs < total) {  // the next tile's rows into L2
          const TileCoord nx = sched.decode(t + npairs);
          for (int kb = 0; kb < kPSlabs; ++kb)
            tma_prefetch_l2_2d(&tmX, kb * kPBK, nx.row0 + (int)rank * kPBM);
        }
        for (int c = 0; c < nch && ok; ++c)
          for (int kb = 0; kb < kPSlabs && ok; ++kb)
            ok = load_pair_slab(ring1, full1, empty1, full_c, kW1Ring, n, &tmW1, kb * kPBK,
                                gw * F + c * kPFC + (int)rank * kPBM, leader, status, 0x401,
                                abort_flag);
      }
      if (leader) {
        drain_ring(full1, kW1Ring, n, status, 0x403);
        if (x_issued > 0)
          mbar_wait_cluster(x_full, (uint32_t)((x_issued - 1) & 1), status, 0x403, nullptr);
      }
    }
  } else if (warp == 2) {
    // ----------------------------------------------------------- W2 producer
    if (lane == 0) {
      uint32_t full_c[kW2Ring];
      for (int s = 0; s < kW2Ring; ++s) full_c[s] = mapa_shared(&full2[s], 0);
      int n = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs) {
        const int gw = sched.decode(t).g % Gw;
        for (int c = 0; c < nch && ok; ++c)
          for (int kb = 0; kb < kPSlabs && ok; ++kb)
            ok = load_pair_slab(ring2, full2, empty2, full_c, kW2Ring, n, &tmW2,
                                c * kPFC + kb * kPBK, gw * kPD + (int)rank * kPBM, leader, status,
                                0x411, abort_flag);
      }
      if (leader) drain_ring(full2, kW2Ring, n, status, 0x412);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(2 * kPBM, 256);  // M 256, N 256 (both GEMMs)
      int n1 = 0, n2 = 0;  // W1 / W2 slabs consumed
      int gc = 0;          // GEMM1s issued (global chunk counter)
      int it = 0;
      bool any = false, ok = true;
      const uint32_t x_addr = smem_u32(sx);
      const uint32_t h_addr = smem_u32(sh);
      const uint32_t ring1_addr = smem_u32(ring1);
      const uint32_t ring2_addr = smem_u32(ring2);
      const uint32_t acc1 = tmem_base + kPAcc1Col;
      for (int t = pair; t < total && ok; t += npairs, ++it) {
        if (!mbar_wait_cluster(x_full, (uint32_t)(it & 1), status, 0x404, abort_flag)) break;
        tc_fence_after();
        for (int c = 0; c <= nch && ok; ++c) {
          if (c < nch) {  // GEMM1(c) into acc1, once both epilogues have drained it
            if (gc > 0 && !mbar_wait_cluster(acc1_free, (uint32_t)((gc - 1) & 1), status, 0x406,
                                             abort_flag)) {
              ok = false;
              break;
            }
            for (int kb = 0; kb < kPSlabs; ++kb) {
              const int slot = n1 % kW1Ring;
              if (!mbar_wait_cluster(&full1[slot], (uint32_t)((n1 / kW1Ring) & 1), status, 0x405,
                                     abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t b0 = ring1_addr + (uint32_t)(slot * kPSlab);
#pragma unroll
              for (int kk = 0; kk < kPBK / 16; ++kk)
                umma_bf16_pair(acc1, smem_desc_sw128(x_addr + kb * kPSlab + kk * 32),
                               smem_desc_sw128(b0 + kk * 32), idesc, (kb | kk) != 0 ? 1u : 0u);
              commit_both(&empty1[slot]);
              ++n1;
            }
            if (!ok) break;
            commit_both(a1_full);
            if (c == nch - 1) commit_both(x_empty);
            ++gc;
            any = true;
          }
          if (c >= 1) {  // GEMM2(c-1): acc2 += H(c-1) @ W2 chunk, slab by slab
            const int cc = c - 1;
            const uint32_t hph = (uint32_t)((it * nch + cc) & 1);  // H of global chunk it*nch+cc
            if (cc == 0 &&
                !mbar_wait_cluster(a2_empty, (uint32_t)(it & 1) ^ 1u, status, 0x407, abort_flag)) {
              ok = false;
              break;
            }
            for (int kb = 0; kb < kPSlabs; ++kb) {
              const int slot = n2 % kW2Ring;
              if (!mbar_wait_cluster(&full2[slot], (uint32_t)((n2 / kW2Ring) & 1), status, 0x413,
                                     abort_flag) ||
                  !mbar_wait_cluster(&h_full[kb], hph, status, 0x408, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t b0 = ring2_addr + (uint32_t)(slot * kPSlab);
#pragma unroll
              for (int kk = 0; kk < kPBK / 16; ++kk)
                umma_bf16_pair(tmem_base, smem_desc_sw128(h_addr + kb * kPSlab + kk * 32),
                               smem_desc_sw128(b0 + kk * 32), idesc,
                               (cc | kb | kk) != 0 ? 1u : 0u);
              commit_both(&empty2[slot]);
              ++n2;
              commit_both(&h_empty[kb]);
            }
            if (!ok) break;
            if (cc == nch - 1) commit_both(a2_full);
          }
        }
      }
      if (any) {
        umma_commit_pair(mapa_shared(drain, 0));
        mbar_wait_cluster(drain, 0, status, 0x409, nullptr);
      }
    } else if (!leader && lane == 0) {
      // ---------------------------------------------- peer: forwarding thread
      // A cluster-scope release arrival costs its thread ~1.7 K cycles; one
      // thread pays it per event instead of each epilogue warp.
      const uint32_t acc1_free_c = mapa_shared(acc1_free, 0);
      const uint32_t a2_empty_c = mapa_shared(a2_empty, 0);
      uint32_t h_full_c[kPSlabs];
      for (int i = 0; i < kPSlabs; ++i) h_full_c[i] = mapa_shared(&h_full[i], 0);
      int gc = 0;
      bool ok = true;
      for (int t = pair, it = 0; t < total && ok; t += npairs, ++it) {
        for (int c = 0; c < nch && ok; ++c, ++gc) {
          if (!mbar_wait(acc1_fwd, (uint32_t)(gc & 1), status, 0x414, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_cluster(acc1_free_c);
          for (int kb = 0; kb < kPSlabs; ++kb) {
            if (!mbar_wait(&h_fwd[kb], (uint32_t)(gc & 1), status, 0x415, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_cluster(h_full_c[kb]);
          }
        }
        if (!ok || !mbar_wait(a2_fwd, (uint32_t)(it & 1), status, 0x416, abort_flag)) break;
        mbar_arrive_cluster(a2_empty_c);
      }
    }
  } else if (warp >= kPEpi0) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - kPEpi0;
    const int q = warp & 3;            // TMEM lane quadrant
    const int sub = ew >> 2;           // columns [16 sub, +16) of every K slab
    const int r = q * 32 + lane;       // row of this CTA's 128
    constexpr int kOutCols = kPD / 4;
    // The leader's warps arrive on its barriers directly; the peer's on local
    // copies that its forwarding thread passes on.
    uint64_t* acc1_sig = leader ? acc1_free : acc1_fwd;
    uint64_t* h_sig = leader ? h_full : h_fwd;
    uint64_t* a2_sig = leader ? a2_empty : a2_fwd;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
    const bool y32 = (reinterpret_cast<uintptr_t>(Y) & 31) == 0;
    int it = 0, gc = 0;
    bool ok = true;
    for (int t = pair; t < total && ok; t += npairs, ++it) {
      const TileCoord tc = sched.decode(t);
      const int gw = tc.g % Gw;
      const int my_row0 = tc.row0 + (int)rank * kPBM;
      const int my_rows = tc.rows - (int)rank * kPBM;  // may be <= 0 in the last tile
      const float* b1e = b1 + (int64_t)gw * F + sub * 16;
      for (int c = 0; c < nch; ++c, ++gc) {
        float4 bias[4];
        load_bias16(bias, b1e + c * kPFC);  // slab 0's, ahead of the accumulator wait
        if (!mbar_wait_cluster(a1_full, (uint32_t)(gc & 1), status, 0x40c, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // Drain this thread's 64 columns of acc1, then hand acc1 back.
        uint32_t v[kPSlabs][16];
#pragma unroll
        for (int kb = 0; kb < kPSlabs; ++kb)
          tmem_ld_32x32b_x16(lane_base + kPAcc1Col + (uint32_t)(kb * kPBK + sub * 16), v[kb]);
        tmem_ld_wait();
        tc_fence_before();
        pair_warp_arrive_local(acc1_sig, lane);
#pragma unroll
        for (int kb = 0; kb < kPSlabs; ++kb) {
          float a[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {  // + b1, two values per packed add
            const float4 bb = bias[i];
            f2_unpack(f2_add(f2_pack(__uint_as_float(v[kb][4 * i + 0]),
                                     __uint_as_float(v[kb][4 * i + 1])),
                             f2_pack(bb.x, bb.y)),
                      a[4 * i + 0], a[4 * i + 1]);
            f2_unpack(f2_add(f2_pack(__uint_as_float(v[kb][4 * i + 2]),
                                     __uint_as_float(v[kb][4 * i + 3])),
                             f2_pack(bb.z, bb.w)),
                      a[4 * i + 2], a[4 * i + 3]);
          }
          if (kb + 1 < kPSlabs) load_bias16(bias, b1e + c * kPFC + (kb + 1) * kPBK);
          act_n<16>(act, a);
          uint4 w0, w1;
          w0.x = pack_bf16x2(a[0], a[1]);
          w0.y = pack_bf16x2(a[2], a[3]);
          w0.z = pack_bf16x2(a[4], a[5]);
          w0.w = pack_bf16x2(a[6], a[7]);
          w1.x = pack_bf16x2(a[8], a[9]);
          w1.y = pack_bf16x2(a[10], a[11]);
          w1.z = pack_bf16x2(a[12], a[13]);
          w1.w = pack_bf16x2(a[14], a[15]);
          // GEMM2 of the previous chunk must be done with slab kb of H.
          if (gc > 0 &&
              !mbar_wait_cluster(&h_empty[kb], (uint32_t)((gc - 1) & 1), status, 0x40d,
                                 abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* slab = sh + kb * kPSlab;
          st_swizzled16(slab, r, 2 * sub, w0);
          st_swizzled16(slab, r, 2 * sub + 1, w1);
          fence_proxy_async_smem();  // visible to the tensor core's operand reads
          pair_warp_arrive_local(&h_sig[kb], lane);
        }
        if (!ok) break;
      }
      if (!ok) break;

      // Output: acc2 + b2 -> bf16 rows of Y (this CTA's rows of the tile).
      // A thread holds kOutCols columns of its row, four units of 16 columns
      // (32 bytes); a transpose of units inside each group of four lanes
      // (two butterfly steps of shuffles) leaves lane i, in slot k, unit
      // i % 4 of row i - i % 4 + k, so four lanes store one row segment.
      const float4* bo4 = reinterpret_cast<const float4*>(b2 + (int64_t)gw * kPD + sub * kOutCols);
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(a2_full, (uint32_t)(it & 1), status, 0x40e,
                                                     abort_flag)))
        break;
      tc_fence_after();
      uint32_t o[kOutCols];
      const uint32_t taddr2 = lane_base + (uint32_t)sub * kOutCols;
#pragma unroll
      for (int j = 0; j < kOutCols / 32; ++j) {
        uint32_t tmp[32];
        tmem_ld_32x32b_x32(taddr2 + 32 * j, tmp);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[32 * j + i] = tmp[i];
      }
      tmem_ld_wait();
      tc_fence_before();
      pair_warp_arrive_local(a2_sig, lane);
      constexpr int kU = kOutCols / 16;
      uint32_t u[kU][8];  // unit j, word w: columns 16j + 2w, 16j + 2w + 1
#pragma unroll
      for (int j = 0; j < kU; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 cb = __ldg(bo4 + 4 * j + i);
          u[j][2 * i] = pack_bf16x2(__uint_as_float(o[16 * j + 4 * i]) + cb.x,
                                    __uint_as_float(o[16 * j + 4 * i + 1]) + cb.y);
          u[j][2 * i + 1] = pack_bf16x2(__uint_as_float(o[16 * j + 4 * i + 2]) + cb.z,
                                        __uint_as_float(o[16 * j + 4 * i + 3]) + cb.w);
        }
#pragma unroll
      for (int m = 1; m < kU; m <<= 1) {
        // Lanes i and i ^ m swap the units whose bit m differs from theirs.
        const bool hi = (lane & m) != 0;
#pragma unroll
        for (int j = 0; j < kU; ++j) {
          if (j & m) continue;
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            const uint32_t got = __shfl_xor_sync(0xffffffffu, hi ? u[j][w] : u[j ^ m][w], m);
            if (hi)
              u[j][w] = got;
            else
              u[j ^ m][w] = got;
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kU; ++k) {
        const int rr = q * 32 + (lane & ~(kU - 1)) + k;
        if (rr < my_rows)
          st_global_32B(Y + ((int64_t)my_row0 + rr) * kPD + sub * kOutCols + 16 * (lane & (kU - 1)),
                        u[k], y32);
      }
    }
  }

  // Neither CTA leaves (or frees the pair's TMEM) while the other may still
  // signal its barriers or read its shared or tensor memory.
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

// The pair kernel (the host checks the shape: d_model 256, d_ff % 256 == 0).
int launch_fused_pair(const void* Xp, const void* W1, const float* b1, const void* W2,
                      const float* b2, const int32_t* offs, int G, int Gw, int64_t rows_total,
                      int F, int act, void* Y, int32_t* status, cudaStream_t s) {
  CUtensorMap tmX, tmW1, tmW2;
  if (!make_tmap_bf16_2d(&tmX, Xp, (uint64_t)rows_total, kPD, kPD, kPBM, kPBK) ||
      !make_tmap_bf16_2d(&tmW1, W1, (uint64_t)Gw * F, kPD, kPD, kPBM, kPBK) ||
      !make_tmap_bf16_2d(&tmW2, W2, (uint64_t)Gw * kPD, (uint64_t)F, (uint64_t)F, kPBM, kPBK))
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
