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
//   GEMM1(c): acc1[c%2] (TMEM, 128 fp32 cols) = X[128, D] @ W1[e][c*128:+128, :]^T
//   epilogue: acc1 -> +b1 -> GELU -> bf16 -> H(c), written back into the
//             same TMEM columns (two bf16 per 32-bit column)
//   GEMM2(c): acc2 (TMEM, D cols) += H(c) @ W2[e][:, c*128:+128]^T, with the
//             A operand read from tensor memory
// GEMM1s and GEMM2s are issued by two threads of their own.  GEMM1(c+2)
// overwrites acc1[c%2], so its thread waits until GEMM2(c) - which read H(c)
// there - has completed (acc1_free[c%2], committed by the GEMM2 thread), and
// the hidden tile never touches shared memory.  While the epilogue turns
// chunk c into H(c), the tensor core runs GEMM1(c+1) and GEMM2(c-1); each
// issuer's barrier waits overlap the other's MMAs (one thread issuing both
// left the tensor core idle during every wait: the issue queue holds only a
// few MMAs).  After the last chunk, acc2 + b2 is written to Y as bf16.
//
// Roles (640 threads; 672 with the row gather below): warp 0 TMA producer of
// the X tile (once per tile, unless warp 20 gathers it) and of W1 in
// half-chunk slots ([128 x D/2], a 3-slot ring), warp 1 TMEM owner and GEMM1
// issuer (tcgen05.mma M=128, N=128, K=16, bf16 -> fp32), warps 2-17 epilogue
// (four warps per TMEM lane quadrant, each owning 32 of a chunk's 128 columns
// and a quarter of the output columns; biases read through the read-only
// cache, the next chunk's prefetched before the accumulator wait), warp 18
// GEMM2 issuer (N=D, A from TMEM), warp 19 TMA producer of W2 in half-chunk
// slots ([D x 64], a 2-slot ring).
//
// TMEM: acc2 in columns [0, D), acc1 buffers at 256 and 384 (512 allocated).
// The epilogue produces H(c) in two halves (chunk columns [0, 64) and
// [64, 128)), each with its own barrier, so GEMM2(c) starts on the first half
// while the GELU of the second is still running.  Epilogue warp group s owns
// fp32 columns [64h + 16s, +16) of each half h and writes their 16 bf16
// values to the first 8 of those columns, so the 16-wide K step k of GEMM2
// reads 8 contiguous columns at 64*(k/4) + 16*(k%4).
// Shared memory: X tile (D/64 slabs of 16 KB) + three W1 and two W2
// half-chunk slots (32 KB each at D=256) + scheduler 2 KB.
// d_ff <= 1024 (one expert's b1 in shared memory).
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
constexpr int kEpiWarps = 16;
constexpr int kMaxF = 1024;
// 128 groups (the library's expert limit) keeps the scheduler's table small
// enough for the weight rings below.
using Sched = GroupSchedT<128>;
constexpr int kEpiThreads = kEpiWarps * 32;
// warps: 0 W1 / X producer, 1 GEMM1 issuer + TMEM owner, 2-17 epilogue,
// 18 GEMM2 issuer, 19 W2 producer (20 row gather in the gather variant)
constexpr int kIssue2Warp = 2 + kEpiWarps;
constexpr int kProd2Warp = 3 + kEpiWarps;
constexpr int kGatherWarp = 4 + kEpiWarps;
constexpr int kThreads = 128 + kEpiThreads;
constexpr uint32_t kAcc1Col = 256;
constexpr int kW1Slots = 3;        // W1 half-chunk slots
constexpr int kW2Slots = 2;        // W2 half-chunk slots

// Weights stream through two rings of half-chunk slots, filled by a
// producer warp each: W1 halves ([128 x D/2], the first or second half of a
// chunk's K) and W2 halves ([D x 64]).  A chunk's weights can be reloaded
// only after the MMAs reading the previous contents of their slot have
// completed, and a reload from L2 takes 1.5-2.3 K cycles; with three W1 and
// two W2 half slots a reload has 1.5-2 K cycles of other MMAs to hide
// behind (with one whole-chunk slot per ring it had 1 K and set the pace).
template <int D>
struct FF {
  static constexpr int XK = D / kBK;                     // X k-slabs
  static constexpr int W1HS = XK / 2;                    // W1 k-slabs [128 x 64] per half
  static constexpr size_t W1H = (size_t)W1HS * kSlab;    // bytes of a W1 half
  static constexpr size_t W2H = (size_t)D * kBK * 2;     // bytes of a W2 half [D x 64]
  static constexpr size_t X_BYTES = (size_t)XK * kSlab;
  static constexpr size_t RING_BYTES = kW1Slots * W1H + kW2Slots * W2H;
  static constexpr size_t SMEM = 1024 + X_BYTES + RING_BYTES + Sched::smem_bytes() + 512;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

// One arrival per warp: the lanes' prior writes are ordered before lane 0's
// (release) arrive by the warp barrier.  Barriers signalled this way count
// warps, not threads.
CTI_DEVICE void warp_arrive(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// Row gather (GATHER = true): instead of TMA loads of the dispatched copy
// Xp, an extra warp copies each tile's 128 rows straight from the token rows
// x[sorted_token[row]] with 16-byte cp.async into the same 128-byte-swizzled
// slabs the TMA would fill (row r of a slab at r*128 B, 16-byte chunk c at
// chunk c ^ (r % 8)); rows at or past rows_total are zero-filled.  It waits
// for its own copies, fences them into the async proxy the tensor core reads
// through, and arrives on x_full.  The dispatch then writes only the
// permutation, not the 2*T*D permuted rows.
CTI_DEVICE void gather_cp16(uint8_t* smem_dst, const void* gmem_src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src), "r"(src_bytes)
               : "memory");
}

CTI_DEVICE void gather_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// L2 prefetch of one contiguous row (bytes a multiple of 16, 16-byte aligned).
CTI_DEVICE void prefetch_row_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// A ring position: slot and the parity of its current use.
struct RingPos {
  int slot = 0;
  uint32_t phase = 0;
  CTI_DEVICE void next(int slots) {
    if (++slot == slots) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

template <int D, bool GATHER>
__global__ void __launch_bounds__(GATHER ? kThreads + 32 : kThreads, 1)
    fused_ffn_kernel(const __grid_constant__ CUtensorMap tmX,
                     const __grid_constant__ CUtensorMap tmW1,
                     const __grid_constant__ CUtensorMap tmW2,
                     const int32_t* __restrict__ group_offsets, int G, int Gw, int64_t rows_total,
                     int F, const float* __restrict__ b1, const float* __restrict__ b2, int act,
                     __nv_bfloat16* __restrict__ Y, int32_t* status,
                     const __nv_bfloat16* __restrict__ x_rows,
                     const int32_t* __restrict__ sorted_token, int64_t n_tokens) {
  using P = FF<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sx = smem;
  uint8_t* ring1 = sx + P::X_BYTES;                   // W1 half slots
  uint8_t* ring2 = ring1 + kW1Slots * P::W1H;         // W2 half slots
  uint8_t* sched_mem = ring2 + kW2Slots * P::W2H;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sched_mem + Sched::smem_bytes());
  uint64_t* full1 = bars;                  // [kW1Slots]
  uint64_t* empty1 = full1 + kW1Slots;     // [kW1Slots]
  uint64_t* full2 = empty1 + kW1Slots;     // [kW2Slots]
  uint64_t* empty2 = full2 + kW2Slots;     // [kW2Slots]
  uint64_t* x_full = empty2 + kW2Slots;
  uint64_t* x_empty = x_full + 1;
  uint64_t* a1_full = x_empty + 1;   // [2] GEMM1(c) done -> epilogue
  uint64_t* h_full = a1_full + 2;    // [2][2] half h of H(c) written -> GEMM2 issuer
  uint64_t* acc1_free = h_full + 4;  // [2] GEMM2 has read H from acc1[b]
  uint64_t* a2_full = acc1_free + 2;
  uint64_t* a2_empty = a2_full + 1;
  uint64_t* drain = a2_empty + 1;    // [2] one per issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int nch = F / kFC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kW1Slots; ++s) {
      mbar_init(&full1[s], 1);
      mbar_init(&empty1[s], 1);
    }
    for (int s = 0; s < kW2Slots; ++s) {
      mbar_init(&full2[s], 1);
      mbar_init(&empty2[s], 1);
    }
    mbar_init(x_full, 1);
    mbar_init(x_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a1_full[i], 1);
      mbar_init(&acc1_free[i], 1);
      mbar_init(&drain[i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&h_full[i], kEpiWarps);
    mbar_init(a2_full, 1);
    mbar_init(a2_empty, kEpiWarps);
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
    // ------------------------------------------------------- W1 / X producer
    if (lane == 0) {
      RingPos w;
      int loads = 0, x_issued = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        const TileCoord tc = sched.decode(t);
        const int gw = tc.g % Gw;
        if (!GATHER) {
          if (!mbar_wait(x_empty, (uint32_t)(it & 1) ^ 1u, status, 0x202, abort_flag)) break;
          mbar_arrive_expect_tx(x_full, (uint32_t)P::X_BYTES);
          for (int kb = 0; kb < P::XK; ++kb)
            tma_load_2d(sx + kb * kSlab, &tmX, x_full, kb * kBK, tc.row0);
          ++x_issued;
          // The next tile's rows come from HBM; pull them into L2 now so that
          // their load at the tile boundary does not stall the tensor core.
          if (t + (int)gridDim.x < total) {
            const TileCoord nx = sched.decode(t + (int)gridDim.x);
            for (int kb = 0; kb < P::XK; ++kb) tma_prefetch_l2_2d(&tmX, kb * kBK, nx.row0);
          }
        }
        for (int c = 0; c < nch && ok; ++c) {
          for (int h = 0; h < 2; ++h) {  // W1 rows [c*128, +128), K slabs of half h
            if (!mbar_wait(&empty1[w.slot], w.phase ^ 1u, status, 0x201, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full1[w.slot], (uint32_t)P::W1H);
            for (int j = 0; j < P::W1HS; ++j)
              tma_load_2d(ring1 + w.slot * P::W1H + j * kSlab, &tmW1, &full1[w.slot],
                          (h * P::W1HS + j) * kBK, gw * F + c * kFC);
            ++loads;
            w.next(kW1Slots);
          }
        }
      }
      // Let every load this thread issued land before the CTA can exit.
      RingPos d = w;
      for (int i = 0; i < kW1Slots && i < loads; ++i) {
        d.slot = (d.slot + kW1Slots - 1) % kW1Slots;
        if (d.slot == kW1Slots - 1) d.phase ^= 1u;
        mbar_wait(&full1[d.slot], d.phase, status, 0x204, nullptr);
      }
      if (x_issued > 0) mbar_wait(x_full, (uint32_t)((x_issued - 1) & 1), status, 0x204, nullptr);
    }
  } else if (warp == kProd2Warp) {
    // ------------------------------------------------------------ W2 producer
    if (lane == 0) {
      RingPos w;
      int loads = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const int gw = sched.decode(t).g % Gw;
        for (int c = 0; c < nch && ok; ++c) {
          for (int h = 0; h < 2; ++h) {  // W2 [D rows, 64 k]: K columns [c*128 + 64h, +64)
            if (!mbar_wait(&empty2[w.slot], w.phase ^ 1u, status, 0x203, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full2[w.slot], (uint32_t)P::W2H);
            tma_load_2d(ring2 + w.slot * P::W2H, &tmW2, &full2[w.slot], c * kFC + h * kBK,
                        gw * D);
            ++loads;
            w.next(kW2Slots);
          }
        }
      }
      RingPos d = w;
      for (int i = 0; i < kW2Slots && i < loads; ++i) {
        d.slot = (d.slot + kW2Slots - 1) % kW2Slots;
        if (d.slot == kW2Slots - 1) d.phase ^= 1u;
        mbar_wait(&full2[d.slot], d.phase, status, 0x204, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ GEMM1 issuer
    if (lane == 0) {
      const uint32_t idesc1 = idesc_bf16_f32(kBM, 128);  // GEMM1: N = d_ff chunk
      RingPos w;
      int it = 0;
      bool any = false, ok = true;
      const uint32_t x_addr = smem_u32(sx);
      const uint32_t ring1_addr = smem_u32(ring1);
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        if (!mbar_wait(x_full, (uint32_t)(it & 1), status, 0x205, abort_flag)) break;
        for (int c = 0; c < nch; ++c) {
          const int gc = it * nch + c;
          const int b = gc & 1;
          // acc1[b] last held H(gc-2): GEMM2(gc-2), issued by the other
          // thread, must have read it.
          if (gc >= 2 && !mbar_wait(&acc1_free[b], (uint32_t)(((gc - 2) >> 1) & 1), status,
                                    0x206, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t d = tmem_base + kAcc1Col + (uint32_t)b * 128u;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!mbar_wait(&full1[w.slot], w.phase, status, 0x207, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t b0 = ring1_addr + (uint32_t)(w.slot * P::W1H);
#pragma unroll
            for (int j = 0; j < P::W1HS; ++j) {
              const uint32_t a0 = x_addr + (h * P::W1HS + j) * kSlab;
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk)
                umma_bf16(d, smem_desc_sw128(a0 + kk * 32),
                          smem_desc_sw128(b0 + j * kSlab + kk * 32), idesc1,
                          (h | j | kk) != 0 ? 1u : 0u);
            }
            umma_commit(&empty1[w.slot]);
            w.next(kW1Slots);
          }
          if (!ok) break;
          any = true;
          umma_commit(&a1_full[b]);
          if (c == nch - 1) umma_commit(x_empty);
        }
      }
      if (any) {
        umma_commit(&drain[0]);
        mbar_wait(&drain[0], 0, status, 0x20b, nullptr);
      }
    }
  } else if (warp == kIssue2Warp) {
    // ------------------------------------------------------------ GEMM2 issuer
    // GEMM2(c), N = D in one instruction, A = H(c) in TMEM.  Issued by its own
    // thread, so that its waits (H from the epilogue, W2 from the producer)
    // overlap the GEMM1s the other thread issues meanwhile.
    if (lane == 0) {
      const uint32_t idesc2 = idesc_bf16_f32(kBM, D);
      RingPos w;
      int it = 0;
      bool any = false, ok = true;
      const uint32_t ring2_addr = smem_u32(ring2);
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        for (int c = 0; c < nch && ok; ++c) {
          const int gc = it * nch + c;
          const int b = gc & 1;
          const uint32_t k = (uint32_t)(gc >> 1);
          if (c == 0 &&
              !mbar_wait(a2_empty, (uint32_t)(it & 1) ^ 1u, status, 0x208, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t h_tmem = tmem_base + kAcc1Col + (uint32_t)b * 128u;
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // K columns [64h, 64h+64) of the chunk
            if (!mbar_wait(&full2[w.slot], w.phase, status, 0x20a, abort_flag) ||
                !mbar_wait(&h_full[2 * b + h], k & 1u, status, 0x209, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t b0 = ring2_addr + (uint32_t)(w.slot * P::W2H);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_bf16_ts(tmem_base, h_tmem + (uint32_t)(h * 64 + kk * 16),
                           smem_desc_sw128(b0 + kk * 32), idesc2, (c | h | kk) != 0 ? 1u : 0u);
            umma_commit(&empty2[w.slot]);
            w.next(kW2Slots);
          }
          if (!ok) break;
          any = true;
          umma_commit(&acc1_free[b]);  // H(gc) read: GEMM1(gc+2) may overwrite acc1[b]
          if (c == nch - 1) umma_commit(a2_full);
        }
      }
      if (any) {
        umma_commit(&drain[1]);
        mbar_wait(&drain[1], 0, status, 0x20b, nullptr);
      }
    }
  } else if (GATHER && warp == kGatherWarp) {
    // ------------------------------------------------------------ row gather
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      bool ok = true;
      if (lane == 0) ok = mbar_wait(x_empty, (uint32_t)(it & 1) ^ 1u, status, 0x211, abort_flag);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      const TileCoord tc = sched.decode(t);
#pragma unroll
      for (int rr = 0; rr < kBM / 32; ++rr) {
        const int r = lane + 32 * rr;
        const int64_t row = (int64_t)tc.row0 + r;
        int64_t tok = -1;
        if (row < rows_total) {
          tok = sorted_token[row];
          if (tok < 0 || tok >= n_tokens) {
            raise_status(status, CTI_ERR_BOUNDS, (int32_t)row);
            tok = -1;
          }
        }
        const uint8_t* src =
            reinterpret_cast<const uint8_t*>(x_rows + (tok >= 0 ? tok : 0) * (int64_t)D);
        const int bytes = tok >= 0 ? 16 : 0;
        uint8_t* dst_row = sx + r * 128;
#pragma unroll
        for (int kb = 0; kb < P::XK; ++kb)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            gather_cp16(dst_row + kb * kSlab + ((c ^ (r & 7)) << 4), src + kb * 128 + c * 16,
                        bytes);
      }
      // The next tile's rows into L2 while this tile's copies land.
      if (t + (int)gridDim.x < total) {
        const TileCoord nx = sched.decode(t + (int)gridDim.x);
#pragma unroll
        for (int rr = 0; rr < kBM / 32; ++rr) {
          const int64_t row = (int64_t)nx.row0 + lane + 32 * rr;
          if (row < rows_total) {
            const int64_t tok = sorted_token[row];
            if (tok >= 0 && tok < n_tokens) prefetch_row_l2(x_rows + tok * D, (uint32_t)(D * 2));
          }
        }
      }
      gather_wait_all();
      fence_proxy_async_smem();
      warp_arrive(x_full, lane);
    }
  } else if (warp >= 2 && warp < 2 + kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    // 16 warps: four per TMEM lane quadrant q; warp group `sub` owns chunk
    // columns [sub*32, sub*32+32) and output columns [sub*D/4, (sub+1)*D/4).
    // Biases come straight from global memory (L1-resident per expert); a
    // chunk's are fetched before its accumulator is waited for.
    const int ew = warp - 2;           // 0..15
    const int q = warp & 3;            // TMEM lane quadrant of this warp
    const int sub = ew >> 2;           // 0..3
    constexpr int kOutCols = D / 4;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
      const TileCoord tc = sched.decode(t);
      const int gw = tc.g % Gw;
      const float* b1e = b1 + (int64_t)gw * F;
      for (int c = 0; c < nch; ++c) {
        const int gc = it * nch + c;
        const int b = gc & 1;
        const uint32_t k = (uint32_t)(gc >> 1);
        float4 bias[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            bias[h][i] = __ldg(reinterpret_cast<const float4*>(b1e + c * kFC + h * 64 + sub * 16) + i);
        if (!mbar_wait(&a1_full[b], k & 1u, status, 0x20c, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + kAcc1Col +
                               (uint32_t)b * 128u + (uint32_t)sub * 16u;
        uint32_t v[2][16];
        tmem_ld_32x32b_x16(tbase, v[0]);        // columns [16s, +16)
        tmem_ld_32x32b_x16(tbase + 64u, v[1]);  // columns [64 + 16s, +16)
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float a[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {  // + b1, two values per packed add
            const float4 bb = bias[h][i];
            f2_unpack(f2_add(f2_pack(__uint_as_float(v[h][4 * i + 0]),
                                     __uint_as_float(v[h][4 * i + 1])),
                             f2_pack(bb.x, bb.y)),
                      a[4 * i + 0], a[4 * i + 1]);
            f2_unpack(f2_add(f2_pack(__uint_as_float(v[h][4 * i + 2]),
                                     __uint_as_float(v[h][4 * i + 3])),
                             f2_pack(bb.z, bb.w)),
                      a[4 * i + 2], a[4 * i + 3]);
          }
          act_n<16>(act, a);
          uint32_t wv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) wv[i] = pack_bf16x2(a[2 * i], a[2 * i + 1]);
          // Half h of H(c): into the first 8 of this thread's 16 columns.
          tmem_st_32x32b_x8(tbase + (uint32_t)(h * 64), wv);
          tmem_st_wait();
          tc_fence_before();
          warp_arrive(&h_full[2 * b + h], lane);
        }
      }
      if (!ok) break;

      // Output: acc2 + b2 -> bf16 rows of Y.  A thread holds kOutCols
      // columns of its row, kU units of 16 columns (32 bytes).  A transpose
      // of units inside each group of kU lanes (log2(kU) butterfly steps of
      // shuffles) leaves lane i, in slot k, unit i % kU of row
      // i - i % kU + k, so that kU lanes store one contiguous row segment
      // together instead of every lane writing to a different row.
      constexpr int kU = kOutCols / 16;  // 4 at D=256, 2 at D=128
      const float4* bo4 = reinterpret_cast<const float4*>(b2 + (int64_t)gw * D + sub * kOutCols);
      if (!__all_sync(0xffffffffu, mbar_wait(a2_full, (uint32_t)(it & 1), status, 0x20e,
                                             abort_flag)))
        break;
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
      const bool y32 = (reinterpret_cast<uintptr_t>(Y) & 31) == 0;
#pragma unroll
      for (int k = 0; k < kU; ++k) {
        const int rr = q * 32 + (lane & ~(kU - 1)) + k;
        if (rr < tc.rows)
          st_global_32B(Y + ((int64_t)tc.row0 + rr) * D + sub * kOutCols + 16 * (lane & (kU - 1)),
                        u[k], y32);
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

// Xp: the dispatched rows (TMA path), or nullptr with x_rows / sorted_token
// (row gather).
template <int D, bool GATHER>
int launch_fused(const void* Xp, const void* W1, const float* b1, const void* W2, const float* b2,
                 const int32_t* offs, int G, int Gw, int64_t rows_total, int F, int act, void* Y,
                 int32_t* status, cudaStream_t s, const void* x_rows = nullptr,
                 const int32_t* sorted_token = nullptr, int64_t n_tokens = 0) {
  using P = FF<D>;
  CUtensorMap tmX, tmW1, tmW2;
  if (!make_tmap_bf16_2d(&tmW1, W1, (uint64_t)Gw * F, D, D, 128, kBK) ||
      !make_tmap_bf16_2d(&tmW2, W2, (uint64_t)Gw * D, (uint64_t)F, (uint64_t)F, D, kBK))
    return CTI_ERR_INVALID_ARG;
  if (GATHER) {
    tmX = tmW1;  // not read in gather mode
  } else if (!make_tmap_bf16_2d(&tmX, Xp, (uint64_t)rows_total, D, D, kBM, kBK)) {
    return CTI_ERR_INVALID_ARG;
  }
  static uint64_t configured = 0;
  if (ensure_smem_limit(fused_ffn_kernel<D, GATHER>, (int)P::SMEM, configured) != cudaSuccess)
    return CTI_ERR_CUDA;
  const int sms = device_sm_count();
  if (sms <= 0) return CTI_ERR_CUDA;
  const int64_t max_tiles = (rows_total + kBM - 1) / kBM + G;
  const int grid = (int)(max_tiles < sms ? max_tiles : sms);
  return launch_dependent(fused_ffn_kernel<D, GATHER>, dim3(grid),
                          dim3(GATHER ? kThreads + 32 : kThreads), P::SMEM, s, tmX, tmW1, tmW2,
                          offs, G, Gw, rows_total, F, b1, b2, act,
                          static_cast<__nv_bfloat16*>(Y), status,
                          static_cast<const __nv_bfloat16*>(x_rows), sorted_token,
                          n_tokens) == cudaSuccess
             ? CTI_OK
             : CTI_ERR_CUDA;
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
    return launch_fused<256, false>(Xp_bf16, W1_bf16, b1, W2_bf16, b2, group_offsets, G, Gw,
                                    rows_total, F, act, Y_bf16, status, s);
  return launch_fused<128, false>(Xp_bf16, W1_bf16, b1, W2_bf16, b2, group_offsets, G, Gw,
                                  rows_total, F, act, Y_bf16, status, s);
}

extern "C" int cti_moe_expert_ffn_fused_supported(int D, int F, int G, int64_t rows_total) {
  using namespace cti;
  return (D == 128 || D == 256) && F > 0 && F % kFC == 0 && F <= kMaxF && G >= 1 &&
                 G <= Sched::kMaxGroups && rows_total >= 0 &&
                 rows_total < ((int64_t)1 << 31) - 256
             ? 1
             : 0;
}

extern "C" int cti_moe_expert_ffn_fused_gather(const void* x_bf16, int64_t T,
                                               const int32_t* sorted_token, const void* W1_bf16,
                                               const float* b1, const void* W2_bf16,
                                               const float* b2, const int32_t* group_offsets,
                                               int G, int Gw, int64_t rows_total, int D, int F,
                                               int act, void* Y_bf16, int32_t* status,
                                               void* stream) {
  using namespace cti;
  if (G < 1 || Gw < 1 || rows_total < 0 || F <= 0 || T < 0) return CTI_ERR_INVALID_ARG;
  if (act < CTI_ACT_NONE || act > CTI_ACT_GELU) return CTI_ERR_INVALID_ARG;
  if ((D != 128 && D != 256) || F % kFC != 0 || F > kMaxF || G > Sched::kMaxGroups)
    return CTI_ERR_UNSUPPORTED;
  if (rows_total >= ((int64_t)1 << 31) - 256) return CTI_ERR_UNSUPPORTED;
  if (!W1_bf16 || !W2_bf16 || !b1 || !b2 || !group_offsets || !Y_bf16) return CTI_ERR_INVALID_ARG;
  if (rows_total == 0) return CTI_OK;
  if (!x_bf16 || !sorted_token || T == 0) return CTI_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) || (reinterpret_cast<uintptr_t>(Y_bf16) & 15) ||
      (reinterpret_cast<uintptr_t>(b1) & 15) || (reinterpret_cast<uintptr_t>(b2) & 15))
    return CTI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 256)
    return launch_fused<256, true>(nullptr, W1_bf16, b1, W2_bf16, b2, group_offsets, G, Gw,
                                   rows_total, F, act, Y_bf16, status, s, x_bf16, sorted_token, T);
  return launch_fused<128, true>(nullptr, W1_bf16, b1, W2_bf16, b2, group_offsets, G, Gw,
                                 rows_total, F, act, Y_bf16, status, s, x_bf16, sorted_token, T);
}
