// Causal attention inside packed variable-length sequences, head_dim 32:
// the attention of the CTR model's layers (baseline/infer.py:267-276
// `scaled_dot_product` with the causal sequence mask of
// get_sequence_causal_mask, :420-427; online_best/infer.py:1132-1202 runs
// SDPA per group of sequences).
//
//   out[t, h, :] = softmax_j( q[t,h,:] . k[j,h,:] / sqrt(32) ) @ v[j,h,:]
//                  over the keys j of t's own sequence with j <= t
//
// One persistent tcgen05 kernel for every sequence length.  Queries are
// tiled flat over the packed token stream: tile (i, h) holds the 128 tokens
// [cu[0] + 128 i, cu[0] + 128 i + 128) of head h, whatever sequences they
// belong to, so short sequences waste no MMA rows.  Row t of a tile attends
// to the key interval [start(t), t], start(t) the first token of t's
// sequence.  The tile's keys come in 64-key blocks, from the block holding
// its last row down to the block holding start(first row).
//
// Per CTA (224 threads, two CTAs per SM):
//   warp 0     tile scheduler and TMA producer: all 32 lanes look up the
//              tile's row starts in cu_seqlens (binary searches) and publish
//              them with the tile's block range in a 4-slot ring in shared
//              memory; lane 0 then loads the tile's Q ([128 x 32] bf16,
//              64-byte swizzle) into a 2-deep ring and each block's K and V
//              ([64 x 32]) into an 8-stage ring.  q, k and v are strided
//              token views ([token][head][32], e.g. the thirds of one qkv
//              projection output), addressed by 2-D tensor maps.
//   warp 1     S issuer (and TMEM owner): S_g = Q K_g^T (M 128, N 64, K 32:
//              two MMAs) into S buffer g % 3, once the buffer's previous PV
//              is done.
//   warp 2     PV issuer: O += P_g V_g (M 128, N 32, K = the block's needed
//              32-key chunks, 16 keys per MMA) with P read from TMEM (the TS
//              form) and V as an MN-major operand, into the tile's O
//              accumulator (two, alternating between tiles).  One thread
//              issues a tcgen05.mma only every ~120 cycles, so S and PV get
//              a thread each.
//   warps 3-6  softmax, thread = query row (one TMEM lane quadrant per
//              warp).  Per block: the row's 64 scores in one TMEM load,
//              masked to the row's keys (chunks every lane needs whole skip
//              the mask), the block max; p = 2^((s - m) log2e / sqrt32) with
//              m the row's exponent offset, P stored over the S buffer as
//              bf16, l += sum(p).  m is set by the row's first keys and only
//              raised (O and l rescaled in place) when a block max exceeds
//              it by more than 2^8 in p, so p <= 2^8.  The tile's output
//              o / l is read from TMEM one block into the next tile, when
//              its last PV has had time to finish.
// TMEM (256 columns): S/P buffers at columns 0, 64 and 128, O accumulators at
// 192 and 224.  Every wait is a bounded mbarrier wait; a wait that runs out
// records its site in the status word and the roles unwind.
#include "common.cuh"
#include "tmap.cuh"

namespace cti {
namespace {

constexpr int kHD = 32;        // head_dim
constexpr int kTile = 128;     // query rows per tile
constexpr int kKB = 64;        // keys per key block
constexpr int kKVStages = 8;   // K/V blocks in flight per CTA
constexpr int kInfoSlots = 4;  // tiles published ahead by the scheduler
constexpr int kNS = 3;         // S/P buffers in TMEM
constexpr int kSoftmaxWarp0 = 3;
constexpr int kAttnThreads = 224;  // scheduler, S issuer, PV issuer, 4 softmax warps
constexpr uint32_t kQBytes = kTile * kHD * 2;   // [128 x 32] bf16, 8 KB
constexpr uint32_t kKVBytes = kKB * kHD * 2;    // [64 x 32] bf16, 4 KB
// TMEM (256 columns): S/P buffers 0-2 at columns 0, 64 and 128 (S: 64 fp32
// columns; P: bf16 pairs over the first 32), O accumulators 0 and 1 (one
// per tile in flight, alternating) at columns 192 and 224.
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kSCols = 64;
constexpr uint32_t kOCol0 = kNS * kSCols;
static_assert(kOCol0 + 2 * kHD <= kTmemCols, "TMEM budget");
// A row's exponent offset m is only raised (and O, l rescaled) when the
// block max exceeds it by more than 2^kSlack in p: p <= 2^kSlack otherwise.
constexpr float kSlack = 8.0f;

// One scheduled tile, as published by the scheduler warp.
struct TileSlot {
  int t0;     // first query token
  int h;      // head
  int st0;    // first key any row needs (start of t0's sequence)
  int tlast;  // last valid query token
  int kbtop;  // first key of the top block; block j starts at kbtop - 64 j
  int nkb;    // key blocks
  int pad[2];
  int row_st[kTile];  // start of each row's sequence (rows past tlast: 0)
};

constexpr size_t kBarBytes = 384;
constexpr size_t kAttnSmem = 1024 + 2 * kQBytes + (size_t)kKVStages * 2 * kKVBytes +
                             kInfoSlots * sizeof(TileSlot) + kBarBytes;
static_assert(2 * kAttnSmem <= 232448, "two CTAs per SM");

// Shared-memory descriptor of a bf16 operand tile with 64-byte rows (32
// elements) in the 64-byte swizzle that the TMA writes: 8-row atoms of 512
// bytes stacked along the tile's rows.  Used K-major for Q and K (each row
// one query or key, its 32 head dims contiguous; a K step of 16 advances the
// start by 32 bytes inside the row) and MN-major for V (each row one key, its
// 32 head dims = N contiguous; a K step of 16 keys advances by 1024 bytes).
// The 8-row stride is 512 bytes in both roles and the tile is one atom wide,
// so both offset fields hold 512.
//   bits 0-13 start >> 4; 16-29 leading byte offset >> 4; 32-45 stride byte
//   offset >> 4; 46-47 version 1; 61-63 layout type (4 = 64-byte swizzle).
CTI_DEVICE uint64_t smem_desc_sw64(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(512u >> 4) << 16) |
         ((uint64_t)(512u >> 4) << 32) | ((uint64_t)1u << 46) | ((uint64_t)4u << 61);
}

CTI_DEVICE float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// First token of the sequences holding tokens t[0..N): cu[s] for the
// largest s in [0, n) with cu[s] <= t (so empty sequences are skipped); the
// N searches run interleaved.  Requires cu[0] <= t < cu[n].
template <int N>
CTI_DEVICE void seq_starts(const int32_t* __restrict__ cu, int n, const int (&t)[N],
                           int (&st)[N]) {
  int lo[N], hi[N];
#pragma unroll
  for (int q = 0; q < N; ++q) {
    lo[q] = 0;
    hi[q] = n;
  }
  for (int span = n; span > 1; span = (span + 1) >> 1) {
#pragma unroll
    for (int q = 0; q < N; ++q) {
      if (hi[q] - lo[q] > 1) {
        const int mid = (lo[q] + hi[q]) >> 1;
        if (__ldg(cu + mid) <= t[q]) lo[q] = mid;
        else hi[q] = mid;
      }
    }
  }
#pragma unroll
  for (int q = 0; q < N; ++q) st[q] = __ldg(cu + lo[q]);
}

// The 32-key chunks [cmin, cmax] (within 0..1) of the block starting at kb
// that some row of the tile needs; the PV MMA covers exactly these keys.
CTI_DEVICE void block_chunks(int st0, int tlast, int kb, int& cmin, int& cmax) {
  cmin = (max(st0, kb) - kb) >> 5;
  cmax = (min(tlast, kb + kKB - 1) - kb) >> 5;
}

// Writes the output rows of a warp's 32 lanes (head h): lane i's row t (or
// -1: none) is o (32 fp32 TMEM columns) / l as bf16, 64 bytes.  Lanes 2j and
// 2j+1 swap 32-byte halves first, so that each store writes one whole row
// piece with two lanes instead of every lane writing half of its own.
CTI_DEVICE void store_rows(__nv_bfloat16* __restrict__ out, int t, int H, int h,
                           const uint32_t (&o)[32], float l, int lane, bool aligned32) {
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
  uint32_t u[2][8];  // half j, word w: columns 16j + 2w, 16j + 2w + 1
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int w = 0; w < 8; ++w)
      u[j][w] = pack_bf16x2(__uint_as_float(o[16 * j + 2 * w]) * inv,
                            __uint_as_float(o[16 * j + 2 * w + 1]) * inv);
  const bool odd = (lane & 1) != 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t got = __shfl_xor_sync(0xffffffffu, odd ? u[0][w] : u[1][w], 1);
    if (odd)
      u[0][w] = got;
    else
      u[1][w] = got;
  }
  // Now slot k holds half (lane & 1) of the row of lane (lane & ~1) + k.
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int tk = __shfl_sync(0xffffffffu, t, (lane & ~1) + k);
    if (tk >= 0) st_global_32B(out + ((int64_t)tk * H + h) * kHD + 16 * (lane & 1), u[k], aligned32);
  }
}

__global__ void __launch_bounds__(kAttnThreads, 2)
    varlen_attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                            const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV,
                            const int32_t* __restrict__ cu, int num_seqs, int tokens, int H,
                            float scale_log2, __nv_bfloat16* __restrict__ out, int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                 // [2] Q tiles
  uint8_t* sKV = smem + 2 * kQBytes;  // [kKVStages] x {K, V}
  TileSlot* slots = reinterpret_cast<TileSlot*>(sKV + (size_t)kKVStages * 2 * kKVBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(slots + kInfoSlots);
  uint64_t* q_full = bars;                        // [2]
  uint64_t* q_empty = q_full + 2;                 // [2]
  uint64_t* kv_full = q_empty + 2;                // [kKVStages]
  uint64_t* kv_empty = kv_full + kKVStages;       // [kKVStages]
  uint64_t* info_full = kv_empty + kKVStages;     // [kInfoSlots] slot published
  uint64_t* info_empty = info_full + kInfoSlots;  // [kInfoSlots] slot read (2 issuers + 4 warps)
  uint64_t* s_full = info_empty + kInfoSlots;     // [kNS] S MMA done
  uint64_t* p_full = s_full + kNS;                // [kNS] P stored (4 softmax warps)
  uint64_t* pv_done = p_full + kNS;               // [kNS] PV MMA done: P consumed, O updated
  uint64_t* drain = pv_done + kNS;                // [2] each issuer's last MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  static_assert((2 * 2 + 2 * kKVStages + 2 * kInfoSlots + 3 * kNS + 2) * 8 + 8 <= kBarBytes,
                "barrier area");

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&drain[i], 1);
    }
    for (int i = 0; i < kNS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < kInfoSlots; ++s) {
      mbar_init(&info_full[s], 1);
      mbar_init(&info_empty[s], 6);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  grid_dependency_wait();  // q, k, v come from the kernels before this one
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int cu0 = __ldg(cu);
  const int tend = min(__ldg(cu + num_seqs), tokens);
  int64_t ntiles = tend > cu0 ? (int64_t)((tend - cu0 + kTile - 1) / kTile) * H : 0;
  if (cu0 < 0) {
    if (threadIdx.x == 0) raise_status(status, CTI_ERR_INVALID_ARG, 0x600);
    ntiles = 0;
  }

  if (warp == 0) {
    // ---------------- scheduler + TMA producer ----------------
    int it = 0, g = 0;
    bool ok = true;
    for (int64_t i = blockIdx.x; ok && i < ntiles; i += gridDim.x, ++it) {
      const int si = it % kInfoSlots;
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&info_empty[si], (uint32_t)((it / kInfoSlots) & 1) ^ 1u, status,
                                0x601, abort_flag));
      if (!ok) break;
      const int h = (int)(i % H);
      const int t0 = cu0 + (int)(i / H) * kTile;
      const int tlast = min(t0 + kTile - 1, tend - 1);
      int tq[5], sq[5];
#pragma unroll
      for (int q = 0; q < 4; ++q) tq[q] = min(t0 + lane + 32 * q, tlast);
      tq[4] = t0;
      seq_starts<5>(cu, num_seqs, tq, sq);
      const int st0 = min(max(sq[4], cu0), t0);
      const int kbtop = t0 + kKB * ((tlast - t0) / kKB);
      const int nkb = 1 + (kbtop - st0 + kKB - 1) / kKB;
      TileSlot& ts = slots[si];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int t = t0 + lane + 32 * q;
        ts.row_st[lane + 32 * q] = t <= tlast ? min(max(sq[q], st0), t) : 0;
      }
      if (lane == 0) {
        ts.t0 = t0;
        ts.h = h;
        ts.st0 = st0;
        ts.tlast = tlast;
        ts.kbtop = kbtop;
        ts.nkb = nkb;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&info_full[si]);
        const int qb = it & 1;
        if (mbar_wait(&q_empty[qb], (uint32_t)((it >> 1) & 1) ^ 1u, status, 0x602, abort_flag)) {
          mbar_arrive_expect_tx(&q_full[qb], kQBytes);
          tma_load_2d(sQ + qb * kQBytes, &tmQ, &q_full[qb], h * kHD, t0);
          for (int j = 0; j < nkb; ++j, ++g) {
            const int s = g % kKVStages;
            if (!mbar_wait(&kv_empty[s], (uint32_t)((g / kKVStages) & 1) ^ 1u, status, 0x603,
                           abort_flag)) {
              ok = false;
              break;
            }
            uint8_t* dst = sKV + (size_t)s * 2 * kKVBytes;
            const int kb = kbtop - kKB * j;
            mbar_arrive_expect_tx(&kv_full[s], 2 * kKVBytes);
            tma_load_2d(dst, &tmK, &kv_full[s], h * kHD, kb);
            tma_load_2d(dst + kKVBytes, &tmV, &kv_full[s], h * kHD, kb);
          }
        } else {
          ok = false;
          --it;  // no Q load issued for this tile
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      it = __shfl_sync(0xffffffffu, it, 0);
    }
    if (lane == 0) {
      // Let the loads in flight land before the CTA can exit.
      for (int q = 1; q <= 2; ++q)
        if (it - q >= 0)
          mbar_wait(&q_full[(it - q) & 1], (uint32_t)(((it - q) >> 1) & 1), status, 0x604,
                    nullptr);
      for (int q = 1; q <= kKVStages; ++q)
        if (g - q >= 0)
          mbar_wait(&kv_full[(g - q) % kKVStages], (uint32_t)(((g - q) / kKVStages) & 1),
                    status, 0x604, nullptr);
    }
  } else if (warp == 1) {
    // ---------------- S issuer ----------------
    // S_g = Q K_g^T into buffer g % 3, once PV_{g-3} (the buffer's last
    // reader) is done.
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16_f32(kTile, kKB);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t kv_addr = smem_u32(sKV);
      bool ok = true, any = false;
      int it = 0, g = 0;
      for (int64_t i = blockIdx.x; ok && i < ntiles; i += gridDim.x, ++it) {
        const int si = it % kInfoSlots;
        if (!mbar_wait(&info_full[si], (uint32_t)((it / kInfoSlots) & 1), status, 0x605,
                       abort_flag))
          break;
        const int nkb = slots[si].nkb;
        mbar_arrive(&info_empty[si]);
        const int qb = it & 1;
        if (!mbar_wait(&q_full[qb], (uint32_t)((it >> 1) & 1), status, 0x606, abort_flag)) break;
        for (int j = 0; j < nkb; ++j, ++g) {
          const int s = g % kKVStages;
          const int b = g % kNS;
          if (!mbar_wait(&kv_full[s], (uint32_t)((g / kKVStages) & 1), status, 0x607,
                         abort_flag) ||
              !mbar_wait(&pv_done[b], (uint32_t)((g / kNS) & 1) ^ 1u, status, 0x608,
                         abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = kv_addr + (uint32_t)s * 2 * kKVBytes;
          const uint32_t qa = q_addr + (uint32_t)qb * kQBytes;
#pragma unroll
          for (int kk = 0; kk < kHD / 16; ++kk)
            umma_bf16(tmem_base + (uint32_t)b * kSCols, smem_desc_sw64(qa + kk * 32),
                      smem_desc_sw64(k_addr + kk * 32), id_s, kk != 0 ? 1u : 0u);
          umma_commit(&s_full[b]);
          if (j == nkb - 1) umma_commit(&q_empty[qb]);
          any = true;
        }
      }
      if (any) {
        umma_commit(&drain[0]);
        mbar_wait(&drain[0], 0, status, 0x609, nullptr);
      }
    }
  } else if (warp == 2) {
    // ---------------- PV issuer ----------------
    // O[tile % 2] (+)= P_g V_g once the softmax has stored P_g, over the
    // 32-key chunks the tile needs; then the K/V stage and the S buffer are
    // free.
    if (lane == 0) {
      const uint32_t id_pv = idesc_bf16_f32(kTile, kHD) | (1u << 16);  // B (V) MN-major
      const uint32_t kv_addr = smem_u32(sKV);
      bool ok = true, any = false;
      int it = 0, g = 0;
      for (int64_t i = blockIdx.x; ok && i < ntiles; i += gridDim.x, ++it) {
        const int si = it % kInfoSlots;
        if (!mbar_wait(&info_full[si], (uint32_t)((it / kInfoSlots) & 1), status, 0x60a,
                       abort_flag))
          break;
        const int st0 = slots[si].st0, tlast = slots[si].tlast;
        const int kbtop = slots[si].kbtop, nkb = slots[si].nkb;
        mbar_arrive(&info_empty[si]);
        const uint32_t ocol = tmem_base + kOCol0 + (uint32_t)(it & 1) * kHD;
        for (int j = 0; j < nkb; ++j, ++g) {
          const int s = g % kKVStages;
          const int b = g % kNS;
          int c0, c1;
          block_chunks(st0, tlast, kbtop - kKB * j, c0, c1);
          if (!mbar_wait(&p_full[b], (uint32_t)((g / kNS) & 1), status, 0x60b, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t pbuf = tmem_base + (uint32_t)b * kSCols;
          const uint32_t v_addr = kv_addr + (uint32_t)s * 2 * kKVBytes + kKVBytes;
          for (int kk = 2 * c0; kk <= 2 * c1 + 1; ++kk)
            umma_bf16_ts(ocol, pbuf + (uint32_t)kk * 8, smem_desc_sw64(v_addr + kk * 1024),
                         id_pv, (j == 0 && kk == 2 * c0) ? 0u : 1u);
          umma_commit(&pv_done[b]);
          umma_commit(&kv_empty[s]);
          any = true;
        }
      }
      if (any) {
        umma_commit(&drain[1]);
        mbar_wait(&drain[1], 0, status, 0x60c, nullptr);
      }
    }
  } else if (warp >= kSoftmaxWarp0) {
    // ---------------- softmax ----------------
    const int wq = warp & 3;  // TMEM lane quadrant of this warp
    const int r = wq * 32 + lane;
    const uint32_t lane_base = tmem_base + ((uint32_t)(wq * 32) << 16);
    const float kNegInf = -INFINITY;
    const uint64_t scale2 = f2_pack(scale_log2, scale_log2);
    const bool out32 = (reinterpret_cast<uintptr_t>(out) & 31) == 0;
    // The previous tile's row, finished once its last PV MMA is done.
    int prev_t = -1, prev_h = 0, prev_o = 0, prev_g = -1;
    float prev_l = 0.0f;
    int it = 0, g = 0;
    bool ok = true;
    // pv_done[b] completes once per use of buffer b.  A thread that has seen
    // s_full for block k knows PV_{k-3} is done (S_k was issued after it),
    // so a wait for PV_k' (k' <= k) on pv_done[k' % 3] has at most that one
    // phase pending and its parity names it.
    auto wait_pv = [&](int k, int where) -> bool {
      return mbar_wait(&pv_done[k % kNS], (uint32_t)((k / kNS) & 1), status, where, abort_flag);
    };
    auto finish_prev = [&]() -> bool {
      if (prev_g < 0) return true;
      // Warp-uniform: the TMEM load and the row exchange below need every lane.
      if (!__all_sync(0xffffffffu, wait_pv(prev_g, 0x60d))) return false;
      tc_fence_after();
      uint32_t o[32];
      tmem_ld_32x32b_x32_sync(lane_base + kOCol0 + (uint32_t)prev_o * kHD, o);
      store_rows(out, prev_t, H, prev_h, o, prev_l, lane, out32);
      prev_g = -1;
      return true;
    };
    for (int64_t i = blockIdx.x; ok && i < ntiles; i += gridDim.x, ++it) {
      const int si = it % kInfoSlots;
      if (!__all_sync(0xffffffffu, mbar_wait(&info_full[si], (uint32_t)((it / kInfoSlots) & 1),
                                             status, 0x60c, abort_flag)))
        break;
      const int t0 = slots[si].t0, h = slots[si].h, st0 = slots[si].st0;
      const int tlast = slots[si].tlast, kbtop = slots[si].kbtop, nkb = slots[si].nkb;
      const int st = slots[si].row_st[r];
      __syncwarp();
      if (lane == 0) mbar_arrive(&info_empty[si]);
      const int t = t0 + r;
      const bool valid = t <= tlast;
      const uint32_t ocol = kOCol0 + (uint32_t)(it & 1) * kHD;
      float m = kNegInf, l = 0.0f;  // exponent offset (raw score units) and sum

      for (int j = 0; j < nkb; ++j, ++g) {
        const int b = g % kNS;
        const int kb = kbtop - kKB * j;
        int cmin, cmax;
        block_chunks(st0, tlast, kb, cmin, cmax);
        // This row's keys in the block, relative to kb: [lo, hi] (empty:
        // lo > hi).
        int lo = kKB, hi = -1;
        if (valid) {
          lo = max(st, kb) - kb;
          hi = min(t, kb + kKB - 1) - kb;
          if (lo > hi) {
            lo = kKB;
            hi = -1;
          }
        }
        const int wlo = __reduce_min_sync(0xffffffffu, lo);
        const int whi = __reduce_max_sync(0xffffffffu, hi);
        const int c_lo = whi >= 0 ? (wlo >> 5) : 2;
        const int c_hi = whi >= 0 ? (whi >> 5) : -1;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (uint32_t)((g / kNS) & 1), status,
                                               0x60e, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sb = lane_base + (uint32_t)b * kSCols;

        // The block's scores of this row (both chunks in one load), masked
        // to the row's keys; the block max.
        uint32_t v[2][32];
        float mx = kNegInf;
        if (c_lo <= c_hi) {
          tmem_ld_32x32b_2x32_sync(sb, sb + 32, v[0], v[1]);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            if (c < c_lo || c > c_hi) continue;
            const int a0 = lo - 32 * c, a1 = hi - 32 * c;
            if (!__all_sync(0xffffffffu, a0 <= 0 && a1 >= 31)) {
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (!(e >= a0 && e <= a1)) v[c][e] = __float_as_uint(kNegInf);
            }
            float mx1 = kNegInf;
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              mx = max3f(mx, __uint_as_float(v[c][e]), __uint_as_float(v[c][e + 1]));
              mx1 = max3f(mx1, __uint_as_float(v[c][e + 2]), __uint_as_float(v[c][e + 3]));
            }
            mx = fmaxf(mx, mx1);
          }
        }
        // Exponent offset: set by the row's first keys; raised (with O and l
        // rescaled) only when this block's max exceeds it by more than
        // 2^kSlack in p.
        float corr = 1.0f;
        if (mx != kNegInf) {
          if (m == kNegInf) {
            m = mx;
          } else if ((mx - m) * scale_log2 > kSlack) {
            corr = ex2_approx((m - mx) * scale_log2);
            m = mx;
          }
        }
        if (__any_sync(0xffffffffu, corr != 1.0f)) {
          // O holds blocks up to g-1 of this tile: wait for PV_{g-1}.
          if (!__all_sync(0xffffffffu, wait_pv(g - 1, 0x60f))) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t o[32];
          tmem_ld_32x32b_x32_sync(lane_base + ocol, o);
#pragma unroll
          for (int d = 0; d < kHD; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * corr);
          tmem_st_32x32b_x32(lane_base + ocol, o);
          l *= corr;
        }
        const float off = m == kNegInf ? 0.0f : m * scale_log2;
        const uint64_t noff2 = f2_pack(-off, -off);

        // p = 2^(s*scale - off) and P (bf16) over the chunks the PV MMA
        // reads; chunks no row of this warp needs are zero.
        uint64_t sum_a = f2_pack(0.0f, 0.0f), sum_b = sum_a;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (c < cmin || c > cmax) continue;
          uint32_t pk[16];
          if (c < c_lo || c > c_hi) {
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[e] = 0u;
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(v[c][2 * e]),
                                       __uint_as_float(v[c][2 * e + 1])),
                               scale2, noff2),
                        x0, x1);
              const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
              if (e & 1) sum_b = f2_add(sum_b, f2_pack(p0, p1));
              else sum_a = f2_add(sum_a, f2_pack(p0, p1));
              pk[e] = pack_bf16x2(p0, p1);
            }
          }
          tmem_st_32x32b_x16(sb + (uint32_t)(16 * c), pk);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[b]);
        float s0, s1;
        f2_unpack(f2_add(sum_a, sum_b), s0, s1);
        l += s0 + s1;
        // The previous tile's output, now that its last PV has had a block's
        // time to finish.
        if (j == 0 && !finish_prev()) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
      prev_t = valid ? t : -1;
      prev_h = h;
      prev_o = it & 1;
      prev_g = g - 1;
      prev_l = l;
    }
    if (ok) finish_prev();
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace
}  // namespace cti

extern "C" int cti_varlen_attention(const void* q_bf16, const void* k_bf16, const void* v_bf16,
                                    int64_t q_stride, int64_t k_stride, int64_t v_stride,
                                    const int32_t* cu_seqlens, int num_seqs, int max_seqlen,
                                    int64_t tokens, int heads, int head_dim, void* out_bf16,
                                    int32_t* status, void* stream) {
  using namespace cti;
  if (num_seqs < 0 || max_seqlen < 0 || heads <= 0 || tokens < 0) return CTI_ERR_INVALID_ARG;
  if (head_dim != kHD) return CTI_ERR_UNSUPPORTED;
  if (num_seqs == 0 || tokens == 0) return CTI_OK;
  if (!q_bf16 || !k_bf16 || !v_bf16 || !cu_seqlens || !out_bf16) return CTI_ERR_INVALID_ARG;
  // Tensor-map rules: 16-byte aligned bases and token strides.
  if ((reinterpret_cast<uintptr_t>(q_bf16) | reinterpret_cast<uintptr_t>(k_bf16) |
       reinterpret_cast<uintptr_t>(v_bf16) | reinterpret_cast<uintptr_t>(out_bf16)) & 15)
    return CTI_ERR_INVALID_ARG;
  if ((q_stride | k_stride | v_stride) % 8 != 0 || q_stride < (int64_t)heads * kHD ||
      k_stride < (int64_t)heads * kHD || v_stride < (int64_t)heads * kHD)
    return CTI_ERR_INVALID_ARG;
  if (tokens > INT32_MAX - 2 * kTile || heads > 65535) return CTI_ERR_UNSUPPORTED;
  const uint64_t cols = (uint64_t)heads * kHD;
  CUtensorMap tmQ, tmK, tmV;
  if (!make_tmap_bf16_2d(&tmQ, q_bf16, (uint64_t)tokens, cols, (uint64_t)q_stride, kTile, kHD,
                         CU_TENSOR_MAP_SWIZZLE_64B) ||
      !make_tmap_bf16_2d(&tmK, k_bf16, (uint64_t)tokens, cols, (uint64_t)k_stride, kKB, kHD,
                         CU_TENSOR_MAP_SWIZZLE_64B) ||
      !make_tmap_bf16_2d(&tmV, v_bf16, (uint64_t)tokens, cols, (uint64_t)v_stride, kKB, kHD,
                         CU_TENSOR_MAP_SWIZZLE_64B))
    return CTI_ERR_INVALID_ARG;
  static uint64_t configured = 0;
  if (ensure_smem_limit(varlen_attention_kernel, (int)kAttnSmem, configured) != cudaSuccess)
    return CTI_ERR_CUDA;
  const int sms = device_sm_count();
  if (sms <= 0) return CTI_ERR_CUDA;
  const int64_t max_tiles = (tokens + kTile - 1) / kTile * heads;
  const int grid = (int)(max_tiles < 2 * sms ? max_tiles : 2 * sms);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)kHD);
  return launch_dependent(varlen_attention_kernel, dim3(grid), dim3(kAttnThreads), kAttnSmem,
                          static_cast<cudaStream_t>(stream), tmQ, tmK, tmV, cu_seqlens, num_seqs,
                          (int)tokens, heads, scale_log2,
                          static_cast<__nv_bfloat16*>(out_bf16), status) == cudaSuccess
             ? CTI_OK
             : CTI_ERR_CUDA;
}
