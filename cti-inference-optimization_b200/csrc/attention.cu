// Causal attention inside packed variable-length sequences, head_dim 32:
// the attention of the CTR model's layers (baseline/infer.py:267-276
// `scaled_dot_product` with the causal sequence mask of
// get_sequence_causal_mask, :420-427; online_best/infer.py:1132-1202 runs
// SDPA per group of sequences).
//
//   out[t, h, :] = softmax_j( q[t,h,:] . k[j,h,:] / sqrt(32) ) @ v[j,h,:]
//                  over the keys j of t's own sequence with j <= t
//
// Two kernels with the same arithmetic per row.  Sequences of at most 256
// tokens (max_seqlen <= 256) take varlen_attention_seq_kernel: one CTA per
// (sequence, head), the whole sequence staged in shared memory.  Longer
// ones take varlen_attention_kernel: one CTA per (sequence, 64-query block,
// head); 4 warps of 16 query rows.  Flash-attention schedule: key blocks of 64 double-buffered in shared
// memory (cp.async, the next block in flight during this one's math), scores
// on the tensor cores (mma.sync m16n8k16 bf16 -> fp32), an online softmax in
// fp32 registers (running max and sum per row), P converted to bf16 straight
// from the score registers into the A fragments of P @ V.  Rows past the
// sequence end are computed on zeros and not stored; keys past the end or
// after the query are masked.  q, k, v are strided views ([token][head][32]
// with a token stride, e.g. the q/k/v thirds of one qkv projection output),
// so no copy is needed.  No barriers other than __syncthreads, no spins.
#include "common.cuh"

namespace cti {
namespace {

constexpr int kHD = 32;
constexpr int kBQ = 64;     // query rows per CTA
constexpr int kBK = 64;     // keys per block
constexpr int kPitch = 40;  // bf16 per shared row (32 + 8 padding: conflict-free ldmatrix)

CTI_DEVICE void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

CTI_DEVICE void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// D[16x8] += A[16x16] * B[16x8], bf16 inputs, fp32 accumulators.
CTI_DEVICE void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Starts the copy of rows [r0, r0 + 64) of a [token][head][32] view into a
// [64][kPitch] tile (16-byte cp.async pieces, 256 of them, two per thread);
// rows >= n are filled with zeros.
CTI_DEVICE void load_tile_async(__nv_bfloat16 (*tile)[kPitch], const __nv_bfloat16* base,
                                int64_t tok_stride, int r0, int n) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int c = threadIdx.x + i * 128;
    const int row = c >> 2;
    const int part = c & 3;
    const bool ok = r0 + row < n;
    const __nv_bfloat16* src = ok ? base + (int64_t)(r0 + row) * tok_stride + part * 8 : base;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(&tile[row][part * 8])),
                 "l"(src), "r"(ok ? 16 : 0)
                 : "memory");
  }
}

CTI_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CTI_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

CTI_DEVICE float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(128)
    varlen_attention_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                            const __nv_bfloat16* __restrict__ v, int64_t q_stride,
                            int64_t k_stride, int64_t v_stride, const int32_t* __restrict__ cu,
                            int qblocks, float scale_log2, __nv_bfloat16* __restrict__ out,
                            int H) {
  __shared__ __align__(16) __nv_bfloat16 sq[kBQ][kPitch];
  __shared__ __align__(16) __nv_bfloat16 sk[2][kBK][kPitch];  // double-buffered key blocks
  __shared__ __align__(16) __nv_bfloat16 sv[2][kBK][kPitch];
  const int seq = blockIdx.x / qblocks;
  const int qb = blockIdx.x % qblocks;
  const int h = blockIdx.y;
  const int start = cu[seq];
  const int L = cu[seq + 1] - start;
  const int q0 = qb * kBQ;
  if (q0 >= L) return;  // the whole CTA leaves together
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const __nv_bfloat16* kbase = k + (int64_t)start * k_stride + h * kHD;
  const __nv_bfloat16* vbase = v + (int64_t)start * v_stride + h * kHD;
  load_tile_async(sq, q + (int64_t)start * q_stride + h * kHD, q_stride, q0, L);
  load_tile_async(sk[0], kbase, k_stride, 0, L);
  load_tile_async(sv[0], vbase, v_stride, 0, L);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  // Q fragments of this warp's 16 rows: two k-steps of 16 head dims.
  uint32_t qa[2][4];
#pragma unroll
  for (int kk = 0; kk < 2; ++kk)
    ldsm_x4(qa[kk], &sq[warp * 16 + (lane & 15)][kk * 16 + (lane >> 4) * 8]);

  float o[4][4] = {};          // O: 4 n-tiles of 8 head dims
  float m_run[2] = {-INFINITY, -INFINITY};  // rows lane/4 and lane/4 + 8
  float l_run[2] = {0.f, 0.f};
  const int row_a = q0 + warp * 16 + (lane >> 2);  // query positions in the sequence
  const int row_b = row_a + 8;

  for (int kb = 0; kb <= qb; ++kb) {
    const int k0 = kb * kBK;
    const int buf = kb & 1;
    // Prefetch the next key block into the other buffer (read two blocks
    // ago; the __syncthreads at the end of the previous step freed it).
    if (kb < qb) {
      load_tile_async(sk[buf ^ 1], kbase, k_stride, k0 + kBK, L);
      load_tile_async(sv[buf ^ 1], vbase, v_stride, k0 + kBK, L);
      cp_async_commit();
    }
    // S = Q K^T for 64 keys: 8 n-tiles of 8 keys.
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    }
#pragma unroll
    for (int np = 0; np < 4; ++np) {  // pairs of n-tiles
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        // B fragments of keys [np*16, np*16+16), head dims [kk*16, kk*16+16):
        // matrices (keys 0-7, d 0-7), (keys 0-7, d 8-15), (keys 8-15, d 0-7), (keys 8-15, d 8-15).
        uint32_t b[4];
        ldsm_x4(b, &sk[buf][np * 16 + (lane & 7) + ((lane >> 4) << 3)][kk * 16 + ((lane >> 3) & 1) * 8]);
        mma_bf16(s[2 * np], qa[kk], b[0], b[1]);
        mma_bf16(s[2 * np + 1], qa[kk], b[2], b[3]);
      }
    }
    // Mask: keys past the sequence end or after the query.
    const bool diag = kb == qb;
    const bool tail = k0 + kBK > L;
    if (diag || tail) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int key = k0 + nt * 8 + (lane & 3) * 2;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (key + e > row_a || key + e >= L) s[nt][e] = -INFINITY;
          if (key + e > row_b || key + e >= L) s[nt][2 + e] = -INFINITY;
        }
      }
    }
    // Online softmax per row (the 4 lanes of a quad share a row).
    float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      mx[0] = fmaxf(mx[0], fmaxf(s[nt][0], s[nt][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[nt][2], s[nt][3]));
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    // Rows with no visible key yet keep max = -inf; use 0 as the offset.
    const float off0 = mx[0] == -INFINITY ? 0.f : mx[0] * scale_log2;
    const float off1 = mx[1] == -INFINITY ? 0.f : mx[1] * scale_log2;
    const float corr0 = fast_exp2(m_run[0] == -INFINITY ? -INFINITY : m_run[0] * scale_log2 - off0);
    const float corr1 = fast_exp2(m_run[1] == -INFINITY ? -INFINITY : m_run[1] * scale_log2 - off1);
    m_run[0] = mx[0];
    m_run[1] = mx[1];
    float ls[2] = {0.f, 0.f};
    uint32_t pa[4][4];  // P as A fragments: 4 k-steps of 16 keys
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = fast_exp2(fmaf(s[nt][0], scale_log2, -off0));
      const float p1 = fast_exp2(fmaf(s[nt][1], scale_log2, -off0));
      const float p2 = fast_exp2(fmaf(s[nt][2], scale_log2, -off1));
      const float p3 = fast_exp2(fmaf(s[nt][3], scale_log2, -off1));
      ls[0] += p0 + p1;
      ls[1] += p2 + p3;
      const int ks = nt >> 1, hi = nt & 1;
      pa[ks][hi * 2 + 0] = pack_bf16x2(p0, p1);  // rows lane/4
      pa[ks][hi * 2 + 1] = pack_bf16x2(p2, p3);  // rows lane/4 + 8
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      ls[i] += __shfl_xor_sync(0xffffffffu, ls[i], 1);
      ls[i] += __shfl_xor_sync(0xffffffffu, ls[i], 2);
    }
    l_run[0] = l_run[0] * corr0 + ls[0];
    l_run[1] = l_run[1] * corr1 + ls[1];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      o[nt][0] *= corr0;
      o[nt][1] *= corr0;
      o[nt][2] *= corr1;
      o[nt][3] *= corr1;
    }
    // O += P V: k = 64 keys (4 steps), n = 32 head dims (4 tiles).
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      // A fragment register order of m16n8k16: (rows 0-7, k 0-7), (rows 8-15, k 0-7),
      // (rows 0-7, k 8-15), (rows 8-15, k 8-15).
      const uint32_t a[4] = {pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3]};
#pragma unroll
      for (int np = 0; np < 2; ++np) {  // pairs of 8-wide head-dim tiles
        // V^T fragments from V[key][d] with .trans: matrices (keys 0-7, d 0-7),
        // (keys 8-15, d 0-7), (keys 0-7, d 8-15), (keys 8-15, d 8-15).
        uint32_t b[4];
        ldsm_x4_t(b, &sv[buf][ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8][np * 16 + (lane >> 4) * 8]);
        mma_bf16(o[2 * np], a, b[0], b[1]);
        mma_bf16(o[2 * np + 1], a, b[2], b[3]);
      }
    }
    // The next block has landed for everyone, and this block's buffer may be
    // overwritten by the prefetch of the step after.
    cp_async_wait<0>();
    __syncthreads();
  }
  // Normalise and store the rows that exist.
  const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
  const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int d = nt * 8 + (lane & 3) * 2;
    if (row_a < L)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)(start + row_a) * H + h) * kHD + d) =
          pack_bf16x2(o[nt][0] * inv0, o[nt][1] * inv0);
    if (row_b < L)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)(start + row_b) * H + h) * kHD + d) =
          pack_bf16x2(o[nt][2] * inv1, o[nt][3] * inv1);
  }
}

// One CTA per (sequence, head) for sequences of at most NB * 64 tokens: the
// sequence's q, k and v rows are all copied into shared memory at once, one
// cp.async group per 64-row block, and the 4 warps then walk the query
// blocks in order; query block qb starts as soon as blocks 0..qb have
// landed, while the later blocks are still in flight.  Compared with one
// CTA per query block, every key/value row is read once per head instead of
// once per query block at or after it, and no CTA is launched for query
// blocks past the sequence end.  Same arithmetic per row as
// varlen_attention_kernel.
template <int NB>
__global__ void __launch_bounds__(128)
    varlen_attention_seq_kernel(const __nv_bfloat16* __restrict__ q,
                                const __nv_bfloat16* __restrict__ k,
                                const __nv_bfloat16* __restrict__ v, int64_t q_stride,
                                int64_t k_stride, int64_t v_stride,
                                const int32_t* __restrict__ cu, float scale_log2,
                                __nv_bfloat16* __restrict__ out, int H) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  auto* sq = reinterpret_cast<__nv_bfloat16(*)[kPitch]>(attn_smem);
  auto* sk = sq + NB * kBK;
  auto* sv = sk + NB * kBK;
  const int seq = blockIdx.x;
  const int h = blockIdx.y;
  const int start = cu[seq];
  const int L = cu[seq + 1] - start;
  if (L <= 0) return;
  // Rows past NB * 64 (a sequence longer than the caller's max_seqlen) are
  // not computed, as in varlen_attention_kernel.
  const int nblk = min((L + kBK - 1) / kBK, NB);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __nv_bfloat16* qbase = q + (int64_t)start * q_stride + h * kHD;
  const __nv_bfloat16* kbase = k + (int64_t)start * k_stride + h * kHD;
  const __nv_bfloat16* vbase = v + (int64_t)start * v_stride + h * kHD;
  for (int b = 0; b < nblk; ++b) {
    load_tile_async(sk + b * kBK, kbase, k_stride, b * kBK, L);
    load_tile_async(sv + b * kBK, vbase, v_stride, b * kBK, L);
    load_tile_async(sq + b * kBK, qbase, q_stride, b * kBK, L);
    cp_async_commit();
  }

  for (int qb = 0; qb < nblk; ++qb) {
    // Blocks 0..qb complete: at most nblk-1-qb groups may still be pending.
    switch (nblk - 1 - qb) {
      case 0: cp_async_wait<0>(); break;
      case 1: cp_async_wait<1>(); break;
      case 2: cp_async_wait<2>(); break;
      default: cp_async_wait<3>(); break;
    }
    __syncthreads();
    uint32_t qa[2][4];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk)
      ldsm_x4(qa[kk], &sq[qb * kBQ + warp * 16 + (lane & 15)][kk * 16 + (lane >> 4) * 8]);

    float o[4][4] = {};
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.f, 0.f};
    const int row_a = qb * kBQ + warp * 16 + (lane >> 2);
    const int row_b = row_a + 8;

    for (int kb = 0; kb <= qb; ++kb) {
      const int k0 = kb * kBK;
      float s[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          uint32_t b[4];
          ldsm_x4(b, &sk[k0 + np * 16 + (lane & 7) + ((lane >> 4) << 3)][kk * 16 + ((lane >> 3) & 1) * 8]);
          mma_bf16(s[2 * np], qa[kk], b[0], b[1]);
          mma_bf16(s[2 * np + 1], qa[kk], b[2], b[3]);
        }
      }
      if (kb == qb || k0 + kBK > L) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int key = k0 + nt * 8 + (lane & 3) * 2;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            if (key + e > row_a || key + e >= L) s[nt][e] = -INFINITY;
            if (key + e > row_b || key + e >= L) s[nt][2 + e] = -INFINITY;
          }
        }
      }
      float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        mx[0] = fmaxf(mx[0], fmaxf(s[nt][0], s[nt][1]));
        mx[1] = fmaxf(mx[1], fmaxf(s[nt][2], s[nt][3]));
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      }
      const float off0 = mx[0] == -INFINITY ? 0.f : mx[0] * scale_log2;
      const float off1 = mx[1] == -INFINITY ? 0.f : mx[1] * scale_log2;
      const float corr0 = fast_exp2(m_run[0] == -INFINITY ? -INFINITY : m_run[0] * scale_log2 - off0);
      const float corr1 = fast_exp2(m_run[1] == -INFINITY ? -INFINITY : m_run[1] * scale_log2 - off1);
      m_run[0] = mx[0];
      m_run[1] = mx[1];
      float ls[2] = {0.f, 0.f};
      uint32_t pa[4][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float p0 = fast_exp2(fmaf(s[nt][0], scale_log2, -off0));
        const float p1 = fast_exp2(fmaf(s[nt][1], scale_log2, -off0));
        const float p2 = fast_exp2(fmaf(s[nt][2], scale_log2, -off1));
        const float p3 = fast_exp2(fmaf(s[nt][3], scale_log2, -off1));
        ls[0] += p0 + p1;
        ls[1] += p2 + p3;
        const int ks = nt >> 1, hi = nt & 1;
        pa[ks][hi * 2 + 0] = pack_bf16x2(p0, p1);
        pa[ks][hi * 2 + 1] = pack_bf16x2(p2, p3);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        ls[i] += __shfl_xor_sync(0xffffffffu, ls[i], 1);
        ls[i] += __shfl_xor_sync(0xffffffffu, ls[i], 2);
      }
      l_run[0] = l_run[0] * corr0 + ls[0];
      l_run[1] = l_run[1] * corr1 + ls[1];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        o[nt][0] *= corr0;
        o[nt][1] *= corr0;
        o[nt][2] *= corr1;
        o[nt][3] *= corr1;
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint32_t a[4] = {pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3]};
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t b[4];
          ldsm_x4_t(b, &sv[k0 + ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8][np * 16 + (lane >> 4) * 8]);
          mma_bf16(o[2 * np], a, b[0], b[1]);
          mma_bf16(o[2 * np + 1], a, b[2], b[3]);
        }
      }
    }
    const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
    const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int d = nt * 8 + (lane & 3) * 2;
      if (row_a < L)
        *reinterpret_cast<uint32_t*>(out + ((int64_t)(start + row_a) * H + h) * kHD + d) =
            pack_bf16x2(o[nt][0] * inv0, o[nt][1] * inv0);
      if (row_b < L)
        *reinterpret_cast<uint32_t*>(out + ((int64_t)(start + row_b) * H + h) * kHD + d) =
            pack_bf16x2(o[nt][2] * inv1, o[nt][3] * inv1);
    }
  }
}

template <int NB>
int launch_seq_attention(const void* q, const void* k, const void* v, int64_t qs, int64_t ks,
                         int64_t vs, const int32_t* cu, int num_seqs, int heads, float scale_log2,
                         void* out, cudaStream_t stream) {
  constexpr int kSmem = 3 * NB * kBK * kPitch * (int)sizeof(__nv_bfloat16);
  static uint64_t configured = 0;
  if (ensure_smem_limit(varlen_attention_seq_kernel<NB>, kSmem, configured) != cudaSuccess)
    return CTI_ERR_CUDA;
  varlen_attention_seq_kernel<NB><<<dim3((unsigned)num_seqs, (unsigned)heads), 128, kSmem,
                                    stream>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(v), qs, ks, vs, cu, scale_log2,
      static_cast<__nv_bfloat16*>(out), heads);
  return cudaGetLastError() == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}

}  // namespace
}  // namespace cti

extern "C" int cti_varlen_attention(const void* q_bf16, const void* k_bf16, const void* v_bf16,
                                    int64_t q_stride, int64_t k_stride, int64_t v_stride,
                                    const int32_t* cu_seqlens, int num_seqs, int max_seqlen,
                                    int heads, int head_dim, void* out_bf16, void* stream) {
  using namespace cti;
  if (num_seqs < 0 || max_seqlen < 0 || heads <= 0) return CTI_ERR_INVALID_ARG;
  if (head_dim != kHD) return CTI_ERR_UNSUPPORTED;
  if (num_seqs == 0 || max_seqlen == 0) return CTI_OK;
  if (!q_bf16 || !k_bf16 || !v_bf16 || !cu_seqlens || !out_bf16) return CTI_ERR_INVALID_ARG;
  // 16-byte row pieces: pointers and token strides (in elements) multiples of 8.
  if ((reinterpret_cast<uintptr_t>(q_bf16) | reinterpret_cast<uintptr_t>(k_bf16) |
       reinterpret_cast<uintptr_t>(v_bf16) | reinterpret_cast<uintptr_t>(out_bf16)) & 15)
    return CTI_ERR_INVALID_ARG;
  if ((q_stride | k_stride | v_stride) % 8 != 0 || q_stride < (int64_t)heads * kHD ||
      k_stride < (int64_t)heads * kHD || v_stride < (int64_t)heads * kHD)
    return CTI_ERR_INVALID_ARG;
  const int qblocks = (max_seqlen + kBQ - 1) / kBQ;
  if ((int64_t)num_seqs * qblocks > INT32_MAX || heads > 65535) return CTI_ERR_UNSUPPORTED;
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)kHD);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Sequences of up to 256 tokens: one CTA per (sequence, head), the whole
  // sequence resident in shared memory (15 KB per 64-token block).
  switch (qblocks) {
    case 1: return launch_seq_attention<1>(q_bf16, k_bf16, v_bf16, q_stride, k_stride, v_stride, cu_seqlens, num_seqs, heads, scale_log2, out_bf16, s);
    case 2: return launch_seq_attention<2>(q_bf16, k_bf16, v_bf16, q_stride, k_stride, v_stride, cu_seqlens, num_seqs, heads, scale_log2, out_bf16, s);
    case 3: return launch_seq_attention<3>(q_bf16, k_bf16, v_bf16, q_stride, k_stride, v_stride, cu_seqlens, num_seqs, heads, scale_log2, out_bf16, s);
    case 4: return launch_seq_attention<4>(q_bf16, k_bf16, v_bf16, q_stride, k_stride, v_stride, cu_seqlens, num_seqs, heads, scale_log2, out_bf16, s);
    default: break;
  }
  varlen_attention_kernel<<<dim3((unsigned)(num_seqs * qblocks), (unsigned)heads), 128, 0, s>>>(
      static_cast<const __nv_bfloat16*>(q_bf16), static_cast<const __nv_bfloat16*>(k_bf16),
      static_cast<const __nv_bfloat16*>(v_bf16), q_stride, k_stride, v_stride, cu_seqlens,
      qblocks, scale_log2, static_cast<__nv_bfloat16*>(out_bf16), heads);
  return cudaGetLastError() == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}
