// Stage 5: the 28-feature embedding-bag sum pooling.
//
// Restates the pooling of RepEncoder.forward (baseline/infer.py:253-263:
// per slot, rows emb(values.clamp(0, V-1)) summed by segment_reduce) and the
// fused_all_slots_embedding_kernel of online_best/infer.py:793-827 (one bag
// per (sample, slot), sequential fp32 accumulation over the bag), over the
// reference's flat 3-tensor batch layout (_flat_values, _flat_row_offsets,
// _val_offsets; online_best/infer.py:130-182, :1029-1033), with one table
// region per feature.
//
// HBM-bound gather.  A group of LPB lanes owns one bag; each lane owns
// VEC 16-byte slices (8 fp16 each) of the row, so a 64-wide fp16 row (128 B,
// one cache line) is read by 8 lanes with one 16-byte load each.  Ids are
// fetched UNROLL at a time and their rows loaded before any of them is
// accumulated, so several row fetches are in flight per lane; the sum itself
// still runs in bag order, element by element, in fp32, which keeps the
// result bit-identical to a sequential fp32 sum.
#include "common.cuh"

namespace cti {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

template <int DIM>
struct EmbCfg {
  static constexpr int LPB = (DIM / 8) < 32 ? (DIM / 8) : 32;  // lanes per bag
  static constexpr int VEC = DIM / 8 / LPB;                     // 16-byte slices per lane
  static constexpr int BAGS_PER_BLOCK = kThreads / LPB;
};

template <typename OutT>
CTI_DEVICE void store8(OutT* dst, const float* v);

template <>
CTI_DEVICE void store8<float>(float* dst, const float* v) {
  float4* d = reinterpret_cast<float4*>(dst);
  d[0] = make_float4(v[0], v[1], v[2], v[3]);
  d[1] = make_float4(v[4], v[5], v[6], v[7]);
}

template <>
CTI_DEVICE void store8<__nv_bfloat16>(__nv_bfloat16* dst, const float* v) {
  uint4 r;
  r.x = pack_bf16x2(v[0], v[1]);
  r.y = pack_bf16x2(v[2], v[3]);
  r.z = pack_bf16x2(v[4], v[5]);
  r.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(dst) = r;
}

template <>
CTI_DEVICE void store8<__half>(__half* dst, const float* v) {
  uint4 r;
  __half2 h[4] = {__floats2half2_rn(v[0], v[1]), __floats2half2_rn(v[2], v[3]),
                  __floats2half2_rn(v[4], v[5]), __floats2half2_rn(v[6], v[7])};
  r = *reinterpret_cast<uint4*>(h);
  *reinterpret_cast<uint4*>(dst) = r;
}

CTI_DEVICE void accumulate8(float* acc, const uint4& raw) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]);
    acc[2 * j] += f.x;
    acc[2 * j + 1] += f.y;
  }
}

template <int DIM, typename OutT>
__global__ void __launch_bounds__(kThreads) embbag_kernel(
    const int64_t* __restrict__ values, int64_t n_values, const int64_t* __restrict__ row_offsets,
    const int64_t* __restrict__ val_offsets, const int64_t* __restrict__ table_row_base,
    const int64_t* __restrict__ vocab, const __half* __restrict__ table, int64_t table_rows,
    int64_t B, int F, OutT* __restrict__ out, int32_t* status) {
  using C = EmbCfg<DIM>;
  const int sub = threadIdx.x % C::LPB;
  const int64_t bag = (int64_t)blockIdx.x * C::BAGS_PER_BLOCK + threadIdx.x / C::LPB;
  if (bag >= B * F) return;
  // Feature-major: the bags of one block are consecutive samples of ONE
  // feature, so a block reads one contiguous range of ids and gathers rows
  // from one table (fewer pages and L2 sets per block; at 204 M ids this is
  // 1.9x faster than the sample-major order, at cfg3 1.5x).
  const int f = (int)(bag / B);
  const int64_t b = bag - (int64_t)f * B;

  const int64_t* roff = row_offsets + (int64_t)f * (B + 1);
  const int64_t start = roff[b];
  const int64_t end = roff[b + 1];
  const int64_t vbase = val_offsets[f];
  const int64_t rbase = table_row_base[f];
  const int64_t vmax = vocab[f] - 1;

  float acc[C::VEC][8];
#pragma unroll
  for (int v = 0; v < C::VEC; ++v)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[v][j] = 0.0f;

  bool ok = start <= end && start >= 0 && vbase >= 0 && vbase + end <= n_values && vmax >= 0 &&
            rbase >= 0 && rbase + vmax < table_rows;
  if (!ok) {
    if (sub == 0) raise_status(status, CTI_ERR_BOUNDS, (int32_t)bag);
  } else {
    const int64_t* vals = values + vbase;
    int64_t i = start;
    for (; i + kUnroll <= end; i += kUnroll) {
      uint4 raw[kUnroll][C::VEC];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        int64_t id = __ldg(vals + i + u);
        id = id < 0 ? 0 : (id > vmax ? vmax : id);
        const uint4* row = reinterpret_cast<const uint4*>(table + (rbase + id) * DIM);
#pragma unroll
        for (int v = 0; v < C::VEC; ++v) raw[u][v] = __ldg(row + v * C::LPB + sub);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
#pragma unroll
        for (int v = 0; v < C::VEC; ++v) accumulate8(acc[v], raw[u][v]);
    }
    for (; i < end; ++i) {
      int64_t id = __ldg(vals + i);
      id = id < 0 ? 0 : (id > vmax ? vmax : id);
      const uint4* row = reinterpret_cast<const uint4*>(table + (rbase + id) * DIM);
#pragma unroll
      for (int v = 0; v < C::VEC; ++v) accumulate8(acc[v], __ldg(row + v * C::LPB + sub));
    }
  }

  OutT* o = out + b * ((int64_t)F * DIM) + (int64_t)f * DIM;
#pragma unroll
  for (int v = 0; v < C::VEC; ++v) store8<OutT>(o + (v * C::LPB + sub) * 8, acc[v]);
}

template <int DIM>
int launch_embbag(const int64_t* values, int64_t n_values, const int64_t* row_offsets,
                  const int64_t* val_offsets, const int64_t* table_row_base,
                  const int64_t* vocab, const __half* table, int64_t table_rows, int64_t B,
                  int F, void* out, int out_dtype, int32_t* status, cudaStream_t s) {
  using C = EmbCfg<DIM>;
  const int64_t bags = B * F;
  const int64_t blocks = (bags + C::BAGS_PER_BLOCK - 1) / C::BAGS_PER_BLOCK;
  if (blocks > INT32_MAX) return CTI_ERR_UNSUPPORTED;
  if (out_dtype == CTI_DTYPE_F32)
    embbag_kernel<DIM, float><<<(unsigned)blocks, kThreads, 0, s>>>(
        values, n_values, row_offsets, val_offsets, table_row_base, vocab, table, table_rows, B,
        F, static_cast<float*>(out), status);
  else if (out_dtype == CTI_DTYPE_BF16)
    embbag_kernel<DIM, __nv_bfloat16><<<(unsigned)blocks, kThreads, 0, s>>>(
        values, n_values, row_offsets, val_offsets, table_row_base, vocab, table, table_rows, B,
        F, static_cast<__nv_bfloat16*>(out), status);
  else if (out_dtype == CTI_DTYPE_F16)
    embbag_kernel<DIM, __half><<<(unsigned)blocks, kThreads, 0, s>>>(
        values, n_values, row_offsets, val_offsets, table_row_base, vocab, table, table_rows, B,
        F, static_cast<__half*>(out), status);
  else
    return CTI_ERR_INVALID_ARG;
  return cudaGetLastError() == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}

}  // namespace
}  // namespace cti

extern "C" int cti_embbag_sum(const int64_t* values, int64_t n_values, const int64_t* row_offsets,
                              const int64_t* val_offsets, const int64_t* table_row_base,
                              const int64_t* vocab, const void* table_f16, int64_t table_rows,
                              int64_t B, int F, int dim, void* out, int out_dtype,
                              int32_t* status, void* stream) {
  using namespace cti;
  if (B < 0 || F <= 0 || n_values < 0 || table_rows < 0) return CTI_ERR_INVALID_ARG;
  if (B == 0) return CTI_OK;
  if (!row_offsets || !val_offsets || !table_row_base || !vocab || !table_f16 || !out)
    return CTI_ERR_INVALID_ARG;
  if (n_values > 0 && !values) return CTI_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(table_f16) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return CTI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* tab = static_cast<const __half*>(table_f16);
  switch (dim) {
    case 32:
      return launch_embbag<32>(values, n_values, row_offsets, val_offsets, table_row_base, vocab,
                               tab, table_rows, B, F, out, out_dtype, status, s);
    case 64:
      return launch_embbag<64>(values, n_values, row_offsets, val_offsets, table_row_base, vocab,
                               tab, table_rows, B, F, out, out_dtype, status, s);
    case 128:
      return launch_embbag<128>(values, n_values, row_offsets, val_offsets, table_row_base,
                                vocab, tab, table_rows, B, F, out, out_dtype, status, s);
    case 256:
      return launch_embbag<256>(values, n_values, row_offsets, val_offsets, table_row_base,
                                vocab, tab, table_rows, B, F, out, out_dtype, status, s);
    case 512:
      return launch_embbag<512>(values, n_values, row_offsets, val_offsets, table_row_base,
                                vocab, tab, table_rows, B, F, out, out_dtype, status, s);
    default:
      return CTI_ERR_UNSUPPORTED;
  }
}
