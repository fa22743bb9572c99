// Residual add + LayerNorm over bf16 rows (the pre-LN steps of the CTR
// model around the MoE layer, baseline/infer.py:388-409, and the RepEncoder's
// LayerNorm over 28*64 columns, :264):
//
//   s   = bf16(x + r)                          (r optional; s written if asked)
//   out = bf16((s - mean(s)) * rsqrt(var(s) + eps) * gamma + beta)
//
// with the sum rounded to bf16 before the statistics, as the reference's
// bf16 `residual + y` followed by `nn.LayerNorm` does, and mean / biased
// variance in fp32 (two passes over the row held in registers).
//
// One warp per row; lane l holds the 8-column vectors l, l+32, ... of the
// row, so every load and store is a coalesced 16-byte access.  cols must be
// a multiple of 8, at most 2048; when it is not a multiple of 256 the lanes
// past the row's last vector sit out of the last step.  HBM-bound:
// 2 (or 3, 4) x rows x cols x 2 bytes per launch.
#include "common.cuh"

namespace cti {
namespace {

constexpr int kWarpsPerBlock = 8;

CTI_DEVICE void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

CTI_DEVICE uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

CTI_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int VPL>  // 16-byte vectors per lane = ceil(cols / 256)
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    add_layernorm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ r,
                         const __nv_bfloat16* __restrict__ gamma,
                         const __nv_bfloat16* __restrict__ beta, int64_t rows, int cols,
                         float eps, __nv_bfloat16* __restrict__ sum_out,
                         __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = cols >> 3;  // 16-byte vectors in the row
  // Vector j*32 + lane of the row exists for every j < VPL-1; for the last
  // step only where it is below nvec.
  auto live = [&](int j) { return j < VPL - 1 || j * 32 + lane < nvec; };
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * cols);
  const uint4* rr = r ? reinterpret_cast<const uint4*>(r + row * cols) : nullptr;
  float v[VPL][8];
  uint4 raw[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) raw[j] = live(j) ? __ldg(xr + j * 32 + lane) : make_uint4(0, 0, 0, 0);
  if (rr) {
    uint4 rv[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j)
      rv[j] = live(j) ? __ldg(rr + j * 32 + lane) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      float a[8], b[8];
      unpack8(raw[j], a);
      unpack8(rv[j], b);
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] += b[i];
      raw[j] = pack8(a);  // the bf16 sum is what the statistics see
    }
    if (sum_out) {
      uint4* so = reinterpret_cast<uint4*>(sum_out + row * cols);
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        if (live(j)) so[j * 32 + lane] = raw[j];
    }
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    unpack8(raw[j], v[j]);  // zero for vectors past the row
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[j][i];
  }
  const float inv_c = 1.0f / (float)cols;
  const float mean = warp_sum(s) * inv_c;
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    if (!live(j)) continue;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = v[j][i] - mean;
      q = fmaf(d, d, q);
    }
  }
  const float rstd = rsqrtf(warp_sum(q) * inv_c + eps);
  const uint4* g4 = reinterpret_cast<const uint4*>(gamma);
  const uint4* b4 = reinterpret_cast<const uint4*>(beta);
  uint4* o4 = reinterpret_cast<uint4*>(out + row * cols);
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    if (!live(j)) continue;
    float g[8], b[8], y[8];
    unpack8(__ldg(g4 + j * 32 + lane), g);
    unpack8(__ldg(b4 + j * 32 + lane), b);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = fmaf((v[j][i] - mean) * rstd, g[i], b[i]);
    o4[j * 32 + lane] = pack8(y);
  }
}

template <int VPL>
int launch_ln(const void* x, const void* r, const void* gamma, const void* beta, int64_t rows,
              int cols, float eps, void* sum_out, void* out, cudaStream_t s) {
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (blocks > INT32_MAX) return CTI_ERR_UNSUPPORTED;
  add_layernorm_kernel<VPL><<<(unsigned)blocks, kWarpsPerBlock * 32, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(r),
      static_cast<const __nv_bfloat16*>(gamma), static_cast<const __nv_bfloat16*>(beta), rows,
      cols, eps, static_cast<__nv_bfloat16*>(sum_out), static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace cti

extern "C" int cti_add_layernorm(const void* x_bf16, const void* residual_bf16,
                                 const void* gamma_bf16, const void* beta_bf16, int64_t rows,
                                 int cols, float eps, void* sum_bf16, void* out_bf16,
                                 void* stream) {
  using namespace cti;
  if (rows < 0 || cols <= 0 || !(eps >= 0.0f)) return CTI_ERR_INVALID_ARG;
  if (cols % 8 != 0 || cols > 2048) return CTI_ERR_UNSUPPORTED;
  if (rows == 0) return CTI_OK;
  if (!x_bf16 || !gamma_bf16 || !beta_bf16 || !out_bf16) return CTI_ERR_INVALID_ARG;
  if (sum_bf16 && !residual_bf16) return CTI_ERR_INVALID_ARG;
  const void* ptrs[] = {x_bf16, residual_bf16, gamma_bf16, beta_bf16, sum_bf16, out_bf16};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return CTI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch ((cols + 255) / 256) {
    case 1: return launch_ln<1>(x_bf16, residual_bf16, gamma_bf16, beta_bf16, rows, cols, eps, sum_bf16, out_bf16, s);
    case 2: return launch_ln<2>(x_bf16, residual_bf16, gamma_bf16, beta_bf16, rows, cols, eps, sum_bf16, out_bf16, s);
    case 3: return launch_ln<3>(x_bf16, residual_bf16, gamma_bf16, beta_bf16, rows, cols, eps, sum_bf16, out_bf16, s);
    case 4: return launch_ln<4>(x_bf16, residual_bf16, gamma_bf16, beta_bf16, rows, cols, eps, sum_bf16, out_bf16, s);
    case 5: return launch_ln<5>(x_bf16, residual_bf16, gamma_bf16, beta_bf16, rows, cols, eps, sum_bf16, out_bf16, s);
    case 6: return launch_ln<6>(x_bf16, residual_bf16, gamma_bf16, beta_bf16, rows, cols, eps, sum_bf16, out_bf16, s);
    case 7: return launch_ln<7>(x_bf16, residual_bf16, gamma_bf16, beta_bf16, rows, cols, eps, sum_bf16, out_bf16, s);
    default: return launch_ln<8>(x_bf16, residual_bf16, gamma_bf16, beta_bf16, rows, cols, eps, sum_bf16, out_bf16, s);
  }
}
