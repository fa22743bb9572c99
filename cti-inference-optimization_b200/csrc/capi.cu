// Library-level entry points: identity, device query, status words, the
// one-call MoE layer (router -> dispatch -> expert FFN -> combine) that
// mirrors SMoE.forward (online_best/infer.py:1910-1954) for C callers, and
// the same layer between host buffers, pipelined over token chunks.
#include <cstring>

#include <vector>

#include "common.cuh"
#include "tmap.cuh"

namespace {

constexpr size_t kAlign = 256;

inline size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

// Workspace carve-up of cti_moe_layer_forward; the same function sizes it
// (base == nullptr) and places the buffers.  The [2T, F] hidden activation
// is reserved only for shapes the fused expert FFN does not take (its
// hidden tile stays on chip).
struct LayerWorkspace {
  int32_t* idx2;
  float* gate2;
  int32_t* rank;
  int32_t* hist;
  int32_t* offsets;
  int32_t* perm_inv;
  int32_t* sorted_token;
  void* xperm;
  void* hidden;  // nullptr when the fused FFN runs
  void* y;
  bool fused;
  size_t bytes;

  LayerWorkspace(void* base, int64_t T, int D, int E, int F) {
    auto* p = static_cast<uint8_t*>(base);
    size_t off = 0;
    auto take = [&](size_t n) -> void* {
      void* r = p ? p + off : nullptr;
      off += align_up(n);
      return r;
    };
    const int64_t R = 2 * T;
    idx2 = static_cast<int32_t*>(take(sizeof(int32_t) * R));
    gate2 = static_cast<float*>(take(sizeof(float) * R));
    rank = static_cast<int32_t*>(take(sizeof(int32_t) * R));
    hist = static_cast<int32_t*>(take(cti_moe_dispatch_workspace_bytes(T, E)));
    offsets = static_cast<int32_t*>(take(sizeof(int32_t) * (E + 1)));
    perm_inv = static_cast<int32_t*>(take(sizeof(int32_t) * R));
    sorted_token = static_cast<int32_t*>(take(sizeof(int32_t) * R));
    xperm = take((size_t)2 * R * D);
    fused = cti_moe_expert_ffn_fused_supported(D, F, E, R) != 0;
    hidden = fused ? nullptr : take((size_t)2 * R * F);
    y = take((size_t)2 * R * D);
    bytes = off;
  }
};

}  // namespace

extern "C" const char* cti_version(void) { return "cti_b200 0.1.0 sm_100a"; }

extern "C" int cti_num_sms(int device, int* num_sms) {
  if (!num_sms) return CTI_ERR_INVALID_ARG;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return CTI_ERR_CUDA;
  *num_sms = n;
  return CTI_OK;
}

namespace cti {
namespace {

// The library's bounded wait (mbar_wait) with a caller-given limit, on a
// barrier whose phase never completes.
__global__ void selftest_wait_kernel(int32_t* status, int64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_barrier_init();
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(&bar, 0)) {
    if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > (uint64_t)limit_ns) {
      raise_status(status, CTI_ERR_TIMEOUT, 0x7f0);
      return;
    }
  }
}

}  // namespace
}  // namespace cti

extern "C" int cti_selftest_wait_timeout(int32_t* status, int64_t limit_ns, void* stream) {
  if (!status || limit_ns < 1000 || limit_ns > 2000000000LL) return CTI_ERR_INVALID_ARG;
  cti::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, limit_ns);
  return cudaGetLastError() == cudaSuccess ? CTI_OK : CTI_ERR_CUDA;
}

extern "C" int cti_status_read(int32_t* status, int clear, int32_t* code, int32_t* detail,
                               void* stream) {
  if (!status) return CTI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t host[2] = {0, 0};
  if (cudaMemcpyAsync(host, status, sizeof(host), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return CTI_ERR_CUDA;
  if (clear && cudaMemsetAsync(status, 0, sizeof(host), s) != cudaSuccess) return CTI_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return CTI_ERR_CUDA;
  if (code) *code = host[0];
  if (detail) *detail = host[1];
  return CTI_OK;
}

extern "C" size_t cti_moe_layer_workspace_bytes(int64_t T, int D, int E, int F) {
  if (T < 0 || D <= 0 || E <= 0 || F <= 0) return 0;
  return LayerWorkspace(nullptr, T, D, E, F).bytes;
}

extern "C" int cti_moe_layer_forward(const void* x_bf16, const float* wg, const float* bg,
                                     const void* W1_bf16, const float* b1, const void* W2_bf16,
                                     const float* b2, int64_t T, int D, int E, int F, int act,
                                     int renorm, void* out_bf16, void* workspace,
                                     size_t workspace_bytes, int32_t* status, void* stream) {
  if (T < 0 || D <= 0 || E < 2 || F <= 0) return CTI_ERR_INVALID_ARG;
  if (T == 0) return CTI_OK;
  if (!workspace || workspace_bytes < cti_moe_layer_workspace_bytes(T, D, E, F))
    return CTI_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0) return CTI_ERR_INVALID_ARG;
  LayerWorkspace ws(workspace, T, D, E, F);
  const int64_t R = 2 * T;
  // The dispatched copy of the rows feeds the fused FFN's TMA loads (measured
  // faster than the fused kernel's in-kernel row gather,
  // cti_moe_expert_ffn_fused_gather, which would skip the copy); shapes the
  // fused kernel does not take run two grouped GEMMs.
  const bool fused = ws.fused;
  int rc = cti_moe_router(x_bf16, wg, bg, T, D, E, renorm, ws.idx2, ws.gate2, ws.rank, ws.hist,
                          status, stream);
  if (rc) return rc;
  rc = cti_moe_dispatch(x_bf16, ws.idx2, ws.rank, ws.hist, T, D, E, ws.offsets, ws.perm_inv,
                        ws.sorted_token, ws.xperm, status, stream);
  if (rc) return rc;
  if (fused) {
    rc = cti_moe_expert_ffn_fused(ws.xperm, W1_bf16, b1, W2_bf16, b2, ws.offsets, E, E, R, D, F,
                                  act, ws.y, status, stream);
  } else {
    rc = cti_moe_grouped_gemm(ws.xperm, W1_bf16, b1, ws.offsets, E, E, R, F, D, act, ws.hidden,
                              status, stream);
    if (rc) return rc;
    rc = cti_moe_grouped_gemm(ws.hidden, W2_bf16, b2, ws.offsets, E, E, R, D, F, CTI_ACT_NONE,
                              ws.y, status, stream);
  }
  if (rc) return rc;
  return cti_moe_combine(ws.y, R, ws.perm_inv, ws.gate2, T, D, out_bf16, status, stream);
}

// The whole layer between pinned host buffers, pipelined over chunks of
// tokens on three streams (four with a second compute stream):
//   copy_in:  H2D of x chunk i            -> record ev_in
//   stream:   wait ev_in; layer on chunk i -> record ev_out
//   copy_out: wait ev_out; D2H of out chunk i
// With compute_stream2, odd chunks' layers run there, on the second half of
// the workspace, so that two chunks' layers overlap: a layer of a few
// thousand tokens fills only part of the GPU and costs ~50 us whatever its
// size, which otherwise sets the pace of small chunks.
// cudaStreamWaitEvent binds to the event's latest record at the time of
// the call, so three events serve every chunk.  Every token's output
// depends only on its own row (router, expert rows and combine are
// per-token), so the result equals one cti_moe_layer_forward over all T.
extern "C" int cti_moe_layer_forward_host(
    const void* x_host, void* out_host, void* x_dev, void* out_dev, const float* wg,
    const float* bg, const void* W1_bf16, const float* b1, const void* W2_bf16, const float* b2,
    int64_t T, int D, int E, int F, int act, int renorm, int64_t chunk_tokens, void* workspace,
    size_t workspace_bytes, int32_t* status, void* stream, void* copy_stream_in,
    void* copy_stream_out, void* compute_stream2) {
  if (T < 0 || D <= 0 || E < 2 || F <= 0 || chunk_tokens <= 0) return CTI_ERR_INVALID_ARG;
  if (T == 0) return CTI_OK;
  if (!x_host || !out_host || !x_dev || !out_dev) return CTI_ERR_INVALID_ARG;
  const int64_t chunk = chunk_tokens < T ? chunk_tokens : T;
  const size_t ws_need = cti_moe_layer_workspace_bytes(chunk, D, E, F);
  const size_t ws_half = align_up(ws_need);  // offset of the second half
  const bool two = compute_stream2 != nullptr;
  if (!workspace || workspace_bytes < (two ? ws_half + ws_need : ws_need))
    return CTI_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaStream_t s2 = two ? static_cast<cudaStream_t>(compute_stream2) : s;
  cudaStream_t s_in = static_cast<cudaStream_t>(copy_stream_in);
  cudaStream_t s_out = static_cast<cudaStream_t>(copy_stream_out);
  const int64_t nchunks = (T + chunk - 1) / chunk;
  if (nchunks > 4096) return CTI_ERR_UNSUPPORTED;
  // ev[0] start, ev[1] out (reused per chunk), ev[2 + i] chunk i copied in.
  std::vector<cudaEvent_t> ev((size_t)nchunks + 2, nullptr);
  for (auto& e : ev)
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      for (auto& d : ev)
        if (d) cudaEventDestroy(d);
      return CTI_ERR_CUDA;
    }
  int rc = CTI_OK;
  auto cuda_ok = [&](cudaError_t err) {
    if (err != cudaSuccess && rc == CTI_OK) rc = CTI_ERR_CUDA;
    return rc == CTI_OK;
  };
  const size_t row_bytes = (size_t)D * 2;
  // The copies start after everything already enqueued on `stream`.
  if (cuda_ok(cudaEventRecord(ev[0], s)) && cuda_ok(cudaStreamWaitEvent(s_in, ev[0], 0)) &&
      cuda_ok(cudaStreamWaitEvent(s_out, ev[0], 0)) && two)
    cuda_ok(cudaStreamWaitEvent(s2, ev[0], 0));
  // Every chunk's copy in first, so that the copy stream runs back to back
  // whatever the host's launch rate for the layers below.
  int64_t copied = 0;
  for (int64_t i = 0; rc == CTI_OK && i < nchunks; ++i) {
    const int64_t t0 = i * chunk;
    const int64_t n = (T - t0) < chunk ? (T - t0) : chunk;
    const size_t off = (size_t)t0 * row_bytes, bytes = (size_t)n * row_bytes;
    if (!cuda_ok(cudaMemcpyAsync(static_cast<uint8_t*>(x_dev) + off,
                                 static_cast<const uint8_t*>(x_host) + off, bytes,
                                 cudaMemcpyHostToDevice, s_in)) ||
        !cuda_ok(cudaEventRecord(ev[2 + i], s_in)))
      break;
    copied = i + 1;
  }
  for (int64_t i = 0; rc == CTI_OK && i < copied; ++i) {
    const int64_t t0 = i * chunk;
    const int64_t n = (T - t0) < chunk ? (T - t0) : chunk;
    const size_t off = (size_t)t0 * row_bytes, bytes = (size_t)n * row_bytes;
    uint8_t* xd = static_cast<uint8_t*>(x_dev) + off;
    uint8_t* od = static_cast<uint8_t*>(out_dev) + off;
    // Layers alternate between the two compute streams and workspace halves;
    // a stream's next layer reuses its half only after its previous one.
    const bool odd = two && (i & 1);
    cudaStream_t sl = odd ? s2 : s;
    void* wsl = odd ? static_cast<void*>(static_cast<uint8_t*>(workspace) + ws_half) : workspace;
    const size_t wsl_bytes = odd ? workspace_bytes - ws_half : (two ? ws_half : workspace_bytes);
    if (!cuda_ok(cudaStreamWaitEvent(sl, ev[2 + i], 0))) break;
    rc = cti_moe_layer_forward(xd, wg, bg, W1_bf16, b1, W2_bf16, b2, n, D, E, F, act, renorm, od,
                               wsl, wsl_bytes, status, sl);
    if (rc != CTI_OK) break;
    if (!cuda_ok(cudaEventRecord(ev[1], sl)) || !cuda_ok(cudaStreamWaitEvent(s_out, ev[1], 0)))
      break;
    cuda_ok(cudaMemcpyAsync(static_cast<uint8_t*>(out_host) + off, od, bytes,
                            cudaMemcpyDeviceToHost, s_out));
  }
  // `stream` resumes after the last copy back and the last copy in (also on
  // an early error, so that nothing enqueued later races the copies already
  // in flight).
  if (cudaEventRecord(ev[1], s_out) == cudaSuccess) cudaStreamWaitEvent(s, ev[1], 0);
  if (cudaEventRecord(ev[0], s_in) == cudaSuccess) cudaStreamWaitEvent(s, ev[0], 0);
  if (two && cudaEventRecord(ev[0], s2) == cudaSuccess) cudaStreamWaitEvent(s, ev[0], 0);
  for (auto& e : ev) cudaEventDestroy(e);
  return rc;
}
