// Routing + dispatch with no allocation at all: cti_moe_route_dispatch_noalloc.
//
// cti_moe_router + cti_moe_dispatch need two scratch arrays between them
// (each route's rank inside its 128-token block, and every block's
// per-expert counts), which the normal entry points take from the caller as
// a device workspace.  Some callers cannot provide one: a host that links
// only this C library (a service written against the C ABI, with no CUDA
// allocator of its own and no torch), or an embedding that must run inside a
// fixed, pre-reserved device-memory budget where a cudaMalloc on the
// inference path is not allowed.  This entry point keeps that scratch in a
// file-scope device array instead, so the caller passes only its inputs and
// outputs.
//
// Limits and sharing rules:
//   * T <= CTI_NOALLOC_MAX_TOKENS and E <= CTI_NOALLOC_MAX_EXPERTS; larger
//     problems are rejected with CTI_ERR_UNSUPPORTED before any launch.
//   * The array (1.5 MiB) is part of the library image: every GPU that loads
//     the library holds it until the process exits.
//   * Every call on a device uses the same array, and it keeps whatever the
//     last call left there.  Nothing in it needs to start at zero (the router
//     writes every rank and every block count before dispatch reads them).
//     Calls that overlap on the GPU (two streams, or two host threads
//     launching concurrently on one device) race on the array and produce
//     wrong results; serialise them.
//   * The first call on each device resolves the device address of the array
//     (cudaGetSymbolAddress, with that device current) and caches it together
//     with the CUDA context that was current.  A later call under a different
//     context on that device (a host that creates its own contexts with the
//     driver API) resolves the address again for that context.  Make the
//     first call on each device, and under each such context, before any
//     stream capture there.  After cudaDeviceReset the cache can only tell a
//     new primary context from the old one if the driver gives it a new
//     handle; call this entry point again only after a fresh first call
//     has been made outside any capture.
#include <mutex>

#include <cudaTypedefs.h>

#include "common.cuh"

namespace {

constexpr int64_t kRankInts = (int64_t)CTI_NOALLOC_MAX_TOKENS * 2;
constexpr int64_t kHistInts = ((int64_t)CTI_NOALLOC_MAX_TOKENS + CTI_ROUTER_BLOCK_TOKENS - 1) /
                              CTI_ROUTER_BLOCK_TOKENS * CTI_NOALLOC_MAX_EXPERTS;

// route_rank [T_max, 2] followed by block_hist [ceil(T_max/128), E_max].
static __device__ __align__(256) int32_t g_route_scratch[kRankInts + kHistInts];

constexpr int kMaxDevices = 64;

struct Resolved {
  CUcontext ctx;  // the context that was current when addr was resolved
  int32_t* addr;  // device address of g_route_scratch in that context
};
std::mutex g_mutex;
Resolved g_resolved[kMaxDevices] = {};

// cuCtxGetCurrent, fetched through the runtime's driver entry-point query
// (the library has no link-time dependency on libcuda).
PFN_cuCtxGetCurrent_v4000 ctx_get_current() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  }
  return fn;
}

// Device address of g_route_scratch on the current device under the current
// context: resolved on the first call there and cached per device with the
// context it belongs to.
int32_t* scratch_on_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  auto get_ctx = ctx_get_current();
  if (get_ctx == nullptr) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return nullptr;
  Resolved& r = g_resolved[dev];
  if (ctx != nullptr && r.addr != nullptr && r.ctx == ctx) return r.addr;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_route_scratch) != cudaSuccess || p == nullptr) return nullptr;
  // The runtime makes the device's primary context current if none was.
  if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return nullptr;
  r.ctx = ctx;
  r.addr = static_cast<int32_t*>(p);
  return r.addr;
}

}  // namespace

extern "C" int cti_moe_route_dispatch_noalloc(const void* x_bf16, const float* wg,
                                              const float* bg, int64_t T, int D, int E,
                                              int renorm, int32_t* idx2, float* gate2,
                                              int32_t* offsets, int32_t* perm_inv,
                                              int32_t* sorted_token, void* xperm_bf16,
                                              int32_t* status, void* stream) {
  if (T < 0 || D <= 0 || E < 2) return CTI_ERR_INVALID_ARG;
  if (T > CTI_NOALLOC_MAX_TOKENS || E > CTI_NOALLOC_MAX_EXPERTS) return CTI_ERR_UNSUPPORTED;
  int32_t* scratch = scratch_on_current_device();
  if (scratch == nullptr) return CTI_ERR_CUDA;
  int32_t* route_rank = scratch;
  int32_t* block_hist = scratch + kRankInts;
  int rc = cti_moe_router(x_bf16, wg, bg, T, D, E, renorm, idx2, gate2, route_rank, block_hist,
                          status, stream);
  if (rc != CTI_OK) return rc;
  return cti_moe_dispatch(x_bf16, idx2, route_rank, block_hist, T, D, E, offsets, perm_inv,
                          sorted_token, xperm_bf16, status, stream);
}
