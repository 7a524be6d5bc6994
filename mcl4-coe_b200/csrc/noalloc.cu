// mcl4moe_route_noalloc: the router entry point with its scratch in a fixed
// device array of this library instead of a caller-provided workspace.
//
// Who needs it: callers that have no device allocator of their own to hand a
// workspace from — a C or cgo/JNI client that owns only the activation and
// weight buffers, or a serving loop whose memory pool is sized once at start
// and must not grow (a cudaMalloc there would also synchronise the device and
// stall the pipeline).  Such a caller routes tokens with only its input and
// output buffers.
//
// Set-up: the first call on a device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress, which also loads this
// module onto the device if lazy loading had not done so yet; it is cached per
// device together with the id of the CUDA context it belongs to.  A call in a
// new context on that device (after cudaDeviceReset, say) looks the address up
// again, because the module is loaded afresh there.  Make the first call on a
// device, and the first after a reset, before any stream capture.  After it, a
// call launches the same kernels as mcl4moe_route and allocates nothing.
//
// Limit: the scratch is kRouteStaticScratchBytes (8 MiB); a shape whose route
// workspace is larger is rejected with MCL4MOE_ERR_WORKSPACE before anything
// touches the device.  One scratch array exists per device, so calls on one
// device must not overlap in time (two streams, or two host threads without
// ordering between their streams): overlapping calls race on the scratch.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.cuh"

using namespace mcl4;

namespace {

constexpr size_t kRouteStaticScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_route_scratch[kRouteStaticScratchBytes];

struct ScratchEntry {
  unsigned long long ctx_id;  // context the address belongs to (0: not looked up)
  void* ptr;
};
ScratchEntry g_scratch[kMaxDevices];
std::mutex g_setup_mutex;

// Id of the calling thread's current CUDA context (0 if it cannot be read).
unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  return get_id(ctx, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of this device's scratch array in the current context (looked
// up once per device and context).
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return MCL4MOE_ERR_UNSUPPORTED;
  unsigned long long ctx = current_context_id();  // 0 before the runtime has made a context current
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  ScratchEntry& e = g_scratch[dev];
  if (ctx == 0 || e.ctx_id != ctx || e.ptr == nullptr) {
    void* p = nullptr;
    // Also initialises the device's primary context when no call has done so yet.
    if (cudaGetSymbolAddress(&p, g_route_scratch) != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      return MCL4MOE_ERR_CUDA;
    }
    ctx = current_context_id();
    if (ctx == 0) return MCL4MOE_ERR_CUDA;
    e.ptr = p;
    e.ctx_id = ctx;
  }
  *out = e.ptr;
  return MCL4MOE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

size_t mcl4moe_route_noalloc_scratch_bytes(void) { return kRouteStaticScratchBytes; }

int mcl4moe_route_noalloc(const uint16_t* x, const float* wr, const float* logit_bias, const float* logits_in,
                          const uint8_t* valid, int T, int d, int E, int k, int norm_topk_prob, int32_t* topk_idx,
                          float* topk_w, float* logits_out, float* sel_mask, int32_t* counts, float* stats,
                          mcl4moe_stream_t stream) {
  // Same argument checks as mcl4moe_route.
  if (T < 0 || E <= 0 || k <= 0 || k > E || !topk_idx || !topk_w) return MCL4MOE_ERR_INVALID;
  if (E > kMaxExperts || k > kMaxTopK) return MCL4MOE_ERR_UNSUPPORTED;
  if (int64_t(T) * k > kMaxRoutedSlots) return MCL4MOE_ERR_UNSUPPORTED;
  if (!logits_in) {
    if (!x || !wr || d <= 0) return MCL4MOE_ERR_INVALID;
    if (d % 64 != 0 || !aligned16(x) || !aligned16(wr)) return MCL4MOE_ERR_UNSUPPORTED;
  }
  const int dd = d > 0 ? d : 0;
  if (route_workspace(nullptr, T, E, k, dd).bytes > kRouteStaticScratchBytes) return MCL4MOE_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch);
  if (st != MCL4MOE_OK) return st;
  const RouteWorkspace ws = route_workspace(scratch, T, E, k, dd);
  cudaStream_t s = stream;
  // The scratch keeps the previous call's contents.  Every region is written
  // before it is read, and the one counter that must start at zero (the scan's
  // finished-expert count) is reset by the first kernel of the chain (or, for
  // T = 0, by launch_route itself), so these are exactly mcl4moe_route's launches.
  return launch_route(x, wr, logit_bias, logits_in, valid, T, d, E, k, norm_topk_prob, topk_idx, topk_w, logits_out,
                      sel_mask, counts, stats, nullptr, nullptr, ws, s);
}

}  // extern "C"
