// noalloc.cu — one-token MoE FFN that allocates no device memory.
//
// Who needs it: callers that cannot call cudaMalloc once inference is running.
// Examples are serving loops that reserve all device memory at start-up and
// treat any later allocation as a fault (an allocation can synchronise the
// device and its latency is unbounded), hosts whose device memory is owned by
// their own pool allocator so that a library-side cudaMalloc would bypass its
// accounting, and plugin hosts that forbid the library from allocating at all.
// uocr_moe_forward (the regular entry point) grows a per-context workspace on
// demand; this variant instead uses a fixed scratch array that is part of the
// library image: every GPU that loads the library holds it until the process
// exits.
//
// Contract:
//  * runs the same decode kernel as uocr_moe_forward with tokens == 1, so
//    results are identical; layers outside the fast decode path are rejected
//    with UOCR_ERR_UNSUPPORTED;
//  * the scratch is kNoAllocScratchFloats floats: the intermediate vector h
//    (shared_width + top_k*width floats, at most UOCR_NOALLOC_MAX_H) plus the
//    token's routing, and four words for the kernel's grid barrier; larger
//    layers are rejected with UOCR_ERR_RESOURCE;
//  * set-up happens on the first call on each device: with that device
//    current, the device address of the scratch array is looked up once with
//    cudaGetSymbolAddress and cached.  That first call may load the library's
//    device code, so it should be made before any stream capture begins;
//  * every call on a device shares the one array and the array keeps the last
//    call's contents.  Nothing has to start at zero (the first kernel writes
//    every element of h and of the routing slots before the second reads
//    them), but calls that overlap on the GPU — two streams, or two contexts
//    on the same device running concurrently — race on it.  Serialise them.
//  * the looked-up addresses are cached for the life of the process: the
//    library must not be used across a cudaDeviceReset (or a new primary
//    context) of a device it has served, whose scratch would then be freed
//    memory.
#include <cuda_runtime.h>

#include <cmath>
#include <limits>
#include <mutex>

#include "../../include/uocr_q8.h"
#include "handles.h"
#include "kernels.h"

namespace uocr {
int record_error(int status, const char* message);  // capi.cu
}

namespace {

constexpr size_t kMaxH = UOCR_NOALLOC_MAX_H;
constexpr size_t kRouteSlots = 64;  // ids then weights, top_k <= 8 used
constexpr size_t kNoAllocScratchFloats = kMaxH + 2 * kRouteSlots;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
// The decode kernel's grid-barrier words (arrival count, generation).  They
// start at zero when the library is loaded and the barrier leaves the count
// at zero after every use.
static __device__ __align__(16) unsigned g_noalloc_sync[4];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};
unsigned* g_sync_ptr[kMaxDevices] = {};

// Set-up, once per device, with that device current.
int scratch_address(int device, float** out, unsigned** sync) {
  if (device < 0 || device >= kMaxDevices)
    return uocr::record_error(UOCR_ERR_UNSUPPORTED, "unsupported configuration: device ordinal");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    void* q = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&q, g_noalloc_sync);
    if (e != cudaSuccess || !p || !q)
      return uocr::record_error(UOCR_ERR_CUDA, cudaGetErrorString(e));
    g_scratch_ptr[device] = static_cast<float*>(p);
    g_sync_ptr[device] = static_cast<unsigned*>(q);
  }
  *out = g_scratch_ptr[device];
  *sync = g_sync_ptr[device];
  return UOCR_OK;
}

struct Device {
  int prev = -1;
  explicit Device(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~Device() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int uocr_moe_forward_decode_noalloc(uocr_ctx* ctx, const uocr_moe* layer, int mode,
                                               const float* x_dev, const float* logits_dev,
                                               float* y_dev) {
  using namespace uocr;
  if (!ctx || !layer || !x_dev || !logits_dev || !y_dev)
    return record_error(UOCR_ERR_INVALID, "null argument");
  if (mode != UOCR_WEIGHTS_ONLY && mode != UOCR_DYNAMIC_ACTIVATIONS && mode != UOCR_DYNAMIC_ROWWISE)
    return record_error(UOCR_ERR_UNSUPPORTED, "unsupported configuration: mode");
  if (layer->device != ctx->device)
    return record_error(UOCR_ERR_UNSUPPORTED, "unsupported configuration: layer on another device");
  // The same element-count rule as every other entry point (CpuContext::
  // check_elements): one row through the shared expert's projections.
  const size_t counts[2] = {static_cast<size_t>(layer->shared_width),
                            static_cast<size_t>(layer->hidden)};
  for (size_t c : counts)
    if (c > ctx->scratch_limit / 4)
      return record_error(UOCR_ERR_RESOURCE, "resource limit: operation exceeds scratch limit");

  MoeDecodeArgs a{};
  a.experts = layer->experts_dev;
  a.shared = layer->shared;
  a.n_experts = static_cast<int>(layer->n_experts);
  a.top_k = static_cast<int>(layer->top_k);
  a.normalize = layer->normalize;
  a.scale = layer->scale;
  a.hidden = layer->hidden;
  a.width = layer->width;
  a.shared_width = layer->shared_width;
  const size_t hn = static_cast<size_t>(a.shared_width) + static_cast<size_t>(a.top_k) * a.width;
  if (hn > kMaxH)
    return record_error(UOCR_ERR_RESOURCE,
                        "resource limit: layer needs more than the fixed no-allocation scratch "
                        "(UOCR_NOALLOC_MAX_H floats)");
  if (!layer->aligned || !moe_decode_supported(a, ctx->sms) || reinterpret_cast<uintptr_t>(x_dev) % 16 != 0)
    return record_error(UOCR_ERR_UNSUPPORTED,
                        "unsupported configuration: layer outside the single-token decode kernels");

  Device guard(ctx->device);
  float* scratch = nullptr;
  unsigned* sync = nullptr;
  int st = scratch_address(ctx->device, &scratch, &sync);
  if (st) return st;
  a.x = x_dev;
  a.logits = logits_dev;
  a.h = scratch;
  a.route_ids = reinterpret_cast<int32_t*>(scratch + kMaxH);
  a.route_weights = scratch + kMaxH + kRouteSlots;
  a.y = y_dev;
  a.status = ctx->status_dev;
  a.grid_sync = sync;
  const cudaError_t e =
      launch_moe_decode(mode == UOCR_WEIGHTS_ONLY ? MODE_FP32 : MODE_INT8, a, ctx->sms, ctx->stream);
  if (e != cudaSuccess) return record_error(UOCR_ERR_CUDA, cudaGetErrorString(e));
  const cudaError_t l = cudaGetLastError();
  if (l != cudaSuccess) return record_error(UOCR_ERR_CUDA, cudaGetErrorString(l));
  return UOCR_OK;
}
