// capi.cu — the C ABI declared in include/uocr_q8.h.
//
// Host-side validation restates the reference's checks (file:line beside each
// rule) so that every entry point fails with the same OcrError variant as the
// Rust method it replaces.  Device work is enqueued on the context's stream;
// *_host entry points copy in, run and copy out synchronously, like the
// reference's Tensor-in / Tensor-out methods.
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <limits>
#include <string>
#include <vector>

#include "../../include/uocr_q8.h"
#include "common.cuh"
#include "kernels.h"

using namespace uocr;

#include "handles.h"

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int ok() { return UOCR_OK; }

#define CUDA_TRY(expr)                                                                  \
  do {                                                                                  \
    cudaError_t e_ = (expr);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return fail(UOCR_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                  __LINE__);                                                            \
  } while (0)

// Switches to the context's device for the lifetime of a call.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

bool mul_ok(size_t a, size_t b, size_t* out) {
  if (a != 0 && b > std::numeric_limits<size_t>::max() / a) return false;
  *out = a * b;
  return true;
}

size_t nblocks(size_t cols) { return (cols + kBlock - 1) / kBlock; }

// CpuContext::check_elements (src/cpu/mod.rs:73-78).
int check_elements(const uocr_ctx* ctx, size_t count) {
  size_t bytes;
  if (!mul_ok(count, 4, &bytes) || bytes > ctx->scratch_limit)
    return fail(UOCR_ERR_RESOURCE, "resource limit: operation exceeds scratch limit");
  return ok();
}

int ensure_ws(uocr_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->ws_bytes) return ok();
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  if (ctx->ws) CUDA_TRY(cudaFree(ctx->ws));
  ctx->ws = nullptr;
  ctx->ws_bytes = 0;
  size_t want = bytes + (bytes >> 2);
  want = (want + 0xFFFFF) & ~static_cast<size_t>(0xFFFFF);
  CUDA_TRY(cudaMalloc(&ctx->ws, want));
  ctx->ws_bytes = want;
  return ok();
}

int ensure_pinned(uocr_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->pinned_bytes) return ok();
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  if (ctx->pinned) CUDA_TRY(cudaFreeHost(ctx->pinned));
  ctx->pinned = nullptr;
  ctx->pinned_bytes = 0;
  size_t want = (bytes + 0xFFFF) & ~static_cast<size_t>(0xFFFF);
  CUDA_TRY(cudaMallocHost(&ctx->pinned, want));
  ctx->pinned_bytes = want;
  return ok();
}

bool is_pinned(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// Maps a device status word to the reference's error variants (clearing the
// context's word when it is set).
int status_result(uocr_ctx* ctx, unsigned st) {
  if (!st) return ok();
  CUDA_TRY(cudaMemsetAsync(ctx->status_dev, 0, sizeof(unsigned), ctx->stream));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  if (st & DEV_TIMEOUT) return fail(UOCR_ERR_TIMEOUT, "a bounded device wait expired");
  if (st & DEV_NONFINITE)
    return fail(UOCR_ERR_NUMERICAL, "nonfinite numerical input: nonfinite quantization input");
  if (st & DEV_UNDERFLOW) return fail(UOCR_ERR_NUMERICAL, "nonfinite numerical input: INT8 scale underflow");
  if (st & DEV_BAD_SCALE)
    return fail(UOCR_ERR_NUMERICAL,
                "nonfinite numerical input: INT8 scales must be finite and nonnegative");
  if (st & DEV_SOFTMAX)
    return fail(UOCR_ERR_NUMERICAL, "nonfinite numerical input: invalid or fully masked softmax row");
  if (st & DEV_RANGE) return fail(UOCR_ERR_FORMAT, "invalid checkpoint: INT8 byte -128");
  if (st & DEV_BAD_ROUTE) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid expert routing");
  if (st & DEV_CAPACITY)
    return fail(UOCR_ERR_RESOURCE, "resource limit exceeded: expert dispatch capacity");
  if (st & DEV_NORM) return fail(UOCR_ERR_NUMERICAL, "nonfinite numerical input: normalization");
  if (st & DEV_POSITION) return fail(UOCR_ERR_RESOURCE, "resource limit: maximum context exceeded");
  if (st & DEV_CACHE) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: cache must be prefilled");
  return fail(UOCR_ERR_CUDA, "unknown device status 0x%x", st);
}

// Reads (synchronously) and maps the context's device status word.
int take_device_status(uocr_ctx* ctx) {
  CUDA_TRY(cudaMemcpyAsync(ctx->status_host, ctx->status_dev, sizeof(unsigned),
                           cudaMemcpyDeviceToHost, ctx->stream));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return status_result(ctx, *ctx->status_host);
}

int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return ok();
}

Q8View view(const uocr_q8* m) {
  return Q8View{m->w, m->s, static_cast<int>(m->rows), static_cast<int>(m->cols)};
}

bool fits_int(size_t v) { return v <= static_cast<size_t>(std::numeric_limits<int>::max()); }

// Host-tensor shape rules shared by the *_host entry points.
int tensor_len(const size_t* shape, size_t ndim, size_t* len) {
  size_t n = 1;
  for (size_t i = 0; i < ndim; ++i)
    if (!mul_ok(n, shape[i], &n)) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: element count overflow");
  *len = n;
  return ok();
}

}  // namespace

namespace uocr {
// Error reporting for entry points defined in other translation units.
int record_error(int status, const char* message) {
  g_last_error = message ? message : "";
  return status;
}
}  // namespace uocr

// ===========================================================================
extern "C" {

int uocr_abi_version(void) { return UOCR_Q8_ABI_VERSION; }

const char* uocr_last_error(void) { return g_last_error.c_str(); }

const char* uocr_status_name(int status) {
  switch (status) {
    case UOCR_OK: return "Ok";
    case UOCR_ERR_IO: return "Io";
    case UOCR_ERR_JSON: return "Json";
    case UOCR_ERR_FORMAT: return "Format";
    case UOCR_ERR_SHAPE: return "Shape";
    case UOCR_ERR_UNSUPPORTED: return "Unsupported";
    case UOCR_ERR_RESOURCE: return "Resource";
    case UOCR_ERR_NUMERICAL: return "Numerical";
    case UOCR_ERR_CUDA: return "Cuda";
    case UOCR_ERR_NCCL: return "Nccl";
    case UOCR_ERR_TIMEOUT: return "Timeout";
    case UOCR_ERR_INVALID: return "Invalid";
    default: return "Unknown";
  }
}

// ---- context ---------------------------------------------------------------
int uocr_ctx_create(int device, size_t scratch_limit, uocr_ctx** out) {
  if (!out) return fail(UOCR_ERR_INVALID, "null output");
  *out = nullptr;
  // CpuContext::new (src/cpu/mod.rs:27-31)
  if (scratch_limit == 0)
    return fail(UOCR_ERR_RESOURCE, "resource limit: threads and scratch limit must be nonzero");
  int count = 0;
  CUDA_TRY(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: no CUDA device %d", device);
  cudaDeviceProp prop{};
  CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: sm_%d%d is not sm_100",
                prop.major, prop.minor);
  DeviceGuard g(device);
  auto* c = new uocr_ctx();
  c->device = device;
  c->sms = prop.multiProcessorCount;
  c->scratch_limit = scratch_limit;
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&c->status_dev, 256);
  if (e == cudaSuccess) e = cudaMemset(c->status_dev, 0, 256);
  if (e == cudaSuccess) e = cudaMallocHost(&c->status_host, sizeof(unsigned) * 4);
  int least_priority = 0, greatest_priority = 0;
  if (e == cudaSuccess) e = cudaDeviceGetStreamPriorityRange(&least_priority, &greatest_priority);
  if (e == cudaSuccess)
    e = cudaStreamCreateWithPriority(&c->side_stream, cudaStreamNonBlocking, greatest_priority);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    uocr_ctx_destroy(c);
    return fail(UOCR_ERR_CUDA, "context: %s", cudaGetErrorString(e));
  }
  c->own_stream = true;
  *out = c;
  return ok();
}

int uocr_ctx_destroy(uocr_ctx* ctx) {
  if (!ctx) return ok();
  DeviceGuard g(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  for (auto& hg : ctx->host_graphs)
    if (hg.exec) cudaGraphExecDestroy(hg.exec);
  if (ctx->capture_stream) cudaStreamDestroy(ctx->capture_stream);
  if (ctx->side_stream) {
    cudaStreamSynchronize(ctx->side_stream);
    cudaStreamDestroy(ctx->side_stream);
  }
  if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
  if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->io) cudaFree(ctx->io);
  if (ctx->pinned) cudaFreeHost(ctx->pinned);
  if (ctx->status_dev) cudaFree(ctx->status_dev);
  if (ctx->status_host) cudaFreeHost(ctx->status_host);
  if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return ok();
}

int uocr_ctx_set_stream(uocr_ctx* ctx, void* stream) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  DeviceGuard g(ctx->device);
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  ctx->own_stream = false;
  ctx->stream = static_cast<cudaStream_t>(stream);
  return ok();
}

int uocr_ctx_sync(uocr_ctx* ctx) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  DeviceGuard g(ctx->device);
  CUDA_TRY(cudaGetLastError());
  return take_device_status(ctx);
}

int uocr_ctx_set_wait_limit(uocr_ctx* ctx, uint64_t ns) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  if (ns > (uint64_t{1} << 40))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: wait limit above 1099 s");
  ctx->wait_ns = ns;
  return ok();
}

int uocr_ctx_hold_decode_barrier(uocr_ctx* ctx, int hold) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  ctx->hold_barrier = hold ? 1 : 0;
  return ok();
}

int uocr_ctx_device(const uocr_ctx* ctx, int* device, int* sm_count) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  if (device) *device = ctx->device;
  if (sm_count) *sm_count = ctx->sms;
  return ok();
}

// ---- matrices --------------------------------------------------------------
int uocr_q8_from_parts(uocr_ctx* ctx, size_t rows, size_t cols, const int8_t* weights,
                       size_t weights_len, const float* scales, size_t scales_len,
                       uocr_q8** out) {
  if (!ctx || !out) return fail(UOCR_ERR_INVALID, "null argument");
  *out = nullptr;
  // src/cpu/quantized.rs:24-30
  size_t n, ns;
  if (rows == 0 || cols == 0 || !mul_ok(rows, cols, &n) || n != weights_len ||
      !mul_ok(rows, nblocks(cols), &ns) || ns != scales_len)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: INT8 matrix storage");
  if (!weights || !scales) return fail(UOCR_ERR_INVALID, "null storage");
  // src/cpu/quantized.rs:31-35 (so -0.0 passes)
  for (size_t i = 0; i < scales_len; ++i)
    if (!std::isfinite(scales[i]) || scales[i] < 0.0f)
      return fail(UOCR_ERR_NUMERICAL,
                  "nonfinite numerical input: INT8 scales must be finite and nonnegative");
  if (!fits_int(rows) || !fits_int(cols))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: matrix extent above 2^31");
  DeviceGuard g(ctx->device);
  auto* m = new uocr_q8();
  m->device = ctx->device;
  m->rows = rows;
  m->cols = cols;
  m->owns = true;
  cudaError_t e = cudaMalloc(&m->w, (n + 15) & ~static_cast<size_t>(15));
  if (e == cudaSuccess) e = cudaMalloc(&m->s, ns * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpy(m->w, weights, n, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(m->s, scales, ns * sizeof(float), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    uocr_q8_free(m);
    return fail(UOCR_ERR_CUDA, "from_parts: %s", cudaGetErrorString(e));
  }
  *out = m;
  return ok();
}

int uocr_q8_from_device(uocr_ctx* ctx, size_t rows, size_t cols, const int8_t* weights_dev,
                        const float* scales_dev, uocr_q8** out) {
  if (!ctx || !out) return fail(UOCR_ERR_INVALID, "null argument");
  *out = nullptr;
  size_t n, ns;
  if (rows == 0 || cols == 0 || !mul_ok(rows, cols, &n) || !mul_ok(rows, nblocks(cols), &ns))
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: INT8 matrix storage");
  if (!weights_dev || !scales_dev) return fail(UOCR_ERR_INVALID, "null storage");
  if (!fits_int(rows) || !fits_int(cols))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: matrix extent above 2^31");
  DeviceGuard g(ctx->device);
  int st = take_device_status(ctx);
  if (st) return st;
  launch_validate_q8(weights_dev, static_cast<long long>(n), scales_dev,
                     static_cast<long long>(ns), 0, ctx->status_dev, ctx->sms, ctx->stream);
  if ((st = check_launch())) return st;
  if ((st = take_device_status(ctx))) return st;
  auto* m = new uocr_q8();
  m->device = ctx->device;
  m->rows = rows;
  m->cols = cols;
  m->w = const_cast<int8_t*>(weights_dev);
  m->s = const_cast<float*>(scales_dev);
  m->owns = false;
  *out = m;
  return ok();
}

int uocr_q8_quantize(uocr_ctx* ctx, size_t rows, size_t cols, const float* values,
                     uocr_q8** out) {
  if (!ctx || !out) return fail(UOCR_ERR_INVALID, "null argument");
  *out = nullptr;
  // src/cpu/quantized.rs:45-49
  size_t n;
  if (rows == 0 || cols == 0 || !mul_ok(rows, cols, &n))
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: quantization expects a nonempty matrix");
  if (!values) return fail(UOCR_ERR_INVALID, "null values");
  if (!fits_int(rows) || !fits_int(cols))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: matrix extent above 2^31");
  DeviceGuard g(ctx->device);
  int st = take_device_status(ctx);
  if (st) return st;
  if ((st = ensure_ws(ctx, n * sizeof(float)))) return st;
  auto* m = new uocr_q8();
  m->device = ctx->device;
  m->rows = rows;
  m->cols = cols;
  m->owns = true;
  const size_t ns = rows * nblocks(cols);
  cudaError_t e = cudaMalloc(&m->w, (n + 15) & ~static_cast<size_t>(15));
  if (e == cudaSuccess) e = cudaMalloc(&m->s, ns * sizeof(float));
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(ctx->ws, values, n * sizeof(float), cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) {
    uocr_q8_free(m);
    return fail(UOCR_ERR_CUDA, "quantize: %s", cudaGetErrorString(e));
  }
  launch_quantize_rows(static_cast<const float*>(ctx->ws), static_cast<long long>(cols),
                       static_cast<int>(rows), static_cast<int>(cols), m->w, m->s, ctx->status_dev,
                       ctx->sms, ctx->stream);
  if ((st = check_launch()) || (st = take_device_status(ctx))) {
    uocr_q8_free(m);
    return st;
  }
  *out = m;
  return ok();
}

int uocr_q8_free(uocr_q8* m) {
  if (!m) return ok();
  DeviceGuard g(m->device);
  if (m->owns) {
    if (m->w) cudaFree(m->w);
    if (m->s) cudaFree(m->s);
  }
  delete m;
  return ok();
}

int uocr_q8_shape(const uocr_q8* m, size_t* rows, size_t* cols) {
  if (!m) return fail(UOCR_ERR_INVALID, "null matrix");
  if (rows) *rows = m->rows;
  if (cols) *cols = m->cols;
  return ok();
}

size_t uocr_q8_storage_bytes(const uocr_q8* m) {
  // src/cpu/quantized.rs:96-98
  return m ? m->rows * m->cols + m->rows * nblocks(m->cols) * 4 : 0;
}

int uocr_q8_device_ptrs(const uocr_q8* m, const int8_t** w, const float** s) {
  if (!m) return fail(UOCR_ERR_INVALID, "null matrix");
  if (w) *w = m->w;
  if (s) *s = m->s;
  return ok();
}

int uocr_q8_download(uocr_ctx* ctx, const uocr_q8* m, int8_t* weights, float* scales) {
  if (!ctx || !m) return fail(UOCR_ERR_INVALID, "null argument");
  DeviceGuard g(ctx->device);
  if (weights)
    CUDA_TRY(cudaMemcpyAsync(weights, m->w, m->rows * m->cols, cudaMemcpyDeviceToHost, ctx->stream));
  if (scales)
    CUDA_TRY(cudaMemcpyAsync(scales, m->s, m->rows * nblocks(m->cols) * 4, cudaMemcpyDeviceToHost,
                             ctx->stream));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return ok();
}

int uocr_q8_dequantize(uocr_ctx* ctx, const uocr_q8* m, float* out_dev) {
  if (!ctx || !m || !out_dev) return fail(UOCR_ERR_INVALID, "null argument");
  DeviceGuard g(ctx->device);
  launch_dequantize(m->w, m->s, static_cast<int>(m->rows), static_cast<int>(m->cols), out_dev,
                    ctx->sms, ctx->stream);
  return check_launch();
}

int uocr_q8_dequantize_host(uocr_ctx* ctx, const uocr_q8* m, float* out, size_t out_len) {
  if (!ctx || !m || !out) return fail(UOCR_ERR_INVALID, "null argument");
  const size_t n = m->rows * m->cols;
  if (out_len != n) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: output length");
  DeviceGuard g(ctx->device);
  int st = ensure_ws(ctx, n * 4);
  if (st) return st;
  launch_dequantize(m->w, m->s, static_cast<int>(m->rows), static_cast<int>(m->cols),
                    static_cast<float*>(ctx->ws), ctx->sms, ctx->stream);
  if ((st = check_launch())) return st;
  CUDA_TRY(cudaMemcpyAsync(out, ctx->ws, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
  return take_device_status(ctx);
}

// Int8Matrix::linear element-count rules (src/cpu/quantized.rs:104-115).
static int linear_checks(const uocr_ctx* ctx, const uocr_q8* m, size_t batch) {
  size_t count;
  if (!mul_ok(batch, m->rows, &count))
    return fail(UOCR_ERR_RESOURCE, "resource limit: INT8 output overflow");
  int st = check_elements(ctx, count);
  if (st) return st;
  if (batch != 1) {
    const size_t w = m->rows * m->cols;
    if (w > std::numeric_limits<size_t>::max() - count)
      return fail(UOCR_ERR_RESOURCE, "resource limit: INT8 scratch overflow");
    if ((st = check_elements(ctx, w + count))) return st;
  }
  return ok();
}

// linear_dynamic_int8 scratch rule (src/cpu/quantized.rs:162-168).
static int dynamic_checks(const uocr_ctx* ctx, const uocr_q8* m) {
  return check_elements(ctx, m->cols * 2 + m->rows + nblocks(m->cols));
}

// Which kernel a linear of `batch` rows runs on: the GEMV kernels for one
// row; for 2..kSmallRowsMax rows the warp-level kernel that streams the
// weights once; beyond that the tensor-core GEMMs.  int8 activations are
// bit-exact on every path; FP32 activations go to the warp-level and
// tensor-core kernels as exact bf16 pieces (FP32 tolerance).
enum class LinearPath { Gemv, SmallInt8, SmallFp32, TcInt8, TcFp32 };

static LinearPath linear_path(const uocr_q8* m, int mode, size_t batch) {
  const bool aligned = reinterpret_cast<uintptr_t>(m->w) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(m->s) % 16 == 0;
  const int rows = static_cast<int>(m->rows), cols = static_cast<int>(m->cols);
  if (batch < 2 || !aligned) return LinearPath::Gemv;
  // up to 16 rows, or up to 64 rows of a matrix small enough that its
  // re-reads by the 8-row chunks come from L2: the warp-level kernel
  const bool small_matrix = static_cast<size_t>(rows) * cols <= (size_t(16) << 20);
  if (batch <= static_cast<size_t>(kSmallRowsMax) || (batch <= 64 && small_matrix)) {
    if (small_rows_supported(rows, cols))
      return mode == MODE_INT8 ? LinearPath::SmallInt8 : LinearPath::SmallFp32;
    if (batch <= static_cast<size_t>(kSmallRowsMax)) return LinearPath::Gemv;
  }
  if (!q8_tc_supported(rows, cols)) return LinearPath::Gemv;
  return mode == MODE_INT8 ? LinearPath::TcInt8 : LinearPath::TcFp32;
}

static size_t al256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

// Device scratch of a linear: quantized rows and their scales, or the pieces.
static size_t linear_scratch_bytes(const uocr_q8* m, int mode, size_t batch) {
  const LinearPath path = linear_path(m, mode, batch);
  if (path == LinearPath::TcFp32 || path == LinearPath::SmallFp32)
    return al256(3 * batch * m->cols * 2) + al256(batch * 4);
  if (mode == MODE_INT8) return al256(batch * m->cols) + al256(batch * nblocks(m->cols) * 4);
  return 0;
}

// x_dev rows of m->cols floats (16-byte aligned for the tensor-core paths),
// y_dev rows of m->rows; `scratch` holds linear_scratch_bytes.
static int linear_launch(uocr_ctx* ctx, const uocr_q8* m, int mode, const float* x_dev,
                         size_t batch, float* y_dev, char* scratch) {
  const int b = static_cast<int>(batch);
  LinearPath path = linear_path(m, mode, batch);
  // the pieces are read as float4 rows
  if ((path == LinearPath::TcFp32 || path == LinearPath::SmallFp32) &&
      reinterpret_cast<uintptr_t>(x_dev) % 16 != 0)
    path = LinearPath::Gemv;
  const Q8View v = view(m);
  if (path == LinearPath::TcFp32 || path == LinearPath::SmallFp32) {
    uint16_t* pieces = reinterpret_cast<uint16_t*>(scratch);
    float* rinv = reinterpret_cast<float*>(scratch + al256(3 * batch * m->cols * 2));
    launch_split_rows(x_dev, static_cast<long long>(m->cols), nullptr, b, static_cast<int>(m->cols),
                      pieces, rinv, ctx->sms, ctx->stream);
    const cudaError_t e =
        path == LinearPath::TcFp32
            ? launch_q8_tc_single_f32(v, pieces, rinv, b, y_dev, static_cast<long long>(m->rows),
                                      ctx->status_dev, ctx->stream)
            : launch_small_rows(false, nullptr, &v, nullptr, nullptr, 1, 1, kSmallRowsMax, b,
                                v.rows, v.cols, pieces, b, rinv, nullptr, nullptr, b, y_dev,
                                static_cast<long long>(m->rows), ctx->status_dev, ctx->stream);
    if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "tensor-core linear: %s", cudaGetErrorString(e));
    return check_launch();
  }
  int8_t* xq = nullptr;
  float* xs = nullptr;
  if (mode == MODE_INT8) {
    xq = reinterpret_cast<int8_t*>(scratch);
    xs = reinterpret_cast<float*>(scratch + al256(batch * m->cols));
  }
  if (path == LinearPath::TcInt8 || path == LinearPath::SmallInt8) {
    // several rows: quantize them, then a tensor-core kernel (bit-exact)
    launch_quantize_rows(x_dev, static_cast<long long>(m->cols), b, static_cast<int>(m->cols), xq,
                         xs, ctx->status_dev, ctx->sms, ctx->stream);
    const cudaError_t e =
        path == LinearPath::TcInt8
            ? launch_q8_tc_single_i8(v, xq, xs, b, y_dev, static_cast<long long>(m->rows),
                                     ctx->status_dev, ctx->stream)
            : launch_small_rows(true, nullptr, &v, nullptr, nullptr, 1, 1, kSmallRowsMax, b,
                                v.rows, v.cols, nullptr, 0, nullptr, xq, xs, b, y_dev,
                                static_cast<long long>(m->rows), ctx->status_dev, ctx->stream);
    if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "tensor-core linear: %s", cudaGetErrorString(e));
    return check_launch();
  }
  launch_gemv(mode, v, x_dev, static_cast<long long>(m->cols), b, y_dev,
              static_cast<long long>(m->rows), xq, xs, ctx->status_dev, ctx->sms, ctx->stream);
  return check_launch();
}

static int run_linear(uocr_ctx* ctx, const uocr_q8* m, int mode, const float* x_dev, size_t batch,
                      float* y_dev) {
  if (batch == 0) return ok();
  if (!fits_int(batch)) return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: batch");
  int st = ensure_ws(ctx, linear_scratch_bytes(m, mode, batch));
  if (st) return st;
  return linear_launch(ctx, m, mode, x_dev, batch, y_dev, static_cast<char*>(ctx->ws));
}

int uocr_q8_linear(uocr_ctx* ctx, const uocr_q8* m, const float* x_dev, size_t batch,
                   float* y_dev) {
  if (!ctx || !m || (batch && (!x_dev || !y_dev))) return fail(UOCR_ERR_INVALID, "null argument");
  int st = linear_checks(ctx, m, batch);
  if (st) return st;
  DeviceGuard g(ctx->device);
  return run_linear(ctx, m, MODE_FP32, x_dev, batch, y_dev);
}

int uocr_q8_linear_dynamic_int8(uocr_ctx* ctx, const uocr_q8* m, const float* x_dev,
                                size_t batch, float* y_dev) {
  if (!ctx || !m || (batch && (!x_dev || !y_dev))) return fail(UOCR_ERR_INVALID, "null argument");
  int st = dynamic_checks(ctx, m);
  if (st) return st;
  DeviceGuard g(ctx->device);
  return run_linear(ctx, m, MODE_INT8, x_dev, batch, y_dev);
}

// Copies x in, runs, copies y out (through pinned staging unless the caller's
// buffers are already pinned), synchronises and reports device errors.
static int host_linear(uocr_ctx* ctx, const uocr_q8* m, int mode, const float* x, size_t batch,
                       float* y) {
  const size_t xn = batch * m->cols, yn = batch * m->rows;
  const size_t xb = al256(xn * 4), yb = al256(yn * 4);
  int st = take_device_status(ctx);
  if (st) return st;
  if ((st = ensure_ws(ctx, xb + yb + linear_scratch_bytes(m, mode, batch)))) return st;
  float* xd = static_cast<float*>(ctx->ws);
  float* yd = reinterpret_cast<float*>(static_cast<char*>(ctx->ws) + xb);
  char* scratch = static_cast<char*>(ctx->ws) + xb + yb;
  const bool xp = is_pinned(x), yp = is_pinned(y);
  if ((!xp || !yp) && (st = ensure_pinned(ctx, (xp ? 0 : xn * 4) + (yp ? 0 : yn * 4) + 256)))
    return st;
  float* xs_h = xp ? const_cast<float*>(x) : static_cast<float*>(ctx->pinned);
  float* ys_h = yp ? y : reinterpret_cast<float*>(static_cast<char*>(ctx->pinned) +
                                                  ((xp ? 0 : xn * 4) + 255) / 256 * 256);
  if (!xp) std::memcpy(xs_h, x, xn * 4);
  CUDA_TRY(cudaMemcpyAsync(xd, xs_h, xn * 4, cudaMemcpyHostToDevice, ctx->stream));
  if ((st = linear_launch(ctx, m, mode, xd, batch, yd, scratch))) return st;
  CUDA_TRY(cudaMemcpyAsync(ys_h, yd, yn * 4, cudaMemcpyDeviceToHost, ctx->stream));
  st = take_device_status(ctx);
  if (st) return st;
  if (!yp) std::memcpy(y, ys_h, yn * 4);
  return ok();
}

int uocr_q8_linear_host(uocr_ctx* ctx, const uocr_q8* m, const float* x, const size_t* x_shape,
                        size_t ndim, float* y, size_t y_len) {
  if (!ctx || !m || (ndim && !x_shape)) return fail(UOCR_ERR_INVALID, "null argument");
  // src/cpu/quantized.rs:101-103
  if (ndim == 0 || x_shape[ndim - 1] != m->cols)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: INT8 linear input width");
  size_t len;
  int st = tensor_len(x_shape, ndim, &len);
  if (st) return st;
  const size_t batch = len / m->cols;
  if ((st = linear_checks(ctx, m, batch))) return st;
  if (y_len != batch * m->rows) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: output length");
  if (batch == 0) return ok();
  if (!x || !y) return fail(UOCR_ERR_INVALID, "null buffer");
  DeviceGuard g(ctx->device);
  return host_linear(ctx, m, MODE_FP32, x, batch, y);
}

int uocr_q8_linear_dynamic_int8_host(uocr_ctx* ctx, const uocr_q8* m, const float* x,
                                     const size_t* x_shape, size_t ndim, float* y,
                                     size_t y_len) {
  if (!ctx || !m || (ndim && !x_shape)) return fail(UOCR_ERR_INVALID, "null argument");
  size_t len;
  int st = tensor_len(x_shape, ndim, &len);
  if (st) return st;
  // src/cpu/quantized.rs:157-161
  if (ndim == 0 || x_shape[ndim - 1] != m->cols || len != m->cols)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: dynamic INT8 requires one input row");
  if ((st = dynamic_checks(ctx, m))) return st;
  if (y_len != m->rows) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: output length");
  if (!x || !y) return fail(UOCR_ERR_INVALID, "null buffer");
  DeviceGuard g(ctx->device);
  return host_linear(ctx, m, MODE_INT8, x, 1, y);
}

int uocr_q8_quantize_rows(uocr_ctx* ctx, const float* x_dev, size_t rows, size_t cols,
                          int8_t* q_dev, float* s_dev) {
  if (!ctx || (rows && cols && (!x_dev || !q_dev || !s_dev)))
    return fail(UOCR_ERR_INVALID, "null argument");
  if (rows == 0 || cols == 0)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: quantization expects a nonempty matrix");
  if (!fits_int(rows) || !fits_int(cols))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: matrix extent above 2^31");
  DeviceGuard g(ctx->device);
  launch_quantize_rows(x_dev, static_cast<long long>(cols), static_cast<int>(rows),
                       static_cast<int>(cols), q_dev, s_dev, ctx->status_dev, ctx->sms,
                       ctx->stream);
  return check_launch();
}

int uocr_q8_linear_multi(uocr_ctx* ctx, const uocr_q8* const* mats, size_t n, int mode,
                         const float* x_dev, float* const* y_dev) {
  if (!ctx || !mats || !y_dev || !x_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (n == 0) return ok();
  if (mode != UOCR_WEIGHTS_ONLY && mode != UOCR_DYNAMIC_ACTIVATIONS && mode != UOCR_DYNAMIC_ROWWISE)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: mode %d", mode);
  std::vector<Q8View> v(n);
  for (size_t i = 0; i < n; ++i) {
    if (!mats[i] || !y_dev[i]) return fail(UOCR_ERR_INVALID, "null matrix or output");
    if (mats[i]->cols != mats[0]->cols)
      return fail(UOCR_ERR_SHAPE, "invalid tensor shape: INT8 linear input width");
    v[i] = view(mats[i]);
  }
  DeviceGuard g(ctx->device);
  const int dmode = mode == UOCR_WEIGHTS_ONLY ? MODE_FP32 : MODE_INT8;
  bool fast = reinterpret_cast<uintptr_t>(x_dev) % 16 == 0;
  for (size_t i = 0; i < n; ++i) fast = fast && gemv_fast_path_ok(v[i]);
  if (fast) {
    launch_gemv_multi(dmode, v.data(), static_cast<int>(n), x_dev, y_dev, ctx->status_dev,
                      ctx->sms, ctx->stream);
    return check_launch();
  }
  for (size_t i = 0; i < n; ++i) {
    int st = run_linear(ctx, mats[i], dmode, x_dev, 1, y_dev[i]);
    if (st) return st;
  }
  return ok();
}

// ---- routing -----------------------------------------------------------------
static int route_checks(size_t n_experts, size_t top_k, float scale) {
  // src/decoder/moe.rs:13-15
  if (top_k == 0 || top_k > n_experts || !std::isfinite(scale) || scale <= 0.0f)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid expert routing");
  if (n_experts > 1024 || top_k > 32)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: routing extent");
  return ok();
}

int uocr_moe_route(uocr_ctx* ctx, const float* logits_dev, size_t tokens, size_t n_experts,
                   size_t top_k, int normalize, float scale, int32_t* ids_dev,
                   float* weights_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  int st = route_checks(n_experts, top_k, scale);
  if (st) return st;
  if (tokens == 0) return ok();
  if (!logits_dev || !ids_dev || !weights_dev) return fail(UOCR_ERR_INVALID, "null argument");
  DeviceGuard g(ctx->device);
  launch_route(logits_dev, static_cast<int>(tokens), static_cast<int>(n_experts),
               static_cast<int>(top_k), normalize, scale, ids_dev, weights_dev, ctx->status_dev,
               ctx->sms, ctx->stream);
  return check_launch();
}

// ---- MoE layer ---------------------------------------------------------------
int uocr_moe_create(uocr_ctx* ctx, const uocr_q8* shared_gate, const uocr_q8* shared_up,
                    const uocr_q8* shared_down, const uocr_q8* const* gate,
                    const uocr_q8* const* up, const uocr_q8* const* down, size_t n_experts,
                    size_t top_k, int normalize_topk, float routed_scale, uocr_moe** out) {
  if (!ctx || !out || !shared_gate || !shared_up || !shared_down || !gate || !up || !down)
    return fail(UOCR_ERR_INVALID, "null argument");
  *out = nullptr;
  if (n_experts == 0) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: no routed experts");
  int st = route_checks(n_experts, top_k, routed_scale);
  if (st) return st;
  if (top_k > 8 || n_experts > 256)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: top_k <= 8, experts <= 256");
  const size_t H = shared_gate->cols, FS = shared_gate->rows;
  // Decoder::new shape expectations (src/decoder/mod.rs:58-80)
  auto expect = [&](const uocr_q8* m, size_t r, size_t c, const char* what) -> int {
    if (!m) return fail(UOCR_ERR_INVALID, "null %s", what);
    if (m->device != ctx->device)
      return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: %s on another device", what);
    if (m->rows != r || m->cols != c)
      return fail(UOCR_ERR_SHAPE, "invalid tensor shape: %s: expected [%zu, %zu], got [%zu, %zu]",
                  what, r, c, m->rows, m->cols);
    return ok();
  };
  if ((st = expect(shared_up, FS, H, "shared_experts.up_proj")) ||
      (st = expect(shared_down, H, FS, "shared_experts.down_proj")))
    return st;
  if (!gate[0]) return fail(UOCR_ERR_INVALID, "null experts.0.gate_proj");
  const size_t F = gate[0]->rows;
  std::vector<FfnView> views(n_experts);
  bool aligned = true;
  auto al = [](const uocr_q8* m) {
    return reinterpret_cast<uintptr_t>(m->w) % 16 == 0 && reinterpret_cast<uintptr_t>(m->s) % 16 == 0;
  };
  for (size_t e = 0; e < n_experts; ++e) {
    if ((st = expect(gate[e], F, H, "experts.gate_proj")) ||
        (st = expect(up[e], F, H, "experts.up_proj")) ||
        (st = expect(down[e], H, F, "experts.down_proj")))
      return st;
    views[e] = FfnView{view(gate[e]), view(up[e]), view(down[e])};
    aligned = aligned && al(gate[e]) && al(up[e]) && al(down[e]);
  }
  aligned = aligned && al(shared_gate) && al(shared_up) && al(shared_down);
  DeviceGuard g(ctx->device);
  static std::atomic<uint64_t> next_serial{1};
  auto* L = new uocr_moe();
  L->serial = next_serial.fetch_add(1);
  L->device = ctx->device;
  L->n_experts = n_experts;
  L->top_k = top_k;
  L->normalize = normalize_topk ? 1 : 0;
  L->scale = routed_scale;
  L->hidden = static_cast<int>(H);
  L->width = static_cast<int>(F);
  L->shared_width = static_cast<int>(FS);
  L->shared = FfnView{view(shared_gate), view(shared_up), view(shared_down)};
  L->aligned = aligned;
  cudaError_t e = cudaMalloc(&L->experts_dev, sizeof(FfnView) * n_experts);
  if (e == cudaSuccess)
    e = cudaMemcpy(L->experts_dev, views.data(), sizeof(FfnView) * n_experts,
                   cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    uocr_moe_free(L);
    return fail(UOCR_ERR_CUDA, "moe_create: %s", cudaGetErrorString(e));
  }
  // TMA maps for the tensor-core prefill, when every matrix qualifies
  if (aligned && q8_tc_supported(static_cast<int>(F), static_cast<int>(H)) &&
      q8_tc_supported(static_cast<int>(H), static_cast<int>(F))) {
    const size_t mb = q8_tc_maps_bytes();
    std::vector<unsigned char> maps(3 * n_experts * mb);
    bool made = true;
    for (size_t i = 0; i < n_experts && made; ++i) {
      const Q8View m3[3] = {views[i].gate, views[i].up, views[i].down};
      for (int j = 0; j < 3 && made; ++j)
        made = q8_tc_weight_maps(maps.data() + (j * n_experts + i) * mb, m3[j]);
    }
    if (!made || cudaMalloc(&L->tc_maps, maps.size()) != cudaSuccess ||
        cudaMemcpy(L->tc_maps, maps.data(), maps.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaGetLastError();
      if (L->tc_maps) cudaFree(L->tc_maps);
      L->tc_maps = nullptr;
    }
  }
  *out = L;
  return ok();
}

int uocr_moe_free(uocr_moe* layer) {
  if (!layer) return ok();
  DeviceGuard g(layer->device);
  if (layer->experts_dev) cudaFree(layer->experts_dev);
  if (layer->tc_maps) cudaFree(layer->tc_maps);
  delete layer;
  return ok();
}

// Reference element-count checks for the shared expert's projections at
// `tokens` rows; the routed groups (<= tokens rows, width <= shared width)
// are bounded by them.
static int moe_checks(const uocr_ctx* ctx, const uocr_moe* L, size_t tokens) {
  const size_t H = L->hidden, FS = L->shared_width;
  const size_t counts[2] = {tokens * FS, tokens * H};
  const size_t mats[2] = {FS * H, H * FS};
  for (int i = 0; i < 2; ++i) {
    int st = check_elements(ctx, counts[i]);
    if (st) return st;
    if (tokens != 1 && (st = check_elements(ctx, counts[i] + mats[i]))) return st;
  }
  return ok();
}

// Arguments of the one-token decode kernel, and whether the layer and x
// qualify for it.  Its workspace: h, plus the routing when the caller does
// not want it back.
static bool decode_args(const uocr_ctx* ctx, const uocr_moe* L, const float* x, MoeDecodeArgs* a) {
  *a = MoeDecodeArgs{};
  a->experts = L->experts_dev;
  a->shared = L->shared;
  a->n_experts = static_cast<int>(L->n_experts);
  a->top_k = static_cast<int>(L->top_k);
  a->normalize = L->normalize;
  a->scale = L->scale;
  a->hidden = L->hidden;
  a->width = L->width;
  a->shared_width = L->shared_width;
  return L->aligned && moe_decode_supported(*a, ctx->sms) &&
         reinterpret_cast<uintptr_t>(x) % 16 == 0;
}

static size_t decode_h_bytes(int shared_width, int top_k, int width) {
  const size_t hn = static_cast<size_t>(shared_width) + static_cast<size_t>(top_k) * width;
  return (hn * 4 + 255) & ~static_cast<size_t>(255);
}

// Launches the decode kernel with `a` from decode_args (workspace present).
static int decode_launch(uocr_ctx* ctx, int mode, MoeDecodeArgs& a, const float* x,
                         const float* logits, float* y, int32_t* ids, float* wts, bool pdl) {
  const size_t hb = decode_h_bytes(a.shared_width, a.top_k, a.width);
  const bool own_route = !ids || !wts;
  a.x = x;
  a.logits = logits;
  a.h = static_cast<float*>(ctx->ws);
  a.route_ids = own_route ? reinterpret_cast<int32_t*>(static_cast<char*>(ctx->ws) + hb) : ids;
  a.route_weights = own_route ? reinterpret_cast<float*>(static_cast<char*>(ctx->ws) + hb + 256)
                              : wts;
  a.y = y;
  a.status = ctx->status_dev;
  a.grid_sync = ctx->status_dev + 16;  // zeroed at context creation, decode-only
  // nanoseconds to SM cycles at the 1.965 GHz maximum clock, rounded up (a
  // lower clock only lengthens the wait)
  a.wait_cycles = ctx->wait_ns ? static_cast<long long>(ctx->wait_ns * 2) : 0;
  a.barrier_extra = ctx->hold_barrier ? 1u : 0u;
  cudaError_t e = launch_moe_decode(mode == UOCR_WEIGHTS_ONLY ? MODE_FP32 : MODE_INT8, a, ctx->sms,
                                    ctx->stream, pdl);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "moe decode launch: %s", cudaGetErrorString(e));
  return check_launch();
}

static int moe_run(uocr_ctx* ctx, const uocr_moe* L, int mode, const float* x, const float* logits,
                   size_t tokens, float* y, int32_t* ids, float* wts) {
  const int k = static_cast<int>(L->top_k);
  // decode fast path: one token, every projection single-row
  if (tokens == 1) {
    MoeDecodeArgs a;
    if (decode_args(ctx, L, x, &a)) {
      int st = ensure_ws(ctx, decode_h_bytes(a.shared_width, a.top_k, a.width) + 512);
      if (st) return st;
      return decode_launch(ctx, mode, a, x, logits, y, ids, wts, true);
    }
  }
  MoePrefillArgs a{};
  a.experts = L->experts_dev;
  a.shared = L->shared;
  a.n_experts = static_cast<int>(L->n_experts);
  a.top_k = k;
  a.normalize = L->normalize;
  a.scale = L->scale;
  a.hidden = L->hidden;
  a.width = L->width;
  a.shared_width = L->shared_width;
  a.tokens = static_cast<int>(tokens);
  a.x = x;
  a.logits = logits;
  a.y = y;
  a.status = ctx->status_dev;
  a.tc_maps = L->tc_maps;
  const size_t rb = (tokens * k * 4 + 255) & ~static_cast<size_t>(255);
  const bool own_route = !ids || !wts;
  const size_t need = moe_prefill_workspace(a, mode) + (own_route ? 2 * rb : 0) + 256;
  int st = ensure_ws(ctx, need);
  if (st) return st;
  char* base = static_cast<char*>(ctx->ws);
  if (own_route) {
    a.route_ids = reinterpret_cast<int32_t*>(base);
    a.route_weights = reinterpret_cast<float*>(base + rb);
    base += 2 * rb;
  } else {
    a.route_ids = ids;
    a.route_weights = wts;
  }
  a.workspace = base;
  a.workspace_bytes = ctx->ws_bytes - (base - static_cast<char*>(ctx->ws));
  a.side = ctx->side_stream;
  a.ev_fork = ctx->ev_fork;
  a.ev_join = ctx->ev_join;
  cudaError_t e = launch_moe_prefill(mode, a, ctx->sms, ctx->stream);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "moe prefill launch: %s", cudaGetErrorString(e));
  return check_launch();
}

int uocr_moe_forward(uocr_ctx* ctx, const uocr_moe* layer, int mode, const float* x_dev,
                     const float* logits_dev, size_t tokens, float* y_dev, int32_t* ids_dev,
                     float* weights_dev) {
  if (!ctx || !layer) return fail(UOCR_ERR_INVALID, "null argument");
  if (mode != UOCR_WEIGHTS_ONLY && mode != UOCR_DYNAMIC_ACTIVATIONS && mode != UOCR_DYNAMIC_ROWWISE)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: mode %d", mode);
  if (layer->device != ctx->device)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: layer on another device");
  if (tokens == 0) return ok();
  if (!x_dev || !logits_dev || !y_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(tokens * layer->top_k)) return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: tokens");
  int st = moe_checks(ctx, layer, tokens);
  if (st) return st;
  DeviceGuard g(ctx->device);
  return moe_run(ctx, layer, mode, x_dev, logits_dev, tokens, y_dev, ids_dev, weights_dev);
}

// One part of the layer over `rows` rows: the routed experts (expert_ids
// given, outputs in row order) or the shared expert (into y).
static int moe_part(uocr_ctx* ctx, const uocr_moe* L, int mode, const float* x, size_t rows,
                    const int32_t* expert_ids, float* out, bool routed) {
  if (!ctx || !L) return fail(UOCR_ERR_INVALID, "null argument");
  if (mode != UOCR_WEIGHTS_ONLY && mode != UOCR_DYNAMIC_ACTIVATIONS && mode != UOCR_DYNAMIC_ROWWISE)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: mode %d", mode);
  if (L->device != ctx->device)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: layer on another device");
  if (rows == 0) return ok();
  if (!x || !out || (routed && !expert_ids)) return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(rows)) return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: rows");
  int st = moe_checks(ctx, L, rows);
  if (st) return st;
  if (routed && (st = check_elements(ctx, rows * L->width))) return st;
  DeviceGuard g(ctx->device);
  MoePrefillArgs a{};
  a.experts = L->experts_dev;
  a.shared = L->shared;
  a.n_experts = static_cast<int>(L->n_experts);
  a.top_k = 1;  // one (row, expert) pair per row
  a.scale = 1.0f;
  a.hidden = L->hidden;
  a.width = L->width;
  a.shared_width = L->shared_width;
  a.tokens = static_cast<int>(rows);
  a.x = x;
  a.status = ctx->status_dev;
  a.tc_maps = L->tc_maps;
  a.route_given = 1;
  if (routed) {
    a.skip_shared = 1;
    a.pair_out = out;
    a.skip_negative_ids = 1;  // padding rows of a fixed-capacity dispatch
  } else {
    a.skip_routed = 1;
    a.y = out;
  }
  const size_t rb = (rows * 4 + 255) & ~static_cast<size_t>(255);
  const size_t need = moe_prefill_workspace(a, mode) + rb + 256;
  if ((st = ensure_ws(ctx, need))) return st;
  char* base = static_cast<char*>(ctx->ws);
  // grouping reads a weight per pair; the routed part never applies it
  a.route_ids = const_cast<int32_t*>(expert_ids);
  a.route_weights = reinterpret_cast<float*>(base);
  a.workspace = base + rb;
  a.workspace_bytes = ctx->ws_bytes - rb;
  cudaError_t e = launch_moe_prefill(mode, a, ctx->sms, ctx->stream);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "moe part launch: %s", cudaGetErrorString(e));
  return check_launch();
}

int uocr_moe_expert_rows(uocr_ctx* ctx, const uocr_moe* layer, int mode, const float* x_dev,
                         const int32_t* expert_ids_dev, size_t rows, float* out_dev) {
  return moe_part(ctx, layer, mode, x_dev, rows, expert_ids_dev, out_dev, true);
}

int uocr_moe_shared_rows(uocr_ctx* ctx, const uocr_moe* layer, int mode, const float* x_dev,
                         size_t rows, float* y_dev) {
  return moe_part(ctx, layer, mode, x_dev, rows, nullptr, y_dev, false);
}

int uocr_moe_dispatch(uocr_ctx* ctx, const float* x_dev, size_t tokens, size_t hidden,
                      const int32_t* ids_dev, size_t top_k, const int32_t* rank_bounds,
                      size_t world, size_t capacity, float* send_x_dev, int32_t* send_ids_dev,
                      int32_t* pair_rows_dev) {
  if (!ctx || !rank_bounds) return fail(UOCR_ERR_INVALID, "null argument");
  if (world < 1 || world > static_cast<size_t>(kMaxDispatchRanks))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: 1 <= world <= %d", kMaxDispatchRanks);
  if (top_k == 0 || top_k > 8 || hidden == 0 || hidden % 4)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: top_k <= 8, hidden % 4 == 0");
  if (capacity == 0 || !fits_int(world * capacity) || !fits_int(tokens * top_k))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: capacity");
  int bounds[kMaxDispatchRanks + 1];
  for (size_t r = 0; r <= world; ++r) {
    bounds[r] = rank_bounds[r];
    if (r > 0 && bounds[r] <= bounds[r - 1])
      return fail(UOCR_ERR_SHAPE, "invalid tensor shape: rank bounds must increase");
  }
  if (bounds[0] != 0) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: rank bounds start at 0");
  if (!send_ids_dev || (tokens && (!x_dev || !ids_dev || !send_x_dev || !pair_rows_dev)))
    return fail(UOCR_ERR_INVALID, "null argument");
  DeviceGuard g(ctx->device);
  const cudaError_t e = launch_moe_dispatch(
      x_dev, static_cast<int>(tokens), static_cast<int>(hidden), ids_dev, static_cast<int>(top_k),
      bounds[world], bounds, static_cast<int>(world), static_cast<int>(capacity), send_x_dev,
      send_ids_dev, pair_rows_dev, ctx->status_dev, ctx->stream);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "dispatch launch: %s", cudaGetErrorString(e));
  return check_launch();
}

int uocr_moe_combine_rows(uocr_ctx* ctx, const int32_t* ids_dev, const float* weights_dev,
                          const float* rows_dev, const int32_t* pair_rows_dev, size_t tokens,
                          size_t top_k, size_t hidden, float* y_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null argument");
  if (top_k == 0 || top_k > 8) return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: top_k <= 8");
  if (tokens == 0 || hidden == 0) return ok();
  if (!ids_dev || !weights_dev || !rows_dev || !pair_rows_dev || !y_dev)
    return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(tokens * top_k) || !fits_int(hidden))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: tokens");
  DeviceGuard g(ctx->device);
  launch_moe_combine_rows(ids_dev, weights_dev, rows_dev, pair_rows_dev, static_cast<int>(tokens),
                          static_cast<int>(top_k), static_cast<int>(hidden), y_dev, ctx->stream);
  return check_launch();
}

int uocr_moe_combine(uocr_ctx* ctx, const int32_t* ids_dev, const float* weights_dev,
                     const float* pair_out_dev, size_t tokens, size_t top_k, size_t hidden,
                     float* y_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null argument");
  if (top_k == 0 || top_k > 8) return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: top_k <= 8");
  if (tokens == 0 || hidden == 0) return ok();
  if (!ids_dev || !weights_dev || !pair_out_dev || !y_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(tokens * top_k) || !fits_int(hidden))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: tokens");
  DeviceGuard g(ctx->device);
  launch_moe_combine_pairs(ids_dev, weights_dev, pair_out_dev, static_cast<int>(tokens),
                           static_cast<int>(top_k), static_cast<int>(hidden), y_dev, ctx->stream);
  return check_launch();
}

// The host-buffer decode call as one captured graph per (layer, mode,
// buffers): copy [x | logits] in, the decode kernel, copy y (and the routing)
// and the status word out.  One launch and one synchronisation per call
// instead of four enqueues.  *done
// is false when the layer does not take the decode kernel or capture is not
// available; the caller then runs the eager path.
constexpr size_t kMaxHostGraphs = 8;

static int host_decode_graph(uocr_ctx* ctx, const uocr_moe* L, int mode, size_t xb, size_t lb,
                             size_t yb, size_t rb, bool outs, bool* done) {
  *done = false;
  HostDecodeGraph* g = nullptr;
  for (auto& e : ctx->host_graphs)
    if (e.layer == L && e.serial == L->serial && e.mode == mode && e.outs == outs &&
        e.io == ctx->io && e.ws == ctx->ws && e.pinned == ctx->pinned) {
      g = &e;
      break;
    }
  if (!g || !g->exec) {
    // the first call for a key runs eagerly (sizing the workspace, configuring
    // the kernel); the second captures the graph
    if (!g) {
      if (ctx->host_graphs.size() >= kMaxHostGraphs) {
        if (ctx->host_graphs.front().exec) cudaGraphExecDestroy(ctx->host_graphs.front().exec);
        ctx->host_graphs.erase(ctx->host_graphs.begin());
      }
      HostDecodeGraph seen;
      seen.layer = L;
      seen.serial = L->serial;
      seen.mode = mode;
      seen.outs = outs;
      seen.io = ctx->io;
      seen.ws = ctx->ws;
      seen.pinned = ctx->pinned;
      ctx->host_graphs.push_back(seen);
      return ok();
    }
    char* d = static_cast<char*>(ctx->io);
    const float* xd = reinterpret_cast<const float*>(d);
    MoeDecodeArgs a;
    if (!decode_args(ctx, L, xd, &a)) return ok();
    int st = ensure_ws(ctx, decode_h_bytes(a.shared_width, a.top_k, a.width) + 512);
    if (st) return st;
    char* hp = static_cast<char*>(ctx->pinned);
    if (!ctx->capture_stream)
      CUDA_TRY(cudaStreamCreateWithFlags(&ctx->capture_stream, cudaStreamNonBlocking));
    cudaStream_t saved = ctx->stream;
    ctx->stream = ctx->capture_stream;
    cudaGraph_t graph = nullptr;
    int lst = UOCR_OK;
    cudaError_t e = cudaStreamBeginCapture(ctx->capture_stream, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      e = cudaMemcpyAsync(d, hp, xb + L->n_experts * 4, cudaMemcpyHostToDevice,
                          ctx->capture_stream);
      if (e == cudaSuccess)
        lst = decode_launch(ctx, mode, a, xd, reinterpret_cast<const float*>(d + xb),
                            reinterpret_cast<float*>(d + xb + lb),
                            outs ? reinterpret_cast<int32_t*>(d + xb + lb + yb) : nullptr,
                            outs ? reinterpret_cast<float*>(d + xb + lb + yb + rb) : nullptr,
                            false);
      // outputs back by one copy node (a measured 4 us faster than the kernel
      // storing them into pinned memory itself)
      if (e == cudaSuccess && !lst)
        e = cudaMemcpyAsync(hp + xb + lb, d + xb + lb,
                            outs ? yb + rb + L->top_k * 4 : static_cast<size_t>(L->hidden) * 4,
                            cudaMemcpyDeviceToHost, ctx->capture_stream);
      if (e == cudaSuccess && !lst)
        e = cudaMemcpyAsync(ctx->status_host, ctx->status_dev, sizeof(unsigned),
                            cudaMemcpyDeviceToHost, ctx->capture_stream);
      const cudaError_t e2 = cudaStreamEndCapture(ctx->capture_stream, &graph);
      if (e == cudaSuccess) e = e2;
    }
    ctx->stream = saved;
    cudaGraphExec_t exec = nullptr;
    if (e == cudaSuccess && !lst && graph) e = cudaGraphInstantiate(&exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (e != cudaSuccess || lst || !exec) {
      cudaGetLastError();
      if (exec) cudaGraphExecDestroy(exec);
      return ok();
    }
    g->ws = ctx->ws;  // ensure_ws above may have grown it
    g->exec = exec;
  }
  CUDA_TRY(cudaGraphLaunch(g->exec, ctx->stream));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  int st = status_result(ctx, *ctx->status_host);
  if (st) return st;
  *done = true;
  return ok();
}

int uocr_moe_forward_host(uocr_ctx* ctx, const uocr_moe* layer, int mode, const float* x,
                          const float* logits, size_t tokens, float* y, int32_t* ids,
                          float* weights) {
  if (!ctx || !layer) return fail(UOCR_ERR_INVALID, "null argument");
  if (mode != UOCR_WEIGHTS_ONLY && mode != UOCR_DYNAMIC_ACTIVATIONS && mode != UOCR_DYNAMIC_ROWWISE)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: mode %d", mode);
  if (tokens == 0) return ok();
  if (!x || !logits || !y) return fail(UOCR_ERR_INVALID, "null argument");
  int st = moe_checks(ctx, layer, tokens);
  if (st) return st;
  DeviceGuard g(ctx->device);
  const size_t H = layer->hidden, E = layer->n_experts, k = layer->top_k;
  auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
  const size_t xb = al(tokens * H * 4), lb = al(tokens * E * 4), yb = al(tokens * H * 4),
               rb = al(tokens * k * 4);
  // Device staging [x | logits | y | ids | weights] has its own allocation so
  // the layer's workspace (ctx->ws) can grow independently.
  const size_t need = xb + lb + yb + 2 * rb;
  if (ctx->io_bytes < need) {
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    if (ctx->io) CUDA_TRY(cudaFree(ctx->io));
    ctx->io = nullptr;
    ctx->io_bytes = 0;
    CUDA_TRY(cudaMalloc(&ctx->io, need));
    ctx->io_bytes = need;
  }
  char* d = static_cast<char*>(ctx->io);
  float* xd = reinterpret_cast<float*>(d);
  float* ld = reinterpret_cast<float*>(d + xb);
  float* yd = reinterpret_cast<float*>(d + xb + lb);
  int32_t* id = reinterpret_cast<int32_t*>(d + xb + lb + yb);
  float* wd = reinterpret_cast<float*>(d + xb + lb + yb + rb);
  // Small calls (decode) go through a pinned mirror of the device staging:
  // one host-to-device copy of [x | logits], one device-to-host copy of the
  // outputs, one synchronisation (with the status word).  Errors of earlier
  // asynchronous calls on this context surface at that synchronisation.
  // Large calls copy straight from/to the caller's buffers when those are
  // pinned, avoiding two host copies of megabytes.
  const bool packed = need <= (size_t(1) << 20);
  const bool pin = !packed && is_pinned(x) && is_pinned(logits) && is_pinned(y) &&
                   (!ids || is_pinned(ids)) && (!weights || is_pinned(weights));
  char* hp = nullptr;
  if (!pin) {
    if ((st = ensure_pinned(ctx, need))) return st;
    hp = static_cast<char*>(ctx->pinned);
    std::memcpy(hp, x, tokens * H * 4);
    std::memcpy(hp + xb, logits, tokens * E * 4);
  }
  // one token, routing returned in full or not at all: the captured graph
  if (packed && tokens == 1 && (!ids) == (!weights)) {
    bool done = false;
    if ((st = host_decode_graph(ctx, layer, mode, xb, lb, yb, rb, ids != nullptr, &done)))
      return st;
    if (done) {
      std::memcpy(y, hp + xb + lb, H * 4);
      if (ids) std::memcpy(ids, hp + xb + lb + yb, k * 4);
      if (weights) std::memcpy(weights, hp + xb + lb + yb + rb, k * 4);
      return ok();
    }
  }
  if (packed) {
    CUDA_TRY(cudaMemcpyAsync(xd, hp, xb + tokens * E * 4, cudaMemcpyHostToDevice, ctx->stream));
  } else {
    CUDA_TRY(cudaMemcpyAsync(xd, pin ? x : reinterpret_cast<float*>(hp), tokens * H * 4,
                             cudaMemcpyHostToDevice, ctx->stream));
    CUDA_TRY(cudaMemcpyAsync(ld, pin ? logits : reinterpret_cast<float*>(hp + xb),
                             tokens * E * 4, cudaMemcpyHostToDevice, ctx->stream));
  }
  if ((st = moe_run(ctx, layer, mode, xd, ld, tokens, yd, id, wd))) return st;
  if (packed) {
    const size_t out = weights ? yb + rb + tokens * k * 4 : ids ? yb + tokens * k * 4 : tokens * H * 4;
    CUDA_TRY(cudaMemcpyAsync(hp + xb + lb, yd, out, cudaMemcpyDeviceToHost, ctx->stream));
  } else {
    CUDA_TRY(cudaMemcpyAsync(pin ? y : reinterpret_cast<float*>(hp + xb + lb), yd, tokens * H * 4,
                             cudaMemcpyDeviceToHost, ctx->stream));
    if (ids)
      CUDA_TRY(cudaMemcpyAsync(pin ? ids : reinterpret_cast<int32_t*>(hp + xb + lb + yb), id,
                               tokens * k * 4, cudaMemcpyDeviceToHost, ctx->stream));
    if (weights)
      CUDA_TRY(cudaMemcpyAsync(pin ? weights : reinterpret_cast<float*>(hp + xb + lb + yb + rb), wd,
                               tokens * k * 4, cudaMemcpyDeviceToHost, ctx->stream));
  }
  if ((st = take_device_status(ctx))) return st;
  if (!pin) {
    std::memcpy(y, hp + xb + lb, tokens * H * 4);
    if (ids) std::memcpy(ids, hp + xb + lb + yb, tokens * k * 4);
    if (weights) std::memcpy(weights, hp + xb + lb + yb + rb, tokens * k * 4);
  }
  return ok();
}


// Decoder::feed_forward (src/decoder/mod.rs:114-122): y = down(silu(gate x) *
// up x) for `rows` rows of x (device), each projection as
// Decoder::projection (:99-112) makes it: int8 activations for a one-row
// input in DynamicActivations mode, for every row in the row-wise mode.
int uocr_feed_forward(uocr_ctx* ctx, const uocr_q8* gate, const uocr_q8* up, const uocr_q8* down,
                      int mode, const float* x_dev, size_t rows, float* y_dev) {
  if (!ctx || !gate || !up || !down) return fail(UOCR_ERR_INVALID, "null argument");
  if (mode != UOCR_WEIGHTS_ONLY && mode != UOCR_DYNAMIC_ACTIVATIONS && mode != UOCR_DYNAMIC_ROWWISE)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: mode %d", mode);
  if (gate->rows != up->rows || gate->cols != up->cols || down->cols != gate->rows)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: feed-forward projections");
  if (rows == 0) return ok();
  if (!x_dev || !y_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(rows)) return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: rows");
  int st;
  if ((st = linear_checks(ctx, gate, rows)) || (st = linear_checks(ctx, down, rows))) return st;
  const int lm = mode == UOCR_DYNAMIC_ROWWISE || (mode == UOCR_DYNAMIC_ACTIVATIONS && rows == 1)
                     ? MODE_INT8
                     : MODE_FP32;
  const size_t F = gate->rows;
  const size_t gb = al256(rows * F * 4);
  size_t sb = linear_scratch_bytes(gate, lm, rows);
  const size_t sd = linear_scratch_bytes(down, lm, rows);
  if (sd > sb) sb = sd;
  DeviceGuard g(ctx->device);
  if ((st = ensure_ws(ctx, 2 * gb + sb))) return st;
  char* base = static_cast<char*>(ctx->ws);
  float* gd = reinterpret_cast<float*>(base);
  float* ud = reinterpret_cast<float*>(base + gb);
  char* scratch = base + 2 * gb;
  if ((st = linear_launch(ctx, gate, lm, x_dev, rows, gd, scratch)) ||
      (st = linear_launch(ctx, up, lm, x_dev, rows, ud, scratch)))
    return st;
  launch_swiglu(gd, ud, static_cast<long long>(rows * F), gd, ctx->sms, ctx->stream);
  if ((st = check_launch())) return st;
  return linear_launch(ctx, down, lm, gd, rows, y_dev, scratch);
}

// ops::linear_weight, BF16 branch (src/cpu/ops.rs:62-133): y [batch x n] =
// x [batch x k] times the BF16 weight [n x k] (device bit patterns), each
// output a left-to-right sum; the router logits of Decoder::experts
// (projection of "mlp.gate.weight", src/decoder/mod.rs:126-130).
int uocr_linear_bf16(uocr_ctx* ctx, const uint16_t* w_dev, size_t n, size_t k, const float* x_dev,
                     size_t batch, float* y_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  if (n == 0 || k == 0) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: linear weight");
  if (batch == 0) return ok();
  if (!w_dev || !x_dev || !y_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(n) || !fits_int(batch) || k > 2400)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: BF16 linear extent");
  int st = check_elements(ctx, batch * n);
  if (st) return st;
  DeviceGuard g(ctx->device);
  cudaError_t e = launch_linear_bf16(w_dev, static_cast<int>(n), static_cast<int>(k), x_dev,
                                     static_cast<int>(batch), y_dev, ctx->status_dev, ctx->stream);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "BF16 linear: %s", cudaGetErrorString(e));
  return ok();
}

// ---- decoder attention at decode --------------------------------------------
// ops::rms_norm (src/cpu/ops.rs:362-414, 419-421)
// ops::linear_weight, BF16 branch (src/cpu/ops.rs:62-133), for large BF16
// weights: exact products on the tensor cores, FP32 accumulation in another
// order than the reference's left-to-right sum (FP32 tolerance).  The
// reference's element-count checks: n for one row, weight + output otherwise.
int uocr_linear_bf16_tc(uocr_ctx* ctx, const uint16_t* w_dev, size_t n, size_t k,
                        const float* x_dev, size_t batch, float* y_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null argument");
  if (n == 0 || k == 0) return fail(UOCR_ERR_SHAPE, "linear weight must be [out,in]");
  if (batch == 0) return ok();
  if (!w_dev || !x_dev || !y_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(n) || !fits_int(k) || !fits_int(batch) || !fits_int(batch * k))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: size");
  if (!linear_bf16_tc_supported(static_cast<int>(n), static_cast<int>(k)))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: k must be a multiple of 64");
  if (reinterpret_cast<uintptr_t>(w_dev) % 16 || reinterpret_cast<uintptr_t>(x_dev) % 16)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: 16-byte aligned weights and rows");
  int st = batch == 1 ? check_elements(ctx, n) : check_elements(ctx, n * k + batch * n);
  if (st) return st;
  DeviceGuard g(ctx->device);
  const size_t pb = al256(3 * batch * k * 2);
  if ((st = ensure_ws(ctx, pb + al256(batch * 4)))) return st;
  uint16_t* pieces = static_cast<uint16_t*>(ctx->ws);
  float* rinv = reinterpret_cast<float*>(static_cast<char*>(ctx->ws) + pb);
  launch_split_rows(x_dev, static_cast<long long>(k), nullptr, static_cast<int>(batch),
                    static_cast<int>(k), pieces, rinv, ctx->sms, ctx->stream);
  const cudaError_t e = launch_linear_bf16_tc(w_dev, static_cast<int>(n), static_cast<int>(k), pieces,
                                              rinv, static_cast<int>(batch), y_dev,
                                              static_cast<long long>(n), ctx->status_dev, ctx->sms,
                                              ctx->stream);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "linear_bf16_tc launch: %s", cudaGetErrorString(e));
  return check_launch();
}

// The fixed-work benchmark's checksum (src/model/benchmark.rs:43-47):
// *acc_dev += the bit patterns of x_dev[0..n) (u64, wrapping).
int uocr_bits_checksum(uocr_ctx* ctx, const float* x_dev, size_t n, uint64_t* acc_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  if (n == 0) return ok();
  if (!x_dev || !acc_dev) return fail(UOCR_ERR_INVALID, "null argument");
  DeviceGuard g(ctx->device);
  launch_bits_checksum(x_dev, static_cast<long long>(n), reinterpret_cast<unsigned long long*>(acc_dev),
                       ctx->sms, ctx->stream);
  return check_launch();
}

int uocr_rms_norm(uocr_ctx* ctx, const float* x_dev, size_t rows, size_t width,
                  const float* weight_dev, float eps, float* out_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  if (width == 0 || !std::isfinite(eps) || eps <= 0.0f)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid normalization parameters");
  if (rows == 0) return ok();
  if (!x_dev || !weight_dev || !out_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(rows) || width > 50000)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: normalization extent");
  DeviceGuard g(ctx->device);
  launch_rms_norm(x_dev, static_cast<long long>(width), static_cast<int>(rows),
                  static_cast<int>(width), weight_dev, eps, out_dev, static_cast<long long>(width),
                  ctx->status_dev, ctx->stream);
  return check_launch();
}

// The residual adds of Decoder::layer (src/decoder/mod.rs:348-349, attention
// output + x; :361-362, + the FFN output) and the RMSNorm of the result that
// follows (:355, or the next layer's input norm) in one launch:
// sum = x + res (one rounding per element; sum may alias x or res), then
// out = rms_norm(sum), each bit-identical to the two separate operations.
int uocr_add_rms_norm(uocr_ctx* ctx, const float* x_dev, const float* res_dev, size_t rows,
                      size_t width, const float* weight_dev, float eps, float* sum_dev,
                      float* out_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  if (width == 0 || !std::isfinite(eps) || eps <= 0.0f)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid normalization parameters");
  if (rows == 0) return ok();
  if (!x_dev || !res_dev || !weight_dev || !sum_dev || !out_dev)
    return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(rows) || width > 50000)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: normalization extent");
  DeviceGuard g(ctx->device);
  launch_rms_norm(x_dev, static_cast<long long>(width), static_cast<int>(rows),
                  static_cast<int>(width), weight_dev, eps, out_dev, static_cast<long long>(width),
                  ctx->status_dev, ctx->stream, res_dev, sum_dev);
  return check_launch();
}

// ops::rope (src/cpu/ops.rs:423-437): the (cos, sin) table of positions
// [0, max_positions) for one head dimension and base.
int uocr_rope_create(uocr_ctx* ctx, size_t head_dim, float theta, size_t max_positions,
                     uocr_rope** out) {
  if (!ctx || !out) return fail(UOCR_ERR_INVALID, "null argument");
  *out = nullptr;
  if (head_dim == 0 || head_dim % 2 || !std::isfinite(theta) || theta <= 0.0f)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid rotary dimensions or base");
  size_t n;
  if (max_positions == 0 || !mul_ok(max_positions, head_dim, &n) || !fits_int(max_positions) ||
      n > (size_t(1) << 31))
    return fail(UOCR_ERR_RESOURCE, "resource limit: rotary table");
  std::vector<float> host(n);  // [max_pos][head_dim/2][2]
  build_rope_table(static_cast<int>(head_dim), theta, static_cast<int>(max_positions), host.data());
  DeviceGuard g(ctx->device);
  auto* r = new uocr_rope();
  r->device = ctx->device;
  r->head_dim = static_cast<int>(head_dim);
  r->max_pos = static_cast<int>(max_positions);
  r->theta = theta;
  cudaError_t e = cudaMalloc(&r->table, n * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpy(r->table, host.data(), n * sizeof(float), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    uocr_rope_free(r);
    return fail(UOCR_ERR_CUDA, "rope table: %s", cudaGetErrorString(e));
  }
  *out = r;
  return ok();
}

int uocr_rope_free(uocr_rope* rope) {
  if (!rope) return ok();
  DeviceGuard g(rope->device);
  if (rope->table) cudaFree(rope->table);
  delete rope;
  return ok();
}

// Rotates q (and k when given) in place: rows x width, heads of head_dim,
// row r at positions_dev[r].  A position outside the table is Resource
// ("maximum context exceeded", src/decoder/mod.rs:259-264) at the next sync.
int uocr_rope_apply(uocr_ctx* ctx, const uocr_rope* rope, float* q_dev, float* k_dev, size_t rows,
                    size_t width, const int32_t* positions_dev) {
  if (!ctx || !rope) return fail(UOCR_ERR_INVALID, "null argument");
  if (width == 0 || width % rope->head_dim)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid rotary dimensions or base");
  if (rows == 0) return ok();
  if (!q_dev || !positions_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(rows)) return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: rows");
  DeviceGuard g(ctx->device);
  launch_rope(q_dev, k_dev, static_cast<long long>(width), static_cast<int>(rows),
              static_cast<int>(width / rope->head_dim), rope->head_dim, positions_dev, nullptr,
              rope->table, rope->max_pos, ctx->status_dev, ctx->sms, ctx->stream);
  return check_launch();
}

// ops::attention_decode (src/cpu/ops.rs:515-606): one query [1 x width] over
// token-major keys/values [tokens x width].
int uocr_attention_decode(uocr_ctx* ctx, const float* q_dev, const float* keys_dev,
                          size_t keys_len, const float* values_dev, size_t values_len,
                          size_t width, size_t heads, float* out_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  if (heads == 0 || width == 0 || width % heads || keys_len == 0 || keys_len % width ||
      keys_len != values_len)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: decode attention layout");
  const size_t tokens = keys_len / width;
  int st = check_elements(ctx, tokens + width);
  if (st) return st;
  if (!q_dev || !keys_dev || !values_dev || !out_dev) return fail(UOCR_ERR_INVALID, "null argument");
  const size_t dim = width / heads;
  if (!fits_int(width) || !fits_int(tokens) ||
      attention_smem_bytes(static_cast<int>(dim), static_cast<int>(tokens)) > kAttnMaxSmem)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: decode attention over %zu tokens",
                tokens);
  DeviceGuard g(ctx->device);
  AttnArgs a{};
  a.q = q_dev;
  a.ld_q = static_cast<long long>(width);
  a.keys = keys_dev;
  a.values = values_dev;
  a.seq_stride = static_cast<long long>(tokens * width);
  a.head_stride = static_cast<long long>(dim);
  a.row_stride = static_cast<long long>(width);
  a.cap = static_cast<long long>(tokens);
  a.width = static_cast<int>(width);
  a.heads = static_cast<int>(heads);
  a.dim = static_cast<int>(dim);
  a.tokens = static_cast<int>(tokens);
  a.scale = 1.0f / std::sqrt(static_cast<float>(dim));  // (dim as f32).sqrt().recip()
  a.out = out_dev;
  a.ld_out = static_cast<long long>(width);
  a.status = ctx->status_dev;
  AttnMaps maps;
  const bool tma = attention_tma_ok(keys_dev, values_dev, static_cast<long long>(tokens),
                                    a.width, a.dim, a.cap) &&
                   attention_tma_maps(&maps, keys_dev, values_dev, static_cast<long long>(tokens),
                                      a.width);
  cudaError_t e = tma ? launch_attention_decode_tma(maps, a, 1, ctx->stream)
                      : launch_attention_decode(a, 1, static_cast<int>(tokens), ctx->stream);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
  return ok();
}

// The prefill branch of Decoder::layer (src/decoder/mod.rs:313-338): causal
// ops::attention (src/cpu/ops.rs:263-360, mask :190-222) of token-major
// q/keys/values [tokens x width] split into heads; query i sees tokens 0..i.
int uocr_attention_prefill(uocr_ctx* ctx, const float* q_dev, const float* keys_dev,
                           const float* values_dev, size_t tokens, size_t width, size_t heads,
                           float* out_dev) {
  if (!ctx) return fail(UOCR_ERR_INVALID, "null context");
  if (heads == 0 || width == 0 || width % heads || tokens == 0)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid attention layout");
  const size_t dim = width / heads;
  // the reference's scratch rule: d * nk + q elements + nk
  int st = check_elements(ctx, dim * tokens + tokens * width + tokens);
  if (st) return st;
  if (!q_dev || !keys_dev || !values_dev || !out_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (!fits_int(width) || tokens > 65535 ||
      attention_smem_bytes(static_cast<int>(dim), static_cast<int>(tokens)) > kAttnMaxSmem)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: prefill attention over %zu tokens",
                tokens);
  DeviceGuard g(ctx->device);
  AttnArgs a{};
  a.q = q_dev;
  a.ld_q = static_cast<long long>(width);
  a.keys = keys_dev;
  a.values = values_dev;
  a.seq_stride = 0;
  a.head_stride = static_cast<long long>(dim);
  a.row_stride = static_cast<long long>(width);
  a.cap = static_cast<long long>(tokens);
  a.width = static_cast<int>(width);
  a.heads = static_cast<int>(heads);
  a.dim = static_cast<int>(dim);
  a.causal = 1;
  a.seq = 0;
  a.scale = 1.0f / std::sqrt(static_cast<float>(dim));
  a.out = out_dev;
  a.ld_out = static_cast<long long>(width);
  a.status = ctx->status_dev;
  AttnMaps maps;
  const bool tma = attention_tma_ok(keys_dev, values_dev, static_cast<long long>(tokens),
                                    a.width, a.dim, a.cap) &&
                   attention_tma_maps(&maps, keys_dev, values_dev, static_cast<long long>(tokens),
                                      a.width);
  const int rows = static_cast<int>(tokens);
  cudaError_t e = tma ? launch_attention_decode_tma(maps, a, rows, ctx->stream)
                      : launch_attention_decode(a, rows, rows, ctx->stream);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
  return ok();
}

// LayerCache::new (src/decoder/cache.rs:14-31) for `batch` sequences, with
// room for a prefix of up to max_prefix tokens.
int uocr_kv_create(uocr_ctx* ctx, size_t batch, size_t heads, size_t head_dim, size_t window,
                   size_t max_prefix, uocr_kv** out) {
  if (!ctx || !out) return fail(UOCR_ERR_INVALID, "null argument");
  *out = nullptr;
  size_t width;
  if (!mul_ok(heads, head_dim, &width) || width == 0)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: cache head dimensions");
  if (window == 0) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: empty cache window");
  if (batch == 0 || max_prefix == 0)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: empty cache batch or prefix");
  size_t cap, rows, n, bytes;
  if (max_prefix > (size_t(1) << 30) || window > (size_t(1) << 30) || !fits_int(width) ||
      !fits_int(batch) || (cap = max_prefix + window) > (size_t(1) << 30))
    return fail(UOCR_ERR_RESOURCE, "resource limit: cache capacity overflow");
  // tiled layout (one TMA box per 32-slot tile) when the TMA attention kernel applies
  const size_t cap_tiled = (cap + 31) & ~static_cast<size_t>(31);
  const bool tiled = attention_tma_ok(nullptr, nullptr, 0, 32, static_cast<int>(head_dim),
                                      static_cast<long long>(cap_tiled));
  if (tiled) cap = cap_tiled;
  if (!mul_ok(batch, cap, &rows) || !mul_ok(rows, width, &n) || !mul_ok(n, 4, &bytes) ||
      n / 32 >= (size_t(1) << 31))
    return fail(UOCR_ERR_RESOURCE, "resource limit: cache capacity overflow");
  DeviceGuard g(ctx->device);
  auto* kv = new uocr_kv();
  kv->device = ctx->device;
  kv->batch = static_cast<int>(batch);
  kv->heads = static_cast<int>(heads);
  kv->head_dim = static_cast<int>(head_dim);
  kv->width = static_cast<int>(width);
  kv->window = static_cast<int>(window);
  kv->max_prefix = static_cast<int>(max_prefix);
  kv->cap = static_cast<long long>(cap);
  kv->layout = KvLayout{kv->heads, kv->head_dim, kv->cap, tiled ? 1 : 0};
  kv->prefix.assign(batch, 0);
  cudaError_t e = cudaMalloc(&kv->keys, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&kv->values, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&kv->state, batch * 2 * sizeof(int));
  if (e == cudaSuccess) e = cudaMemsetAsync(kv->state, 0, batch * 2 * sizeof(int), ctx->stream);
  if (e == cudaSuccess && tiled) e = cudaMalloc(&kv->scores, rows * heads * sizeof(float));
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    uocr_kv_free(kv);
    cudaGetLastError();
    return fail(e == cudaErrorMemoryAllocation ? UOCR_ERR_RESOURCE : UOCR_ERR_CUDA,
                "cache allocation: %s", cudaGetErrorString(e));
  }
  kv->tma = tiled && attention_tma_maps_tiled(&kv->maps, kv->keys, kv->values,
                                              static_cast<long long>(n), kv->head_dim);
  if (tiled && !kv->tma) {
    uocr_kv_free(kv);
    return fail(UOCR_ERR_CUDA, "cache tensor maps could not be built");
  }
  *out = kv;
  return ok();
}

int uocr_kv_free(uocr_kv* kv) {
  if (!kv) return ok();
  DeviceGuard g(kv->device);
  if (kv->keys) cudaFree(kv->keys);
  if (kv->values) cudaFree(kv->values);
  if (kv->state) cudaFree(kv->state);
  if (kv->scores) cudaFree(kv->scores);
  delete kv;
  return ok();
}

// Attention form of uocr_kv_attention: 0 chooses by batch size, 1 one CTA per
// (head, sequence), 2 split over tokens (tiled caches only).  Same results.
int uocr_kv_set_attention_form(uocr_kv* kv, int form) {
  if (!kv) return fail(UOCR_ERR_INVALID, "null argument");
  if (form < 0 || form > 2 || (form == 2 && !kv->scores))
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: attention form");
  kv->split = form;
  return ok();
}

// LayerCache::prefill (src/decoder/cache.rs:33-57) of sequence `seq`:
// tokens rows of width floats (device).
int uocr_kv_prefill(uocr_ctx* ctx, uocr_kv* kv, size_t seq, const float* keys_dev,
                    const float* values_dev, size_t tokens) {
  if (!ctx || !kv) return fail(UOCR_ERR_INVALID, "null argument");
  if (seq >= static_cast<size_t>(kv->batch)) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: cache sequence");
  if (kv->prefix[seq] || tokens == 0)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid cache prefill");
  if (tokens > static_cast<size_t>(kv->max_prefix))
    return fail(UOCR_ERR_RESOURCE, "resource limit: cache capacity overflow");
  if (!keys_dev || !values_dev) return fail(UOCR_ERR_INVALID, "null argument");
  DeviceGuard g(ctx->device);
  launch_kv_prefill(kv->keys, kv->values, kv->layout, static_cast<int>(seq), keys_dev, values_dev,
                    static_cast<int>(tokens), ctx->stream);
  launch_kv_set_prefix(kv->state, static_cast<int>(seq), static_cast<int>(tokens), ctx->stream);
  int st = check_launch();
  if (st) return st;
  kv->prefix[seq] = static_cast<int>(tokens);
  return ok();
}

static int kv_ready(const uocr_kv* kv) {
  for (int p : kv->prefix)
    if (!p) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: cache must be prefilled");
  return ok();
}

// LayerCache::push (src/decoder/cache.rs:59-80) for every sequence: row b of
// k_dev / v_dev ([batch x width]) into sequence b.
int uocr_kv_push(uocr_ctx* ctx, uocr_kv* kv, const float* k_dev, const float* v_dev) {
  if (!ctx || !kv) return fail(UOCR_ERR_INVALID, "null argument");
  int st = kv_ready(kv);
  if (st) return st;
  if (!k_dev || !v_dev) return fail(UOCR_ERR_INVALID, "null argument");
  DeviceGuard g(ctx->device);
  launch_kv_push(kv->keys, kv->values, kv->state, kv->batch, kv->layout, kv->window, k_dev, v_dev,
                 kv->width, ctx->status_dev, ctx->stream);
  return check_launch();
}

// ops::rope of q and k ([batch x width]) at each sequence's position
// (LayerCache::position before this token's push).
int uocr_kv_rope(uocr_ctx* ctx, const uocr_kv* kv, const uocr_rope* rope, float* q_dev, float* k_dev) {
  if (!ctx || !kv || !rope) return fail(UOCR_ERR_INVALID, "null argument");
  if (rope->head_dim != kv->head_dim)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid rotary dimensions or base");
  int st = kv_ready(kv);
  if (st) return st;
  if (!q_dev) return fail(UOCR_ERR_INVALID, "null argument");
  DeviceGuard g(ctx->device);
  launch_rope(q_dev, k_dev, kv->width, kv->batch, kv->heads, kv->head_dim, nullptr, kv->state,
              rope->table, rope->max_pos, ctx->status_dev, ctx->sms, ctx->stream);
  return check_launch();
}

// ops::rope of q and k at each sequence's position and LayerCache::push of
// k and v, from the fused projection rows [q | k | v] (batch x 3*width,
// device): q rotated into q_out (batch x width).  One launch for what
// uocr_kv_rope then uocr_kv_push do, with the same results.
int uocr_kv_rope_push_qkv(uocr_ctx* ctx, uocr_kv* kv, const uocr_rope* rope, const float* qkv_dev,
                          float* q_out_dev) {
  if (!ctx || !kv || !rope) return fail(UOCR_ERR_INVALID, "null argument");
  if (rope->head_dim != kv->head_dim)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: invalid rotary dimensions or base");
  int st = kv_ready(kv);
  if (st) return st;
  if (!qkv_dev || !q_out_dev) return fail(UOCR_ERR_INVALID, "null argument");
  DeviceGuard g(ctx->device);
  launch_kv_rope_push(kv->keys, kv->values, kv->state, kv->batch, kv->layout, kv->window, qkv_dev,
                      q_out_dev, rope->table, rope->max_pos, ctx->status_dev, ctx->stream);
  return check_launch();
}

// ops::attention_decode of q row b over sequence b's cache, for every b.
int uocr_kv_attention(uocr_ctx* ctx, const uocr_kv* kv, const float* q_dev, float* out_dev) {
  if (!ctx || !kv) return fail(UOCR_ERR_INVALID, "null argument");
  int st = kv_ready(kv);
  if (st) return st;
  if (!q_dev || !out_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if ((st = check_elements(ctx, static_cast<size_t>(kv->cap) + kv->width))) return st;
  if (attention_smem_bytes(kv->head_dim, static_cast<int>(kv->cap)) > kAttnMaxSmem)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: decode attention over %lld tokens",
                kv->cap);
  DeviceGuard g(ctx->device);
  AttnArgs a{};
  a.q = q_dev;
  a.ld_q = kv->width;
  a.keys = kv->keys;
  a.values = kv->values;
  a.head_stride = kv->cap * kv->head_dim;
  a.seq_stride = a.head_stride * kv->heads;
  a.row_stride = kv->head_dim;
  a.cap = kv->cap;
  a.tiled = kv->layout.tiled;
  a.width = kv->width;
  a.heads = kv->heads;
  a.dim = kv->head_dim;
  a.state = kv->state;
  a.window = kv->window;
  a.scale = 1.0f / std::sqrt(static_cast<float>(kv->head_dim));
  a.out = out_dev;
  a.ld_out = kv->width;
  a.status = ctx->status_dev;
  a.scores = kv->scores;
  // few CTAs with one per (head, sequence): each would stream its head alone,
  // latency-bound; the split form spreads every head over many CTAs
  const bool split = attention_split_ok(a) &&
                     (kv->split == 2 ||
                      (kv->split == 0 && static_cast<long long>(kv->batch) * kv->heads <= ctx->sms));
  cudaError_t e = split     ? launch_attention_split(a, kv->batch, static_cast<int>(kv->cap), ctx->stream)
                  : kv->tma ? launch_attention_decode_tma(kv->maps, a, kv->batch, ctx->stream)
                            : launch_attention_decode(a, kv->batch, static_cast<int>(kv->cap),
                                                      ctx->stream);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
  return ok();
}

// The prefill branch of Decoder::layer (src/decoder/mod.rs:313-338) on the
// cache: right after uocr_kv_prefill of `rows` tokens, query row i of q
// ([rows x width], position i) attends to the sequence's tokens 0..i.
int uocr_kv_attention_prefill(uocr_ctx* ctx, const uocr_kv* kv, size_t seq, const float* q_dev,
                              size_t rows, float* out_dev) {
  if (!ctx || !kv) return fail(UOCR_ERR_INVALID, "null argument");
  if (seq >= static_cast<size_t>(kv->batch)) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: cache sequence");
  if (rows == 0 || static_cast<size_t>(kv->prefix[seq]) != rows)
    return fail(UOCR_ERR_SHAPE, "invalid tensor shape: prefill attention needs the prefilled rows");
  int st = check_elements(ctx, static_cast<size_t>(kv->head_dim) * rows +
                                   rows * static_cast<size_t>(kv->width) + rows);
  if (st) return st;
  if (!q_dev || !out_dev) return fail(UOCR_ERR_INVALID, "null argument");
  if (rows > 65535 || attention_smem_bytes(kv->head_dim, static_cast<int>(kv->cap)) > kAttnMaxSmem)
    return fail(UOCR_ERR_UNSUPPORTED, "unsupported configuration: prefill attention over %zu tokens",
                rows);
  DeviceGuard g(ctx->device);
  AttnArgs a{};
  a.q = q_dev;
  a.ld_q = kv->width;
  a.keys = kv->keys;
  a.values = kv->values;
  a.head_stride = kv->cap * kv->head_dim;
  a.seq_stride = a.head_stride * kv->heads;
  a.row_stride = kv->head_dim;
  a.cap = kv->cap;
  a.tiled = kv->layout.tiled;
  a.width = kv->width;
  a.heads = kv->heads;
  a.dim = kv->head_dim;
  a.causal = 1;
  a.seq = static_cast<int>(seq);
  a.tokens = static_cast<int>(rows);
  a.scale = 1.0f / std::sqrt(static_cast<float>(kv->head_dim));
  a.out = out_dev;
  a.ld_out = kv->width;
  a.status = ctx->status_dev;
  const int n = static_cast<int>(rows);
  // 16 rows per CTA where it applies (head_dim 128, prefix up to ~2,500
  // tokens), else one row per CTA; the same bits either way
  const bool blocked = kv->tma && kv->split != 1 && attention_prefill_ok(a);
  cudaError_t e = blocked   ? launch_attention_prefill(kv->maps, a, ctx->stream)
                  : kv->tma ? launch_attention_decode_tma(kv->maps, a, n, ctx->stream)
                            : launch_attention_decode(a, n, static_cast<int>(kv->cap), ctx->stream);
  if (e != cudaSuccess) return fail(UOCR_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
  return ok();
}

// LayerCache::new (src/decoder/cache.rs:14-31) again for sequence `seq`:
// empty, to be prefilled anew (the reference's prefill makes new caches).
int uocr_kv_reset(uocr_ctx* ctx, uocr_kv* kv, size_t seq) {
  if (!ctx || !kv) return fail(UOCR_ERR_INVALID, "null argument");
  if (seq >= static_cast<size_t>(kv->batch)) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: cache sequence");
  DeviceGuard g(ctx->device);
  launch_kv_set_prefix(kv->state, static_cast<int>(seq), 0, ctx->stream);
  int st = check_launch();
  if (st) return st;
  kv->prefix[seq] = 0;
  return ok();
}

// LayerCache::tokens / position of sequence `seq` (synchronous read).
int uocr_kv_state(uocr_ctx* ctx, const uocr_kv* kv, size_t seq, size_t* tokens, size_t* position) {
  if (!ctx || !kv) return fail(UOCR_ERR_INVALID, "null argument");
  if (seq >= static_cast<size_t>(kv->batch)) return fail(UOCR_ERR_SHAPE, "invalid tensor shape: cache sequence");
  DeviceGuard g(ctx->device);
  int h[2];
  CUDA_TRY(cudaMemcpyAsync(h, kv->state + 2 * seq, sizeof h, cudaMemcpyDeviceToHost, ctx->stream));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  const size_t gen = static_cast<size_t>(h[1]), win = static_cast<size_t>(kv->window);
  if (tokens) *tokens = static_cast<size_t>(h[0]) + (gen < win ? gen : win);
  if (position) *position = static_cast<size_t>(h[0]) + gen;
  return take_device_status(ctx);
}

// Slots [0, tokens) of sequence seq, where tokens = LayerCache::tokens, as
// token-major rows (keys_out / values_out: tokens * width floats each, device).
int uocr_kv_export(uocr_ctx* ctx, const uocr_kv* kv, size_t seq, float* keys_out,
                   float* values_out, size_t* tokens) {
  if (!ctx || !kv || !tokens) return fail(UOCR_ERR_INVALID, "null argument");
  size_t n = 0;
  int st = uocr_kv_state(ctx, kv, seq, &n, nullptr);
  if (st) return st;
  *tokens = n;
  if (!keys_out || !values_out) return ok();  // size query
  DeviceGuard g(ctx->device);
  launch_kv_export(kv->keys, kv->values, kv->layout, static_cast<int>(seq), static_cast<int>(n),
                   keys_out, values_out, ctx->stream);
  return check_launch();
}

}  // extern "C"
