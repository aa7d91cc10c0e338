// ep_peer.cu — expert parallelism of Decoder::experts over NVLink peer memory.
//
// The reference runs every routed expert of a MoE layer on the device that
// holds the tokens (src/decoder/mod.rs:124-220).  Here the routed experts of
// a layer are spread over `world` GPUs in contiguous blocks, every GPU holds
// the shared expert and brings its own tokens, and the (token, expert) rows
// move between GPUs as stores into the other GPUs' memory: no collective
// library, no padding, and no host synchronisation, so a whole step can be
// captured in a CUDA graph.
//
// Every rank owns one device region (cudaMalloc'd, exported as a CUDA IPC
// handle, or shared directly between contexts of one process):
//   recv_x     [world][cap][hidden]  rows sent to this rank, one block per source
//   recv_ids   [world][cap]          their expert ids, local to this rank
//   recv_pair  [world][cap]          their pair index t*top_k + j on the source
//   recv_count [world]               rows each source sent this step
//   recv_flag  [world]               step number of each source's last dispatch
//   ret_rows   [max_tokens*top_k][hidden]  expert outputs of this rank's pairs
//   ret_flag   [world]               step number of each owner's last return
// with cap = max_tokens * top_k (a source can send all of its pairs to one
// rank).  One step (stream order, step number e = previous + 1):
//   dispatch  route this rank's tokens (moe::route, one warp per token, in
//             the same kernel); every pair's row of x is stored into its
//             owner's recv_x block at a slot claimed from a counter per owner,
//             with its local expert id and pair index; the last CTA to finish
//             stores each owner's count and then, with release semantics at
//             system scope, the flag = e.
//   wait      the owner waits (bounded) until every source's flag is e, reads
//             the counts and marks the unused slots of each block (id -1).
//   experts   the owner's grouped SwiGLU projections over all received rows
//             (the prefill machinery of moe_prefill.cu, rows of one expert in
//             one group; in QuantizationMode::DynamicActivations one call per
//             source block, because a group's row count selects int8 or FP32).
//   return    every received row's output is stored into its source's
//             ret_rows at its pair index; the last CTA publishes ret_flag = e
//             on every source.
//   combine   the source waits (bounded) until every owner's ret_flag is e and
//             adds p * output to the shared expert's output in ascending
//             expert id (src/decoder/mod.rs:208-217); the last CTA advances
//             the step number.
// Ranks move in lock step: a rank starts step e+1 only after every owner
// returned step e, and an owner returns step e only after its experts have
// read every row of step e, so a block of recv_x is never overwritten while
// it is read.  The result on each rank is uocr_moe_forward of its own tokens:
// routing and int8-activation outputs bit for bit, FP32-activation outputs
// within the FP32 tolerance (a group of rows from several ranks may take
// another projection kernel than the same rows on one GPU).
//
// The buffers are written only by plain stores and read after an acquire at
// system scope; no bulk or tensor-map copy ever reads peer memory.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <string>
#include <mutex>
#include <vector>

#include "../../include/uocr_q8.h"
#include "common.cuh"
#include "handles.h"
#include "kernels.h"
#include "route.cuh"

namespace uocr {
int record_error(int status, const char* message);  // capi.cu
}

using namespace uocr;

// The exchange's kernels and device helpers live in namespace uocr like every
// other kernel of the library (a profiler or a graph's node list shows them
// as uocr::...).
namespace uocr {
namespace {

constexpr int kEpThreads = 256;
constexpr int kEpWarps = kEpThreads / 32;
constexpr int kEpMaxWorld = kMaxDispatchRanks;
constexpr unsigned long long kEpDefaultWaitNs = 2000000000ull;  // 2 s

size_t al256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

// Byte offsets of the arrays in a rank's shared region.
struct EpLayout {
  long long recv_x, recv_ids, recv_pair, recv_count, recv_flag, ret_rows, ret_flag, bytes;
};

EpLayout ep_layout(int world, int cap, int hidden) {
  EpLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = al256(off + bytes);
    return static_cast<long long>(o);
  };
  const size_t rows = static_cast<size_t>(world) * cap;
  L.recv_x = take(sizeof(float) * rows * hidden);
  L.recv_ids = take(sizeof(int) * rows);
  L.recv_pair = take(sizeof(int) * rows);
  L.recv_count = take(sizeof(int) * world);
  L.recv_flag = take(sizeof(unsigned) * world);
  L.ret_rows = take(sizeof(float) * static_cast<size_t>(cap) * hidden);
  L.ret_flag = take(sizeof(unsigned) * world);
  L.bytes = static_cast<long long>(off);
  return L;
}

// Local step state: [0] step number, [1] dispatch arrivals, [2] return
// arrivals, [3] combine arrivals.
enum : int { kCtrStep = 0, kCtrDispatch = 1, kCtrReturn = 2, kCtrCombine = 3, kCtrWords = 8 };

// What every kernel of the exchange needs.
struct EpDev {
  char* const* peers;  // [world] base of every rank's region (this rank's own included)
  EpLayout L;
  int world, rank, cap, hidden, top_k, n_experts;
  const int* owner_of;  // [n_experts] rank holding each expert
  const int* local_of;  // [n_experts] its index among that rank's experts
  unsigned* ctr;        // kCtrWords local words
  int* live;            // [world] rows received from each source this step
  unsigned* status;
  unsigned long long wait_ns;
  int sys;  // some peer is another GPU: fences at system scope, else GPU scope
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_volatile_i32(const int* p) {
  return *reinterpret_cast<const volatile int*>(p);
}

// Bounded wait until *p == want (a value another GPU stores with release
// semantics); false when limit_ns passed first.
__device__ bool wait_flag_sys(const unsigned* p, unsigned want, unsigned long long limit_ns) {
  if (ld_acquire_sys(p) == want) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    __nanosleep(64);
    if (ld_acquire_sys(p) == want) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
}

__device__ __forceinline__ void fence_for(const EpDev& d) {
  if (d.sys)
    __threadfence_system();
  else
    __threadfence();
}

// The last CTA of a grid to arrive on counter *c.  The CTA barrier orders the
// CTA's stores (peer memory included) before its first thread's system-scope
// fence and arrival; the last CTA's fence after the arrival orders every
// CTA's stores before what it stores next (the pattern of a grid barrier,
// one fence per CTA instead of one per thread).
__device__ __forceinline__ bool last_to_arrive(const EpDev& d, unsigned* c) {
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_for(d);
    last = atomicAdd(c, 1u) == gridDim.x - 1u;
    if (last) fence_for(d);
  }
  __syncthreads();
  return last != 0;
}

// Route and dispatch: one warp per token runs moe::route (route.cuh), writes
// the token's routing, claims a slot in each selected expert's owner block
// (a counter per owner; the slot order within a block does not change any
// result, every row is computed on its own) and stores the token's row of x
// there with the expert id local to the owner and the pair index.  The last
// CTA to finish publishes each owner's count and then, with release
// semantics at system scope, the step number.
constexpr int kRdWarps = 4;
// A warp moves a row of up to 32 * kRowRegs float4 through registers: every
// load issued before the first store (a copy loop `dst[c] = src[c]` waits for
// each load in turn, since the stores may alias the source).
constexpr int kRowRegs = 16;

__device__ __forceinline__ void row_to_regs(const float4* src, int h4, int lane, float4 (&v)[kRowRegs]) {
#pragma unroll
  for (int u = 0; u < kRowRegs; ++u) {
    const int c = lane + 32 * u;
    if (c < h4) v[u] = __ldcg(src + c);
  }
}

__device__ __forceinline__ void regs_to_row(float4* dst, int h4, int lane, const float4 (&v)[kRowRegs]) {
#pragma unroll
  for (int u = 0; u < kRowRegs; ++u) {
    const int c = lane + 32 * u;
    if (c < h4) dst[c] = v[u];
  }
}

__global__ void __launch_bounds__(kRdWarps * 32) ep_route_dispatch_kernel(
    const __grid_constant__ EpDev d, const float* __restrict__ x, const float* __restrict__ logits,
    int tokens, int normalize, float scale, int32_t* __restrict__ ids, float* __restrict__ wts,
    unsigned* __restrict__ send_cnt) {
  extern __shared__ float rd_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, k = d.top_k;
  // up to 64 experts: the warp-collective form (route_row_warp64, the same
  // IEEE sequence with the max, the selection and the sums on the warp's
  // reductions instead of shared-memory loops); otherwise the general form
  const bool warp64 = d.n_experts <= 64;  // top_k <= 8 (uocr_ep_create)
  __shared__ __align__(16) float r64p[kRdWarps][64];
  __shared__ int r64ids[kRdWarps][8], r64sorted[kRdWarps][8];
  __shared__ float r64wts[kRdWarps][8], r64sorted_w[kRdWarps][8];
  float* p = rd_smem + warp * (d.n_experts + 2 * k);
  int* sel = warp64 ? r64ids[warp] : reinterpret_cast<int*>(p + d.n_experts);
  float* sw = warp64 ? r64wts[warp] : p + d.n_experts + k;
  __shared__ unsigned cta_cnt[kEpMaxWorld], cta_base[kEpMaxWorld];
  const unsigned step = d.ctr[kCtrStep] + 1u;
  const int h4 = d.hidden >> 2;
  for (int r = threadIdx.x; r < d.world; r += blockDim.x) cta_cnt[r] = 0u;
  __syncthreads();
  // one token per warp (the grid covers the tokens); slots are claimed per
  // CTA: shared-memory counts per owner, then one global reservation per
  // (CTA, owner).  One global atomic per pair serialised 384 of them on one
  // address at one GPU.  A block's slot order carries no meaning: each row's
  // output depends on that row alone, and the combine orders by expert id.
  const int t = blockIdx.x * kRdWarps + warp;
  bool ok = false;
  int e = 0, o = 0, local = 0;
  if (t < tokens) {
    const float* lrow = logits + static_cast<long long>(t) * d.n_experts;
    ok = warp64 ? route_row_warp64(lrow, d.n_experts, k, normalize, scale, r64p[warp], sel, sw,
                                   r64sorted[warp], r64sorted_w[warp], d.status)
                : route_row_warp(lrow, d.n_experts, k, normalize, scale, p, sel, sw, d.status);
    for (int r = lane; r < k; r += 32) {
      ids[static_cast<long long>(t) * k + r] = ok ? sel[r] : -1;
      wts[static_cast<long long>(t) * k + r] = ok ? sw[r] : 0.0f;
    }
    if (ok && lane < k) {
      e = sel[lane];
      o = d.owner_of[e];
      local = static_cast<int>(atomicAdd(&cta_cnt[o], 1u));
    }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < d.world; r += blockDim.x)
    cta_base[r] = cta_cnt[r] ? atomicAdd(send_cnt + r, cta_cnt[r]) : 0u;
  __syncthreads();
  if (t < tokens) {
    if (ok) {
      const int slot = lane < k ? static_cast<int>(cta_base[o]) + local : 0;
      const float4* src = reinterpret_cast<const float4*>(x) + static_cast<long long>(t) * h4;
      // the token's row once into registers, then stored to each owner
      const bool in_regs = h4 <= 32 * kRowRegs;
      float4 v[kRowRegs];
      if (in_regs) row_to_regs(src, h4, lane, v);
      for (int j = 0; j < k; ++j) {
        const int oj = __shfl_sync(0xffffffffu, o, j);
        const int sj = __shfl_sync(0xffffffffu, slot, j);
        const int ej = __shfl_sync(0xffffffffu, e, j);
        if (sj >= d.cap) {  // cannot happen while every step completes; never write past a block
          if (lane == 0) flag(d.status, DEV_CAPACITY);
          continue;
        }
        char* base = d.peers[oj];
        const long long row = static_cast<long long>(d.rank) * d.cap + sj;
        float4* dst = reinterpret_cast<float4*>(base + d.L.recv_x) + row * h4;
        if (in_regs)
          regs_to_row(dst, h4, lane, v);
        else
          for (int c = lane; c < h4; c += 32) dst[c] = src[c];
        if (lane == 0) {
          reinterpret_cast<int*>(base + d.L.recv_ids)[row] = d.local_of[ej];
          reinterpret_cast<int*>(base + d.L.recv_pair)[row] = t * k + j;
        }
      }
    }
    __syncwarp();
  }
  if (!last_to_arrive(d, d.ctr + kCtrDispatch)) return;
  for (int r = threadIdx.x; r < d.world; r += blockDim.x) {
    const unsigned c = atomicExch(send_cnt + r, 0u);
    char* base = d.peers[r];
    reinterpret_cast<volatile int*>(base + d.L.recv_count)[d.rank] =
        c < static_cast<unsigned>(d.cap) ? static_cast<int>(c) : d.cap;
    st_release_sys(reinterpret_cast<unsigned*>(base + d.L.recv_flag) + d.rank, step);
  }
  if (threadIdx.x == 0) d.ctr[kCtrDispatch] = 0u;
}

// Owner side: wait for every source's dispatch of this step, take the counts,
// mark the unused slots of each source block with id -1.  One CTA.
__global__ void __launch_bounds__(kEpThreads) ep_recv_wait_kernel(const __grid_constant__ EpDev d) {
  pdl_launch_dependents();  // launched as a programmatic dependent (launch_dependent):
  pdl_wait_prior_grids();   // nothing is touched before the previous kernel completes
  __shared__ int cnt[kEpMaxWorld];
  const int tid = threadIdx.x;
  const unsigned step = d.ctr[kCtrStep] + 1u;
  char* own = d.peers[d.rank];
  if (tid < d.world) {
    int c = 0;
    if (wait_flag_sys(reinterpret_cast<const unsigned*>(own + d.L.recv_flag) + tid, step,
                      d.wait_ns)) {
      c = ld_volatile_i32(reinterpret_cast<const int*>(own + d.L.recv_count) + tid);
      if (c < 0 || c > d.cap) {
        flag(d.status, DEV_BAD_ROUTE);
        c = 0;
      }
    } else {
      flag(d.status, DEV_TIMEOUT);
    }
    cnt[tid] = c;
    d.live[tid] = c;
  }
  __syncthreads();
  int* rid = reinterpret_cast<int*>(own + d.L.recv_ids);
  const int total = d.world * d.cap;
  for (int i = tid; i < total; i += kEpThreads)
    if (i % d.cap >= cnt[i / d.cap]) rid[i] = -1;
}

// Return: the output row of every received pair into its source's ret_rows
// at the pair index; one warp per row.  The row of slot i is row
// token_pos[i] of `rows` (the experts' grouped outputs), or row i when
// token_pos is null (outputs already in slot order).
__global__ void __launch_bounds__(kEpThreads) ep_return_kernel(const __grid_constant__ EpDev d,
                                                               const float* __restrict__ rows,
                                                               const int* __restrict__ token_pos) {
  pdl_launch_dependents();  // launched as a programmatic dependent (launch_dependent):
  pdl_wait_prior_grids();   // nothing is touched before the previous kernel completes
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned step = d.ctr[kCtrStep] + 1u;
  const int* pair = reinterpret_cast<const int*>(d.peers[d.rank] + d.L.recv_pair);
  const int total = d.world * d.cap, h4 = d.hidden >> 2;
  for (int i = blockIdx.x * kEpWarps + warp; i < total; i += gridDim.x * kEpWarps) {
    const int s = i / d.cap, j = i - s * d.cap;
    if (j >= d.live[s]) continue;
    const int p = __ldcg(pair + i);
    if (p < 0 || p >= d.cap) {
      if (lane == 0) flag(d.status, DEV_BAD_ROUTE);
      continue;
    }
    const int src_row = token_pos ? token_pos[i] : i;
    if (src_row < 0) {
      if (lane == 0) flag(d.status, DEV_BAD_ROUTE);
      continue;
    }
    float4* dst = reinterpret_cast<float4*>(d.peers[s] + d.L.ret_rows) + static_cast<long long>(p) * h4;
    const float4* src = reinterpret_cast<const float4*>(rows) + static_cast<long long>(src_row) * h4;
    if (h4 <= 32 * kRowRegs) {
      float4 v[kRowRegs];
      row_to_regs(src, h4, lane, v);
      regs_to_row(dst, h4, lane, v);
    } else {
      for (int c = lane; c < h4; c += 32) dst[c] = src[c];
    }
  }
  if (!last_to_arrive(d, d.ctr + kCtrReturn)) return;
  for (int r = threadIdx.x; r < d.world; r += kEpThreads)
    st_release_sys(reinterpret_cast<unsigned*>(d.peers[r] + d.L.ret_flag) + d.rank, step);
  if (threadIdx.x == 0) d.ctr[kCtrReturn] = 0u;
}

// Source side: wait for every owner's return of this step, then y[t] += p *
// out over t's pairs in ascending expert id, one rounding per operation (y
// holds the shared expert's output).  Grid (max(tokens, 1), column blocks of
// 128 float4); the last CTA advances the step number.
__global__ void __launch_bounds__(128) ep_combine_kernel(const __grid_constant__ EpDev d,
                                                         const int32_t* __restrict__ ids,
                                                         const float* __restrict__ wts, int tokens,
                                                         float* __restrict__ y) {
  pdl_launch_dependents();  // launched as a programmatic dependent (launch_dependent):
  pdl_wait_prior_grids();   // nothing is touched before the previous kernel completes
  const unsigned step = d.ctr[kCtrStep] + 1u;
  const char* own = d.peers[d.rank];
  for (int r = threadIdx.x; r < d.world; r += blockDim.x)
    if (!wait_flag_sys(reinterpret_cast<const unsigned*>(own + d.L.ret_flag) + r, step, d.wait_ns))
      flag(d.status, DEV_TIMEOUT);
  __syncthreads();
  const int t = blockIdx.x, k = d.top_k, h4 = d.hidden >> 2;
  if (t < tokens) {
    int e[8], p[8];
    float w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool used = j < k;
      e[j] = used ? ids[t * k + j] : 0x7fffffff;
      p[j] = t * k + j;
      w[j] = used ? wts[t * k + j] : 0.0f;
      if (used && e[j] < 0) e[j] = 0x7ffffffe;  // an invalid router row (flagged): no pair
    }
#pragma unroll
    for (int i = 1; i < 8; ++i)
#pragma unroll
      for (int j = i; j > 0; --j)
        if (e[j - 1] > e[j]) {
          const int te = e[j]; e[j] = e[j - 1]; e[j - 1] = te;
          const int tp = p[j]; p[j] = p[j - 1]; p[j - 1] = tp;
          const float tw = w[j]; w[j] = w[j - 1]; w[j - 1] = tw;
        }
    const int c = blockIdx.y * blockDim.x + threadIdx.x;
    if (c < h4) {
      const float4* rows = reinterpret_cast<const float4*>(own + d.L.ret_rows);
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < k && e[j] < 0x7ffffffe) v[j] = __ldcg(rows + static_cast<long long>(p[j]) * h4 + c);
      float4* yr = reinterpret_cast<float4*>(y + static_cast<long long>(t) * d.hidden) + c;
      float4 acc = *yr;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < k && e[j] < 0x7ffffffe) {
          acc.x = __fadd_rn(acc.x, __fmul_rn(w[j], v[j].x));
          acc.y = __fadd_rn(acc.y, __fmul_rn(w[j], v[j].y));
          acc.z = __fadd_rn(acc.z, __fmul_rn(w[j], v[j].z));
          acc.w = __fadd_rn(acc.w, __fmul_rn(w[j], v[j].w));
        }
      *yr = acc;
    }
  }
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(d.ctr + kCtrCombine, 1u) == gridDim.x * gridDim.y - 1u;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    d.ctr[kCtrCombine] = 0u;
    d.ctr[kCtrStep] = step;
  }
}

// Serialised handle of a rank's region.
struct EpHandle {
  char magic[8];
  int32_t world, rank, max_tokens, hidden, top_k, n_experts;
  uint64_t bytes;
  cudaIpcMemHandle_t ipc;
};
static_assert(sizeof(EpHandle) <= UOCR_EP_HANDLE_BYTES, "EpHandle too large");
const char kEpMagic[8] = {'U', 'O', 'C', 'R', 'E', 'P', '1', 0};

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

int err(int status, const char* msg) { return record_error(status, msg); }

int cuda_err(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorString(e);
  return record_error(UOCR_ERR_CUDA, m.c_str());
}

}  // namespace
}  // namespace uocr

struct uocr_ep {
  int device = 0;
  int world = 0, rank = 0, max_tokens = 0, cap = 0;
  int hidden = 0, width = 0, shared_width = 0, top_k = 0, n_experts = 0, local_experts = 0;
  int normalize = 0;
  float scale = 1.0f;
  const uocr_moe* layer = nullptr;
  EpLayout L{};
  char* region = nullptr;
  std::vector<char*> peers;
  std::vector<bool> opened;  // peers[r] came from cudaIpcOpenMemHandle
  char** peers_dev = nullptr;
  bool connected = false;
  int* owner_of = nullptr;
  int* local_of = nullptr;
  unsigned* ctr = nullptr;
  int* live = nullptr;
  unsigned* send_cnt = nullptr;  // [world] rows claimed per owner in the step's dispatch
  int32_t* ids = nullptr;
  float* wts = nullptr;
  float* pair_w = nullptr;  // grouping reads a weight per received row; never applied
  float* out_slots = nullptr;
  void* ws_routed = nullptr;
  size_t ws_routed_bytes = 0;
  void* ws_shared = nullptr;
  size_t ws_shared_bytes = 0;
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  unsigned long long wait_ns = kEpDefaultWaitNs;
  // uocr_ep_forward_host: device [x | logits | y] and a pinned mirror
  char* io = nullptr;
  char* io_host = nullptr;
  size_t io_x = 0, io_l = 0;  // byte offsets of logits and y
  bool cross_device = false;  // some peer is another GPU (set when connecting)
  // the step begun by uocr_ep_dispatch
  int step_tokens = -1;
  int step_mode = 0;
};

namespace {

EpDev ep_dev(const uocr_ep* ep, const uocr_ctx* ctx) {
  EpDev d{};
  d.peers = ep->peers_dev;
  d.L = ep->L;
  d.world = ep->world;
  d.rank = ep->rank;
  d.cap = ep->cap;
  d.hidden = ep->hidden;
  d.top_k = ep->top_k;
  d.n_experts = ep->n_experts;
  d.owner_of = ep->owner_of;
  d.local_of = ep->local_of;
  d.ctr = ep->ctr;
  d.live = ep->live;
  d.status = ctx->status_dev;
  d.wait_ns = ep->wait_ns;
  d.sys = ep->cross_device ? 1 : 0;
  return d;
}

// Arguments of one part of the local layer (moe_prefill.cu).
MoePrefillArgs part_args(const uocr_ep* ep, const uocr_ctx* ctx) {
  const uocr_moe* Lr = ep->layer;
  MoePrefillArgs a{};
  a.experts = Lr->experts_dev;
  a.shared = Lr->shared;
  a.n_experts = static_cast<int>(Lr->n_experts);
  a.top_k = 1;
  a.scale = 1.0f;
  a.hidden = Lr->hidden;
  a.width = Lr->width;
  a.shared_width = Lr->shared_width;
  a.status = ctx->status_dev;
  a.tc_maps = Lr->tc_maps;
  a.route_given = 1;
  return a;
}

// The routed rows of `rows` consecutive receive slots from `first`.
MoePrefillArgs routed_args(const uocr_ep* ep, const uocr_ctx* ctx, int first, int rows, int max_group) {
  MoePrefillArgs a = part_args(ep, ctx);
  a.tokens = rows;
  a.x = reinterpret_cast<const float*>(ep->region + ep->L.recv_x) +
        static_cast<long long>(first) * ep->hidden;
  a.route_ids = reinterpret_cast<int32_t*>(ep->region + ep->L.recv_ids) + first;
  a.route_weights = ep->pair_w;
  a.skip_shared = 1;
  a.skip_negative_ids = 1;
  a.pair_out = ep->out_slots + static_cast<long long>(first) * ep->hidden;
  a.max_group_rows = max_group;
  // every group on the warp-level kernel, one CTA per 8-row chunk (at decode
  // batch sizes groups hold tens of rows; a large group re-reads its
  // weights from L2 once per chunk)
  a.small_max = max_group;
  a.workspace = ep->ws_routed;
  a.workspace_bytes = ep->ws_routed_bytes;
  return a;
}

MoePrefillArgs shared_args(const uocr_ep* ep, const uocr_ctx* ctx, const float* x, int tokens,
                           float* y) {
  MoePrefillArgs a = part_args(ep, ctx);
  a.tokens = tokens;
  a.x = x;
  a.y = y;
  a.route_ids = ep->ids;
  a.route_weights = ep->pair_w;
  a.skip_routed = 1;
  a.workspace = ep->ws_shared;
  a.workspace_bytes = ep->ws_shared_bytes;
  return a;
}

int check_ctx(const uocr_ctx* ctx, const uocr_ep* ep) {
  if (!ctx || !ep) return err(UOCR_ERR_INVALID, "null argument");
  if (ctx->device != ep->device)
    return err(UOCR_ERR_UNSUPPORTED, "unsupported configuration: expert-parallel layer on another device");
  if (!ep->connected) return err(UOCR_ERR_INVALID, "expert-parallel layer is not connected to its peers");
  return UOCR_OK;
}

int check_mode(int mode) {
  if (mode != UOCR_WEIGHTS_ONLY && mode != UOCR_DYNAMIC_ACTIVATIONS && mode != UOCR_DYNAMIC_ROWWISE)
    return err(UOCR_ERR_UNSUPPORTED, "unsupported configuration: mode");
  return UOCR_OK;
}

// CpuContext::check_elements (src/cpu/mod.rs:73-78) for the shared expert's
// projections at `tokens` rows, as uocr_moe_forward applies it.
int check_scratch(const uocr_ctx* ctx, const uocr_ep* ep, size_t tokens) {
  const size_t H = ep->hidden, FS = ep->shared_width;
  const size_t counts[2] = {tokens * FS, tokens * H};
  const size_t mats[2] = {FS * H, H * FS};
  for (int i = 0; i < 2; ++i) {
    size_t c = counts[i] + (tokens != 1 ? mats[i] : 0);
    if (c > ctx->scratch_limit / 4)
      return err(UOCR_ERR_RESOURCE, "resource limit: operation exceeds scratch limit");
  }
  return UOCR_OK;
}

// Enqueues route + dispatch on `rs` and the shared expert on `ss`.
int enqueue_dispatch(uocr_ctx* ctx, uocr_ep* ep, int mode, const float* x, const float* logits,
                     int tokens, float* y, cudaStream_t rs, cudaStream_t ss) {
  const EpDev d = ep_dev(ep, ctx);
  const int grid = tokens > 0 ? (tokens + kRdWarps - 1) / kRdWarps : 1;
  const size_t smem = sizeof(float) * kRdWarps * (ep->n_experts + 2 * ep->top_k);
  ep_route_dispatch_kernel<<<grid, kRdWarps * 32, smem, rs>>>(
      d, x, logits, tokens, ep->normalize, ep->scale, ep->ids, ep->wts, ep->send_cnt);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(e, "expert-parallel dispatch");
  if (tokens > 0) {
    e = launch_moe_prefill(mode, shared_args(ep, ctx, x, tokens, y), ctx->sms, ss);
    if (e != cudaSuccess) return cuda_err(e, "expert-parallel shared expert");
  }
  return UOCR_OK;
}

// Enqueues wait + routed experts + return on `rs`.
int enqueue_experts(uocr_ctx* ctx, uocr_ep* ep, int mode, cudaStream_t rs) {
  const EpDev d = ep_dev(ep, ctx);
  cudaError_t e = launch_dependent(ep_recv_wait_kernel, dim3(1), dim3(kEpThreads), 0, rs, d);
  if (e != cudaSuccess) return cuda_err(e, "expert-parallel wait");
  const float* rows = ep->out_slots;
  const int* token_pos = nullptr;
  if (mode == UOCR_DYNAMIC_ACTIVATIONS) {
    // a group's row count selects its arithmetic: one call per source block,
    // outputs into out_slots in slot order
    for (int s = 0; s < ep->world && e == cudaSuccess; ++s)
      e = launch_moe_prefill(mode, routed_args(ep, ctx, s * ep->cap, ep->cap, ep->max_tokens),
                             ctx->sms, rs);
  } else {
    // one call over every source block; the return reads the grouped outputs
    MoePrefillArgs a =
        routed_args(ep, ctx, 0, ep->world * ep->cap, ep->world * ep->max_tokens);
    a.pair_out = nullptr;
    a.keep_grouped = 1;
    e = launch_moe_prefill(mode, a, ctx->sms, rs);
    moe_prefill_grouped(a, mode, &token_pos, &rows);
  }
  if (e != cudaSuccess) return cuda_err(e, "expert-parallel experts");
  const int total_warps = ep->world * ep->cap;
  int grid = (total_warps + kEpWarps - 1) / kEpWarps;
  if (grid > 2 * ctx->sms) grid = 2 * ctx->sms;
  e = launch_dependent(ep_return_kernel, dim3(grid), dim3(kEpThreads), 0, rs, d, rows, token_pos);
  if (e != cudaSuccess) return cuda_err(e, "expert-parallel return");
  return UOCR_OK;
}

int enqueue_combine(uocr_ctx* ctx, uocr_ep* ep, int tokens, float* y, int32_t* ids_out,
                    float* wts_out, cudaStream_t st) {
  const EpDev d = ep_dev(ep, ctx);
  const dim3 grid(tokens > 0 ? tokens : 1, (ep->hidden / 4 + 127) / 128);
  cudaError_t e = launch_dependent(ep_combine_kernel, grid, dim3(128), 0, st, d,
                                   static_cast<const int32_t*>(ep->ids),
                                   static_cast<const float*>(ep->wts), tokens, y);
  if (e != cudaSuccess) return cuda_err(e, "expert-parallel combine");
  const size_t rb = sizeof(float) * static_cast<size_t>(tokens) * ep->top_k;
  if (ids_out && tokens > 0) e = cudaMemcpyAsync(ids_out, ep->ids, rb, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && wts_out && tokens > 0)
    e = cudaMemcpyAsync(wts_out, ep->wts, rb, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return cuda_err(e, "expert-parallel routing copy");
  return UOCR_OK;
}

int step_checks(const uocr_ctx* ctx, const uocr_ep* ep, int mode, const float* x,
                const float* logits, size_t tokens, const float* y) {
  int st = check_ctx(ctx, ep);
  if (st || (st = check_mode(mode))) return st;
  if (tokens > static_cast<size_t>(ep->max_tokens))
    return err(UOCR_ERR_RESOURCE, "resource limit exceeded: more tokens than the expert-parallel layer's max_tokens");
  if (tokens > 0) {
    if (!x || !logits || !y) return err(UOCR_ERR_INVALID, "null argument");
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(y) % 16)
      return err(UOCR_ERR_UNSUPPORTED, "unsupported configuration: x and y must be 16-byte aligned");
  }
  return check_scratch(ctx, ep, tokens);
}

void release(uocr_ep* ep) {
  Device g(ep->device);
  for (size_t r = 0; r < ep->peers.size(); ++r)
    if (ep->opened[r] && ep->peers[r]) cudaIpcCloseMemHandle(ep->peers[r]);
  if (ep->side) {
    cudaStreamSynchronize(ep->side);
    cudaStreamDestroy(ep->side);
  }
  if (ep->ev_fork) cudaEventDestroy(ep->ev_fork);
  if (ep->ev_join) cudaEventDestroy(ep->ev_join);
  void* bufs[] = {ep->region, ep->peers_dev, ep->owner_of, ep->local_of, ep->ctr, ep->live,
                  ep->send_cnt,
                  ep->ids, ep->wts, ep->pair_w, ep->out_slots, ep->ws_routed, ep->ws_shared,
                  ep->io};
  for (void* b : bufs)
    if (b) cudaFree(b);
  if (ep->io_host) cudaFreeHost(ep->io_host);
  delete ep;
}

}  // namespace

extern "C" {

int uocr_ep_create(uocr_ctx* ctx, const uocr_moe* local_layer, size_t n_experts, size_t top_k,
                   int normalize_topk, float routed_scale, const int32_t* rank_bounds, size_t world,
                   size_t rank, size_t max_tokens, uocr_ep** out) {
  if (!ctx || !local_layer || !rank_bounds || !out) return err(UOCR_ERR_INVALID, "null argument");
  *out = nullptr;
  if (world < 1 || world > static_cast<size_t>(kEpMaxWorld) || rank >= world)
    return err(UOCR_ERR_UNSUPPORTED, "unsupported configuration: 1 <= world <= 64, rank < world");
  if (n_experts == 0 || n_experts > 256 || top_k == 0 || top_k > 8 || top_k > n_experts)
    return err(UOCR_ERR_SHAPE, "invalid tensor shape: top_k must be in 1..=n_experts (<= 8 of <= 256)");
  if (!(routed_scale > 0.0f) || !std::isfinite(routed_scale))
    return err(UOCR_ERR_SHAPE, "invalid tensor shape: routed scaling factor must be finite and positive");
  if (max_tokens == 0 || max_tokens > 65536)
    return err(UOCR_ERR_UNSUPPORTED, "unsupported configuration: 1 <= max_tokens <= 65536");
  if (local_layer->device != ctx->device)
    return err(UOCR_ERR_UNSUPPORTED, "unsupported configuration: layer on another device");
  if (local_layer->hidden % 4)
    return err(UOCR_ERR_UNSUPPORTED, "unsupported configuration: hidden % 4 == 0");
  std::vector<int> bounds(world + 1);
  for (size_t r = 0; r <= world; ++r) {
    bounds[r] = rank_bounds[r];
    if (r > 0 && bounds[r] <= bounds[r - 1])
      return err(UOCR_ERR_SHAPE, "invalid tensor shape: rank bounds must increase");
  }
  if (bounds[0] != 0 || bounds[world] != static_cast<int>(n_experts))
    return err(UOCR_ERR_SHAPE, "invalid tensor shape: rank bounds must run from 0 to n_experts");
  if (static_cast<size_t>(bounds[rank + 1] - bounds[rank]) != local_layer->n_experts)
    return err(UOCR_ERR_SHAPE, "invalid tensor shape: the local layer must hold this rank's block of experts");
  Device g(ctx->device);
  auto* ep = new uocr_ep();
  ep->device = ctx->device;
  ep->world = static_cast<int>(world);
  ep->rank = static_cast<int>(rank);
  ep->max_tokens = static_cast<int>(max_tokens);
  ep->cap = static_cast<int>(max_tokens * top_k);
  ep->hidden = local_layer->hidden;
  ep->width = local_layer->width;
  ep->shared_width = local_layer->shared_width;
  ep->top_k = static_cast<int>(top_k);
  ep->n_experts = static_cast<int>(n_experts);
  ep->local_experts = static_cast<int>(local_layer->n_experts);
  ep->normalize = normalize_topk ? 1 : 0;
  ep->scale = routed_scale;
  ep->layer = local_layer;
  ep->L = ep_layout(ep->world, ep->cap, ep->hidden);
  ep->peers.assign(world, nullptr);
  ep->opened.assign(world, false);
  std::vector<int> owner(n_experts), local(n_experts);
  for (size_t r = 0; r < world; ++r)
    for (int e = bounds[r]; e < bounds[r + 1]; ++e) {
      owner[e] = static_cast<int>(r);
      local[e] = e - bounds[r];
    }
  const size_t rows = static_cast<size_t>(ep->world) * ep->cap;
  // workspaces of the two parts, sized for the largest mode
  MoePrefillArgs ra = part_args(ep, ctx);
  ra.tokens = static_cast<int>(rows);
  ra.skip_shared = 1;
  ra.skip_negative_ids = 1;
  ra.max_group_rows = ep->world * ep->max_tokens;
  MoePrefillArgs sa = part_args(ep, ctx);
  sa.tokens = ep->max_tokens;
  sa.skip_routed = 1;
  for (int m = 0; m < 3; ++m) {
    ep->ws_routed_bytes = std::max(ep->ws_routed_bytes, moe_prefill_workspace(ra, m));
    ep->ws_shared_bytes = std::max(ep->ws_shared_bytes, moe_prefill_workspace(sa, m));
  }
  cudaError_t e = cudaMalloc(&ep->region, ep->L.bytes);
  if (e == cudaSuccess) e = cudaMemset(ep->region, 0, ep->L.bytes);
  if (e == cudaSuccess) e = cudaMalloc(&ep->peers_dev, sizeof(char*) * world);
  if (e == cudaSuccess) e = cudaMalloc(&ep->owner_of, sizeof(int) * n_experts);
  if (e == cudaSuccess) e = cudaMalloc(&ep->local_of, sizeof(int) * n_experts);
  if (e == cudaSuccess)
    e = cudaMemcpy(ep->owner_of, owner.data(), sizeof(int) * n_experts, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(ep->local_of, local.data(), sizeof(int) * n_experts, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&ep->ctr, sizeof(unsigned) * kCtrWords);
  if (e == cudaSuccess) e = cudaMemset(ep->ctr, 0, sizeof(unsigned) * kCtrWords);
  if (e == cudaSuccess) e = cudaMalloc(&ep->live, sizeof(int) * world);
  if (e == cudaSuccess) e = cudaMemset(ep->live, 0, sizeof(int) * world);
  if (e == cudaSuccess) e = cudaMalloc(&ep->send_cnt, sizeof(unsigned) * world);
  if (e == cudaSuccess) e = cudaMemset(ep->send_cnt, 0, sizeof(unsigned) * world);
  if (e == cudaSuccess) e = cudaMalloc(&ep->ids, sizeof(int32_t) * ep->cap);
  if (e == cudaSuccess) e = cudaMalloc(&ep->wts, sizeof(float) * ep->cap);
  if (e == cudaSuccess) e = cudaMalloc(&ep->pair_w, sizeof(float) * rows);
  if (e == cudaSuccess) e = cudaMemset(ep->pair_w, 0, sizeof(float) * rows);
  if (e == cudaSuccess) e = cudaMalloc(&ep->out_slots, sizeof(float) * rows * ep->hidden);
  if (e == cudaSuccess) e = cudaMalloc(&ep->ws_routed, ep->ws_routed_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&ep->ws_shared, ep->ws_shared_bytes);
  ep->io_x = al256(sizeof(float) * max_tokens * ep->hidden);
  ep->io_l = ep->io_x + al256(sizeof(float) * max_tokens * n_experts);
  const size_t io_bytes = ep->io_l + al256(sizeof(float) * max_tokens * ep->hidden);
  if (e == cudaSuccess) e = cudaMalloc(&ep->io, io_bytes);
  if (e == cudaSuccess) e = cudaMallocHost(&ep->io_host, io_bytes);
  int least = 0, greatest = 0;
  if (e == cudaSuccess) e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&ep->side, cudaStreamNonBlocking, greatest);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ep->ev_fork, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ep->ev_join, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    release(ep);
    return cuda_err(e, "uocr_ep_create");
  }
  ep->peers[ep->rank] = ep->region;
  *out = ep;
  return UOCR_OK;
}

int uocr_ep_free(uocr_ep* ep) {
  if (ep) release(ep);
  return UOCR_OK;
}

int uocr_ep_handle(const uocr_ep* ep, void* handle_out) {
  if (!ep || !handle_out) return err(UOCR_ERR_INVALID, "null argument");
  EpHandle h{};
  std::memcpy(h.magic, kEpMagic, sizeof h.magic);
  h.world = ep->world;
  h.rank = ep->rank;
  h.max_tokens = ep->max_tokens;
  h.hidden = ep->hidden;
  h.top_k = ep->top_k;
  h.n_experts = ep->n_experts;
  h.bytes = static_cast<uint64_t>(ep->L.bytes);
  Device g(ep->device);
  const cudaError_t e = cudaIpcGetMemHandle(&h.ipc, ep->region);
  if (e != cudaSuccess) return cuda_err(e, "cudaIpcGetMemHandle");
  std::memset(handle_out, 0, UOCR_EP_HANDLE_BYTES);
  std::memcpy(handle_out, &h, sizeof h);
  return UOCR_OK;
}

static int finish_connect(uocr_ep* ep) {
  Device g(ep->device);
  const cudaError_t e = cudaMemcpy(ep->peers_dev, ep->peers.data(), sizeof(char*) * ep->world,
                                   cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_err(e, "expert-parallel peer table");
  ep->connected = true;
  return UOCR_OK;
}

int uocr_ep_connect(uocr_ep* ep, const void* handles) {
  if (!ep || !handles) return err(UOCR_ERR_INVALID, "null argument");
  if (ep->connected) return err(UOCR_ERR_INVALID, "expert-parallel layer is already connected");
  const unsigned char* hb = static_cast<const unsigned char*>(handles);
  std::vector<EpHandle> hs(ep->world);
  for (int r = 0; r < ep->world; ++r) {
    std::memcpy(&hs[r], hb + static_cast<size_t>(r) * UOCR_EP_HANDLE_BYTES, sizeof(EpHandle));
    const EpHandle& h = hs[r];
    if (std::memcmp(h.magic, kEpMagic, sizeof h.magic) != 0)
      return err(UOCR_ERR_FORMAT, "invalid expert-parallel handle");
    if (h.world != ep->world || h.rank != r || h.max_tokens != ep->max_tokens ||
        h.hidden != ep->hidden || h.top_k != ep->top_k || h.n_experts != ep->n_experts ||
        h.bytes != static_cast<uint64_t>(ep->L.bytes))
      return err(UOCR_ERR_SHAPE,
                 "invalid tensor shape: expert-parallel handles disagree (world, rank order, max_tokens, hidden, top_k or experts)");
  }
  Device g(ep->device);
  for (int r = 0; r < ep->world; ++r) {
    if (r == ep->rank) continue;
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, hs[r].ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (ep->opened[q]) {
          cudaIpcCloseMemHandle(ep->peers[q]);
          ep->peers[q] = nullptr;
          ep->opened[q] = false;
        }
      return cuda_err(e, "cudaIpcOpenMemHandle");
    }
    ep->peers[r] = static_cast<char*>(p);
    ep->opened[r] = true;
    ep->cross_device = true;  // another process: fences at system scope
  }
  return finish_connect(ep);
}

int uocr_ep_connect_local(uocr_ep* const* eps, size_t world) {
  if (!eps || world == 0) return err(UOCR_ERR_INVALID, "null argument");
  for (size_t r = 0; r < world; ++r) {
    const uocr_ep* ep = eps[r];
    if (!ep) return err(UOCR_ERR_INVALID, "null argument");
    if (static_cast<size_t>(ep->world) != world || ep->rank != static_cast<int>(r) ||
        ep->max_tokens != eps[0]->max_tokens || ep->hidden != eps[0]->hidden ||
        ep->top_k != eps[0]->top_k || ep->n_experts != eps[0]->n_experts)
      return err(UOCR_ERR_SHAPE,
                 "invalid tensor shape: expert-parallel layers disagree (world, rank order, max_tokens, hidden, top_k or experts)");
    if (ep->connected) return err(UOCR_ERR_INVALID, "expert-parallel layer is already connected");
  }
  for (size_t r = 0; r < world; ++r) {
    uocr_ep* ep = eps[r];
    Device g(ep->device);
    for (size_t q = 0; q < world; ++q) {
      ep->peers[q] = eps[q]->region;
      if (eps[q]->device != ep->device) {
        ep->cross_device = true;
        const cudaError_t e = cudaDeviceEnablePeerAccess(eps[q]->device, 0);
        if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
          return cuda_err(e, "cudaDeviceEnablePeerAccess");
        cudaGetLastError();
      }
    }
  }
  for (size_t r = 0; r < world; ++r) {
    const int st = finish_connect(eps[r]);
    if (st) return st;
  }
  return UOCR_OK;
}

int uocr_ep_set_wait_limit(uocr_ep* ep, uint64_t ns) {
  if (!ep) return err(UOCR_ERR_INVALID, "null argument");
  if (ns == 0) return err(UOCR_ERR_UNSUPPORTED, "unsupported configuration: wait limit 0");
  ep->wait_ns = ns;
  return UOCR_OK;
}

int uocr_ep_forward(uocr_ctx* ctx, uocr_ep* ep, int mode, const float* x_dev,
                    const float* logits_dev, size_t tokens, float* y_dev, int32_t* ids_dev,
                    float* weights_dev) {
  int st = step_checks(ctx, ep, mode, x_dev, logits_dev, tokens, y_dev);
  if (st) return st;
  if (ep->step_tokens >= 0)
    return err(UOCR_ERR_INVALID, "an expert-parallel step begun by uocr_ep_dispatch is not finished");
  Device g(ctx->device);
  const int T = static_cast<int>(tokens);
  // the exchange chain on the high-priority side stream, the shared expert on
  // the context's stream, joined before the combine
  cudaError_t e = cudaEventRecord(ep->ev_fork, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ep->side, ep->ev_fork, 0);
  if (e != cudaSuccess) return cuda_err(e, "expert-parallel fork");
  if ((st = enqueue_dispatch(ctx, ep, mode, x_dev, logits_dev, T, y_dev, ep->side, ctx->stream)) ||
      (st = enqueue_experts(ctx, ep, mode, ep->side)))
    return st;
  e = cudaEventRecord(ep->ev_join, ep->side);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, ep->ev_join, 0);
  if (e != cudaSuccess) return cuda_err(e, "expert-parallel join");
  return enqueue_combine(ctx, ep, T, y_dev, ids_dev, weights_dev, ctx->stream);
}

int uocr_ep_forward_host(uocr_ctx* ctx, uocr_ep* ep, int mode, const float* x,
                         const float* logits, size_t tokens, float* y) {
  int st = check_ctx(ctx, ep);
  if (st || (st = check_mode(mode))) return st;
  if (tokens > static_cast<size_t>(ep->max_tokens))
    return err(UOCR_ERR_RESOURCE, "resource limit exceeded: more tokens than the expert-parallel layer's max_tokens");
  if (tokens > 0 && (!x || !logits || !y)) return err(UOCR_ERR_INVALID, "null argument");
  Device g(ctx->device);
  const size_t xb = sizeof(float) * tokens * ep->hidden;
  const size_t lb = sizeof(float) * tokens * ep->n_experts;
  float* xd = reinterpret_cast<float*>(ep->io);
  float* ld = reinterpret_cast<float*>(ep->io + ep->io_x);
  float* yd = reinterpret_cast<float*>(ep->io + ep->io_l);
  // pinned caller buffers are copied directly, others through the mirror
  auto pinned = [](const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return a.type == cudaMemoryTypeHost;
  };
  const bool direct = tokens > 0 && pinned(x) && pinned(logits) && pinned(y);
  cudaError_t e = cudaSuccess;
  if (tokens > 0) {
    const void* hx = x;
    const void* hl = logits;
    if (!direct) {
      std::memcpy(ep->io_host, x, xb);
      std::memcpy(ep->io_host + ep->io_x, logits, lb);
      hx = ep->io_host;
      hl = ep->io_host + ep->io_x;
    }
    e = cudaMemcpyAsync(xd, hx, xb, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ld, hl, lb, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_err(e, "expert-parallel input copy");
  }
  if ((st = uocr_ep_forward(ctx, ep, mode, xd, ld, tokens, yd, nullptr, nullptr))) return st;
  if (tokens > 0) {
    e = cudaMemcpyAsync(direct ? static_cast<void*>(y) : ep->io_host + ep->io_l, yd, xb,
                        cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_err(e, "expert-parallel output copy");
  }
  if ((st = uocr_ctx_sync(ctx))) return st;
  if (tokens > 0 && !direct) std::memcpy(y, ep->io_host + ep->io_l, xb);
  return UOCR_OK;
}

int uocr_ep_dispatch(uocr_ctx* ctx, uocr_ep* ep, int mode, const float* x_dev,
                     const float* logits_dev, size_t tokens, float* y_dev) {
  int st = step_checks(ctx, ep, mode, x_dev, logits_dev, tokens, y_dev);
  if (st) return st;
  if (ep->step_tokens >= 0) return err(UOCR_ERR_INVALID, "expert-parallel step already begun");
  Device g(ctx->device);
  if ((st = enqueue_dispatch(ctx, ep, mode, x_dev, logits_dev, static_cast<int>(tokens), y_dev,
                             ctx->stream, ctx->stream)))
    return st;
  ep->step_tokens = static_cast<int>(tokens);
  ep->step_mode = mode;
  return UOCR_OK;
}

int uocr_ep_experts(uocr_ctx* ctx, uocr_ep* ep) {
  int st = check_ctx(ctx, ep);
  if (st) return st;
  if (ep->step_tokens < 0) return err(UOCR_ERR_INVALID, "no expert-parallel step begun");
  Device g(ctx->device);
  return enqueue_experts(ctx, ep, ep->step_mode, ctx->stream);
}

int uocr_ep_combine(uocr_ctx* ctx, uocr_ep* ep, float* y_dev, int32_t* ids_dev, float* weights_dev) {
  int st = check_ctx(ctx, ep);
  if (st) return st;
  if (ep->step_tokens < 0) return err(UOCR_ERR_INVALID, "no expert-parallel step begun");
  if (ep->step_tokens > 0 && !y_dev) return err(UOCR_ERR_INVALID, "null argument");
  Device g(ctx->device);
  const int T = ep->step_tokens;
  ep->step_tokens = -1;
  return enqueue_combine(ctx, ep, T, y_dev, ids_dev, weights_dev, ctx->stream);
}

}  // extern "C"
