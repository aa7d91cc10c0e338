// moe_decode.cu — Decoder::experts for one token (src/decoder/mod.rs:124-220)
// as two kernels chained with programmatic dependent launch (PDL).
//
// Units: unit 0 is the fused shared-expert FFN (width shared_width, the
// reference's n_shared_experts*moe_intermediate_size fusion,
// src/decoder/mod.rs:71-75); units 1..top_k are the selected routed experts
// in ascending expert id, which is the order Decoder::experts adds them.
//
// moe_up_kernel (grid = #SMs, 1 producer + 8 consumer warps)
//   Each CTA owns an equal slice of the shared expert's rows and an equal
//   slice of the routed units' rows (so every CTA can start streaming shared
//   weights before routing is known).  A producer warp moves stages of up to
//   8 gate rows + the same 8 up rows (+ their block scales) into a 4-stage
//   shared-memory ring with 1-D bulk async copies; it computes moe::route for
//   the token meanwhile.  Consumer warps compute gate and up dots from shared
//   memory and write h = silu(gate) * up (Decoder::feed_forward,
//   src/decoder/mod.rs:114-122) to a global scratch vector.
// moe_down_kernel (grid = #SMs, 8 warps)
//   Launched as a PDL dependent of moe_up_kernel, so it becomes resident
//   while moe_up_kernel streams: each CTA recomputes the routing, then
//   prefetches its rows [i0, i1) of every unit's down matrix into shared
//   memory before griddepcontrol.wait.  After the wait it loads all of h (and
//   block-quantizes it in int8 mode, as projection() does for the down input
//   in DynamicActivations mode), computes the unit outputs for its rows and
//   combines them in the reference's order: r = shared; r += p_e * out_e for
//   e ascending, one rounding per multiply and per add.
#include "common.cuh"
#include "kernels.h"
#include "route.cuh"

namespace uocr {

constexpr int kUpConsumerWarps = 8;
constexpr int kUpThreads = (kUpConsumerWarps + 1) * 32;
constexpr int kUpStages = 4;
constexpr int kUpTileRows = 8;
constexpr int kDownThreads = 256;
constexpr int kMaxTopK = 8;
constexpr int kMaxRouteExperts = 256;

struct StageDesc {
  int unit, j0, nr;
};

// Deterministic enumeration of one CTA's stages, replayed identically by the
// producer and the consumers.
struct StageIter {
  int s_cur, s_end, r_cur, r_end, width;
  __device__ void init(int cta, int grid, int shared_width, int routed_rows, int w) {
    s_cur = static_cast<int>(static_cast<long long>(shared_width) * cta / grid);
    s_end = static_cast<int>(static_cast<long long>(shared_width) * (cta + 1) / grid);
    r_cur = static_cast<int>(static_cast<long long>(routed_rows) * cta / grid);
    r_end = static_cast<int>(static_cast<long long>(routed_rows) * (cta + 1) / grid);
    width = w;
  }
  __device__ bool next(StageDesc& d) {
    if (s_cur < s_end) {
      d.unit = 0;
      d.j0 = s_cur;
      d.nr = min(kUpTileRows, s_end - s_cur);
      s_cur += d.nr;
      return true;
    }
    if (r_cur < r_end) {
      const int u = r_cur / width, j = r_cur - u * width;
      d.unit = 1 + u;
      d.j0 = j;
      d.nr = min(kUpTileRows, min(r_end - r_cur, width - j));
      r_cur += d.nr;
      return true;
    }
    return false;
  }
  __device__ bool next_is_shared() const { return s_cur < s_end; }
};

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Two FP32-mode dots sharing x (gate and up rows of the same index).
__device__ __forceinline__ void pair_dot_fp32(const int8_t* g, const float* gs, const int8_t* u,
                                              const float* us, const float* xsm, int cols,
                                              int lane, float& og, float& ou) {
  float ag = 0.0f, au = 0.0f;
#pragma unroll 2
  for (int k0 = lane * 4; k0 < cols; k0 += 128) {
    const float4 xv = *reinterpret_cast<const float4*>(xsm + k0);
    const int b = k0 >> 5;
    ag = fmaf(gs[b], dot4_i8_f32(*reinterpret_cast<const uint32_t*>(g + k0), xv), ag);
    au = fmaf(us[b], dot4_i8_f32(*reinterpret_cast<const uint32_t*>(u + k0), xv), au);
  }
  og = warp_sum(ag);
  ou = warp_sum(au);
}

// Ordered int8-mode dot (bit-exact linear_dynamic_int8 row).
__device__ __forceinline__ float dot_int8_ordered(const int8_t* wrow, const float* srow,
                                                  const int8_t* xq, const float* xs, int cols,
                                                  int lane) {
  float acc = -0.0f;
  for (int k0 = lane * 4; k0 < cols; k0 += 128) {
    const int b = k0 >> 5;
    int p = __dp4a(*reinterpret_cast<const int*>(wrow + k0),
                   *reinterpret_cast<const int*>(xq + k0), 0);
    p += __shfl_xor_sync(0xffffffffu, p, 1);
    p += __shfl_xor_sync(0xffffffffu, p, 2);
    p += __shfl_xor_sync(0xffffffffu, p, 4);
    const float t = __fmul_rn(__fmul_rn(static_cast<float>(p), srow[b]), xs[b]);
    acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, t, 0));
    acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, t, 8));
    acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, t, 16));
    acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, t, 24));
  }
  return acc;
}

__device__ __forceinline__ float dot_fp32_smem(const int8_t* wrow, const float* srow,
                                               const float* xsm, int cols, int lane) {
  float acc = 0.0f;
#pragma unroll 2
  for (int k0 = lane * 4; k0 < cols; k0 += 128) {
    const float4 xv = *reinterpret_cast<const float4*>(xsm + k0);
    acc = fmaf(srow[k0 >> 5], dot4_i8_f32(*reinterpret_cast<const uint32_t*>(wrow + k0), xv), acc);
  }
  return warp_sum(acc);
}

// Block quantization of a float vector in shared memory by `nw` warps
// starting at warp `w0` (the activation step of linear_dynamic_int8).
__device__ __forceinline__ void quantize_vec_smem(const float* v, int n, int8_t* q, float* s,
                                                 int warp, int nw, unsigned* status) {
  const int lane = threadIdx.x & 31;
  const int nb = blocks_of(n);
  for (int b = warp; b < nb; b += nw) {
    const int k = b * kBlock + lane;
    const bool in = k < n;
    const float x = in ? v[k] : 0.0f;
    const bool bad = in && !isfinite(x);
    if (__any_sync(0xffffffffu, bad) && lane == 0) flag(status, DEV_NONFINITE);
    const float mx = warp_max(in ? fabsf(x) : 0.0f);
    const float scale = __fdiv_rn(mx, 127.0f);
    if (lane == 0) {
      if (mx > 0.0f && scale == 0.0f) flag(status, DEV_UNDERFLOW);
      s[b] = scale;
    }
    if (in) q[k] = quantize_elem(x, scale);
  }
}

__device__ __forceinline__ int h_base(int unit, int shared_width, int width) {
  return unit == 0 ? 0 : shared_width + (unit - 1) * width;
}

// ---------------------------------------------------------------------------
template <int MODE, int CPL>
__global__ void __launch_bounds__(kUpThreads, 1) moe_up_kernel(const __grid_constant__ MoeDecodeArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.hidden, nbH = H >> 5;
  const int stage_w = kUpTileRows * H, stage_s = kUpTileRows * nbH * 4;
  const int stage_bytes = 2 * stage_w + 2 * stage_s;
  unsigned char* ring = smem;
  float* xsm = reinterpret_cast<float*>(smem + kUpStages * stage_bytes);
  int8_t* xq = reinterpret_cast<int8_t*>(xsm + H);
  float* xs = reinterpret_cast<float*>(xq + H);
  float* rp = xs + nbH;                                  // routing scratch [n_experts]
  float* red = rp + a.n_experts;                         // [32]
  int* bad = reinterpret_cast<int*>(red + 32);           // [1] (+3 pad)
  int* sel = bad + 4;                                    // [kMaxTopK] route order
  float* selw = reinterpret_cast<float*>(sel + kMaxTopK);
  int* sorted = reinterpret_cast<int*>(selw + kMaxTopK); // [kMaxTopK] ascending id
  float* sortedw = reinterpret_cast<float*>(sorted + kMaxTopK);
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(sortedw + kMaxTopK) + 15) & ~static_cast<uintptr_t>(15));
  uint64_t* empty = full + kUpStages;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool producer = warp == kUpConsumerWarps && lane == 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kUpStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kUpConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // Producer state (used by one thread).
  StageIter itp;
  itp.init(blockIdx.x, gridDim.x, a.shared_width, a.top_k * a.width, a.width);
  int it = 0;
  bool ok = true;
  auto issue = [&](const StageDesc& d) {
    const FfnView fv = d.unit == 0 ? a.shared : a.experts[sorted[d.unit - 1]];
    const int stage = it % kUpStages;
    if (it >= kUpStages) ok = mbar_wait(&empty[stage], ((it / kUpStages) - 1) & 1, a.status);
    if (!ok) return;
    unsigned char* dst = ring + stage * stage_bytes;
    const int wb = d.nr * H, sb = d.nr * nbH * 4;
    mbar_arrive_expect_tx(&full[stage], 2 * wb + 2 * sb);
    bulk_g2s(dst, fv.gate.w + static_cast<long long>(d.j0) * H, wb, &full[stage]);
    bulk_g2s(dst + stage_w, fv.up.w + static_cast<long long>(d.j0) * H, wb, &full[stage]);
    bulk_g2s(dst + 2 * stage_w, fv.gate.s + static_cast<long long>(d.j0) * nbH, sb, &full[stage]);
    bulk_g2s(dst + 2 * stage_w + stage_s, fv.up.s + static_cast<long long>(d.j0) * nbH, sb,
             &full[stage]);
    ++it;
  };
  StageDesc d;
  // 1. shared-expert stages need neither routing nor the previous kernel's
  //    output: start streaming them immediately.
  if (producer)
    while (ok && it < kUpStages && itp.next_is_shared() && itp.next(d)) issue(d);

  // 2. x and the router logits may come from the previous kernel.
  pdl_wait_prior_grids();
  for (int k = threadIdx.x; k < H; k += blockDim.x) xsm[k] = a.x[k];
  const bool routed = route_row_block(a.logits, a.n_experts, a.top_k, a.normalize, a.scale, rp,
                                      red, sel, selw, bad, a.status);
  if (threadIdx.x == 0) {
    for (int r = 0; r < a.top_k; ++r) {
      sorted[r] = routed ? sel[r] : r;  // invalid row: keep addresses valid, status flagged
      sortedw[r] = routed ? selw[r] : 0.0f;
    }
    sort_by_id(sorted, sortedw, a.top_k);
    if (blockIdx.x == 0)
      for (int r = 0; r < a.top_k; ++r) {
        a.route_ids[r] = routed ? sel[r] : -1;
        a.route_weights[r] = routed ? selw[r] : 0.0f;
      }
  }
  __syncthreads();
  // Every prerequisite of this grid is complete: the dependent down kernel
  // may now launch and read the logits.
  pdl_launch_dependents();
  if (MODE == MODE_INT8) {
    quantize_vec_smem(xsm, H, xq, xs, warp, blockDim.x >> 5, a.status);
    __syncthreads();
  }

  if (warp == kUpConsumerWarps) {
    // 3. the remaining stages
    if (producer) {
      while (ok && itp.next(d)) issue(d);
      const int issued = it;
      for (int j = issued - kUpStages; j < issued; ++j)
        if (j >= 0) mbar_wait(&full[j % kUpStages], (j / kUpStages) & 1, a.status);
    }
    return;
  }

  // ---------------- consumer warps ----------------
  // FP32 mode with hidden = 256*CPL: this lane's x chunks live in registers.
  float4 xr[CPL > 0 ? CPL : 1][4];
  if constexpr (CPL > 0)
    if (MODE == MODE_FP32) load_pair_x<CPL>(xsm, H, lane, xr);
  StageIter itc;
  itc.init(blockIdx.x, gridDim.x, a.shared_width, a.top_k * a.width, a.width);
  int ct = 0;
  while (itc.next(d)) {
    const int stage = ct % kUpStages;
    if (!mbar_wait(&full[stage], (ct / kUpStages) & 1, a.status)) break;
    const unsigned char* base = ring + stage * stage_bytes;
    const int8_t* gw = reinterpret_cast<const int8_t*>(base);
    const int8_t* uw = reinterpret_cast<const int8_t*>(base + stage_w);
    const float* gs = reinterpret_cast<const float*>(base + 2 * stage_w);
    const float* us = reinterpret_cast<const float*>(base + 2 * stage_w + stage_s);
    for (int r = warp; r < d.nr; r += kUpConsumerWarps) {
      float g, u;
      if (MODE == MODE_FP32) {
        if constexpr (CPL > 0)
          pair_dot_xregs<CPL>(gw + r * H, gs + r * nbH, uw + r * H, us + r * nbH, H, xr, lane, g, u);
        else
          pair_dot_fp32(gw + r * H, gs + r * nbH, uw + r * H, us + r * nbH, xsm, H, lane, g, u);
      } else {
        g = dot_int8_ordered(gw + r * H, gs + r * nbH, xq, xs, H, lane);
        u = dot_int8_ordered(uw + r * H, us + r * nbH, xq, xs, H, lane);
      }
      if (lane == 0)
        a.h[h_base(d.unit, a.shared_width, a.width) + d.j0 + r] = __fmul_rn(silu_ref(g), u);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    ++ct;
  }
}

// ---------------------------------------------------------------------------
struct DownLayout {
  int rows_max;             // rows of the output owned by one CTA (max)
  int w_off[kMaxTopK + 1];  // byte offset of unit u's weight rows
  int s_off[kMaxTopK + 1];  // byte offset of unit u's scale rows
  int h_off, hq_off, hs_off, out_off, route_off, bar_off, total;
};

__host__ __device__ inline int unit_width(int u, int shared_width, int width) {
  return u == 0 ? shared_width : width;
}

static DownLayout down_layout(const MoeDecodeArgs& a, int grid) {
  DownLayout L{};
  L.rows_max = (a.hidden + grid - 1) / grid;
  int off = 0;
  for (int u = 0; u <= a.top_k; ++u) {
    L.w_off[u] = off;
    off += L.rows_max * unit_width(u, a.shared_width, a.width);
  }
  for (int u = 0; u <= a.top_k; ++u) {
    L.s_off[u] = off;
    off += L.rows_max * (unit_width(u, a.shared_width, a.width) / 32) * 4;
  }
  const int hn = a.shared_width + a.top_k * a.width;
  L.h_off = off;
  off += hn * 4;
  L.hq_off = off;
  off += hn;
  L.hs_off = off;
  off += (hn / 32) * 4;
  L.out_off = off;
  off += (a.top_k + 1) * L.rows_max * 4;
  L.route_off = off;
  off += (a.n_experts + 36 + 4 * kMaxTopK) * 4;
  off = (off + 15) & ~15;
  L.bar_off = off;
  off += 16;
  L.total = off;
  return L;
}

template <int MODE>
__global__ void __launch_bounds__(kDownThreads, 1) moe_down_kernel(const __grid_constant__ MoeDecodeArgs a,
                                                                   const __grid_constant__ DownLayout L) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i0 = static_cast<int>(static_cast<long long>(a.hidden) * blockIdx.x / gridDim.x);
  const int i1 = static_cast<int>(static_cast<long long>(a.hidden) * (blockIdx.x + 1) / gridDim.x);
  const int nr = i1 - i0;
  const int units = a.top_k + 1;
  const int hn = a.shared_width + a.top_k * a.width;
  float* hsm = reinterpret_cast<float*>(smem + L.h_off);
  int8_t* hq = reinterpret_cast<int8_t*>(smem + L.hq_off);
  float* hs = reinterpret_cast<float*>(smem + L.hs_off);
  float* outs = reinterpret_cast<float*>(smem + L.out_off);
  float* rp = reinterpret_cast<float*>(smem + L.route_off);
  float* red = rp + a.n_experts;
  int* bad = reinterpret_cast<int*>(red + 32);
  int* sel = bad + 4;
  float* selw = reinterpret_cast<float*>(sel + kMaxTopK);
  int* sorted = reinterpret_cast<int*>(selw + kMaxTopK);
  float* sortedw = reinterpret_cast<float*>(sorted + kMaxTopK);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);

  if (threadIdx.x == 0) {
    mbar_init(bar, 2);  // one arrival for the shared rows, one for the routed rows
    fence_mbar_init();
  }
  __syncthreads();
  auto issue_unit = [&](int u) {
    const Q8View& dm = u == 0 ? a.shared.down : a.experts[sorted[u - 1]].down;
    const int K = dm.cols, nbK = K / 32;
    bulk_g2s(smem + L.w_off[u], dm.w + static_cast<long long>(i0) * K, nr * K, bar);
    bulk_g2s(smem + L.s_off[u], dm.s + static_cast<long long>(i0) * nbK, nr * nbK * 4, bar);
  };
  // The shared expert's down rows do not depend on routing: fetch them first.
  if (threadIdx.x == 0 && nr > 0) {
    mbar_arrive_expect_tx(bar, nr * a.shared_width + nr * (a.shared_width / 32) * 4);
    issue_unit(0);
  }
  // Routing again (identical arithmetic, so identical result): this CTA
  // needs the selected experts to prefetch their down rows.  The logits were
  // complete before moe_up_kernel triggered this launch.
  const bool routed = route_row_block(a.logits, a.n_experts, a.top_k, a.normalize, a.scale, rp,
                                      red, sel, selw, bad, nullptr);
  if (threadIdx.x == 0) {
    for (int r = 0; r < a.top_k; ++r) {
      sorted[r] = routed ? sel[r] : r;
      sortedw[r] = routed ? selw[r] : 0.0f;
    }
    sort_by_id(sorted, sortedw, a.top_k);
    if (nr > 0) {
      mbar_arrive_expect_tx(bar, a.top_k * (nr * a.width + nr * (a.width / 32) * 4));
      for (int u = 1; u < units; ++u) issue_unit(u);
    }
  }
  // h is written by moe_up_kernel.
  pdl_wait_prior_grids();
  for (int k = threadIdx.x * 4; k < hn; k += kDownThreads * 4)
    *reinterpret_cast<float4*>(hsm + k) = *reinterpret_cast<const float4*>(a.h + k);
  __syncthreads();
  if (MODE == MODE_INT8) {
    // unit boundaries are multiples of 32, so flat 32-blocks are unit blocks
    quantize_vec_smem(hsm, hn, hq, hs, warp, kDownThreads / 32, a.status);
    __syncthreads();
  }
  bool ready = true;
  if (nr > 0) ready = mbar_wait(bar, 0, a.status);
  if (ready) {
    for (int t = warp; t < units * nr; t += kDownThreads / 32) {
      const int u = t / nr, r = t - u * nr;
      const int K = unit_width(u, a.shared_width, a.width), nbK = K / 32;
      const int8_t* wrow = reinterpret_cast<const int8_t*>(smem + L.w_off[u]) + r * K;
      const float* srow = reinterpret_cast<const float*>(smem + L.s_off[u]) + r * nbK;
      const int hb = h_base(u, a.shared_width, a.width);
      float v;
      if (MODE == MODE_FP32)
        v = row_dot_xsmem(wrow, srow, hsm + hb, K, lane);
      else
        v = dot_int8_ordered(wrow, srow, hq + hb, hs + hb / 32, K, lane);
      if (lane == 0) outs[u * L.rows_max + r] = v;
    }
  }
  __syncthreads();
  if (ready)
    for (int r = threadIdx.x; r < nr; r += kDownThreads) {
      float acc = outs[r];
      for (int u = 1; u < units; ++u)
        acc = __fadd_rn(acc, __fmul_rn(sortedw[u - 1], outs[u * L.rows_max + r]));
      a.y[i0 + r] = acc;
    }
}

// ---------------------------------------------------------------------------
static size_t up_smem(const MoeDecodeArgs& a) {
  const int H = a.hidden, nbH = H / 32;
  const size_t stage = 2 * static_cast<size_t>(kUpTileRows) * H + 2 * kUpTileRows * nbH * 4;
  return kUpStages * stage + H * 4 + H + nbH * 4 + (a.n_experts + 36 + 4 * kMaxTopK) * 4 + 16 +
         2 * kUpStages * 8 + 16;
}

bool moe_decode_supported(const MoeDecodeArgs& a) {
  if (a.hidden % 128 || a.width % 128 || a.shared_width % 128) return false;
  if (a.top_k < 1 || a.top_k > kMaxTopK || a.n_experts > kMaxRouteExperts) return false;
  if (a.hidden > 4096 || a.width > 8192 || a.shared_width > 8192) return false;
  if (up_smem(a) > 200 * 1024) return false;
  return true;
}

static void set_smem_attr(const void* fn, int bytes) {
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

cudaError_t launch_moe_decode(int mode, const MoeDecodeArgs& a, int sms, cudaStream_t st) {
  const int grid_up = sms;
  const int grid_down = a.hidden < sms ? a.hidden : sms;
  const DownLayout L = down_layout(a, grid_down);
  if (L.total > 200 * 1024) return cudaErrorInvalidConfiguration;
  const size_t us = up_smem(a);

  // Up kernel variants: FP32 with x in registers (hidden = 256*CPL), FP32
  // generic, int8.
  const int cpl = (a.hidden % 256 == 0) ? a.hidden / 256 : 0;
  using UpFn = void (*)(MoeDecodeArgs);
  UpFn up = mode == MODE_INT8 ? moe_up_kernel<MODE_INT8, 0>
            : cpl == 4        ? moe_up_kernel<MODE_FP32, 4>
            : cpl == 5        ? moe_up_kernel<MODE_FP32, 5>
                              : moe_up_kernel<MODE_FP32, 0>;

  static unsigned configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1u << (dev & 31)))) {
    const void* fns[] = {reinterpret_cast<const void*>(moe_up_kernel<MODE_FP32, 0>),
                         reinterpret_cast<const void*>(moe_up_kernel<MODE_FP32, 4>),
                         reinterpret_cast<const void*>(moe_up_kernel<MODE_FP32, 5>),
                         reinterpret_cast<const void*>(moe_up_kernel<MODE_INT8, 0>),
                         reinterpret_cast<const void*>(moe_down_kernel<MODE_FP32>),
                         reinterpret_cast<const void*>(moe_down_kernel<MODE_INT8>)};
    for (const void* f : fns) set_smem_attr(f, 200 * 1024);
    configured |= 1u << (dev & 31);
  }

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid_up);
  cfg.blockDim = dim3(kUpThreads);
  cfg.dynamicSmemBytes = us;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, up, a);
  if (e != cudaSuccess) return e;

  cudaLaunchConfig_t cfg2{};
  cfg2.gridDim = dim3(grid_down);
  cfg2.blockDim = dim3(kDownThreads);
  cfg2.dynamicSmemBytes = L.total;
  cfg2.stream = st;
  cfg2.attrs = attr;
  cfg2.numAttrs = 1;
  return mode == MODE_FP32 ? cudaLaunchKernelEx(&cfg2, moe_down_kernel<MODE_FP32>, a, L)
                           : cudaLaunchKernelEx(&cfg2, moe_down_kernel<MODE_INT8>, a, L);
}

}  // namespace uocr
