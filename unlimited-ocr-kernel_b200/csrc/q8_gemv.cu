// q8_gemv.cu — q8-block32 matrix-vector products (decode, M = 1).
//
// Two paths:
//  * gemv_tma_kernel  — the HBM-streaming path.  Persistent CTAs walk row
//    tiles of one or more matrices that share the input row.  A producer warp
//    moves each tile (int8 rows + their fp32 block scales, both contiguous in
//    HBM) into a ring of shared-memory stages with 1-D bulk async copies
//    completed on mbarriers; sixteen consumer warps (four groups) compute from
//    shared memory.  Requires cols % 128 == 0 and 16-byte aligned storage.
//  * gemv_generic_kernel — any shape and any batch; one warp per output row.
//
// Lane mapping of the fast path: FP32 mode — lane l owns the 16-byte chunks
// l, l+32, ... of a row (a chunk never straddles a 32-column scale block) and
// four rows share each x chunk; int8 mode — lane l owns bytes [4l, 4l+4) of
// every 128-byte window (block = window*4 + l/8).
//
// FP32-activation mode (Int8Matrix::linear, src/cpu/quantized.rs:99-149):
//   y = sum_b s_b * sum_{k in b} w_k x_k, fp32 FMA accumulation, reordered
//   relative to the reference's left-to-right sum (tolerance-checked).
// int8-activation mode (linear_dynamic_int8, src/cpu/quantized.rs:155-236):
//   S_b = sum_{k in b} w_k xq_k exactly in int32 (dp4a), then
//   acc = acc + (float(S_b) * ws_b) * xs_b over b = 0,1,2,... with _rn
//   intrinsics starting from -0.0: the reference's exact rounding sequence.
#include "common.cuh"
#include "device_once.h"
#include "kernels.h"

namespace uocr {

// ---------------------------------------------------------------------------
// generic path
template <int MODE>
__global__ void __launch_bounds__(256) gemv_generic_kernel(Q8View m, const float* __restrict__ x,
                                                           long long ld_x,
                                                           const int8_t* __restrict__ xq,
                                                           const float* __restrict__ xs,
                                                           int batch, float* __restrict__ y,
                                                           long long ld_y) {
  const int lane = threadIdx.x & 31;
  const int nb = blocks_of(m.cols);
  const long long warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long n = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5;
       n < m.rows; n += warps) {
    const int8_t* wr = m.w + n * m.cols;
    const float* sr = m.s + n * nb;
    for (int r = 0; r < batch; ++r) {
      if (MODE == MODE_FP32) {
        const float* xr = x + r * ld_x;
        float acc = 0.0f;
        for (int k = lane; k < m.cols; k += 32)
          acc = fmaf(__fmul_rn(static_cast<float>(wr[k]), sr[k >> 5]), xr[k], acc);
        acc = warp_sum(acc);
        if (lane == 0) y[r * ld_y + n] = acc;
      } else {
        const int8_t* qr = xq + static_cast<long long>(r) * m.cols;
        const float* sx = xs + static_cast<long long>(r) * nb;
        float acc = -0.0f;
        for (int b0 = 0; b0 < nb; b0 += 32) {
          const int b = b0 + lane;
          float t = 0.0f;
          if (b < nb) {
            const int k0 = b * kBlock, k1 = min(k0 + kBlock, m.cols);
            int sum = 0;
            for (int k = k0; k < k1; ++k) sum += static_cast<int>(wr[k]) * static_cast<int>(qr[k]);
            t = __fmul_rn(__fmul_rn(static_cast<float>(sum), sr[b]), sx[b]);
          }
          const int lim = min(32, nb - b0);
          for (int i = 0; i < lim; ++i) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, t, i));
        }
        if (lane == 0) y[r * ld_y + n] = acc;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// fast path
// ---------------------------------------------------------------------------
// fast path
//
// 16 consumer warps form 4 groups of 4.  The CTA's i-th tile goes to ring stage
// i % kGemvStages and is consumed by group i % 4, so each group owns two stages
// and double-buffers while the other groups work on theirs.  Inside a group,
// each warp takes 4 rows of the tile at a time (rows4_dot_xsmem).
constexpr int kGemvGroups = 4;
constexpr int kGemvWarpsPerGroup = 4;
constexpr int kGemvConsumerWarps = kGemvGroups * kGemvWarpsPerGroup;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kGemvStages = 8;
constexpr int kGemvMaxMats = 64;
constexpr int kGemvStageBudget = 24 * 1024;  // bytes of one stage (weights + scales)

struct GemvTmaParams {
  const int8_t* w[kGemvMaxMats];
  const float* s[kGemvMaxMats];
  float* y[kGemvMaxMats];
  int tile_begin[kGemvMaxMats + 1];  // prefix of tiles per matrix
  int rows[kGemvMaxMats];
  int n_mats, cols, tile_rows, total_tiles;
  int uniform_tiles;  // tiles per matrix when every matrix has the same rows, else 0
  const float* x;
  unsigned* status;
};


template <int MODE>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_tma_kernel(const __grid_constant__ GemvTmaParams p) {
  pdl_launch_dependents();  // launched as a programmatic dependent (launch_dependent):
  pdl_wait_prior_grids();   // nothing is touched before the previous kernel completes
  extern __shared__ __align__(128) unsigned char smem[];
  const int cols = p.cols, nb = cols >> 5, TR = p.tile_rows;
  const int w_bytes = TR * cols, s_bytes = TR * nb * 4;
  const int stage_bytes = w_bytes + s_bytes;
  unsigned char* ring = smem;
  float* xsm = reinterpret_cast<float*>(smem + kGemvStages * stage_bytes);
  int8_t* xq = reinterpret_cast<int8_t*>(xsm + cols);
  float* xs = reinterpret_cast<float*>(xq + cols);
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(xs + nb) + 15) & ~static_cast<uintptr_t>(15));
  uint64_t* empty = full + kGemvStages;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGemvStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGemvWarpsPerGroup);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kGemvConsumerWarps) {
    // producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x, ++it) {
        const int stage = it % kGemvStages;
        if (it >= kGemvStages) ok = mbar_wait(&empty[stage], ((it / kGemvStages) - 1) & 1, p.status);
        if (!ok) break;
        int mi = 0;
        if (p.uniform_tiles)
          mi = tile / p.uniform_tiles;
        else
          while (tile >= p.tile_begin[mi + 1]) ++mi;
        const int r0 = (tile - p.tile_begin[mi]) * TR;
        const int nr = min(TR, p.rows[mi] - r0);
        unsigned char* dst = ring + stage * stage_bytes;
        mbar_arrive_expect_tx(&full[stage], nr * cols + nr * nb * 4);
        bulk_g2s(dst, p.w[mi] + static_cast<long long>(r0) * cols, nr * cols, &full[stage]);
        bulk_g2s(dst + w_bytes, p.s[mi] + static_cast<long long>(r0) * nb, nr * nb * 4, &full[stage]);
      }
      // drain: every issued copy has landed before the CTA may exit
      const int issued = it;
      for (int j = issued - kGemvStages; j < issued; ++j)
        if (j >= 0) mbar_wait(&full[j % kGemvStages], (j / kGemvStages) & 1, p.status);
    }
    return;
  }

  // consumers: x staged (and quantized) while the producer's first copies
  // are in flight, then group g takes this CTA's tiles g, g+4, g+8, ...
  constexpr int kConsumerThreads = kGemvConsumerWarps * 32;
  if (MODE == MODE_FP32) {
    stage_x_transposed(xsm, p.x, cols, threadIdx.x, kConsumerThreads);
    named_barrier(1, kConsumerThreads);
  } else {
    for (int k = threadIdx.x; k < cols; k += kConsumerThreads) xsm[k] = p.x[k];
    named_barrier(1, kConsumerThreads);
    quantize_blocks_smem(xsm, cols, xq, xs, threadIdx.x, kConsumerThreads, 1, p.status);
    named_barrier(1, kConsumerThreads);
  }
  const int group = warp / kGemvWarpsPerGroup, wg = warp % kGemvWarpsPerGroup;
  for (int it = group, tile = blockIdx.x + group * gridDim.x; tile < p.total_tiles;
       it += kGemvGroups, tile += kGemvGroups * gridDim.x) {
    const int stage = it % kGemvStages;
    if (!mbar_wait(&full[stage], (it / kGemvStages) & 1, p.status)) break;
    int mi = 0;
    if (p.uniform_tiles)
      mi = tile / p.uniform_tiles;
    else
      while (tile >= p.tile_begin[mi + 1]) ++mi;
    const int r0 = (tile - p.tile_begin[mi]) * TR;
    const int nr = min(TR, p.rows[mi] - r0);
    const int8_t* wt = reinterpret_cast<const int8_t*>(ring + stage * stage_bytes);
    const float* st = reinterpret_cast<const float*>(ring + stage * stage_bytes + w_bytes);
    float* y = p.y[mi] + r0;
    for (int r = 4 * wg; r < nr; r += 4 * kGemvWarpsPerGroup) {
      const int q1 = min(r + 1, nr - 1), q2 = min(r + 2, nr - 1), q3 = min(r + 3, nr - 1);
      if (MODE == MODE_FP32) {
        const float v = rows4_dot_xsmem(wt + r * cols, wt + q1 * cols, wt + q2 * cols,
                                        wt + q3 * cols, st + r * nb, st + q1 * nb, st + q2 * nb,
                                        st + q3 * nb, xsm, cols, lane);
        const int j = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
        if ((lane & 7) == 0 && r + j < nr) y[r + j] = v;
      } else {
        const int8_t* const wr[4] = {wt + r * cols, wt + q1 * cols, wt + q2 * cols,
                                     wt + q3 * cols};
        const float* const sr[4] = {st + r * nb, st + q1 * nb, st + q2 * nb, st + q3 * nb};
        float v[4];
        rows4_dot_int8(wr, sr, xq, xs, cols, lane, v);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (lane == 0 && r + j < nr) y[r + j] = v[j];
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }
}


static int gemv_tile_rows(int cols) {
  int tr = kGemvStageBudget / (cols + cols / 8);
  tr = tr > 32 ? 32 : tr;
  tr &= ~3;
  return tr < 4 ? 4 : tr;
}

static size_t gemv_tma_smem(int cols, int tile_rows) {
  const int nb = cols / 32;
  const size_t stage = static_cast<size_t>(tile_rows) * cols + static_cast<size_t>(tile_rows) * nb * 4;
  return kGemvStages * stage + cols * 4 + cols + nb * 4 + 16 + 2 * kGemvStages * 8 + 16;
}

constexpr size_t kGemvSmemLimit = 220 * 1024;  // the kernels' dynamic shared-memory opt-in

// The streaming kernel takes a matrix whose ring of kGemvStages tiles (at
// least four rows each) and staged x fit the opt-in; wider rows (above about
// 5000 columns) go to the generic kernel.
bool gemv_fast_path_ok(const Q8View& m) {
  return m.cols % 128 == 0 && m.cols <= 8192 && reinterpret_cast<uintptr_t>(m.w) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(m.s) % 16 == 0 &&
         gemv_tma_smem(m.cols, gemv_tile_rows(m.cols)) <= kGemvSmemLimit;
}

template <int MODE>
static void launch_gemv_tma(const Q8View* mats, int n, const float* x, float* const* ys,
                            unsigned* status, int sms, cudaStream_t st) {
  GemvTmaParams p{};
  const int cols = mats[0].cols;
  const int tr = gemv_tile_rows(cols);
  p.n_mats = n;
  p.cols = cols;
  p.tile_rows = tr;
  p.x = x;
  p.status = status;
  int tiles = 0;
  for (int i = 0; i < n; ++i) {
    p.w[i] = mats[i].w;
    p.s[i] = mats[i].s;
    p.y[i] = ys[i];
    p.rows[i] = mats[i].rows;
    p.tile_begin[i] = tiles;
    tiles += (mats[i].rows + tr - 1) / tr;
  }
  for (int i = n; i <= kGemvMaxMats; ++i) p.tile_begin[i] = tiles;
  p.total_tiles = tiles;
  p.uniform_tiles = (mats[0].rows + tr - 1) / tr;
  for (int i = 1; i < n; ++i)
    if (mats[i].rows != mats[0].rows) p.uniform_tiles = 0;
  const size_t smem = gemv_tma_smem(cols, tr);
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(gemv_tma_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kGemvSmemLimit));
  });
  const int grid = tiles < sms ? tiles : sms;
  launch_dependent(gemv_tma_kernel<MODE>, dim3(grid), dim3(kGemvThreads), smem, st, p);
}

static void dispatch_gemv_tma(int mode, const Q8View* mats, int n, const float* x,
                              float* const* ys, unsigned* status, int sms, cudaStream_t st) {
  if (mode == MODE_INT8)
    launch_gemv_tma<MODE_INT8>(mats, n, x, ys, status, sms, st);
  else
    launch_gemv_tma<MODE_FP32>(mats, n, x, ys, status, sms, st);
}

void launch_gemv_multi(int mode, const Q8View* mats, int n, const float* x, float* const* ys,
                       unsigned* status, int sms, cudaStream_t st) {
  for (int base = 0; base < n; base += kGemvMaxMats) {
    const int cnt = n - base < kGemvMaxMats ? n - base : kGemvMaxMats;
    dispatch_gemv_tma(mode, mats + base, cnt, x, ys + base, status, sms, st);
  }
}

void launch_gemv(int mode, const Q8View& m, const float* x, long long ld_x, int batch, float* y,
                 long long ld_y, int8_t* xq, float* xs, unsigned* status, int sms,
                 cudaStream_t st) {
  if (batch == 1 && gemv_fast_path_ok(m) && reinterpret_cast<uintptr_t>(x) % 16 == 0) {
    float* ys[1] = {y};
    dispatch_gemv_tma(mode, &m, 1, x, ys, status, sms, st);
    return;
  }
  long long grid = (static_cast<long long>(m.rows) + 7) / 8;
  grid = grid < 1 ? 1 : (grid > sms * 16LL ? sms * 16LL : grid);
  if (mode == MODE_INT8) launch_quantize_rows(x, ld_x, batch, m.cols, xq, xs, status, sms, st);
  if (mode == MODE_FP32)
    gemv_generic_kernel<MODE_FP32><<<static_cast<int>(grid), 256, 0, st>>>(m, x, ld_x, xq, xs,
                                                                          batch, y, ld_y);
  else
    gemv_generic_kernel<MODE_INT8><<<static_cast<int>(grid), 256, 0, st>>>(m, x, ld_x, xq, xs,
                                                                          batch, y, ld_y);
}

}  // namespace uocr
