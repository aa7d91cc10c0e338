// moe_decode.cu — Decoder::experts for one token (src/decoder/mod.rs:124-220)
// as ONE cooperative kernel with an in-kernel grid barrier.
//
// Units: unit 0 is the fused shared-expert FFN (width shared_width, the
// reference's n_shared_experts*moe_intermediate_size fusion,
// src/decoder/mod.rs:71-75); units 1..top_k are the selected routed experts
// in ascending expert id, which is the order Decoder::experts adds them.
//
// grid = #SMs (one CTA per SM, all co-resident: cooperative launch),
// block = 16 consumer warps + 1 producer warp + 1 router warp.
//
// Producer warp, before anything token-dependent is known: 1-D bulk async
// copies of (a) the expert descriptor table, (b) this CTA's rows [i0, i1) of
// the shared expert's down matrix into a dedicated shared-memory region,
// (c) the first stages of this CTA's slice of the shared expert's gate/up
// rows into a ring of up to 6 stages.  None of these depend on the token.
// Router warp, at the same time: griddepcontrol.wait (the logits may come
// from the previous kernel), then moe::route (src/decoder/moe.rs:7-30) with
// the logits in registers; it publishes the selection through shared memory.
// Phase A: the producer fills the ring's free slots with the selected
// experts' gate/up rows, starts the copies of their down rows [i0, i1), then
// streams the rest of this CTA's slice.  Four groups of four consumer warps
// compute from the ring (a warp does two gate/up pairs: 4 rows sharing each x
// chunk) and write h = silu(gate) * up (Decoder::feed_forward,
// src/decoder/mod.rs:114-122) to global scratch.
// Grid barrier (bounded wait), then Phase B: every CTA loads all of h (int8
// mode: block-quantizes it, as projection() does for the down input in
// DynamicActivations mode) and computes its output rows of every unit from
// the prefetched down rows.  The down work is cut into pieces (unit, range of
// 32-element blocks) of equal size so that every consumer warp streams the
// same number of weights; each lane keeps one 16-element chunk of h in
// registers for all rows.  Weights-only mode sums a row's pieces in a fixed
// order; int8 mode stores every block term and sums them in block order, the
// reference's rounding sequence.  Finally the rows are combined in the
// reference's order: r = shared; r += p_e * out_e for e ascending, one
// rounding per op.
#include "common.cuh"
#include "device_once.h"
#include "kernels.h"
#include "route.cuh"

namespace uocr {

constexpr int kGroups = 4;
constexpr int kWarpsPerGroup = 4;
constexpr int kConsumerWarps = kGroups * kWarpsPerGroup;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kRouterWarp = kConsumerWarps + 1;
constexpr int kThreads = kConsumerThreads + 64;
constexpr int kMaxStages = 6;  // ring slots: as many as shared memory allows
// At least one ring slot per consumer group: a group waits on its slot's fill
// by phase parity, which is only sound while no group can wait more than one
// phase ahead of a slot's first fill.
constexpr int kMinStages = 4;
static_assert(kMinStages >= kGroups, "one ring slot per consumer group at least");
constexpr int kSmemBudget = 220 * 1024;
constexpr int kTileRows = 8;
constexpr int kMaxTopK = 8;
constexpr int kMaxDecodeExperts = 64;

struct StageDesc {
  int unit, j0, nr;
};

// Even split of n items over `parts`: the start of part i (32-bit: every
// product here is below 2^31).
__host__ __device__ __forceinline__ int split_at(int n, int i, int parts) {
  return static_cast<int>(static_cast<unsigned>(n) * static_cast<unsigned>(i) /
                          static_cast<unsigned>(parts));
}

// Deterministic enumeration of one CTA's stages, replayed identically by the
// producer and the consumers.
struct StageIter {
  int s_cur, s_end, r_cur, r_end, width;
  __device__ void init(int cta, int grid, int shared_width, int routed_rows, int w) {
    s_cur = split_at(shared_width, cta, grid);
    s_end = split_at(shared_width, cta + 1, grid);
    r_cur = split_at(routed_rows, cta, grid);
    r_end = split_at(routed_rows, cta + 1, grid);
    width = w;
  }
  __device__ bool next(StageDesc& d) {
    if (s_cur < s_end) {
      d.unit = 0;
      d.j0 = s_cur;
      d.nr = min(kTileRows, s_end - s_cur);
      s_cur += d.nr;
      return true;
    }
    if (r_cur < r_end) {
      const int u = r_cur / width, j = r_cur - u * width;
      d.unit = 1 + u;
      d.j0 = j;
      d.nr = min(kTileRows, min(r_end - r_cur, width - j));
      r_cur += d.nr;
      return true;
    }
    return false;
  }
  __device__ bool next_is_shared() const { return s_cur < s_end; }
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid-wide barrier for a co-resident grid.  Words: sync[1] is the
// generation g, sync[2 + (g & 1)] the arrival counter of generation g.
// Every CTA reads g (after the previous kernel in the stream completed,
// i.e. before any CTA of this grid can arrive); CTA 0 zeroes the other
// generation's counter for the next launch and, once past the barrier,
// publishes g + 1.  An arrival is one release reduction (it carries the
// CTA's prior global writes, ordered before it by the CTA barrier); the
// waiters poll the counter until it reaches the grid size.  On the critical
// path: the last arrival's one-way trip to L2 and one observed load.  A
// launch that timed out still leaves the words ready for the next one.
__device__ __forceinline__ bool grid_barrier(unsigned* sync, unsigned gen, unsigned nblocks,
                                             unsigned* status, long long limit) {
  unsigned* cnt = sync + 2 + (gen & 1u);
  red_release_gpu_add(cnt, 1u);
  const long long t0 = clock64();
  while (ld_acquire_gpu(cnt) < nblocks) {
    if (clock64() - t0 > limit) {
      flag(status, DEV_TIMEOUT);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

// Sum of N row partials over the warp, N rows at once (transposed butterfly:
// N/2 + N/4 + ... + 1 shuffles to split the rows over lane groups, then a
// plain butterfly inside each group).  Afterwards every lane of group
// lane / (32 / N) holds the total of that row.  `v` is clobbered.
template <int N>
__device__ __forceinline__ float reduce_rows(float (&v)[N], int lane) {
  int o = 16;
#pragma unroll
  for (int n = N; n > 1; n >>= 1, o >>= 1) {
    const bool hi = lane & o;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float keep = hi ? v[i + n / 2] : v[i];
      const float send = hi ? v[i] : v[i + n / 2];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float t = v[0];
#pragma unroll
  for (; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// Weights-only phase B, rows [r0, r0 + N) of one piece: lane's 16 weights of
// each row against its h chunk; the piece's row sums go to part[row].
template <int N>
__device__ __forceinline__ void piece_rows_fp32(const int8_t* wu, const float* su, int K, int nbK,
                                                int c, bool act, const float4 (&xv)[4], int r0,
                                                int nr, float* part, int lane) {
  float v[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int r = min(r0 + i, nr - 1);
    const float t =
        su[r * nbK + (c >> 1)] * chunk16_dot(*reinterpret_cast<const uint4*>(wu + r * K + 16 * c), xv);
    v[i] = act ? t : 0.0f;
  }
  const float t = reduce_rows<N>(v, lane);
  const int i = lane / (32 / N);
  if (lane % (32 / N) == 0 && r0 + i < nr) part[r0 + i] = t;
}

__host__ __device__ __forceinline__ int h_base(int unit, int shared_width, int width) {
  return unit == 0 ? 0 : shared_width + (unit - 1) * width;
}

__host__ __device__ inline int unit_width(int u, int shared_width, int width) {
  return u == 0 ? shared_width : width;
}

// Phase-B piece size in 32-element blocks: the h vector's blocks spread
// evenly over the consumer warps, at most 16 blocks (one 16-float chunk per
// lane).  Unit u is cut into ceil(nb_u / piece) pieces of near-equal size.
__host__ __device__ __forceinline__ int piece_blocks(int hn) {
  const int per_warp = (hn / 32 + kConsumerWarps - 1) / kConsumerWarps;
  return per_warp < 16 ? per_warp : 16;
}

// ---------------------------------------------------------------------------
struct DecodeLayout {
  int rows_max;             // output rows owned by one CTA (max)
  int stage_bytes;          // one ring stage (gate + up rows and scales)
  int slots;                // ring stages
  int x_off, xq_off, xs_off;
  // Down rows of unit u at w_off(u), their block scales at s_off(u): unit 0
  // (rows_max x shared_width), then the routed units (rows_max x width
  // each).  Computed, not tabulated: a kernel-parameter array indexed at run
  // time is read through the constant cache one serialised access at a time.
  int w_base, s_base, w_shared, w_unit, s_shared, s_unit;
  __device__ __forceinline__ int w_off(int u) const {
    return u == 0 ? w_base : w_base + w_shared + (u - 1) * w_unit;
  }
  __device__ __forceinline__ int s_off(int u) const {
    return u == 0 ? s_base : s_base + s_shared + (u - 1) * s_unit;
  }
  int part_off;             // phase-B partials (inside the ring, after h)
  int hq_off, hs_off, out_off, route_off, rp_off, desc_off, bar_off, total;
};

static int align16(int v) { return (v + 15) & ~15; }

static DecodeLayout decode_layout_with(const MoeDecodeArgs& a, int grid, int slots) {
  DecodeLayout L{};
  const int H = a.hidden, nbH = H / 32;
  L.rows_max = (H + grid - 1) / grid;
  L.stage_bytes = 2 * kTileRows * H + 2 * kTileRows * nbH * 4;
  L.slots = slots;
  int off = slots * L.stage_bytes;  // ring; phase B stages h (float) here
  L.x_off = off;
  off += H * 4;
  L.xq_off = off;
  off += H;
  L.xs_off = align16(off);
  off = align16(L.xs_off + nbH * 4);
  L.w_shared = L.rows_max * a.shared_width;
  L.w_unit = L.rows_max * a.width;
  L.s_shared = L.rows_max * (a.shared_width / 32) * 4;
  L.s_unit = L.rows_max * (a.width / 32) * 4;
  L.w_base = off;
  off += L.w_shared + a.top_k * L.w_unit;
  L.s_base = off;
  off += L.s_shared + a.top_k * L.s_unit;
  const int hn = a.shared_width + a.top_k * a.width;
  L.part_off = align16(hn * 4);
  L.hq_off = align16(off);
  off = L.hq_off + hn;
  L.hs_off = align16(off);
  off = L.hs_off + (hn / 32) * 4;
  L.out_off = align16(off);
  off = L.out_off + (a.top_k + 1) * L.rows_max * 4;
  L.rp_off = align16(off);
  off = L.rp_off + 64 * 4;  // router scratch
  L.route_off = align16(off);
  off = L.route_off + 4 * kMaxTopK * 4;  // sel, selw, sorted, sortedw
  L.desc_off = align16(off);
  off = L.desc_off + a.n_experts * static_cast<int>(sizeof(FfnView));
  L.bar_off = align16(off);
  off = L.bar_off + (2 * kMaxStages + 3) * 8;
  L.total = align16(off);
  return L;
}

// The layout with as many ring slots (up to kMaxStages) as the budget allows.
static DecodeLayout decode_layout(const MoeDecodeArgs& a, int grid) {
  const DecodeLayout base = decode_layout_with(a, grid, 0);
  const int room = (kSmemBudget - base.total) / base.stage_bytes;
  return decode_layout_with(a, grid, room < kMaxStages ? room : kMaxStages);
}

// Phase-B partial storage: weights-only keeps one float per (piece, row),
// int8 mode one per (block, row).
static int part_bytes(const MoeDecodeArgs& a, int rows_max) {
  const int hn = a.shared_width + a.top_k * a.width, pb = piece_blocks(hn);
  int pieces = 0;
  for (int u = 0; u <= a.top_k; ++u) {
    const int nb = unit_width(u, a.shared_width, a.width) / 32;
    pieces += (nb + pb - 1) / pb;
  }
  const int per_row = pieces > hn / 32 ? pieces : hn / 32;
  return per_row * rows_max * 4;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) moe_decode_kernel(const __grid_constant__ MoeDecodeArgs a,
                                                                 const __grid_constant__ DecodeLayout L) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.hidden, nbH = H >> 5;
  const int stage_w = kTileRows * H, stage_s = kTileRows * nbH * 4;
  const int i0 = split_at(H, blockIdx.x, gridDim.x);
  const int i1 = split_at(H, blockIdx.x + 1, gridDim.x);
  const int nr = i1 - i0;
  const int units = a.top_k + 1;
  const int hn = a.shared_width + a.top_k * a.width;
  const int slots = L.slots;
  unsigned char* ring = smem;
  float* xsm = reinterpret_cast<float*>(smem + L.x_off);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + L.xq_off);
  float* xs = reinterpret_cast<float*>(smem + L.xs_off);
  float* hsm = reinterpret_cast<float*>(smem);  // phase B: aliases the ring
  float* part = reinterpret_cast<float*>(smem + L.part_off);  // phase B, in the ring
  int8_t* hq = reinterpret_cast<int8_t*>(smem + L.hq_off);
  float* hs = reinterpret_cast<float*>(smem + L.hs_off);
  float* outs = reinterpret_cast<float*>(smem + L.out_off);
  float* rp = reinterpret_cast<float*>(smem + L.rp_off);
  int* sel = reinterpret_cast<int*>(smem + L.route_off);
  float* selw = reinterpret_cast<float*>(sel + kMaxTopK);
  int* sorted = reinterpret_cast<int*>(selw + kMaxTopK);
  float* sortedw = reinterpret_cast<float*>(sorted + kMaxTopK);
  FfnView* edesc = reinterpret_cast<FfnView*>(smem + L.desc_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + kMaxStages;
  uint64_t* down_bar = empty + kMaxStages;  // down rows landed (2 arrivals)
  uint64_t* desc_bar = down_bar + 1;     // descriptor table landed
  uint64_t* route_bar = desc_bar + 1;    // routing result in shared memory

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < slots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarpsPerGroup);
    }
    mbar_init(down_bar, 2);
    mbar_init(desc_bar, 1);
    mbar_init(route_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  StageDesc d;
  if (warp == kRouterWarp) {
    // ======================= router warp =======================
    pdl_wait_prior_grids();  // the router logits may come from the previous kernel
    pdl_launch_dependents();
    const bool routed = route_row_warp64(a.logits, a.n_experts, a.top_k, a.normalize, a.scale, rp,
                                         sel, selw, sorted, sortedw, a.status);
    if (!routed && lane < a.top_k) {  // invalid row: keep addresses valid, status flagged
      sorted[lane] = lane;
      sortedw[lane] = 0.0f;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(route_bar);
    if (blockIdx.x == 0 && lane < a.top_k) {
      a.route_ids[lane] = routed ? sel[lane] : -1;
      a.route_weights[lane] = routed ? selw[lane] : 0.0f;
    }
    return;
  }
  if (warp == kProducerWarp) {
    // ======================= producer warp =======================
    if (lane != 0) return;
    StageIter itp;
    itp.init(blockIdx.x, gridDim.x, a.shared_width, a.top_k * a.width, a.width);
    int it = 0;
    bool ok = true;
    auto issue = [&](const StageDesc& sd) {
      const FfnView fv = sd.unit == 0 ? a.shared : edesc[sorted[sd.unit - 1]];
      const int stage = it % slots;
      if (it >= slots) ok = mbar_wait(&empty[stage], ((it / slots) - 1) & 1, a.status);
      if (!ok) return;
      unsigned char* dst = ring + stage * L.stage_bytes;
      const int wb = sd.nr * H, sb = sd.nr * nbH * 4;
      mbar_arrive_expect_tx(&full[stage], 2 * wb + 2 * sb);
      bulk_g2s(dst, fv.gate.w + static_cast<long long>(sd.j0) * H, wb, &full[stage]);
      bulk_g2s(dst + stage_w, fv.up.w + static_cast<long long>(sd.j0) * H, wb, &full[stage]);
      bulk_g2s(dst + 2 * stage_w, fv.gate.s + static_cast<long long>(sd.j0) * nbH, sb,
               &full[stage]);
      bulk_g2s(dst + 2 * stage_w + stage_s, fv.up.s + static_cast<long long>(sd.j0) * nbH, sb,
               &full[stage]);
      ++it;
    };
    auto issue_down = [&](const Q8View& dm, int u) {
      const int K = dm.cols, nbK = K / 32;
      bulk_g2s(smem + L.w_off(u), dm.w + static_cast<long long>(i0) * K, nr * K, down_bar);
      bulk_g2s(smem + L.s_off(u), dm.s + static_cast<long long>(i0) * nbK, nr * nbK * 4, down_bar);
    };
    // Token-independent copies first, before any wait for the previous
    // kernel: the descriptor table and the weights are written only when the
    // layer and its matrices are created (matrices are immutable while their
    // handles live), never by a kernel this launch may overlap.
    const int desc_bytes = a.n_experts * static_cast<int>(sizeof(FfnView));
    mbar_arrive_expect_tx(desc_bar, desc_bytes);
    bulk_g2s(edesc, a.experts, desc_bytes, desc_bar);
    while (ok && it < slots && itp.next_is_shared() && itp.next(d)) issue(d);
    mbar_arrive_expect_tx(down_bar, nr * a.shared_width + nr * (a.shared_width / 32) * 4);
    if (nr > 0) issue_down(a.shared.down, 0);
    // Then the selected experts: free ring slots, their down rows, the rest.
    ok = mbar_wait(route_bar, 0, a.status) && mbar_wait(desc_bar, 0, a.status);
    while (ok && it < slots && itp.next(d)) issue(d);
    mbar_arrive_expect_tx(down_bar, a.top_k * (nr * a.width + nr * (a.width / 32) * 4));
    if (ok && nr > 0)
      for (int u = 1; u < units; ++u) issue_down(edesc[sorted[u - 1]].down, u);
    while (ok && itp.next(d)) issue(d);
    const int issued = it;
    for (int j = issued - slots; j < issued; ++j)
      if (j >= 0) mbar_wait(&full[j % slots], (j / slots) & 1, a.status);
    return;
  }

  // ======================= consumer warps =======================
  pdl_wait_prior_grids();  // x may come from the previous kernel
  pdl_launch_dependents();
  // The previous grid (which may have used the barrier words) is complete.
  const unsigned barrier_gen = threadIdx.x == 0 ? ld_acquire_gpu(a.grid_sync + 1) : 0u;
  if (threadIdx.x == 0 && blockIdx.x == 0) a.grid_sync[2 + ((barrier_gen + 1u) & 1u)] = 0u;
  if (MODE == MODE_FP32) {
    stage_x_transposed(xsm, a.x, H, threadIdx.x, kConsumerThreads);
    named_barrier(1, kConsumerThreads);
  } else {
    for (int k = threadIdx.x; k < H; k += kConsumerThreads) xsm[k] = a.x[k];
    named_barrier(1, kConsumerThreads);
    quantize_blocks_smem(xsm, H, xq, xs, threadIdx.x, kConsumerThreads, 1, a.status);
    named_barrier(1, kConsumerThreads);
  }
  // ---- phase A: group g consumes this CTA's stages g, g+4, ...
  {
    const int group = warp / kWarpsPerGroup, wg = warp % kWarpsPerGroup;
    StageIter itc;
    itc.init(blockIdx.x, gridDim.x, a.shared_width, a.top_k * a.width, a.width);
    for (int ct = 0; itc.next(d); ++ct) {
      if (ct % kGroups != group) continue;
      const int stage = ct % slots;
      if (!mbar_wait(&full[stage], (ct / slots) & 1, a.status)) break;
      const unsigned char* base = ring + stage * L.stage_bytes;
      const int8_t* gw = reinterpret_cast<const int8_t*>(base);
      const int8_t* uw = reinterpret_cast<const int8_t*>(base + stage_w);
      const float* gs = reinterpret_cast<const float*>(base + 2 * stage_w);
      const float* us = reinterpret_cast<const float*>(base + 2 * stage_w + stage_s);
      float* h = a.h + h_base(d.unit, a.shared_width, a.width) + d.j0;
      for (int r = 2 * wg; r < d.nr; r += 2 * kWarpsPerGroup) {
        const int r1 = r + 1 < d.nr ? r + 1 : r;
        if (MODE == MODE_FP32) {
          // lanes 0-7: gate r, 8-15: up r, 16-23: gate r1, 24-31: up r1
          const float v = rows4_dot_xsmem(gw + r * H, uw + r * H, gw + r1 * H, uw + r1 * H,
                                          gs + r * nbH, us + r * nbH, gs + r1 * nbH,
                                          us + r1 * nbH, xsm, H, lane);
          const float u = __shfl_down_sync(0xffffffffu, v, 8);
          if (lane == 0) h[r] = __fmul_rn(silu_ref(v), u);
          if (lane == 16 && r1 != r) h[r1] = __fmul_rn(silu_ref(v), u);
        } else {
          // gate r, up r, gate r1, up r1 as four interleaved ordered chains
          const int8_t* const wr[4] = {gw + r * H, uw + r * H, gw + r1 * H, uw + r1 * H};
          const float* const sr[4] = {gs + r * nbH, us + r * nbH, gs + r1 * nbH, us + r1 * nbH};
          float v[4];
          rows4_dot_int8(wr, sr, xq, xs, H, lane, v);
          if (lane == 0) {
            h[r] = __fmul_rn(silu_ref(v[0]), v[1]);
            if (r1 != r) h[r1] = __fmul_rn(silu_ref(v[2]), v[3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }
  }
  // ---- every CTA's slice of h is in global memory
  named_barrier(1, kConsumerThreads);
  if (threadIdx.x == 0) {
    grid_barrier(a.grid_sync, barrier_gen, gridDim.x + a.barrier_extra, a.status,
                 a.wait_cycles > 0 ? a.wait_cycles : kWaitLimitCycles);
    if (blockIdx.x == 0) a.grid_sync[1] = barrier_gen + 1u;
  }
  named_barrier(1, kConsumerThreads);

  // ---- phase B: stage h (the ring is idle: every issued stage was consumed)
  {
    const float4* h4 = reinterpret_cast<const float4*>(a.h);
    float4* d4 = reinterpret_cast<float4*>(hsm);
    const int n4 = hn >> 2, fs4 = a.shared_width >> 2, f4 = a.width >> 2;
    for (int i = threadIdx.x; i < n4; i += 4 * kConsumerThreads) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i + u * kConsumerThreads < n4) v[u] = __ldcg(h4 + i + u * kConsumerThreads);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int k = i + u * kConsumerThreads;
        if (k >= n4) break;
        if (MODE == MODE_FP32) {  // chunk-transposed per unit
          const int base = k < fs4 ? 0 : fs4 + ((k - fs4) / f4) * f4;
          const int C = (k < fs4 ? fs4 : f4) >> 2;
          const int loc = k - base;
          d4[base + (loc & 3) * C + (loc >> 2)] = v[u];
        } else {
          d4[k] = v[u];
        }
      }
    }
  }
  named_barrier(1, kConsumerThreads);
  if (MODE == MODE_INT8) {
    // unit boundaries are multiples of 32, so flat 32-blocks are unit blocks
    quantize_blocks_smem(hsm, hn, hq, hs, threadIdx.x, kConsumerThreads, 1, a.status);
    named_barrier(1, kConsumerThreads);
  }
  const bool ready = nr > 0 && mbar_wait(down_bar, 0, a.status);
  const int pb = piece_blocks(hn);
  // pieces: unit 0 has np0 of them, every routed unit npe (same width)
  const int nbS = a.shared_width >> 5, nbE = a.width >> 5;
  const int np0 = (nbS + pb - 1) / pb, npe = (nbE + pb - 1) / pb;
  if (ready) {
    // piece p = (unit u, blocks [b0, b1) of the unit); warp w takes p = w, w + 16, ...
    for (int p = warp; p < np0 + a.top_k * npe; p += kConsumerWarps) {
      const int u = p < np0 ? 0 : 1 + (p - np0) / npe;
      const int j = p < np0 ? p : (p - np0) - (u - 1) * npe;
      const int np = u == 0 ? np0 : npe;
      const int nbK = u == 0 ? nbS : nbE, K = nbK << 5, C = nbK << 1;
      const int hb = h_base(u, a.shared_width, a.width);
      const int8_t* wu = reinterpret_cast<const int8_t*>(smem + L.w_off(u));
      const float* su = reinterpret_cast<const float*>(smem + L.s_off(u));
      const int b0 = split_at(nbK, j, np), b1 = split_at(nbK, j + 1, np);
      // this lane's 16-element chunk of the unit; idle lanes address the
      // piece's first chunk and contribute zeros
      const bool act = 2 * b0 + lane < 2 * b1;
      const int c = act ? 2 * b0 + lane : 2 * b0;
      if (MODE == MODE_FP32) {
        float4 xv[4];
        const float4* x4 = reinterpret_cast<const float4*>(hsm + hb);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          xv[q] = x4[q * C + c];
        float* pp = part + p * L.rows_max;
        int r0 = 0;
        for (; r0 + 8 <= nr; r0 += 8)
          piece_rows_fp32<8>(wu, su, K, nbK, c, act, xv, r0, nr, pp, lane);
        if (nr - r0 >= 4) {
          piece_rows_fp32<4>(wu, su, K, nbK, c, act, xv, r0, nr, pp, lane);
          r0 += 4;
        }
        if (nr - r0 >= 2) {
          piece_rows_fp32<2>(wu, su, K, nbK, c, act, xv, r0, nr, pp, lane);
          r0 += 2;
        }
        if (nr - r0 >= 1) piece_rows_fp32<1>(wu, su, K, nbK, c, act, xv, r0, nr, pp, lane);
      } else {
        // a lane pair forms one block's exact int32 sum; the even lane
        // stores the block term (S * w_scale) * h_scale
        const int4 xq4 = *reinterpret_cast<const int4*>(hq + hb + 16 * c);
        const float hsc = hs[(hb >> 5) + (c >> 1)];
        float* tb = part + (hb >> 5) * L.rows_max;  // [row][block] of unit u
        for (int r = 0; r < nr; ++r) {
          const int4 w4 = *reinterpret_cast<const int4*>(wu + r * K + 16 * c);
          int S = __dp4a(w4.x, xq4.x, 0);
          S = __dp4a(w4.y, xq4.y, S);
          S = __dp4a(w4.z, xq4.z, S);
          S = __dp4a(w4.w, xq4.w, S);
          S += __shfl_xor_sync(0xffffffffu, S, 1);
          if (act && !(lane & 1))
            tb[r * nbK + (c >> 1)] =
                __fmul_rn(__fmul_rn(static_cast<float>(S), su[r * nbK + (c >> 1)]), hsc);
        }
      }
    }
  }
  named_barrier(1, kConsumerThreads);
  if (ready) {
    // per (unit, row) totals in a fixed order
    for (int t = threadIdx.x; t < units * nr; t += kConsumerThreads) {
      const int u = t / nr, r = t - u * nr;
      const int K = unit_width(u, a.shared_width, a.width), nbK = K >> 5;
      float acc;
      if (MODE == MODE_FP32) {
        const int p0 = u == 0 ? 0 : np0 + (u - 1) * npe;
        const int np = u == 0 ? np0 : npe;
        acc = part[p0 * L.rows_max + r];
        for (int j = 1; j < np; ++j) acc += part[(p0 + j) * L.rows_max + r];
      } else {
        // linear_dynamic_int8: block terms added in block order from -0.0
        const float* tb = part + (h_base(u, a.shared_width, a.width) >> 5) * L.rows_max + r * nbK;
        acc = -0.0f;
        for (int b = 0; b < nbK; ++b) acc = __fadd_rn(acc, tb[b]);
      }
      outs[u * L.rows_max + r] = acc;
    }
  }
  named_barrier(1, kConsumerThreads);
  if (ready && mbar_wait(route_bar, 0, a.status))
    for (int r = threadIdx.x; r < nr; r += kConsumerThreads) {
      float acc = outs[r];
      for (int u = 1; u < units; ++u)
        acc = __fadd_rn(acc, __fmul_rn(sortedw[u - 1], outs[u * L.rows_max + r]));
      a.y[i0 + r] = acc;
    }
}

// ---------------------------------------------------------------------------
bool moe_decode_supported(const MoeDecodeArgs& a, int sms) {
  if (a.hidden % 128 || a.width % 128 || a.shared_width % 128) return false;
  if (a.top_k < 1 || a.top_k > kMaxTopK || a.n_experts > kMaxDecodeExperts) return false;
  if (a.top_k > a.n_experts) return false;
  if (a.hidden > 4096 || a.width > 8192 || a.shared_width > 8192) return false;
  // the descriptor table is fetched with one bulk copy: 16-byte multiple
  if ((a.n_experts * static_cast<int>(sizeof(FfnView))) % 16) return false;
  const int grid = a.hidden < sms ? a.hidden : sms;
  if (grid < 1) return false;
  const DecodeLayout L = decode_layout(a, grid);
  // shared memory, and h plus the phase-B partials inside the idle ring
  return L.slots >= kMinStages && L.total <= kSmemBudget &&
         L.part_off + part_bytes(a, L.rows_max) <= L.slots * L.stage_bytes;
}

cudaError_t launch_moe_decode(int mode, const MoeDecodeArgs& a, int sms, cudaStream_t st, bool pdl) {
  if (!moe_decode_supported(a, sms) || !a.grid_sync) return cudaErrorInvalidValue;
  const int grid = a.hidden < sms ? a.hidden : sms;
  const DecodeLayout L = decode_layout(a, grid);
  // Every shared-memory region accessed with 16-byte vectors or by a bulk
  // copy must start on a 16-byte boundary, and so must x and h.
  int misaligned = L.stage_bytes | L.x_off | L.xs_off | L.hq_off | L.rp_off | L.desc_off |
                   L.bar_off | L.part_off;
  // every unit's region: the bases and the strides (rows_max * widths, widths % 128 == 0)
  misaligned |= L.w_base | L.s_base | L.w_shared | L.w_unit | L.s_shared | L.s_unit;
  if ((misaligned & 15) || reinterpret_cast<uintptr_t>(a.x) % 16 ||
      reinterpret_cast<uintptr_t>(a.h) % 16 || reinterpret_cast<uintptr_t>(a.experts) % 16)
    return cudaErrorMisalignedAddress;

  using Fn = void (*)(MoeDecodeArgs, DecodeLayout);
  Fn fn = mode == MODE_INT8 ? moe_decode_kernel<MODE_INT8> : moe_decode_kernel<MODE_FP32>;
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(moe_decode_kernel<MODE_FP32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemBudget);
    cudaFuncSetAttribute(moe_decode_kernel<MODE_INT8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemBudget);
  });
  // Cooperative: all CTAs co-resident (the grid barrier needs it).  PDL: the
  // next step's kernel may launch early; its CTAs wait in
  // griddepcontrol.wait before reading anything this one writes.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a, L);
  if (e != cudaSuccess && pdl) {
    cudaGetLastError();
    cfg.numAttrs = 1;  // cooperative only
    e = cudaLaunchKernelEx(&cfg, fn, a, L);
  }
  return e;
}

}  // namespace uocr
