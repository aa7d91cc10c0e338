// moe_prefill.cu — Decoder::experts for many tokens (src/decoder/mod.rs:124-220,
// serial branch :197-219): route every token, group the (token, expert) pairs
// by expert with tokens ascending inside a group (the order in which
// `assignments[expert].push((row, p))` fills them), run each expert's SwiGLU
// FFN on its gathered rows, and add p * out to the shared expert's output in
// ascending expert id.
//
// Projection dispatch per group follows Decoder::projection
// (src/decoder/mod.rs:99-112):
//   mode WEIGHTS_ONLY        -> FP32 activations for every group;
//   mode DYNAMIC (reference) -> int8 activations only for a group of exactly
//                               one row, FP32 otherwise (so the shared expert
//                               is FP32 whenever tokens > 1);
//   mode DYNAMIC_ROWWISE     -> int8 activations for every row (extension).
//
// This file holds the grouping, combine and a CUDA-core grouped projection
// kernel that serves every shape.  In int8 mode for every row, layers whose
// shapes qualify run every projection on the tensor cores instead
// (q8_tc.cu): rows gathered per expert, one grouped launch per projection.
#include "common.cuh"
#include "kernels.h"

namespace uocr {

constexpr int kGroupThreads = 1024;
constexpr int kMaxGroupExperts = 256;

// Stable counting sort of the tokens*top_k (token, expert) pairs by expert.
// Pair i = t*top_k + j is visited in increasing i, i.e. increasing token, so
// each expert's slice lists its tokens in ascending order.  With
// skip_negative, a negative id marks an unused pair (a padding row of a
// fixed-capacity dispatch): it joins no group and its token_pos is -1.
__global__ void __launch_bounds__(kGroupThreads) group_pairs_kernel(
    const int32_t* __restrict__ ids, const float* __restrict__ wts, int tokens, int top_k,
    int n_experts, int skip_negative, int* __restrict__ counts, int* __restrict__ offsets,
    int* __restrict__ pair_token, float* __restrict__ pair_weight, int* __restrict__ token_pos,
    int* __restrict__ items, int items_max, unsigned* status) {
  pdl_launch_dependents();  // launched as a programmatic dependent (launch_dependent):
  pdl_wait_prior_grids();   // nothing is touched before the previous kernel completes
  // per-warp counts, padded so that a warp reading one expert's column (a
  // lane per source warp) touches 32 banks
  __shared__ int cnt[kGroupThreads / 32][kMaxGroupExperts + 1];
  __shared__ int base[kMaxGroupExperts];
  __shared__ int off[kMaxGroupExperts + 1];
  __shared__ int first[kMaxGroupExperts + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int npairs = tokens * top_k;
  for (int e = tid; e < n_experts; e += blockDim.x) base[e] = 0;
  for (int i = tid; i < (kGroupThreads / 32) * (kMaxGroupExperts + 1); i += blockDim.x)
    (&cnt[0][0])[i] = 0;
  __syncthreads();
  // pass 1: histogram
  for (int i = tid; i < npairs; i += blockDim.x) {
    int e = ids[i];
    if (e < 0 && skip_negative) continue;
    if (e < 0 || e >= n_experts) {
      flag(status, DEV_BAD_ROUTE);
      e = 0;
    }
    atomicAdd(&base[e], 1);
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive prefix sums over the experts of the group sizes and of the
    // groups' 8-row chunk counts (first list position of each group's chunks;
    // groups of more than items_max rows have none: the tensor-core GEMMs).
    // Lane l sums experts [8l, 8l + 8) in order, a warp scan adds the lanes.
    constexpr int kPer = kMaxGroupExperts / 32;
    int c[kPer];
    int s = 0, sc = 0;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = kPer * lane + u;
      c[u] = e < n_experts ? base[e] : 0;
      s += c[u];
      sc += c[u] <= items_max ? (c[u] + 7) / 8 : 0;
    }
    int is = s, isc = sc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, is, o);
      const int w = __shfl_up_sync(0xffffffffu, isc, o);
      if (lane >= o) {
        is += v;
        isc += w;
      }
    }
    int run = is - s, chunks = isc - sc;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = kPer * lane + u;
      if (e < n_experts) {
        off[e] = run;
        counts[e] = c[u];
        offsets[e] = run;
        first[e] = chunks;
        base[e] = 0;
      }
      run += c[u];
      chunks += c[u] <= items_max ? (c[u] + 7) / 8 : 0;
    }
    if (lane == 31) {  // the totals
      off[n_experts] = is;
      offsets[n_experts] = is;
      first[n_experts] = isc;
    }
  }
  __syncthreads();
  if (items) {
    // the list of 8-row chunks of every group of at most items_max rows
    // (small_rows_kernel's work)
    if (tid == 0) items[0] = first[n_experts];
    for (int e = warp; e < n_experts; e += kGroupThreads / 32)
      for (int c = lane; c < first[e + 1] - first[e]; c += 32) items[1 + first[e] + c] = c << 8 | e;
  }
  // pass 2: stable positions, chunk by chunk
  for (int c0 = 0; c0 < npairs; c0 += blockDim.x) {
    const int i = c0 + tid;
    int e = i < npairs ? ids[i] : -1;
    if (i < npairs && e < 0 && skip_negative) token_pos[i] = -1;
    const bool valid = i < npairs && !(e < 0 && skip_negative);
    if (valid && (e < 0 || e >= n_experts)) e = 0;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1));
    if (valid && rank == 0) cnt[warp][e] = __popc(peers);
    __syncthreads();
    // expert x's running base over the warps in order: a warp per expert,
    // lane w holding warp w's count, an exclusive warp scan
    for (int x = warp; x < n_experts; x += kGroupThreads / 32) {
      const int v = cnt[lane][x];
      const int b = base[x];
      int inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
      }
      cnt[lane][x] = b + inc - v;
      __syncwarp();
      if (lane == 31) base[x] = b + inc;
    }
    __syncthreads();
    if (valid) {
      const int pos = off[e] + cnt[warp][e] + rank;
      pair_token[pos] = i / top_k;
      pair_weight[pos] = wts[i];
      token_pos[i] = pos;
    }
    __syncthreads();
    for (int x = tid; x < (kGroupThreads / 32) * n_experts; x += blockDim.x)
      cnt[x / n_experts][x % n_experts] = 0;
    __syncthreads();
  }
  // positions past the grouped pairs (unused pairs were skipped): the gathers
  // that walk every position (split_rows, gather_rows) read row 0 there, a
  // valid row that no group consumes
  for (int i = off[n_experts] + tid; i < npairs; i += blockDim.x) {
    pair_token[i] = 0;
    pair_weight[i] = 0.0f;
  }
}

// y[t] = shared_out[t] (already in y); then for t's experts in ascending id:
// y[t] += p * out[pos] — src/decoder/mod.rs:208-217, one rounding per op.
// Grid (tokens, column blocks); the top_k (<= 8) pairs sit in fixed-size
// register arrays (unused slots sort last), a thread's loads of all pairs
// are issued before its ordered sums.
template <bool VEC4>
__global__ void __launch_bounds__(128) combine_kernel(
    const int32_t* __restrict__ ids, const int* __restrict__ token_pos,
    const float* __restrict__ pair_weight, const float* __restrict__ out_routed, int tokens,
    int top_k, int hidden, float* __restrict__ y) {
  const int t = blockIdx.x;
  if (t >= tokens) return;
  int e[8], pos[8];
  float w[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const bool used = j < top_k;
    e[j] = used ? ids[t * top_k + j] : 0x7fffffff;
    pos[j] = used ? token_pos[t * top_k + j] : 0;
    w[j] = used ? pair_weight[pos[j]] : 0.0f;
  }
#pragma unroll
  for (int i = 1; i < 8; ++i)
#pragma unroll
    for (int j = i; j > 0; --j)
      if (e[j - 1] > e[j]) {
        const int te = e[j]; e[j] = e[j - 1]; e[j - 1] = te;
        const int tp = pos[j]; pos[j] = pos[j - 1]; pos[j - 1] = tp;
        const float tw = w[j]; w[j] = w[j - 1]; w[j - 1] = tw;
      }
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (VEC4) {
    if (4 * c >= hidden) return;
    float4* yr = reinterpret_cast<float4*>(y + static_cast<long long>(t) * hidden) + c;
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < top_k)
        v[j] = reinterpret_cast<const float4*>(out_routed + static_cast<long long>(pos[j]) * hidden)[c];
    float4 acc = *yr;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < top_k) {
        acc.x = __fadd_rn(acc.x, __fmul_rn(w[j], v[j].x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(w[j], v[j].y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(w[j], v[j].z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(w[j], v[j].w));
      }
    *yr = acc;
  } else {
    if (c >= hidden) return;
    float acc = y[static_cast<long long>(t) * hidden + c];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < top_k)
        acc = __fadd_rn(acc, __fmul_rn(w[j], out_routed[static_cast<long long>(pos[j]) * hidden + c]));
    y[static_cast<long long>(t) * hidden + c] = acc;
  }
}

// The same combine for outputs in pair order (row t*top_k + j).
__global__ void combine_pairs_kernel(const int32_t* __restrict__ ids,
                                     const float* __restrict__ weights,
                                     const float* __restrict__ pair_out, int tokens, int top_k,
                                     int hidden, float* __restrict__ y) {
  const int t = blockIdx.x;
  if (t >= tokens) return;
  int e[8], j[8];
  for (int i = 0; i < top_k; ++i) {
    e[i] = ids[t * top_k + i];
    j[i] = i;
  }
  for (int i = 1; i < top_k; ++i)
    for (int m = i; m > 0 && e[m - 1] > e[m]; --m) {
      int te = e[m]; e[m] = e[m - 1]; e[m - 1] = te;
      int tj = j[m]; j[m] = j[m - 1]; j[m - 1] = tj;
    }
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    float acc = y[static_cast<long long>(t) * hidden + c];
    for (int i = 0; i < top_k; ++i) {
      const long long row = static_cast<long long>(t) * top_k + j[i];
      acc = __fadd_rn(acc, __fmul_rn(weights[row], pair_out[row * hidden + c]));
    }
    y[static_cast<long long>(t) * hidden + c] = acc;
  }
}

// pair_out[i] = out_r[token_pos[i]]: routed outputs back in pair order
// (unused pairs, token_pos -1, are left as they are).
__global__ void unpermute_kernel(const int* __restrict__ token_pos, const float* __restrict__ out_r,
                                 int pairs, int hidden, float* __restrict__ pair_out) {
  const int i = blockIdx.x;
  if (i >= pairs || token_pos[i] < 0) return;
  const float* src = out_r + static_cast<long long>(token_pos[i]) * hidden;
  float* dst = pair_out + static_cast<long long>(i) * hidden;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) dst[c] = src[c];
}

void launch_moe_combine_pairs(const int32_t* ids, const float* weights, const float* pair_out,
                              int tokens, int top_k, int hidden, float* y, cudaStream_t st) {
  if (tokens > 0)
    combine_pairs_kernel<<<tokens, 256, 0, st>>>(ids, weights, pair_out, tokens, top_k, hidden, y);
}

// ---------------------------------------------------------------------------
// Fixed-capacity dispatch for expert parallelism.  Pair i = t*top_k + j goes
// to the rank r that owns its expert (bounds[r] <= e < bounds[r+1]), slot =
// the number of earlier pairs (in pair order) for r: send_ids[r][slot] = e -
// bounds[r] (-1 marks an unused slot), pair_rows[i] = r * capacity + slot.
__global__ void __launch_bounds__(kGroupThreads) dispatch_plan_kernel(
    const int32_t* __restrict__ ids, int pairs, int n_experts, DispatchBounds bd, int capacity,
    int32_t* __restrict__ send_ids, int32_t* __restrict__ pair_rows, unsigned* status) {
  __shared__ int cnt[kGroupThreads / 32][kMaxDispatchRanks];
  __shared__ int base[kMaxDispatchRanks];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, world = bd.world;
  for (int i = tid; i < world * capacity; i += blockDim.x) send_ids[i] = -1;
  for (int r = tid; r < world; r += blockDim.x) base[r] = 0;
  for (int i = tid; i < (kGroupThreads / 32) * kMaxDispatchRanks; i += blockDim.x)
    (&cnt[0][0])[i] = 0;
  __syncthreads();
  for (int c0 = 0; c0 < pairs; c0 += blockDim.x) {
    const int i = c0 + tid;
    int e = i < pairs ? ids[i] : -1, r = -1;
    if (i < pairs) {
      if (e < 0 || e >= n_experts) {
        flag(status, DEV_BAD_ROUTE);
        e = 0;
      }
      r = 0;
      while (r + 1 < world && e >= bd.b[r + 1]) ++r;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, r);
    const int rank_in_warp = __popc(peers & ((1u << lane) - 1));
    if (r >= 0 && rank_in_warp == 0) cnt[warp][r] = __popc(peers);
    __syncthreads();
    for (int x = tid; x < world; x += blockDim.x) {
      int run = base[x];
      for (int w = 0; w < kGroupThreads / 32; ++w) {
        const int v = cnt[w][x];
        cnt[w][x] = run;
        run += v;
      }
      base[x] = run;
    }
    __syncthreads();
    if (r >= 0) {
      const int slot = cnt[warp][r] + rank_in_warp;
      if (slot < capacity) {
        send_ids[r * capacity + slot] = e - bd.b[r];
        pair_rows[i] = r * capacity + slot;
      } else {
        flag(status, DEV_CAPACITY);
        pair_rows[i] = -1;
      }
    }
    __syncthreads();
    for (int x = tid; x < (kGroupThreads / 32) * world; x += blockDim.x)
      cnt[x / world][x % world] = 0;
    __syncthreads();
  }
}

// send_x[pair_rows[i]] = x[i / top_k], one CTA per pair.
__global__ void dispatch_rows_kernel(const float* __restrict__ x, int hidden, int top_k,
                                     const int32_t* __restrict__ pair_rows, int pairs,
                                     float* __restrict__ send_x) {
  const int i = blockIdx.x;
  if (i >= pairs) return;
  const int row = pair_rows[i];
  if (row < 0) return;
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<long long>(i / top_k) * hidden);
  float4* dst = reinterpret_cast<float4*>(send_x + static_cast<long long>(row) * hidden);
  for (int c = threadIdx.x; c < hidden / 4; c += blockDim.x) dst[c] = src[c];
}

// y[t] += w * rows[pair_rows[t*top_k + j]] over t's pairs in ascending expert
// id (y holds the shared expert's output), one rounding per operation.
__global__ void combine_rows_kernel(const int32_t* __restrict__ ids,
                                    const float* __restrict__ weights,
                                    const float* __restrict__ rows,
                                    const int32_t* __restrict__ pair_rows, int tokens, int top_k,
                                    int hidden, float* __restrict__ y) {
  const int t = blockIdx.x;
  if (t >= tokens) return;
  int e[8], j[8];
  for (int i = 0; i < top_k; ++i) {
    e[i] = ids[t * top_k + i];
    j[i] = i;
  }
  for (int i = 1; i < top_k; ++i)
    for (int m = i; m > 0 && e[m - 1] > e[m]; --m) {
      int te = e[m]; e[m] = e[m - 1]; e[m - 1] = te;
      int tj = j[m]; j[m] = j[m - 1]; j[m - 1] = tj;
    }
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    float acc = y[static_cast<long long>(t) * hidden + c];
    for (int i = 0; i < top_k; ++i) {
      const int p = t * top_k + j[i];
      const int row = pair_rows[p];
      if (row < 0) continue;  // over capacity: reported through the status word
      acc = __fadd_rn(acc, __fmul_rn(weights[p], rows[static_cast<long long>(row) * hidden + c]));
    }
    y[static_cast<long long>(t) * hidden + c] = acc;
  }
}

cudaError_t launch_moe_dispatch(const float* x, int tokens, int hidden, const int32_t* ids,
                                int top_k, int n_experts, const int* bounds, int world,
                                int capacity, float* send_x, int32_t* send_ids,
                                int32_t* pair_rows, unsigned* status, cudaStream_t st) {
  if (world < 1 || world > kMaxDispatchRanks || capacity < 1 || hidden % 4) return cudaErrorInvalidValue;
  DispatchBounds bd{};
  bd.world = world;
  for (int r = 0; r <= world; ++r) bd.b[r] = bounds[r];
  const int pairs = tokens * top_k;
  // unused slots travel as zero rows (quantizing them raises nothing)
  cudaMemsetAsync(send_x, 0, sizeof(float) * static_cast<size_t>(world) * capacity * hidden, st);
  dispatch_plan_kernel<<<1, kGroupThreads, 0, st>>>(ids, pairs, n_experts, bd, capacity, send_ids,
                                                    pair_rows, status);
  if (pairs > 0)
    dispatch_rows_kernel<<<pairs, 128, 0, st>>>(x, hidden, top_k, pair_rows, pairs, send_x);
  return cudaGetLastError();
}

void launch_moe_combine_rows(const int32_t* ids, const float* weights, const float* rows,
                             const int32_t* pair_rows, int tokens, int top_k, int hidden, float* y,
                             cudaStream_t st) {
  if (tokens > 0)
    combine_rows_kernel<<<tokens, 256, 0, st>>>(ids, weights, rows, pair_rows, tokens, top_k,
                                                hidden, y);
}

// ---------------------------------------------------------------------------
// CUDA-core grouped projection.  Problem p < E is expert p over its pair
// slice; p == E is the shared expert over all tokens.
struct GroupSet {
  const FfnView* experts;
  FfnView shared;
  int E, T, H, F, FS, mode, stage;  // stage 0: gate/up -> h, stage 1: down -> out
  const int* counts;
  const int* offsets;
  const int* pair_token;
  // stage 0 inputs: x rows by token (float / block-quantized)
  const float* x;
  const int8_t* xq;
  const float* xs;
  // stage 0 outputs / stage 1 inputs: h rows (routed by pair slot, shared by token)
  float* h_r;
  float* h_s;
  const int8_t* hq_r;
  const float* hs_r;
  const int8_t* hq_s;
  const float* hs_s;
  // stage 1 outputs
  float* out_r;
  float* y;
};

constexpr int kTM = 32, kTN = 64, kCCThreads = 256;

__device__ __forceinline__ bool group_int8(int mode, int count) {
  return mode == 2 || (mode == 1 && count == 1);
}

// Locate the m-tile `bx` among problems 0..E (tiles of kTM rows).
__device__ __forceinline__ bool find_tile(const GroupSet& g, int bx, int& p, int& m0, int& count) {
  int run = 0;
  for (int q = 0; q <= g.E; ++q) {
    const int c = q < g.E ? g.counts[q] : g.T;
    const int tiles = (c + kTM - 1) / kTM;
    if (bx < run + tiles) {
      p = q;
      m0 = (bx - run) * kTM;
      count = c;
      return true;
    }
    run += tiles;
  }
  return false;
}

template <bool PAIRED>
__global__ void __launch_bounds__(kCCThreads) grouped_cc_kernel(const __grid_constant__ GroupSet g) {
  __shared__ int s_p, s_m0, s_count;
  __shared__ __align__(16) float xt[kTM][kBlock + 1];
  __shared__ __align__(16) int8_t xqt[kTM][kBlock];
  __shared__ float xst[kTM];
  __shared__ __align__(16) int8_t wt[2][kTN][kBlock];
  __shared__ float wst[2][kTN];
  __shared__ int rowsrc[kTM];
  if (threadIdx.x == 0) {
    int p, m0, c;
    if (!find_tile(g, blockIdx.x, p, m0, c)) p = -1;
    s_p = p;
    s_m0 = m0;
    s_count = c;
  }
  __syncthreads();
  const int p = s_p;
  if (p < 0) return;
  const int m0 = s_m0, count = s_count;
  const bool is_shared = p == g.E;
  const FfnView& f = is_shared ? g.shared : g.experts[p];
  const Q8View& A = g.stage == 0 ? f.gate : f.down;
  const Q8View& B = f.up;  // only used when PAIRED
  const int N = A.rows, K = A.cols, nbK = blocks_of(K);
  const int n0 = blockIdx.y * kTN;
  if (n0 >= N) return;
  const bool i8 = group_int8(g.mode, count);
  const int off = is_shared ? 0 : g.offsets[p];
  // row sources
  if (threadIdx.x < kTM) {
    const int i = m0 + threadIdx.x;
    int src = -1;
    if (i < count) src = g.stage == 0 ? (is_shared ? i : g.pair_token[off + i]) : i;
    rowsrc[threadIdx.x] = src;
  }
  __syncthreads();
  // input row pointers
  const float* in_f = nullptr;
  const int8_t* in_q = nullptr;
  const float* in_s = nullptr;
  long long in_ld = K;
  if (g.stage == 0) {
    in_f = g.x;
    in_q = g.xq;
    in_s = g.xs;
  } else if (is_shared) {
    in_f = g.h_s;
    in_q = g.hq_s;
    in_s = g.hs_s;
  } else {
    in_f = g.h_r + static_cast<long long>(off) * K;
    in_q = g.hq_r + static_cast<long long>(off) * K;
    in_s = g.hs_r + static_cast<long long>(off) * nbK;
  }
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 4 n-rows x 2 tokens
  float acc[2][2][4];
  for (int a = 0; a < 2; ++a)
    for (int b = 0; b < 2; ++b)
      for (int c = 0; c < 4; ++c) acc[a][b][c] = i8 ? -0.0f : 0.0f;
  for (int blk = 0; blk < nbK; ++blk) {
    const int k0 = blk * kBlock, kw = min(kBlock, K - k0);
    // stage X tile
    for (int e = threadIdx.x; e < kTM * kBlock; e += kCCThreads) {
      const int r = e / kBlock, c = e % kBlock;
      const int src = rowsrc[r];
      if (i8) {
        xqt[r][c] = (src >= 0 && c < kw) ? in_q[src * in_ld + k0 + c] : 0;
        if (c == 0) xst[r] = src >= 0 ? in_s[src * static_cast<long long>(nbK) + blk] : 0.0f;
      } else {
        xt[r][c] = (src >= 0 && c < kw) ? in_f[src * in_ld + k0 + c] : 0.0f;
      }
    }
    // stage W tiles
    for (int e = threadIdx.x; e < kTN * kBlock; e += kCCThreads) {
      const int r = e / kBlock, c = e % kBlock;
      const int n = n0 + r;
      wt[0][r][c] = (n < N && c < kw) ? A.w[static_cast<long long>(n) * K + k0 + c] : 0;
      if (PAIRED) wt[1][r][c] = (n < N && c < kw) ? B.w[static_cast<long long>(n) * K + k0 + c] : 0;
      if (c == 0) {
        wst[0][r] = n < N ? A.s[static_cast<long long>(n) * nbK + blk] : 0.0f;
        if (PAIRED) wst[1][r] = n < N ? B.s[static_cast<long long>(n) * nbK + blk] : 0.0f;
      }
    }
    __syncthreads();
    for (int mat = 0; mat < (PAIRED ? 2 : 1); ++mat)
      for (int a = 0; a < 2; ++a) {
        const int r = ty * 2 + a;
        for (int c = 0; c < 4; ++c) {
          const int nr = tx * 4 + c;
          if (i8) {
            int S = 0;
            const int* wq = reinterpret_cast<const int*>(&wt[mat][nr][0]);
            const int* xqq = reinterpret_cast<const int*>(&xqt[r][0]);
#pragma unroll
            for (int q = 0; q < 8; ++q) S = __dp4a(wq[q], xqq[q], S);
            acc[mat][a][c] = __fadd_rn(acc[mat][a][c],
                                       __fmul_rn(__fmul_rn(static_cast<float>(S), wst[mat][nr]), xst[r]));
          } else {
            float d = 0.0f;
#pragma unroll 8
            for (int q = 0; q < kBlock; ++q) d = fmaf(static_cast<float>(wt[mat][nr][q]), xt[r][q], d);
            acc[mat][a][c] = fmaf(wst[mat][nr], d, acc[mat][a][c]);
          }
        }
      }
    __syncthreads();
  }
  for (int a = 0; a < 2; ++a) {
    const int r = ty * 2 + a;
    const int i = m0 + r;
    if (i >= count) continue;
    for (int c = 0; c < 4; ++c) {
      const int n = n0 + tx * 4 + c;
      if (n >= N) continue;
      if (g.stage == 0) {
        const float h = __fmul_rn(silu_ref(acc[0][a][c]), acc[PAIRED ? 1 : 0][a][c]);
        if (is_shared)
          g.h_s[static_cast<long long>(i) * N + n] = h;
        else
          g.h_r[static_cast<long long>(off + i) * N + n] = h;
      } else {
        if (is_shared)
          g.y[static_cast<long long>(i) * N + n] = acc[0][a][c];
        else
          g.out_r[static_cast<long long>(off + i) * N + n] = acc[0][a][c];
      }
    }
  }
}

// ---------------------------------------------------------------------------
static size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

struct PrefillWs {
  int* counts;
  int* offsets;
  int* pair_token;
  float* pair_weight;
  int* token_pos;
  int8_t* xq;
  float* xs;
  float* h_r;
  float* h_s;
  int8_t* hq_r;
  float* hs_r;
  int8_t* hq_s;
  float* hs_s;
  float* out_r;
  // tensor-core paths
  float* u_r;
  float* u_s;
  int8_t* xq_p;  // int8: gathered rows
  float* xs_p;
  uint16_t* xp_r;  // FP32 activations: bf16 pieces of the gathered rows,
  uint16_t* hp_r;  // of the routed hidden rows,
  uint16_t* xp_s;  // of the tokens,
  uint16_t* hp_s;  // of the shared hidden rows
  float* xr_r;     // their rows' 2^-e
  float* hr_r;
  float* xr_s;
  float* hr_s;
  int* counts_big;  // tensor-core paths: groups of more than kSmallRowsMax rows
  int* items;       // 8-row chunks of the groups (count first)
  int max_items;
  size_t bytes;
};

// Which kernels run the projections.  TcMixed is QuantizationMode::
// DynamicActivations (src/decoder/mod.rs:103-106): int8 activations for a
// group of one row, FP32 for the others, each on its tensor-core kernel.
enum class Path { CudaCore, TcInt8, TcFp32, TcMixed };

static Path prefill_path(const MoePrefillArgs& a, int mode) {
  const bool shapes = a.tc_maps && q8_tc_supported(a.shared_width, a.hidden) &&
                      q8_tc_supported(a.hidden, a.shared_width) &&
                      q8_tc_supported(a.width, a.hidden) && q8_tc_supported(a.hidden, a.width);
  if (!shapes) return Path::CudaCore;
  if (mode == 2) return Path::TcInt8;
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0) return Path::CudaCore;
  return mode == 0 ? Path::TcFp32 : Path::TcMixed;
}

static PrefillWs carve(const MoePrefillArgs& a, void* base, Path path) {
  PrefillWs w{};
  const size_t T = a.tokens, P = static_cast<size_t>(a.tokens) * a.top_k;
  const size_t H = a.hidden, F = a.width, FS = a.shared_width;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return base ? static_cast<char*>(base) + o : nullptr;
  };
  w.counts = reinterpret_cast<int*>(take(sizeof(int) * (a.n_experts + 1)));
  w.offsets = reinterpret_cast<int*>(take(sizeof(int) * (a.n_experts + 1)));
  w.pair_token = reinterpret_cast<int*>(take(sizeof(int) * P));
  w.pair_weight = reinterpret_cast<float*>(take(sizeof(float) * P));
  w.token_pos = reinterpret_cast<int*>(take(sizeof(int) * P));
  w.max_items = small_chunk_items(static_cast<int>(P), a.n_experts);
  w.items = reinterpret_cast<int*>(take(sizeof(int) * (w.max_items + 1)));
  w.h_r = reinterpret_cast<float*>(take(sizeof(float) * P * F));
  w.h_s = reinterpret_cast<float*>(take(sizeof(float) * T * FS));
  w.out_r = reinterpret_cast<float*>(take(sizeof(float) * P * H));
  if (path != Path::TcFp32) {  // int8 activations somewhere
    w.xq = reinterpret_cast<int8_t*>(take(T * H));
    w.xs = reinterpret_cast<float*>(take(sizeof(float) * T * blocks_of(a.hidden)));
    w.hq_r = reinterpret_cast<int8_t*>(take(P * F));
    w.hs_r = reinterpret_cast<float*>(take(sizeof(float) * P * blocks_of(a.width)));
    w.hq_s = reinterpret_cast<int8_t*>(take(T * FS));
    w.hs_s = reinterpret_cast<float*>(take(sizeof(float) * T * blocks_of(a.shared_width)));
  }
  if (path != Path::CudaCore) {
    w.u_r = reinterpret_cast<float*>(take(sizeof(float) * P * F));
    w.u_s = reinterpret_cast<float*>(take(sizeof(float) * T * FS));
  }
  if (path == Path::TcInt8 || path == Path::TcMixed) {
    w.xq_p = reinterpret_cast<int8_t*>(take(P * H));
    w.xs_p = reinterpret_cast<float*>(take(sizeof(float) * P * blocks_of(a.hidden)));
  }
  if (path != Path::CudaCore)
    w.counts_big = reinterpret_cast<int*>(take(sizeof(int) * (a.n_experts + 1)));
  if (path == Path::TcFp32 || path == Path::TcMixed) {
    w.xp_r = reinterpret_cast<uint16_t*>(take(2 * 3 * P * H));
    w.hp_r = reinterpret_cast<uint16_t*>(take(2 * 3 * P * F));
    w.xp_s = reinterpret_cast<uint16_t*>(take(2 * 3 * T * H));
    w.hp_s = reinterpret_cast<uint16_t*>(take(2 * 3 * T * FS));
    w.xr_r = reinterpret_cast<float*>(take(sizeof(float) * P));
    w.hr_r = reinterpret_cast<float*>(take(sizeof(float) * P));
    w.xr_s = reinterpret_cast<float*>(take(sizeof(float) * T));
    w.hr_s = reinterpret_cast<float*>(take(sizeof(float) * T));
  }
  w.bytes = off;
  return w;
}

size_t moe_prefill_workspace(const MoePrefillArgs& a, int mode) {
  return carve(a, nullptr, prefill_path(a, mode)).bytes;
}

void moe_prefill_grouped(const MoePrefillArgs& a, int mode, const int** token_pos,
                         const float** out_rows) {
  const PrefillWs w = carve(a, a.workspace, prefill_path(a, mode));
  *token_pos = w.token_pos;
  *out_rows = w.out_r;
}

// Token counts up to which the shared expert (one matrix, every token) runs on
// the warp-level kernel: its tcgen05 tiles would occupy only N / 128 SMs.
constexpr int kSmallShared = 64;

// counts_big[g] = counts[g] when it exceeds `small` rows, else 0 (the
// tensor-core GEMMs take the big groups, the warp-level kernel the others).
__global__ void big_counts_kernel(const int* __restrict__ counts, int groups, int small,
                                  int* __restrict__ counts_big) {
  for (int g = threadIdx.x; g < groups; g += blockDim.x) {
    const int c = counts[g];
    counts_big[g] = c > small ? c : 0;
  }
}

static void launch_big_counts(const int* counts, int groups, int small, int* counts_big,
                              cudaStream_t st) {
  big_counts_kernel<<<1, 256, 0, st>>>(counts, groups, small, counts_big);
}

// Upper bound on the 64-row tiles of the groups the tensor-core GEMMs take
// (more than kSmallRowsMax rows each, so at most P / (kSmallRowsMax + 1) of
// them): sum over those groups of ceil(count / 64) <= P / 64 + their number.
// The grid has a slot per possible tile; a tight bound keeps the slots that
// find no tile (every one, at decode batch sizes) few.
static int big_group_tiles(int P, int E) {
  const int groups = P / (kSmallRowsMax + 1) < E ? P / (kSmallRowsMax + 1) : E;
  return P / 64 + groups + 1;
}

// The largest group a call can form: tokens, or the caller's bound.
static int max_group_rows(const MoePrefillArgs& a) {
  return a.max_group_rows > 0 && a.max_group_rows < a.tokens ? a.max_group_rows : a.tokens;
}

// Groups of up to this many rows run on the warp-level kernel (from the chunk
// list, one CTA per 8-row chunk), larger ones on the tensor-core GEMMs: every
// group when no group can exceed kSmallChunkedMax rows, else the caller's
// bound or kSmallRowsMax.
static int small_group_rows(const MoePrefillArgs& a) {
  const int G = max_group_rows(a);
  if (G <= kSmallChunkedMax) return G > 1 ? G : 1;
  if (a.small_max > 0) return a.small_max;
  return kSmallRowsMax;
}

// Grid rows of a chunk-list launch: the list holds the chunks of groups of at
// most R rows, so with larger groups possible (tc) at most n_experts * R/8.
static int items_bound(const MoePrefillArgs& a, const PrefillWs& w, int R, bool tc) {
  const int by_groups = a.n_experts * ((R + 7) / 8);
  return tc && by_groups < w.max_items ? by_groups : w.max_items;
}

// With unused rows (negative ids) the grouped rows in use are the first
// offsets[n_experts]; the row passes over grouped rows stop there.
static const int* grouped_live(const MoePrefillArgs& a, const PrefillWs& w) {
  return a.skip_negative_ids ? w.offsets + a.n_experts : nullptr;
}

// The shared expert over T <= kSmallShared tokens with FP32 activations, as
// chunks of 8 rows on the warp-level kernel (the tokens' pieces are in
// w.xp_s / w.xr_s); its down projection writes y.
static cudaError_t shared_small_f32(const MoePrefillArgs& a, const PrefillWs& w, int sms,
                                    cudaStream_t st) {
  const int T = a.tokens, H = a.hidden, FS = a.shared_width;
  cudaError_t e;
  // gate and up in one launch
  if ((e = launch_small_rows(false, nullptr, &a.shared.gate, nullptr, nullptr, 1, 1, kSmallRowsMax, T, FS,
                             H, w.xp_s, T, w.xr_s, nullptr, nullptr, T, w.h_s, FS,
                             a.status, st, nullptr, 0, nullptr, &a.shared.up, w.u_s)))
    return e;
  launch_swiglu_split(w.h_s, w.u_s, T, FS, w.hp_s, w.hr_s, sms, st);
  return launch_small_rows(false, nullptr, &a.shared.down, nullptr, nullptr, 1, 1, kSmallRowsMax, T, H,
                             FS, w.hp_s, T, w.hr_s, nullptr, nullptr, T, a.y, H,
                             a.status, st);
}

// FP32 activations, all projections on the tensor cores (exact bf16 pieces).
static cudaError_t prefill_tc_f32(const MoePrefillArgs& a, const PrefillWs& w, int sms,
                                  cudaStream_t st) {
  const int T = a.tokens, k = a.top_k, E = a.n_experts, P = T * k;
  const int H = a.hidden, F = a.width, FS = a.shared_width;
  const int max_tiles = big_group_tiles(P, E);
  const unsigned char* maps = static_cast<const unsigned char*>(a.tc_maps);
  const size_t mb = q8_tc_maps_bytes();
  cudaError_t e;
  // no group exceeds T rows: up to kSmallChunkedMax tokens every group runs on
  // the warp-level kernel and the tensor-core launches are skipped
  const int R = small_group_rows(a);
  const bool tc = max_group_rows(a) > R;
  const int* live = grouped_live(a, w);
  const int ni = items_bound(a, w, R, tc);
  if (!a.skip_routed) {
    if (tc) launch_big_counts(w.counts, E, R, w.counts_big, st);
    launch_split_rows(a.x, H, w.pair_token, P, H, w.xp_r, w.xr_r, sms, st, live);
    // gate and up of the small groups in one launch
    if ((e = launch_small_rows(false, maps, nullptr, w.counts, w.offsets, E, 1, R, 0, F, H, w.xp_r,
                               P, w.xr_r, nullptr, nullptr, P, w.h_r, F, a.status, st,
                               w.items, ni, maps + E * mb, nullptr, w.u_r)))
      return e;
    for (int j = 0; tc && j < 2; ++j)  // gate, up of the larger groups
      if ((e = launch_q8_tc_grouped_f32(maps + j * E * mb, E, w.counts_big, w.offsets, max_tiles,
                                        F, H, w.xp_r, w.xr_r, P, j == 0 ? w.h_r : w.u_r, F,
                                        a.status, st)))
        return e;
    launch_swiglu_split(w.h_r, w.u_r, P, F, w.hp_r, w.hr_r, sms, st, live);
    if ((e = launch_small_rows(false, maps + 2 * E * mb, nullptr, w.counts, w.offsets, E, 1, R, 0, H,
                                 F, w.hp_r, P, w.hr_r, nullptr, nullptr, P, w.out_r, H,
                                 a.status, st, w.items, ni)) ||
        (tc && (e = launch_q8_tc_grouped_f32(maps + 2 * E * mb, E, w.counts_big, w.offsets,
                                             max_tiles, H, F, w.hp_r, w.hr_r, P, w.out_r, H,
                                             a.status, st))))
      return e;
  }
  if (a.skip_shared) return cudaSuccess;
  launch_split_rows(a.x, H, nullptr, T, H, w.xp_s, w.xr_s, sms, st);
  if (T <= kSmallShared) return shared_small_f32(a, w, sms, st);
  if ((e = launch_q8_tc_single_f32(a.shared.gate, w.xp_s, w.xr_s, T, w.h_s, FS, a.status, st)) ||
      (e = launch_q8_tc_single_f32(a.shared.up, w.xp_s, w.xr_s, T, w.u_s, FS, a.status, st)))
    return e;
  launch_swiglu_split(w.h_s, w.u_s, T, FS, w.hp_s, w.hr_s, sms, st);
  return launch_q8_tc_single_f32(a.shared.down, w.hp_s, w.hr_s, T, a.y, H, a.status, st);
}

// Int8 activations for every row, all projections on the tensor cores.
static cudaError_t prefill_tc(const MoePrefillArgs& a, const PrefillWs& w, int sms, cudaStream_t st) {
  const int T = a.tokens, k = a.top_k, E = a.n_experts, P = T * k;
  const int H = a.hidden, F = a.width, FS = a.shared_width;
  const int max_tiles = big_group_tiles(P, E);
  const unsigned char* maps = static_cast<const unsigned char*>(a.tc_maps);
  const size_t mb = q8_tc_maps_bytes();  // per matrix
  cudaError_t e;
  const int R = small_group_rows(a);
  const bool tc = max_group_rows(a) > R;
  const int* live = grouped_live(a, w);
  const int ni = items_bound(a, w, R, tc);
  if (!a.skip_routed) {
    // routed experts: rows gathered per expert; groups of <= R rows on the
    // warp-level kernel, larger ones on the tensor-core GEMM
    if (tc) launch_big_counts(w.counts, E, R, w.counts_big, st);
    launch_gather_rows(w.xq, w.xs, w.pair_token, P, H, w.xq_p, w.xs_p, sms, st, live);
    // gate and up of the small groups in one launch
    if ((e = launch_small_rows(true, maps, nullptr, w.counts, w.offsets, E, 1, R, 0, F, H, nullptr,
                               0, nullptr, w.xq_p, w.xs_p, P, w.h_r, F, a.status, st,
                               w.items, ni, maps + E * mb, nullptr, w.u_r)))
      return e;
    for (int j = 0; tc && j < 2; ++j)  // gate, up of the larger groups
      if ((e = launch_q8_tc_grouped_i8(maps + j * E * mb, E, w.counts_big, w.offsets, max_tiles,
                                       F, H, w.xq_p, w.xs_p, P, j == 0 ? w.h_r : w.u_r, F,
                                       a.status, st)))
        return e;
    launch_swiglu_quantize(w.h_r, w.u_r, P, F, w.hq_r, w.hs_r, a.status, sms, st, live);
    if ((e = launch_small_rows(true, maps + 2 * E * mb, nullptr, w.counts, w.offsets, E, 1, R, 0, H,
                                 F, nullptr, 0, nullptr, w.hq_r, w.hs_r, P, w.out_r, H,
                                 a.status, st, w.items, ni)) ||
        (tc && (e = launch_q8_tc_grouped_i8(maps + 2 * E * mb, E, w.counts_big, w.offsets,
                                            max_tiles, H, F, w.hq_r, w.hs_r, P, w.out_r, H,
                                            a.status, st))))
      return e;
  }
  if (a.skip_shared) return cudaSuccess;
  // shared expert over every token; its down projection writes y
  if (T <= kSmallShared) {
    if ((e = launch_small_rows(true, nullptr, &a.shared.gate, nullptr, nullptr, 1, 1, kSmallRowsMax, T, FS,
                             H, nullptr, 0, nullptr, w.xq, w.xs, T, w.h_s, FS,
                             a.status, st, nullptr, 0, nullptr, &a.shared.up, w.u_s)))
      return e;
    launch_swiglu_quantize(w.h_s, w.u_s, T, FS, w.hq_s, w.hs_s, a.status, sms, st);
    return launch_small_rows(true, nullptr, &a.shared.down, nullptr, nullptr, 1, 1, kSmallRowsMax, T, H,
                             FS, nullptr, 0, nullptr, w.hq_s, w.hs_s, T, a.y, H,
                             a.status, st);
  }
  if ((e = launch_q8_tc_single_i8(a.shared.gate, w.xq, w.xs, T, w.h_s, FS, a.status, st)) ||
      (e = launch_q8_tc_single_i8(a.shared.up, w.xq, w.xs, T, w.u_s, FS, a.status, st)))
    return e;
  launch_swiglu_quantize(w.h_s, w.u_s, T, FS, w.hq_s, w.hs_s, a.status, sms, st);
  return launch_q8_tc_single_i8(a.shared.down, w.hq_s, w.hs_s, T, a.y, H, a.status, st);
}

// QuantizationMode::DynamicActivations on the tensor cores: a group of one
// row (src/decoder/mod.rs:103-106: projection of a single-row input) takes the
// bit-exact int8 arithmetic, every other group FP32: groups of 2..R rows on
// the warp-level kernel, larger ones on the FP32 GEMM; the launches write
// disjoint rows.  Both SwiGLU forms run over all rows (each down projection
// reads its own).  The shared expert sees every token: int8 for one token.
static cudaError_t prefill_tc_mixed(const MoePrefillArgs& a, const PrefillWs& w, int sms,
                                    cudaStream_t st) {
  const int T = a.tokens, k = a.top_k, E = a.n_experts, P = T * k;
  const int H = a.hidden, F = a.width, FS = a.shared_width;
  const int max_tiles = big_group_tiles(P, E);
  const unsigned char* maps = static_cast<const unsigned char*>(a.tc_maps);
  const size_t mb = q8_tc_maps_bytes();
  const int R0 = small_group_rows(a);
  const int R = R0 > 2 ? R0 : 2;
  const bool tc = max_group_rows(a) > R0;
  const int* live = grouped_live(a, w);
  const int ni = items_bound(a, w, R, tc);
  cudaError_t e;
  if (!a.skip_routed) {
    if (tc) launch_big_counts(w.counts, E, R, w.counts_big, st);
    launch_gather_rows(w.xq, w.xs, w.pair_token, P, H, w.xq_p, w.xs_p, sms, st, live);
    launch_split_rows(a.x, H, w.pair_token, P, H, w.xp_r, w.xr_r, sms, st, live);
    // gate and up together: one-row groups int8, 2..R rows FP32, larger on the GEMM
    if ((e = launch_small_rows(true, maps, nullptr, w.counts, w.offsets, E, 1, 1, 0, F, H, nullptr,
                               0, nullptr, w.xq_p, w.xs_p, P, w.h_r, F, a.status, st,
                               w.items, ni, maps + E * mb, nullptr, w.u_r)) ||
        (e = launch_small_rows(false, maps, nullptr, w.counts, w.offsets, E, 2, R, 0, F, H, w.xp_r,
                               P, w.xr_r, nullptr, nullptr, P, w.h_r, F, a.status, st,
                               w.items, ni, maps + E * mb, nullptr, w.u_r)))
      return e;
    for (int j = 0; tc && j < 2; ++j)
      if ((e = launch_q8_tc_grouped_f32(maps + j * E * mb, E, w.counts_big, w.offsets, max_tiles,
                                        F, H, w.xp_r, w.xr_r, P, j == 0 ? w.h_r : w.u_r, F,
                                        a.status, st)))
        return e;
    launch_swiglu_quantize(w.h_r, w.u_r, P, F, w.hq_r, w.hs_r, a.status, sms, st, live);
    launch_swiglu_split(w.h_r, w.u_r, P, F, w.hp_r, w.hr_r, sms, st, live);
    if ((e = launch_small_rows(true, maps + 2 * E * mb, nullptr, w.counts, w.offsets, E, 1, 1, 0, H,
                                 F, nullptr, 0, nullptr, w.hq_r, w.hs_r, P, w.out_r, H,
                                 a.status, st, w.items, ni)) ||
        (e = launch_small_rows(false, maps + 2 * E * mb, nullptr, w.counts, w.offsets, E, 2, R, 0, H,
                                 F, w.hp_r, P, w.hr_r, nullptr, nullptr, P, w.out_r, H,
                                 a.status, st, w.items, ni)) ||
        (tc && (e = launch_q8_tc_grouped_f32(maps + 2 * E * mb, E, w.counts_big, w.offsets,
                                             max_tiles, H, F, w.hp_r, w.hr_r, P, w.out_r, H,
                                             a.status, st))))
      return e;
  }
  if (a.skip_shared) return cudaSuccess;
  if (T == 1) {
    if ((e = launch_small_rows(true, nullptr, &a.shared.gate, nullptr, nullptr, 1, 1, 1, 1, FS,
                             H, nullptr, 0, nullptr, w.xq, w.xs, T, w.h_s, FS,
                             a.status, st, nullptr, 0, nullptr, &a.shared.up, w.u_s)))
      return e;
    launch_swiglu_quantize(w.h_s, w.u_s, T, FS, w.hq_s, w.hs_s, a.status, sms, st);
    return launch_small_rows(true, nullptr, &a.shared.down, nullptr, nullptr, 1, 1, 1, 1, H,
                             FS, nullptr, 0, nullptr, w.hq_s, w.hs_s, T, a.y, H,
                             a.status, st);
  }
  launch_split_rows(a.x, H, nullptr, T, H, w.xp_s, w.xr_s, sms, st);
  if (T <= kSmallShared) return shared_small_f32(a, w, sms, st);
  if ((e = launch_q8_tc_single_f32(a.shared.gate, w.xp_s, w.xr_s, T, w.h_s, FS, a.status, st)) ||
      (e = launch_q8_tc_single_f32(a.shared.up, w.xp_s, w.xr_s, T, w.u_s, FS, a.status, st)))
    return e;
  launch_swiglu_split(w.h_s, w.u_s, T, FS, w.hp_s, w.hr_s, sms, st);
  return launch_q8_tc_single_f32(a.shared.down, w.hp_s, w.hr_s, T, a.y, H, a.status, st);
}

cudaError_t launch_moe_prefill(int mode, const MoePrefillArgs& a, int sms, cudaStream_t st) {
  if (a.n_experts > kMaxGroupExperts || a.top_k > 8) return cudaErrorInvalidValue;
  if (a.skip_shared && a.skip_routed) return cudaErrorInvalidValue;
  if (a.skip_shared && !a.skip_routed && !a.pair_out && !a.keep_grouped)
    return cudaErrorInvalidValue;
  const Path path = prefill_path(a, mode);
  PrefillWs w = carve(a, a.workspace, path);
  if (w.bytes > a.workspace_bytes) return cudaErrorInvalidValue;
  const int T = a.tokens, k = a.top_k, E = a.n_experts;
  if (mode != 0) launch_quantize_rows(a.x, a.hidden, T, a.hidden, w.xq, w.xs, a.status, sms, st);
  // the shared expert needs only x: it runs on the call's stream while the
  // routing and the routed experts (the longer chain) run on the high-priority
  // side stream, when both parts run on the warp-level kernel
  const bool fork = a.side && a.ev_fork && a.ev_join && !a.skip_shared && !a.skip_routed &&
                    !a.pair_out && !a.skip_negative_ids && path != Path::CudaCore &&
                    T <= kSmallShared && T <= kSmallChunkedMax;
  auto run_path = [&](const MoePrefillArgs& pa, cudaStream_t s) {
    return path == Path::TcInt8   ? prefill_tc(pa, w, sms, s)
           : path == Path::TcFp32 ? prefill_tc_f32(pa, w, sms, s)
                                  : prefill_tc_mixed(pa, w, sms, s);
  };
  const cudaStream_t rs = fork ? a.side : st;  // the routed chain's stream
  if (fork) {
    cudaError_t e = cudaEventRecord(a.ev_fork, st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(rs, a.ev_fork, 0);
    if (e != cudaSuccess) return e;
  }
  if (!a.skip_routed) {
    if (!a.route_given)
      launch_route(a.logits, T, E, k, a.normalize, a.scale, a.route_ids, a.route_weights,
                   a.status, sms, rs);
    launch_dependent(group_pairs_kernel, dim3(1), dim3(kGroupThreads), 0, rs, a.route_ids,
                     a.route_weights, T, k, E, static_cast<int>(a.skip_negative_ids), w.counts,
                     w.offsets, w.pair_token, w.pair_weight, w.token_pos,
                     path == Path::CudaCore ? nullptr : w.items,
                     path == Path::TcMixed ? (small_group_rows(a) > 2 ? small_group_rows(a) : 2)
                                           : small_group_rows(a),
                     a.status);
  }
  if (a.skip_negative_ids && !a.skip_routed && path == Path::CudaCore) {
    // unused rows belong to no group and are never written by the projections:
    // zero them so that the SwiGLU and quantization passes over all rows see 0
    // (the tensor-core paths stop their row passes at the grouped count)
    const size_t hb = sizeof(float) * static_cast<size_t>(T) * k * a.width;
    cudaMemsetAsync(w.h_r, 0, hb, st);
    if (w.u_r) cudaMemsetAsync(w.u_r, 0, hb, st);
  }
  if (fork) {
    MoePrefillArgs routed_only = a, shared_only = a;
    routed_only.skip_shared = 1;
    shared_only.skip_routed = 1;
    cudaError_t e = run_path(routed_only, rs);
    const cudaError_t ej = cudaEventRecord(a.ev_join, rs);
    const cudaError_t es = e == cudaSuccess ? run_path(shared_only, st) : cudaSuccess;
    const cudaError_t ew = cudaStreamWaitEvent(st, a.ev_join, 0);  // the routed outputs
    if (e == cudaSuccess) e = ej != cudaSuccess ? ej : es != cudaSuccess ? es : ew;
    if (e != cudaSuccess) return e;
  } else if (path != Path::CudaCore) {
    const cudaError_t e = path == Path::TcInt8   ? prefill_tc(a, w, sms, st)
                          : path == Path::TcFp32 ? prefill_tc_f32(a, w, sms, st)
                                                 : prefill_tc_mixed(a, w, sms, st);
    if (e != cudaSuccess) return e;
  } else {
    GroupSet g{};
    g.experts = a.experts;
    g.shared = a.shared;
    g.E = a.skip_routed ? 0 : E;      // no routed problems
    g.T = a.skip_shared ? 0 : T;      // the shared problem has no rows
    g.H = a.hidden;
    g.F = a.width;
    g.FS = a.shared_width;
    g.mode = mode;
    g.counts = w.counts;
    g.offsets = w.offsets;
    g.pair_token = w.pair_token;
    g.x = a.x;
    g.xq = w.xq;
    g.xs = w.xs;
    g.h_r = w.h_r;
    g.h_s = w.h_s;
    g.hq_r = w.hq_r;
    g.hs_r = w.hs_r;
    g.hq_s = w.hq_s;
    g.hs_s = w.hs_s;
    g.out_r = w.out_r;
    g.y = a.y;
    // an upper bound on m-tiles over all problems
    const int mtiles = (T * k) / kTM + E + (T + kTM - 1) / kTM + 1;
    const int wmax = a.width > a.shared_width ? a.width : a.shared_width;
    g.stage = 0;
    grouped_cc_kernel<true><<<dim3(mtiles, (wmax + kTN - 1) / kTN), kCCThreads, 0, st>>>(g);
    if (mode != 0) {
      if (!a.skip_routed)
        launch_quantize_rows(w.h_r, a.width, T * k, a.width, w.hq_r, w.hs_r, a.status, sms, st);
      if (!a.skip_shared)
        launch_quantize_rows(w.h_s, a.shared_width, T, a.shared_width, w.hq_s, w.hs_s, a.status,
                             sms, st);
    }
    g.stage = 1;
    grouped_cc_kernel<false><<<dim3(mtiles, (a.hidden + kTN - 1) / kTN), kCCThreads, 0, st>>>(g);
  }
  if (!a.skip_routed && !a.keep_grouped) {
    if (a.pair_out)
      unpermute_kernel<<<T * k, 256, 0, st>>>(w.token_pos, w.out_r, T * k, a.hidden, a.pair_out);
    else
    {
      // float4 columns when rows stay 16-byte aligned
      const bool v4 = a.hidden % 4 == 0 && reinterpret_cast<uintptr_t>(a.y) % 16 == 0;
      const int cols = v4 ? a.hidden / 4 : a.hidden;
      const dim3 grid(T, (cols + 127) / 128);
      if (v4)
        combine_kernel<true><<<grid, 128, 0, st>>>(a.route_ids, w.token_pos, w.pair_weight,
                                                   w.out_r, T, k, a.hidden, a.y);
      else
        combine_kernel<false><<<grid, 128, 0, st>>>(a.route_ids, w.token_pos, w.pair_weight,
                                                    w.out_r, T, k, a.hidden, a.y);
    }
  }
  return cudaGetLastError();
}

}  // namespace uocr
