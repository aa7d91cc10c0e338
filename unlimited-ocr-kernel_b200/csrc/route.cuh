// route.cuh — moe::route for one token, computed by one warp.
//
// Restates src/decoder/moe.rs:7-30 with ops::softmax (src/cpu/ops.rs:135-187):
//   reject NaN / +inf, max must be finite; subtract the max; exp; sum left to
//   right from -0.0; divide; order by probability descending then expert id
//   ascending; keep top_k; optional renormalisation by the (rank-ordered) sum
//   of the kept probabilities + 1e-20; multiply by the routed scale.
// Every step uses the same IEEE operation sequence as the reference, so the
// selection and weights match it bit for bit except where an exp value rounds
// differently (exp_f32_via_f64), which can only move a weight by one ulp.
// The rank of element i is #{j : p_j > p_i or (p_j == p_i and j < i)}; the
// kept elements are those of rank < top_k, so no sort is needed.
#pragma once

#include "common.cuh"

namespace uocr {

// `p` is warp-private shared scratch of n floats; ids/wts receive top_k
// entries in route order.  Returns false (status flagged) for an invalid row.
__device__ __forceinline__ bool route_row_warp(const float* __restrict__ logits, int n, int top_k,
                                               int normalize, float scale, float* p, int* ids,
                                               float* wts, unsigned* status) {
  const int lane = threadIdx.x & 31;
  bool bad = false;
  float mx = -INFINITY;
  for (int i = lane; i < n; i += 32) {
    const float v = logits[i];
    p[i] = v;
    bad |= isnan(v) || v == INFINITY;
    mx = fmaxf(mx, v);
  }
  bad = __any_sync(0xffffffffu, bad);
  mx = warp_max(mx);
  if (bad || !isfinite(mx)) {
    if (lane == 0) flag(status, DEV_SOFTMAX);
    return false;
  }
  __syncwarp();
  for (int i = lane; i < n; i += 32) p[i] = exp_f32_via_f64(__fsub_rn(p[i], mx));
  __syncwarp();
  float sum = -0.0f;
  if (lane == 0)
    for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, p[i]);
  sum = __shfl_sync(0xffffffffu, sum, 0);
  for (int i = lane; i < n; i += 32) p[i] = __fdiv_rn(p[i], sum);
  __syncwarp();
  for (int i = lane; i < n; i += 32) {
    const float pi = p[i];
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const float pj = p[j];
      rank += (pj > pi) || (pj == pi && j < i);
    }
    if (rank < top_k) {
      ids[rank] = i;
      wts[rank] = pi;
    }
  }
  __syncwarp();
  if (lane == 0) {
    float denominator = 1.0f;
    if (normalize) {
      float s = -0.0f;
      for (int r = 0; r < top_k; ++r) s = __fadd_rn(s, wts[r]);
      denominator = __fadd_rn(s, 1e-20f);
    }
    for (int r = 0; r < top_k; ++r) wts[r] = __fmul_rn(__fdiv_rn(wts[r], denominator), scale);
  }
  __syncwarp();
  return true;
}

// Low-latency single-warp form for up to 64 experts (the decode kernels).
// Lane l holds experts l and l+32.  Same arithmetic as route_row_warp,
// arranged around the warp's latency:
//  * the max is one redux.sync over order-preserving integer keys;
//  * lane 0 sums the exponentials in index order from vector loads out of
//    `p` (64 floats of 16-byte-aligned warp-private shared scratch);
//  * the top_k experts are taken one per round, already in route order: a
//    redux.sync max over the remaining probabilities (all >= +0, so their bit
//    patterns order like their values; a taken or absent expert has key 0,
//    the others bits + 1), then the lowest expert id holding that key from
//    two ballots (ids 0-31 come before 32-63);
//  * the renormalisation sum accumulates in the same rank order.
// Writes ids/wts (route order) and sorted_ids/sorted_wts (ascending id, the
// order Decoder::experts adds the routed outputs), top_k entries each.
// Requires top_k <= n <= 64 and top_k <= 32.  Every lane must call it.
__device__ __forceinline__ int float_order_key(float v) {
  const int b = __float_as_int(v);
  return b >= 0 ? b : b ^ 0x7FFFFFFF;
}

__device__ __forceinline__ bool route_row_warp64(const float* __restrict__ logits, int n,
                                                 int top_k, int normalize, float scale, float* p,
                                                 int* ids, float* wts, int* sorted_ids,
                                                 float* sorted_wts, unsigned* status) {
  const int lane = threadIdx.x & 31;
  const bool in0 = lane < n, in1 = lane + 32 < n;
  const float v0 = in0 ? logits[lane] : -INFINITY;
  const float v1 = in1 ? logits[lane + 32] : -INFINITY;
  const bool bad = __any_sync(0xffffffffu, (in0 && (isnan(v0) || v0 == INFINITY)) ||
                                               (in1 && (isnan(v1) || v1 == INFINITY)));
  if (bad) {
    if (lane == 0) flag(status, DEV_SOFTMAX);
    return false;
  }
  const int mk = __reduce_max_sync(0xffffffffu, max(float_order_key(v0), float_order_key(v1)));
  const float mx = __int_as_float(mk >= 0 ? mk : mk ^ 0x7FFFFFFF);
  if (!isfinite(mx)) {  // every logit is -inf
    if (lane == 0) flag(status, DEV_SOFTMAX);
    return false;
  }
  const float e0 = in0 ? exp_f32_via_f64(__fsub_rn(v0, mx)) : 0.0f;
  const float e1 = in1 ? exp_f32_via_f64(__fsub_rn(v1, mx)) : 0.0f;
  p[lane] = e0;
  p[lane + 32] = e1;
  __syncwarp();
  float sum = -0.0f;  // left to right over expert ids
  if (lane == 0) {
    const float4* p4 = reinterpret_cast<const float4*>(p);
    float4 t[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) t[q] = p4[q];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      if (4 * q < n) sum = __fadd_rn(sum, t[q].x);
      if (4 * q + 1 < n) sum = __fadd_rn(sum, t[q].y);
      if (4 * q + 2 < n) sum = __fadd_rn(sum, t[q].z);
      if (4 * q + 3 < n) sum = __fadd_rn(sum, t[q].w);
    }
  }
  sum = __shfl_sync(0xffffffffu, sum, 0);
  unsigned k0 = in0 ? __float_as_uint(__fdiv_rn(e0, sum)) + 1u : 0u;
  unsigned k1 = in1 ? __float_as_uint(__fdiv_rn(e1, sum)) + 1u : 0u;
  int my_id = 0;
  float my_p = 0.0f, kept = -0.0f;
  for (int r = 0; r < top_k; ++r) {
    const unsigned m = __reduce_max_sync(0xffffffffu, max(k0, k1));
    const unsigned b0 = __ballot_sync(0xffffffffu, k0 == m);
    const unsigned b1 = __ballot_sync(0xffffffffu, k1 == m);
    const int id = b0 ? __ffs(b0) - 1 : 31 + __ffs(b1);
    const float pr = __uint_as_float(m - 1u);
    if (lane == (id & 31)) {
      if (id < 32) k0 = 0u;
      else k1 = 0u;
    }
    if (lane == r) {
      my_id = id;
      my_p = pr;
    }
    kept = __fadd_rn(kept, pr);  // rank order, from -0.0
  }
  // The selected experts are exactly the present ones whose key is now 0.
  const unsigned lo = __ballot_sync(0xffffffffu, in0 && k0 == 0u);
  const unsigned hi = __ballot_sync(0xffffffffu, in1 && k1 == 0u);
  if (lane < top_k) {
    const float denominator = normalize ? __fadd_rn(kept, 1e-20f) : 1.0f;
    const float w = __fmul_rn(__fdiv_rn(my_p, denominator), scale);
    const unsigned long long sel = (static_cast<unsigned long long>(hi) << 32) | lo;
    const int pos = __popcll(sel & ((1ull << my_id) - 1ull));
    ids[lane] = my_id;
    wts[lane] = w;
    sorted_ids[pos] = my_id;
    sorted_wts[pos] = w;
  }
  __syncwarp();
  return true;
}

}  // namespace uocr
