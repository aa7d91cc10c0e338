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

// CTA-wide form of route_row_warp for the decode kernels: thread i owns
// expert i (n <= blockDim.x), so max, exp, division and the rank count run in
// parallel; only the sum stays sequential (thread 0, left to right) because
// its rounding order is part of the result.  Every thread of the block must
// call it.  Shared scratch: p[n], red[32], ids/wts[top_k], flag[1].
__device__ __forceinline__ bool route_row_block(const float* __restrict__ logits, int n,
                                                int top_k, int normalize, float scale, float* p,
                                                float* red, int* ids, float* wts, int* bad_flag,
                                                unsigned* status) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  if (tid == 0) *bad_flag = 0;
  const bool mine = tid < n;
  const float v = mine ? logits[tid] : -INFINITY;
  const bool bad = mine && (isnan(v) || v == INFINITY);
  const float wm = warp_max(v);
  const bool wbad = __any_sync(0xffffffffu, bad);
  __syncthreads();
  if (lane == 0) {
    red[warp] = wm;
    if (wbad) *bad_flag = 1;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int w = 0; w < nwarps; ++w) mx = fmaxf(mx, red[w]);
  if (*bad_flag || !isfinite(mx)) {
    if (tid == 0) flag(status, DEV_SOFTMAX);
    return false;
  }
  if (mine) p[tid] = exp_f32_via_f64(__fsub_rn(v, mx));
  __syncthreads();
  if (tid == 0) {
    float s = -0.0f;
    for (int i = 0; i < n; ++i) s = __fadd_rn(s, p[i]);
    red[0] = s;
  }
  __syncthreads();
  const float pi = mine ? __fdiv_rn(p[tid], red[0]) : 0.0f;
  __syncthreads();
  if (mine) p[tid] = pi;
  __syncthreads();
  if (mine) {
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const float pj = p[j];
      rank += (pj > pi) || (pj == pi && j < tid);
    }
    if (rank < top_k) {
      ids[rank] = tid;
      wts[rank] = pi;
    }
  }
  __syncthreads();
  if (tid == 0) {
    float denominator = 1.0f;
    if (normalize) {
      float s = -0.0f;
      for (int r = 0; r < top_k; ++r) s = __fadd_rn(s, wts[r]);
      denominator = __fadd_rn(s, 1e-20f);
    }
    for (int r = 0; r < top_k; ++r) wts[r] = __fmul_rn(__fdiv_rn(wts[r], denominator), scale);
  }
  __syncthreads();
  return true;
}

// Sort the top_k (id, weight) pairs by ascending id: the order in which
// Decoder::experts adds routed outputs (src/decoder/mod.rs:186-194,198-218).
__device__ __forceinline__ void sort_by_id(int* ids, float* wts, int k) {
  for (int i = 1; i < k; ++i) {
    const int id = ids[i];
    const float w = wts[i];
    int j = i - 1;
    while (j >= 0 && ids[j] > id) {
      ids[j + 1] = ids[j];
      wts[j + 1] = wts[j];
      --j;
    }
    ids[j + 1] = id;
    wts[j + 1] = w;
  }
}

}  // namespace uocr
