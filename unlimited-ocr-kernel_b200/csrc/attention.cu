// attention.cu — the attention half of a decoder layer at decode, on the
// device: RMSNorm (ops::rms_norm, src/cpu/ops.rs:362-414), the rotary
// embedding (ops::rope, :420-437), the token-major KV cache with an
// immutable prefix and a bounded ring (LayerCache, src/decoder/cache.rs:3-95)
// and single-query attention over it (ops::attention_decode, :515-606); the
// causal attention of a prefill (ops::attention, :263-360) runs the same
// kernels with one query per row, row i over tokens 0..i of one sequence.
//
// Arithmetic follows the reference's order so that results are bit-identical
// to it except where exp rounds differently (exp_f32_via_f64, rarely one ulp):
//  * RMSNorm: squares in parallel, one thread sums them left to right from
//    -0.0, IEEE division by the width, sqrt then reciprocal, then
//    ((x * scale) * w) + 0.0 per element;
//  * rope: cos/sin from a table the host builds with the same single-precision
//    operations as the reference (powf, division, sinf/cosf), then
//    a*cos - b*sin and b*cos + a*sin with one rounding per operation;
//  * attention: per head, each token's score is a left-to-right sum over the
//    head dimension (one thread per token, -0.0 start), times the scale;
//    softmax as the reference's (max, subtract, exp, left-to-right sum by one
//    thread, divide); each output element is a left-to-right sum over the
//    tokens in physical cache order (one thread per element, +0.0 start).
//
// Cache layout: head-major keys/values [batch][heads][cap][dim], so that one
// head's tokens are one contiguous stream (the reference stores token-major
// rows; the physical token order per head is the same, so sums run in the
// same order); per-sequence state {prefix, generated} in device memory, so
// pushes and attention can run inside captured graphs.  Slot of the next
// token: prefix + generated % window; tokens present: prefix +
// min(generated, window).  The single-query entry point takes the
// reference's token-major buffers.
#include <cuda_runtime.h>

#include "common.cuh"
#include "device_once.h"
#include "kernels.h"
#include "tc_maps.cuh"

namespace uocr {

// Left-to-right sum from -0.0 of n floats in shared memory (16-byte aligned),
// one thread: 16-byte loads, unrolled so that they run ahead of the chain of
// dependent adds (the order, and so the result, is the sequential one).
__device__ __forceinline__ float serial_sum_smem(const float* v, int n) {
  float acc = -0.0f;
  const float4* v4 = reinterpret_cast<const float4*>(v);
  const int n4 = n >> 2;
#pragma unroll 8
  for (int i = 0; i < n4; ++i) {
    const float4 c = v4[i];
    acc = __fadd_rn(acc, c.x);
    acc = __fadd_rn(acc, c.y);
    acc = __fadd_rn(acc, c.z);
    acc = __fadd_rn(acc, c.w);
  }
  for (int i = n4 << 2; i < n; ++i) acc = __fadd_rn(acc, v[i]);
  return acc;
}

// ---- RMSNorm -----------------------------------------------------------------
constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads)
    rms_norm_kernel(const float* x, long long ld_x, int width, const float* __restrict__ w,
                    float eps, float* out, long long ld_out, const float* res, float* sum,
                    unsigned* status) {
  pdl_launch_dependents();  // launched as a programmatic dependent (launch_dependent):
  pdl_wait_prior_grids();   // nothing is touched before the previous kernel completes
  extern __shared__ __align__(16) float sq[];  // width squares
  __shared__ float s_scale;
  const long long row = blockIdx.x;
  const float* xr = x + row * ld_x;
  // with a residual: the row normalised is sum = x + res (one rounding),
  // written to `sum` (which may alias x or res: each element is read and
  // written by the same thread)
  const float* rr = res ? res + row * ld_x : nullptr;
  float* sr = res ? sum + row * ld_x : nullptr;
  bool bad = false;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    float v = xr[i];
    if (rr) {
      v = __fadd_rn(v, rr[i]);
      sr[i] = v;
    }
    bad |= !isfinite(v) || !isfinite(w[i]);
    sq[i] = __fmul_rn(v, v);
  }
  if (__syncthreads_or(bad)) {
    if (threadIdx.x == 0) flag(status, DEV_NORM);
    return;
  }
  if (threadIdx.x == 0) {
    const float acc = serial_sum_smem(sq, width);
    const float var = __fdiv_rn(acc, static_cast<float>(width));
    s_scale = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
  }
  __syncthreads();
  const float scale = s_scale;
  float* o = out + row * ld_out;
  const float* src = sr ? sr : xr;  // this thread's own writes of `sum`
  for (int i = threadIdx.x; i < width; i += blockDim.x)
    o[i] = __fadd_rn(__fmul_rn(__fmul_rn(src[i], scale), w[i]), 0.0f);
}

void launch_rms_norm(const float* x, long long ld_x, int rows, int width, const float* w, float eps,
                     float* out, long long ld_out, unsigned* status, cudaStream_t st,
                     const float* res, float* sum) {
  if (rows <= 0) return;
  const size_t smem = static_cast<size_t>(width) * 4;
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  launch_dependent(rms_norm_kernel, dim3(rows), dim3(kNormThreads), smem, st, x, ld_x, width, w,
                   eps, out, ld_out, res, sum, status);
}

// ---- rotary embedding ---------------------------------------------------------
// Pairs (i, i + dim/2) of every head of `rows` rows of a (and of b when
// given, the keys beside the queries).  Position of row r: positions[r], or
// from the cache state (prefix + generated) when positions is null.
__global__ void rope_kernel(float* a, float* b, long long ld, int rows, int heads, int dim,
                            const int* __restrict__ positions, const int* __restrict__ state,
                            const float2* __restrict__ table, int max_pos, unsigned* status) {
  const int half = dim >> 1;
  const long long per_row = static_cast<long long>(heads) * half;
  const long long n = rows * per_row;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(idx / per_row);
    const int rem = static_cast<int>(idx % per_row);
    const int head = rem / half, i = rem % half;
    const int pos = positions ? positions[row] : state[2 * row] + state[2 * row + 1];
    if (pos < 0 || pos >= max_pos) {
      flag(status, DEV_POSITION);
      continue;
    }
    const float2 cs = table[static_cast<long long>(pos) * half + i];
    float* ptrs[2] = {a, b};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (!ptrs[k]) continue;
      float* h = ptrs[k] + row * ld + static_cast<long long>(head) * dim;
      const float x0 = h[i], x1 = h[i + half];
      h[i] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
      h[i + half] = __fadd_rn(__fmul_rn(x1, cs.x), __fmul_rn(x0, cs.y));
    }
  }
}

void launch_rope(float* a, float* b, long long ld, int rows, int heads, int dim,
                 const int* positions, const int* state, const float2* table, int max_pos,
                 unsigned* status, int sms, cudaStream_t st) {
  const long long n = static_cast<long long>(rows) * heads * (dim / 2);
  if (n <= 0) return;
  long long blocks = (n + 255) / 256;
  if (blocks > 8LL * sms) blocks = 8LL * sms;
  rope_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(a, b, ld, rows, heads, dim, positions,
                                                         state, table, max_pos, status);
}

// ---- KV cache ------------------------------------------------------------------
__global__ void kv_set_prefix_kernel(int* state, int seq, int tokens) {
  state[2 * seq] = tokens;
  state[2 * seq + 1] = 0;
}

void launch_kv_set_prefix(int* state, int seq, int tokens, cudaStream_t st) {
  kv_set_prefix_kernel<<<1, 1, 0, st>>>(state, seq, tokens);
}

__device__ __forceinline__ long long kv_index(const KvLayout& L, int b, int h, long long slot,
                                              int d) {
  const long long base = (static_cast<long long>(b) * L.heads + h) * L.cap * L.dim;
  if (!L.tiled) return base + slot * L.dim + d;
  const long long tile = slot >> 5;
  const int t = static_cast<int>(slot & 31), j = d >> 5, f = d & 31;
  return base + ((tile * (L.dim >> 5) + j) * 32 + t) * 32 + f;
}

// LayerCache::push for every sequence: row b of k/v into its next slot.
__global__ void kv_push_kernel(float* keys, float* values, int* state, const KvLayout L,
                               int window, const float* __restrict__ k,
                               const float* __restrict__ v, long long ld, unsigned* status) {
  const int b = blockIdx.x;
  const int prefix = state[2 * b], gen = state[2 * b + 1];
  if (prefix <= 0) {
    if (threadIdx.x == 0) flag(status, DEV_CACHE);
    return;
  }
  const long long slot = prefix + gen % window;
  const float* ks = k + b * ld;
  const float* vs = v + b * ld;
  for (int i = threadIdx.x; i < L.heads * L.dim; i += blockDim.x) {
    const int h = i / L.dim, d = i - h * L.dim;
    const long long o = kv_index(L, b, h, slot, d);
    keys[o] = ks[i];
    values[o] = vs[i];
  }
  __syncthreads();  // every thread has read `gen`
  if (threadIdx.x == 0) state[2 * b + 1] = gen + 1;
}

void launch_kv_push(float* keys, float* values, int* state, int batch, const KvLayout& L,
                    int window, const float* k, const float* v, long long ld, unsigned* status,
                    cudaStream_t st) {
  if (batch <= 0) return;
  kv_push_kernel<<<batch, 256, 0, st>>>(keys, values, state, L, window, k, v, ld, status);
}

// ops::rope of q and k and LayerCache::push of k and v for every sequence,
// straight from the fused projection output: row b of qkv is [q | k | v]
// (3 * heads * dim floats).  q is rotated into q_out (row b), k rotated and v
// copied into sequence b's next slot, then the sequence's counter advances —
// the same results as uocr_kv_rope followed by uocr_kv_push.
__global__ void kv_rope_push_kernel(float* keys, float* values, int* state, const KvLayout L,
                                    int window, const float* __restrict__ qkv, float* q_out,
                                    const float2* __restrict__ table, int max_pos,
                                    unsigned* status) {
  pdl_launch_dependents();  // launched as a programmatic dependent (launch_dependent):
  pdl_wait_prior_grids();   // nothing is touched before the previous kernel completes
  const int b = blockIdx.x;
  const int prefix = state[2 * b], gen = state[2 * b + 1];
  if (prefix <= 0) {
    if (threadIdx.x == 0) flag(status, DEV_CACHE);
    return;
  }
  const int width = L.heads * L.dim, half = L.dim >> 1;
  const int pos = prefix + gen;
  const long long slot = prefix + gen % window;
  const float* q = qkv + static_cast<long long>(b) * 3 * width;
  const float* k = q + width;
  const float* v = k + width;
  float* qo = q_out + static_cast<long long>(b) * width;
  const bool in_table = pos >= 0 && pos < max_pos;
  if (!in_table && threadIdx.x == 0) flag(status, DEV_POSITION);
  for (int p = threadIdx.x; p < L.heads * half; p += blockDim.x) {
    const int h = p / half, i = p - h * half;
    const int d0 = h * L.dim + i, d1 = d0 + half;
    float q0 = q[d0], q1 = q[d1], k0 = k[d0], k1 = k[d1];
    if (in_table) {
      const float2 cs = table[static_cast<long long>(pos) * half + i];
      const float rq0 = __fsub_rn(__fmul_rn(q0, cs.x), __fmul_rn(q1, cs.y));
      const float rq1 = __fadd_rn(__fmul_rn(q1, cs.x), __fmul_rn(q0, cs.y));
      const float rk0 = __fsub_rn(__fmul_rn(k0, cs.x), __fmul_rn(k1, cs.y));
      const float rk1 = __fadd_rn(__fmul_rn(k1, cs.x), __fmul_rn(k0, cs.y));
      q0 = rq0;
      q1 = rq1;
      k0 = rk0;
      k1 = rk1;
    }
    qo[d0] = q0;
    qo[d1] = q1;
    keys[kv_index(L, b, h, slot, i)] = k0;
    keys[kv_index(L, b, h, slot, i + half)] = k1;
    values[kv_index(L, b, h, slot, i)] = v[d0];
    values[kv_index(L, b, h, slot, i + half)] = v[d1];
  }
  __syncthreads();  // every thread has read `gen`
  if (threadIdx.x == 0) state[2 * b + 1] = gen + 1;
}

void launch_kv_rope_push(float* keys, float* values, int* state, int batch, const KvLayout& L,
                         int window, const float* qkv, float* q_out, const float2* table,
                         int max_pos, unsigned* status, cudaStream_t st) {
  if (batch <= 0) return;
  launch_dependent(kv_rope_push_kernel, dim3(batch), dim3(256), 0, st, keys, values, state, L,
                   window, qkv, q_out, table, max_pos, status);
}

// One block per token row: token-major [tokens][heads*dim] into the layout.
__global__ void kv_prefill_kernel(float* keys, float* values, const KvLayout L, int seq,
                                  const float* __restrict__ k, const float* __restrict__ v) {
  const long long t = blockIdx.x;
  const int width = L.heads * L.dim;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const int h = i / L.dim, d = i - h * L.dim;
    const long long o = kv_index(L, seq, h, t, d);
    keys[o] = k[t * width + i];
    values[o] = v[t * width + i];
  }
}

void launch_kv_prefill(float* keys, float* values, const KvLayout& L, int seq, const float* k,
                       const float* v, int tokens, cudaStream_t st) {
  if (tokens <= 0) return;
  kv_prefill_kernel<<<tokens, 256, 0, st>>>(keys, values, L, seq, k, v);
}

__global__ void kv_export_kernel(const float* __restrict__ keys, const float* __restrict__ values,
                                 const KvLayout L, int seq, float* k, float* v) {
  const long long t = blockIdx.x;
  const int width = L.heads * L.dim;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const int h = i / L.dim, d = i - h * L.dim;
    const long long o = kv_index(L, seq, h, t, d);
    k[t * width + i] = keys[o];
    v[t * width + i] = values[o];
  }
}

void launch_kv_export(const float* keys, const float* values, const KvLayout& L, int seq,
                      int tokens, float* k_out, float* v_out, cudaStream_t st) {
  if (tokens <= 0) return;
  kv_export_kernel<<<tokens, 256, 0, st>>>(keys, values, L, seq, k_out, v_out);
}

// ---- single-query attention ---------------------------------------------------------
constexpr int kAttnThreads = 256;

// Score of one token: left-to-right over the head dimension from -0.0.
template <bool VEC>
__device__ __forceinline__ float token_score(const float* __restrict__ kr, const float* qs, int dim) {
  float acc = -0.0f;
  if (VEC) {
    const float4* q4 = reinterpret_cast<const float4*>(qs);
    const float4* k4 = reinterpret_cast<const float4*>(kr);
#pragma unroll 8
    for (int d = 0; d < dim / 4; ++d) {
      const float4 kv = __ldg(k4 + d);
      const float4 qv = q4[d];
      acc = __fadd_rn(acc, __fmul_rn(qv.x, kv.x));
      acc = __fadd_rn(acc, __fmul_rn(qv.y, kv.y));
      acc = __fadd_rn(acc, __fmul_rn(qv.z, kv.z));
      acc = __fadd_rn(acc, __fmul_rn(qv.w, kv.w));
    }
  } else {
    for (int d = 0; d < dim; ++d) acc = __fadd_rn(acc, __fmul_rn(qs[d], __ldg(kr + d)));
  }
  return acc;
}

template <bool VEC>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float smem_f[];
  __shared__ float red[kAttnThreads / 32];
  __shared__ int red_bad[kAttnThreads / 32];
  __shared__ float s_max, s_sum;
  __shared__ int s_bad;
  const int h = blockIdx.x;
  // causal: the longest rows first, so that the short ones fill the tail
  const int b = a.causal ? static_cast<int>(gridDim.y - 1 - blockIdx.y) : static_cast<int>(blockIdx.y);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int dim = a.dim;
  float* qs = smem_f;                              // dim floats
  float* sc = smem_f + ((dim + 3) & ~3);           // tokens floats
  int T = a.tokens;
  if (a.causal) {
    T = b + 1;
  } else if (a.state) {
    const int prefix = a.state[2 * b], gen = a.state[2 * b + 1];
    if (prefix <= 0) {
      if (tid == 0) flag(a.status, DEV_CACHE);
      return;
    }
    T = prefix + (gen < a.window ? gen : a.window);
  }
  const long long off = (a.causal ? a.seq : b) * a.seq_stride + h * a.head_stride,
                  rs = a.row_stride;
  const float* kb = a.keys + off;
  const float* vb = a.values + off;
  for (int d = tid; d < dim; d += kAttnThreads) qs[d] = a.q[b * a.ld_q + static_cast<long long>(h) * dim + d];
  __syncthreads();

  // scores: one thread per token, two tokens in flight per thread
  for (int t = tid; t < T; t += 2 * kAttnThreads) {
    const int t2 = t + kAttnThreads;
    const float s1 = token_score<VEC>(kb + t * rs, qs, dim);
    if (t2 < T) {
      const float s2 = token_score<VEC>(kb + t2 * rs, qs, dim);
      sc[t2] = __fmul_rn(s2, a.scale);
    }
    sc[t] = __fmul_rn(s1, a.scale);
  }
  __syncthreads();

  // softmax_backend (src/cpu/ops.rs:139-187)
  float mx = -INFINITY;
  int bad = 0;
  for (int t = tid; t < T; t += kAttnThreads) {
    const float v = sc[t];
    bad |= isnan(v) || v == INFINITY;
    mx = fmaxf(mx, v);
  }
  mx = warp_max(mx);
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    red[warp] = mx;
    red_bad[warp] = bad;
  }
  __syncthreads();
  if (tid == 0) {
    float m = red[0];
    int bd = red_bad[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) {
      m = fmaxf(m, red[w]);
      bd |= red_bad[w];
    }
    s_max = m;
    s_bad = bd || !isfinite(m);
  }
  __syncthreads();
  if (s_bad) {
    if (tid == 0) flag(a.status, DEV_SOFTMAX);
    return;
  }
  mx = s_max;
  for (int t = tid; t < T; t += kAttnThreads) sc[t] = exp_f32_via_f64(__fsub_rn(sc[t], mx));
  __syncthreads();
  if (tid == 0) s_sum = serial_sum_smem(sc, T);
  __syncthreads();
  const float sum = s_sum;
  for (int t = tid; t < T; t += kAttnThreads) sc[t] = __fdiv_rn(sc[t], sum);
  __syncthreads();

  // output: one thread per element, tokens in order from +0.0
  // (ops::attention_decode) or from -0.0 (the Sum of ops::attention)
  float* ob = a.out + b * a.ld_out + static_cast<long long>(h) * dim;
  const float zero = a.causal ? -0.0f : 0.0f;
  for (int d = tid; d < dim; d += kAttnThreads) {
    const float* vc = vb + d;
    float acc = zero;
    int t = 0;
    for (; t + 16 <= T; t += 16) {
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = __ldg(vc + (t + j) * rs);
#pragma unroll
      for (int j = 0; j < 16; ++j) acc = __fadd_rn(acc, __fmul_rn(sc[t + j], v[j]));
    }
    for (; t < T; ++t) acc = __fadd_rn(acc, __fmul_rn(sc[t], __ldg(vc + t * rs)));
    ob[d] = acc;
  }
}

size_t attention_smem_bytes(int dim, int max_tokens) {
  return static_cast<size_t>((dim + 3) & ~3) * 4 + static_cast<size_t>(max_tokens) * 4;
}

cudaError_t launch_attention_decode(const AttnArgs& a, int batch, int max_tokens, cudaStream_t st) {
  const size_t smem = attention_smem_bytes(a.dim, max_tokens);
  if (smem > kAttnMaxSmem || batch <= 0 || a.heads <= 0) return cudaErrorInvalidValue;
  // 16-byte key loads: every row and head start aligned
  const bool vec = a.dim % 4 == 0 && a.row_stride % 4 == 0 && a.head_stride % 4 == 0 &&
                   a.seq_stride % 4 == 0 && reinterpret_cast<uintptr_t>(a.keys) % 16 == 0;
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(attn_decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kAttnMaxSmem));
    cudaFuncSetAttribute(attn_decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kAttnMaxSmem));
  });
  const dim3 grid(a.heads, batch);
  if (vec)
    attn_decode_kernel<true><<<grid, kAttnThreads, smem, st>>>(a);
  else
    attn_decode_kernel<false><<<grid, kAttnThreads, smem, st>>>(a);
  return cudaGetLastError();
}


// ---- single-query attention, TMA pipeline ----------------------------------------
// For head_dim % 32 == 0 (<= 256) and 16-byte-aligned rows: one CTA per
// (head, sequence) of two warps.  The producer warp streams the head's key
// rows, then its value rows, as 32-token tiles of head_dim/32 boxes of
// 32 x 32 floats (128-byte swizzle) through a two-stage ring; the consumer
// warp computes from shared memory with the same arithmetic as
// attn_decode_kernel: lane = token for the scores (a swizzled row is read
// conflict-free by eight lanes at a time), one warp for the softmax, lane =
// four output elements for the value sums.  The ring keeps two tiles in
// flight per CTA while five CTAs share an SM, and the value tiles stream in
// while the softmax runs.
constexpr int kTmaTile = 32;
constexpr int kTmaStages = 2;
constexpr int kTmaBoxBytes = 32 * 32 * 4;

__host__ __device__ inline size_t attn_tma_smem(int dim, long long max_tokens) {
  const size_t stage = static_cast<size_t>(dim / 32) * kTmaBoxBytes;
  return 1024 + kTmaStages * stage + static_cast<size_t>(dim) * 4 +
         ((static_cast<size_t>(max_tokens) * 4 + 15) & ~static_cast<size_t>(15)) + 64;
}

// D128 (head dim 128): the consumer copies its part of a tile (its token's
// key row, or its four output columns of the tile's 32 value rows: 128 floats
// either way) into registers and frees the stage before computing on it, so
// that both stages are in flight while it computes.
template <bool D128>
__global__ void __launch_bounds__(64, 5)
    attn_decode_tma_kernel(const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, const AttnArgs a) {
  extern __shared__ unsigned char smem_raw[];
  // aligned through an integer cast (the pointers below are generic): measured
  // 7% faster here than shared-space pointers (6.57 vs 6.09 TB/s at batch 64)
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int dim = a.dim, nb = dim / 32;
  const int stage_bytes = nb * kTmaBoxBytes;
  float* qs = reinterpret_cast<float*>(base + kTmaStages * stage_bytes);
  float* sc = qs + dim;
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(sc + a.cap) + 15) & ~static_cast<uintptr_t>(15));
  uint64_t* empty = full + kTmaStages;
  const int h = blockIdx.x;
  const int b = a.causal ? static_cast<int>(gridDim.y - 1 - blockIdx.y) : static_cast<int>(blockIdx.y);
  const int kvs = a.causal ? a.seq : b;  // the sequence whose keys/values are read
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int T = a.tokens;
  if (a.causal) {
    T = b + 1;
  } else if (a.state) {
    const int prefix = a.state[2 * b], gen = a.state[2 * b + 1];
    if (prefix <= 0) {
      if (threadIdx.x == 0) flag(a.status, DEV_CACHE);
      return;
    }
    T = prefix + (gen < a.window ? gen : a.window);
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTmaStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 0)
    for (int d = lane; d < dim; d += 32) qs[d] = a.q[b * a.ld_q + static_cast<long long>(h) * dim + d];
  __syncthreads();
  const int ntiles = (T + kTmaTile - 1) / kTmaTile;
  if (warp == 1) {
    // ---- producer
    if (lane == 0) {
      // tiled cache: the map's rows are 128-byte rows of the cache, a tile is
      // one box of 32 * nb of them; token-major buffers ([rows][width]): a
      // tile is nb boxes of 32 rows at x = h*dim + 32j
      const long long tiled_y0 = (static_cast<long long>(kvs) * a.heads + h) * a.cap * nb;
      const int y0 = static_cast<int>(static_cast<long long>(kvs) * a.cap);
      const int x0 = h * dim;
      int it = 0;
      for (; it < 2 * ntiles; ++it) {
        const int st = it & 1;
        if (it >= kTmaStages && !mbar_wait(&empty[st], ((it >> 1) - 1) & 1, a.status)) break;
        const bool keys = it < ntiles;
        const int tile = keys ? it : it - ntiles;
        unsigned char* dst = base + st * stage_bytes;
        mbar_arrive_expect_tx(&full[st], stage_bytes);
        if (a.tiled) {
          tma_load_2d(dst, keys ? &kmap : &vmap, 0,
                      static_cast<int>(tiled_y0 + static_cast<long long>(tile) * kTmaTile * nb),
                      &full[st]);
        } else {
          for (int j = 0; j < nb; ++j)
            tma_load_2d(dst + j * kTmaBoxBytes, keys ? &kmap : &vmap, x0 + 32 * j,
                        y0 + tile * kTmaTile, &full[st]);
        }
      }
      for (int j = it - kTmaStages; j < it; ++j)  // every issued copy lands before exit
        if (j >= 0) mbar_wait(&full[j & 1], (j >> 1) & 1, a.status);
    }
    return;
  }
  // ---- consumer: scores
  const float4* q4 = reinterpret_cast<const float4*>(qs);
  if (D128) {
    for (int i = 0; i < ntiles; ++i) {
      const int st = i & 1;
      mbar_wait(&full[st], (i >> 1) & 1, a.status);
      const unsigned char* row = base + st * stage_bytes + lane * 128;
      float4 kr[32];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int c = 0; c < 8; ++c)
          kr[j * 8 + c] =
              *reinterpret_cast<const float4*>(row + j * kTmaBoxBytes + ((c ^ (lane & 7)) << 4));
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      const int t = i * kTmaTile + lane;
      if (t < T) {
        float acc = -0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float4 qv = q4[j];
          acc = __fadd_rn(acc, __fmul_rn(qv.x, kr[j].x));
          acc = __fadd_rn(acc, __fmul_rn(qv.y, kr[j].y));
          acc = __fadd_rn(acc, __fmul_rn(qv.z, kr[j].z));
          acc = __fadd_rn(acc, __fmul_rn(qv.w, kr[j].w));
        }
        sc[t] = __fmul_rn(acc, a.scale);
      }
    }
  }
  for (int i = 0; !D128 && i < ntiles; ++i) {
    const int st = i & 1;
    mbar_wait(&full[st], (i >> 1) & 1, a.status);
    const int t = i * kTmaTile + lane;
    if (t < T) {
      const unsigned char* row = base + st * stage_bytes + lane * 128;
      float acc = -0.0f;
      for (int j = 0; j < nb; ++j) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 kv =
              *reinterpret_cast<const float4*>(row + j * kTmaBoxBytes + ((c ^ (lane & 7)) << 4));
          const float4 qv = q4[j * 8 + c];
          acc = __fadd_rn(acc, __fmul_rn(qv.x, kv.x));
          acc = __fadd_rn(acc, __fmul_rn(qv.y, kv.y));
          acc = __fadd_rn(acc, __fmul_rn(qv.z, kv.z));
          acc = __fadd_rn(acc, __fmul_rn(qv.w, kv.w));
        }
      }
      sc[t] = __fmul_rn(acc, a.scale);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  __syncwarp();
  // ---- softmax_backend (src/cpu/ops.rs:139-187)
  float mx = -INFINITY;
  int bad = 0;
  for (int t = lane; t < T; t += 32) {
    const float v = sc[t];
    bad |= isnan(v) || v == INFINITY;
    mx = fmaxf(mx, v);
  }
  mx = warp_max(mx);
  bad = __any_sync(0xffffffffu, bad) || !isfinite(mx);
  if (!bad) {
    for (int t = lane; t < T; t += 32) sc[t] = exp_f32_via_f64(__fsub_rn(sc[t], mx));
    __syncwarp();
    float sum = -0.0f;
    if (lane == 0) sum = serial_sum_smem(sc, T);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int t = lane; t < T; t += 32) sc[t] = __fdiv_rn(sc[t], sum);
    __syncwarp();
  } else if (lane == 0) {
    flag(a.status, DEV_SOFTMAX);
  }
  // ---- values: lane owns 16-byte chunks g = lane, lane + 32 of the head row
  const int chunks = dim / 4;
  const float zero = a.causal ? -0.0f : 0.0f;  // see attn_decode_kernel
  float4 acc0 = make_float4(zero, zero, zero, zero), acc1 = acc0;
  const int g0 = lane, g1 = lane + 32;
  if (D128) {
    // chunks == 32: lane owns chunk g0 = lane, in box lane / 8
    for (int i = 0; i < ntiles; ++i) {
      const int it = ntiles + i, st = it & 1;
      mbar_wait(&full[st], (it >> 1) & 1, a.status);
      const unsigned char* tile = base + st * stage_bytes + (lane >> 3) * kTmaBoxBytes;
      float4 vr[32];
#pragma unroll
      for (int r = 0; r < 32; ++r)
        vr[r] = *reinterpret_cast<const float4*>(tile + r * 128 + (((lane & 7) ^ (r & 7)) << 4));
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (!bad) {
        const int rows = T - i * kTmaTile < kTmaTile ? T - i * kTmaTile : kTmaTile;
#pragma unroll
        for (int r = 0; r < 32; ++r)
          if (r < rows) {
            const float p = sc[i * kTmaTile + r];
            acc0.x = __fadd_rn(acc0.x, __fmul_rn(p, vr[r].x));
            acc0.y = __fadd_rn(acc0.y, __fmul_rn(p, vr[r].y));
            acc0.z = __fadd_rn(acc0.z, __fmul_rn(p, vr[r].z));
            acc0.w = __fadd_rn(acc0.w, __fmul_rn(p, vr[r].w));
          }
      }
    }
  }
  for (int i = 0; !D128 && i < ntiles; ++i) {
    const int it = ntiles + i, st = it & 1;
    mbar_wait(&full[st], (it >> 1) & 1, a.status);
    if (!bad) {
      const unsigned char* tile = base + st * stage_bytes;
      const int rows = T - i * kTmaTile < kTmaTile ? T - i * kTmaTile : kTmaTile;
      for (int r = 0; r < rows; ++r) {
        const float p = sc[i * kTmaTile + r];
        const unsigned char* row = tile + r * 128;
        if (g0 < chunks) {
          const float4 v = *reinterpret_cast<const float4*>(
              row + (g0 >> 3) * kTmaBoxBytes + (((g0 & 7) ^ (r & 7)) << 4));
          acc0.x = __fadd_rn(acc0.x, __fmul_rn(p, v.x));
          acc0.y = __fadd_rn(acc0.y, __fmul_rn(p, v.y));
          acc0.z = __fadd_rn(acc0.z, __fmul_rn(p, v.z));
          acc0.w = __fadd_rn(acc0.w, __fmul_rn(p, v.w));
        }
        if (g1 < chunks) {
          const float4 v = *reinterpret_cast<const float4*>(
              row + (g1 >> 3) * kTmaBoxBytes + (((g1 & 7) ^ (r & 7)) << 4));
          acc1.x = __fadd_rn(acc1.x, __fmul_rn(p, v.x));
          acc1.y = __fadd_rn(acc1.y, __fmul_rn(p, v.y));
          acc1.z = __fadd_rn(acc1.z, __fmul_rn(p, v.z));
          acc1.w = __fadd_rn(acc1.w, __fmul_rn(p, v.w));
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (bad) return;
  float* ob = a.out + b * a.ld_out + static_cast<long long>(h) * dim;
  if (g0 < chunks) {
    ob[4 * g0] = acc0.x;
    ob[4 * g0 + 1] = acc0.y;
    ob[4 * g0 + 2] = acc0.z;
    ob[4 * g0 + 3] = acc0.w;
  }
  if (g1 < chunks) {
    ob[4 * g1] = acc1.x;
    ob[4 * g1 + 1] = acc1.y;
    ob[4 * g1 + 2] = acc1.z;
    ob[4 * g1 + 3] = acc1.w;
  }
}

bool attention_tma_ok(const float* keys, const float* values, long long rows, int cols, int dim,
                      long long cap) {
  return dim % 32 == 0 && dim <= 256 && cols % 4 == 0 && rows < (1LL << 31) &&
         reinterpret_cast<uintptr_t>(keys) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(values) % 16 == 0 && attn_tma_smem(dim, cap) <= kAttnMaxSmem;
}

bool attention_tma_maps(AttnMaps* m, const float* keys, const float* values, long long rows,
                        int cols) {
  return make_map_f32_sw128(reinterpret_cast<CUtensorMap*>(m->k), keys, rows, cols) &&
         make_map_f32_sw128(reinterpret_cast<CUtensorMap*>(m->v), values, rows, cols);
}

bool attention_tma_maps_tiled(AttnMaps* m, const float* keys, const float* values,
                              long long elements, int dim) {
  const long long rows = elements / 32;  // 128-byte rows
  return make_map_f32_sw128(reinterpret_cast<CUtensorMap*>(m->k), keys, rows, 32, dim) &&
         make_map_f32_sw128(reinterpret_cast<CUtensorMap*>(m->v), values, rows, 32, dim);
}

cudaError_t launch_attention_decode_tma(const AttnMaps& m, const AttnArgs& a, int batch,
                                        cudaStream_t st) {
  const size_t smem = attn_tma_smem(a.dim, a.cap);
  if (smem > kAttnMaxSmem || batch <= 0 || a.heads <= 0) return cudaErrorInvalidValue;
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(attn_decode_tma_kernel<false>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kAttnMaxSmem));
    cudaFuncSetAttribute(attn_decode_tma_kernel<true>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kAttnMaxSmem));
  });
  const CUtensorMap* km = reinterpret_cast<const CUtensorMap*>(m.k);
  const CUtensorMap* vm = reinterpret_cast<const CUtensorMap*>(m.v);
  if (a.dim == 128)
    attn_decode_tma_kernel<true><<<dim3(a.heads, batch), 64, smem, st>>>(*km, *vm, a);
  else
    attn_decode_tma_kernel<false><<<dim3(a.heads, batch), 64, smem, st>>>(*km, *vm, a);
  return cudaGetLastError();
}

// ---- single-query attention, split over tokens (few sequences) -------------------
// With one CTA per (head, sequence) a small batch leaves most SMs idle and
// each CTA is bound by its own latency (one sequential stream of its head's
// keys and values).  This form splits the work without changing a single
// rounding:
//  * scores kernel, grid (chunks of 128 tokens, heads, batch): thread = token,
//    the left-to-right dot from -0.0 over the head dimension, times the
//    scale, into scratch [batch][heads][cap];
//  * values kernel, grid (head_dim / 32 column slices, heads, batch), launched
//    as a programmatic dependent of the scores kernel: its producer warp
//    starts streaming the slice's value sub-blocks (32 tokens x 32 floats,
//    4 KB contiguous in the tiled cache) through a bulk-copy ring at once;
//    three warps wait for the scores, take the max, the exps, the
//    left-to-right sum (one thread) and the divisions; then lane c of warp 0
//    runs column c's left-to-right sum over the tokens from +0.0 out of the
//    ring.
constexpr int kSplitChunk = 128;
constexpr int kSplitStages = 16;
constexpr int kSplitThreads = 128;  // warps 0-2 softmax (warp 0 the sums), warp 3 producer
constexpr int kSplitSubBytes = 32 * 32 * 4;

__device__ __forceinline__ int split_tokens(const AttnArgs& a, int b, bool* ok) {
  *ok = true;
  if (!a.state) return a.tokens;
  const int prefix = a.state[2 * b], gen = a.state[2 * b + 1];
  if (prefix <= 0) {
    *ok = false;
    return 0;
  }
  return prefix + (gen < a.window ? gen : a.window);
}

__global__ void __launch_bounds__(kSplitChunk) attn_split_scores_kernel(const AttnArgs a) {
  __shared__ __align__(16) float qs[256];
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  pdl_launch_dependents();  // the values kernel waits for this grid before reading scores
  if (threadIdx.x == 0 && a.tiled) {
    // this chunk's keys (contiguous in the tiled layout) into L2 while the
    // push finishes (prefetch_l2_bulk: safe before the wait)
    const int t0 = c * kSplitChunk, t1 = min(t0 + kSplitChunk, static_cast<int>(a.cap));
    if (t1 > t0)
      prefetch_l2_bulk(a.keys + b * a.seq_stride + h * a.head_stride + static_cast<long long>(t0) * a.dim,
                       static_cast<uint32_t>(t1 - t0) * a.dim * 4);
  }
  pdl_wait_prior_grids();   // launched as a programmatic dependent itself (launch_dependent)
  bool ok;
  const int T = split_tokens(a, b, &ok);
  if (!ok) {
    if (c == 0 && threadIdx.x == 0) flag(a.status, DEV_CACHE);
    return;
  }
  const int t0 = c * kSplitChunk;
  if (t0 >= T) return;
  const int dim = a.dim, nb = dim >> 5;
  for (int d = threadIdx.x; d < dim; d += kSplitChunk)
    qs[d] = a.q[b * a.ld_q + static_cast<long long>(h) * dim + d];
  __syncthreads();
  const int t = t0 + threadIdx.x;
  if (t >= T) return;
  const float* kh = a.keys + b * a.seq_stride + h * a.head_stride;
  const float4* q4 = reinterpret_cast<const float4*>(qs);
  float acc = -0.0f;
  // four 32-float pieces of the key row per round, all loads issued before
  // the chain of adds that consumes them
  for (int j0 = 0; j0 < nb; j0 += 4) {
    float4 kr[32];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = j0 + jj;
      if (j < nb) {
        const float* row = a.tiled
                               ? kh + ((static_cast<long long>(t >> 5) * nb + j) * 32 + (t & 31)) * 32
                               : kh + t * a.row_stride + 32 * j;
        const float4* k4 = reinterpret_cast<const float4*>(row);
#pragma unroll
        for (int i = 0; i < 8; ++i) kr[jj * 8 + i] = __ldg(k4 + i);
      }
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      if (j0 + jj < nb) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 kv = kr[jj * 8 + i];
          const float4 qv = q4[(j0 + jj) * 8 + i];
          acc = __fadd_rn(acc, __fmul_rn(qv.x, kv.x));
          acc = __fadd_rn(acc, __fmul_rn(qv.y, kv.y));
          acc = __fadd_rn(acc, __fmul_rn(qv.z, kv.z));
          acc = __fadd_rn(acc, __fmul_rn(qv.w, kv.w));
        }
      }
    }
  }
  a.scores[(static_cast<long long>(b) * a.heads + h) * a.cap + t] = __fmul_rn(acc, a.scale);
}

__device__ __forceinline__ void softmax_bar() {  // warps 0-2 only
  asm volatile("bar.sync 1, 96;" ::: "memory");
}

__global__ void __launch_bounds__(kSplitThreads) attn_split_values_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) unsigned char split_raw[];
  float* ring = reinterpret_cast<float*>(split_raw);  // kSplitStages x 32 x 32
  float* sc = ring + kSplitStages * 1024;              // cap floats
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(sc + a.cap) + 15) & ~static_cast<uintptr_t>(15));
  uint64_t* empty = full + kSplitStages;
  __shared__ float red[3];
  __shared__ int red_bad[3];
  __shared__ float s_max, s_sum;
  __shared__ int s_bad;
  const int j = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = a.dim >> 5;
  const float* vh = a.values + b * a.seq_stride + h * a.head_stride;
  // This kernel may start while the cache push two launches back is still
  // running (the scores kernel between them lets it launch before waiting for
  // the push itself), so nothing of the cache is read before the wait.  Before
  // it, the slice's value sub-blocks only go into L2 (prefetch_l2_bulk), sized
  // by a state read that may predate the push (L2-only load, not reused).
  if (warp == 3 && lane == 0 && a.state && a.cap >= 32) {
    const int prefix = __ldcg(a.state + 2 * b), gen = __ldcg(a.state + 2 * b + 1);
    const int t_est = prefix + (gen < a.window ? gen : a.window) + 1;
    const int n0 = prefix > 0 ? min((t_est + 31) >> 5, static_cast<int>(a.cap >> 5)) : 0;
    for (int it = 0; it < n0; ++it)
      prefetch_l2_bulk(vh + (static_cast<long long>(it) * nb + j) * 1024, kSplitSubBytes);
  }
  // the scores grid has completed, and with it the push it waited for
  pdl_wait_prior_grids();
  bool ok;
  const int T = split_tokens(a, b, &ok);
  if (!ok) return;  // flagged by the scores kernel
  const int ntiles = (T + 31) >> 5;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSplitStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 3) {
    // ---- producer: the slice's sub-blocks in token order
    if (lane == 0) {
      int it = 0;
      for (; it < ntiles; ++it) {
        const int st = it % kSplitStages;
        if (it >= kSplitStages &&
            !mbar_wait(&empty[st], ((it / kSplitStages) - 1) & 1, a.status))
          break;
        mbar_arrive_expect_tx(&full[st], kSplitSubBytes);
        bulk_g2s(ring + st * 1024, vh + (static_cast<long long>(it) * nb + j) * 1024,
                 kSplitSubBytes, &full[st]);
      }
      for (int i = it - kSplitStages; i < it; ++i)  // every issued copy lands before exit
        if (i >= 0) mbar_wait(&full[i % kSplitStages], (i / kSplitStages) & 1, a.status);
    }
    return;
  }
  // ---- softmax_backend (src/cpu/ops.rs:139-187) over the scores
  // the scores row (16-byte aligned: cap is a multiple of 32), four 16-byte
  // loads in flight per thread
  const float4* src4 =
      reinterpret_cast<const float4*>(a.scores + (static_cast<long long>(b) * a.heads + h) * a.cap);
  float4* sc4 = reinterpret_cast<float4*>(sc);
  const int n4 = (T + 3) >> 2;
  float mx = -INFINITY;
  int bad = 0;
  for (int g0 = threadIdx.x; g0 < n4; g0 += 4 * 96) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (g0 + u * 96 < n4) v[u] = __ldcg(src4 + g0 + u * 96);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int g = g0 + u * 96;
      if (g < n4) {
        sc4[g] = v[u];
        const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (4 * g + c < T) {
            bad |= isnan(e[c]) || e[c] == INFINITY;
            mx = fmaxf(mx, e[c]);
          }
      }
    }
  }
  mx = warp_max(mx);
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    red[warp] = mx;
    red_bad[warp] = bad;
  }
  softmax_bar();
  if (threadIdx.x == 0) {
    const float m = fmaxf(fmaxf(red[0], red[1]), red[2]);
    s_max = m;
    s_bad = red_bad[0] | red_bad[1] | red_bad[2] | !isfinite(m);
  }
  softmax_bar();
  bad = s_bad;
  if (!bad) {
    mx = s_max;
#pragma unroll 4
    for (int t = threadIdx.x; t < T; t += 96) sc[t] = exp_f32_via_f64(__fsub_rn(sc[t], mx));
    softmax_bar();
    if (threadIdx.x == 0) s_sum = serial_sum_smem(sc, T);
    softmax_bar();
    const float sum = s_sum;
#pragma unroll 4
    for (int t = threadIdx.x; t < T; t += 96) sc[t] = __fdiv_rn(sc[t], sum);
    softmax_bar();
  } else if (threadIdx.x == 0 && j == 0) {
    flag(a.status, DEV_SOFTMAX);
  }
  if (warp != 0) return;
  // ---- column sums: lane = column 32 j + lane, tokens in order from +0.0;
  // every tile is consumed (and its slot released) even after an error, so
  // that the producer never waits for a slot that is not coming
  float acc = 0.0f;
  for (int i = 0; i < ntiles; ++i) {
    const int st = i % kSplitStages;
    mbar_wait(&full[st], (i / kSplitStages) & 1, a.status);
    if (!bad) {
      const float* tile = ring + st * 1024 + lane;
      const float* p = sc + i * 32;
      const int rows = T - i * 32 < 32 ? T - i * 32 : 32;
      if (rows == 32) {
#pragma unroll
        for (int r = 0; r < 32; ++r) acc = __fadd_rn(acc, __fmul_rn(p[r], tile[r * 32]));
      } else {
        for (int r = 0; r < rows; ++r) acc = __fadd_rn(acc, __fmul_rn(p[r], tile[r * 32]));
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (!bad) a.out[b * a.ld_out + static_cast<long long>(h) * a.dim + 32 * j + lane] = acc;
}

static size_t split_smem(long long cap) {
  return static_cast<size_t>(kSplitStages) * kSplitSubBytes +
         ((static_cast<size_t>(cap) * 4 + 15) & ~static_cast<size_t>(15)) +
         2 * kSplitStages * sizeof(uint64_t) + 16;
}

bool attention_split_ok(const AttnArgs& a) {
  return a.tiled && !a.causal && a.scores && a.dim % 32 == 0 && a.dim <= 256 &&
         split_smem(a.cap) <= kAttnMaxSmem;
}

cudaError_t launch_attention_split(const AttnArgs& a, int batch, int max_tokens, cudaStream_t st) {
  if (!attention_split_ok(a) || batch <= 0 || a.heads <= 0 || max_tokens <= 0 || batch > 65535 ||
      a.heads > 65535)
    return cudaErrorInvalidValue;
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(attn_split_values_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kAttnMaxSmem));
  });
  const int chunks = (max_tokens + kSplitChunk - 1) / kSplitChunk;
  cudaError_t e = launch_dependent(attn_split_scores_kernel, dim3(chunks, a.heads, batch),
                                   dim3(kSplitChunk), 0, st, a);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.dim / 32, a.heads, batch);
  cfg.blockDim = dim3(kSplitThreads);
  cfg.dynamicSmemBytes = split_smem(a.cap);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, attn_split_values_kernel, a);
  if (e != cudaSuccess) {  // without the early start
    cudaGetLastError();
    cfg.numAttrs = 0;
    e = cudaLaunchKernelEx(&cfg, attn_split_values_kernel, a);
  }
  return e;
}

// ---- causal attention of a prefill, 16 query rows per CTA (head_dim 128) ---------
// ops::attention with its mask (src/cpu/ops.rs:263-360) over the tiled cache:
// CTA = (head, 16 consecutive query rows), so that each 32-token key or value
// tile crosses from L2 once per 16 rows instead of once per row.  A producer
// warp streams the head's key tiles, then its value tiles (tokens 0 .. the
// block's last row), through a four-slot TMA ring; warp q owns query row
// i = i0 + q:
//  * scores: lane = token of the tile, the left-to-right dot from -0.0 over
//    the head dimension (products in pairs, each rounded on its own, added
//    one by one), times the scale, for tokens 0..i only;
//  * softmax over tokens 0..i: max, exps, lane 0's left-to-right sum, the
//    divisions;
//  * values: lane = four output columns, tokens 0..i in order from -0.0.
// The same operations in the same order as the one-query-per-CTA causal form,
// so the same bits.
constexpr int kPfRows = 16;
constexpr int kPfStages = 4;
constexpr int kPfThreads = (kPfRows + 1) * 32;
constexpr int kPfTileBytes = 4 * kTmaBoxBytes;  // 32 tokens x 128 floats

__host__ __device__ inline size_t attn_prefill_smem(long long tokens) {
  const size_t tpad = static_cast<size_t>((tokens + 3) & ~3LL);
  return 1024 + kPfStages * kPfTileBytes + kPfRows * 128 * 4 + kPfRows * tpad * 4 +
         2 * kPfStages * 8 + 16;
}

__global__ void __launch_bounds__(kPfThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const AttnArgs a) {
  extern __shared__ __align__(1024) unsigned char pf_raw[];
  // offset from the shared array itself (not through an integer cast), so
  // that every pointer below stays a shared-memory pointer to the compiler
  unsigned char* ring = pf_raw + ((1024u - (smem_addr(pf_raw) & 1023u)) & 1023u);
  const int T = a.tokens, tpad = (T + 3) & ~3;
  float* qs = reinterpret_cast<float*>(ring + kPfStages * kPfTileBytes);  // [16][128]
  float* sc_all = qs + kPfRows * 128;                                      // [16][tpad]
  uint64_t* full = reinterpret_cast<uint64_t*>(sc_all + kPfRows * tpad);
  uint64_t* empty = full + kPfStages;
  const int h = blockIdx.y;
  const int i0 = static_cast<int>(gridDim.x - 1 - blockIdx.x) * kPfRows;  // longest first
  const int last = min(i0 + kPfRows, T);  // rows [i0, last)
  const int ntk = (last + 31) >> 5;       // key tiles 0 .. ntk-1 cover tokens 0 .. last-1
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPfStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kPfRows);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kPfRows) {
    // ---- producer: key tiles, then value tiles
    if (lane == 0) {
      const long long y0 = (static_cast<long long>(a.seq) * a.heads + h) * a.cap * 4;
      int it = 0;
      for (; it < 2 * ntk; ++it) {
        const int st = it % kPfStages;
        if (it >= kPfStages && !mbar_wait(&empty[st], ((it / kPfStages) - 1) & 1, a.status)) break;
        const bool keys = it < ntk;
        const int tile = keys ? it : it - ntk;
        mbar_arrive_expect_tx(&full[st], kPfTileBytes);
        tma_load_2d(ring + st * kPfTileBytes, keys ? &kmap : &vmap, 0,
                    static_cast<int>(y0 + static_cast<long long>(tile) * 32 * 4), &full[st]);
      }
      for (int j = it - kPfStages; j < it; ++j)  // every issued copy lands before exit
        if (j >= 0) mbar_wait(&full[j % kPfStages], (j / kPfStages) & 1, a.status);
    }
    return;
  }
  const int i = i0 + warp;
  const bool valid = i < T;
  float* qrow = qs + warp * 128;
  float* sc = sc_all + warp * tpad;
  {
    const float4 v = valid ? *reinterpret_cast<const float4*>(a.q + static_cast<long long>(i) * a.ld_q +
                                                              static_cast<long long>(h) * 128 + 4 * lane)
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    reinterpret_cast<float4*>(qrow)[lane] = v;
  }
  __syncwarp();
  const float4* q4 = reinterpret_cast<const float4*>(qrow);
  // ---- scores
  for (int j = 0; j < ntk; ++j) {
    const int st = j % kPfStages;
    mbar_wait(&full[st], (j / kPfStages) & 1, a.status);
    const int t = 32 * j + lane;
    if (valid && t <= i) {
      const unsigned char* row = ring + st * kPfTileBytes + lane * 128;
      float acc = -0.0f;
#pragma unroll
      for (int b = 0; b < 4; ++b)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 kv =
              *reinterpret_cast<const float4*>(row + b * kTmaBoxBytes + ((c ^ (lane & 7)) << 4));
          const float4 qv = q4[b * 8 + c];
          const float2 p0 = f2_mul(make_float2(qv.x, qv.y), make_float2(kv.x, kv.y));
          const float2 p1 = f2_mul(make_float2(qv.z, qv.w), make_float2(kv.z, kv.w));
          acc = __fadd_rn(acc, p0.x);
          acc = __fadd_rn(acc, p0.y);
          acc = __fadd_rn(acc, p1.x);
          acc = __fadd_rn(acc, p1.y);
        }
      sc[t] = __fmul_rn(acc, a.scale);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  // ---- softmax_backend (src/cpu/ops.rs:139-187) over tokens 0..i
  const int L = i + 1;
  bool bad = false;
  if (valid) {
    float mx = -INFINITY;
    int b = 0;
    for (int t = lane; t < L; t += 32) {
      const float v = sc[t];
      b |= isnan(v) || v == INFINITY;
      mx = fmaxf(mx, v);
    }
    mx = warp_max(mx);
    bad = __any_sync(0xffffffffu, b) || !isfinite(mx);
    if (!bad) {
      for (int t = lane; t < L; t += 32) sc[t] = exp_f32_via_f64(__fsub_rn(sc[t], mx));
      __syncwarp();
      float sum = -0.0f;
      if (lane == 0) sum = serial_sum_smem(sc, L);
      sum = __shfl_sync(0xffffffffu, sum, 0);
      for (int t = lane; t < L; t += 32) sc[t] = __fdiv_rn(sc[t], sum);
      __syncwarp();
    } else if (lane == 0) {
      flag(a.status, DEV_SOFTMAX);
    }
  }
  // ---- values: lane owns columns 4 lane .. 4 lane + 3 (box lane / 8)
  float4 acc = make_float4(-0.0f, -0.0f, -0.0f, -0.0f);
  for (int j = 0; j < ntk; ++j) {
    const int it = ntk + j, st = it % kPfStages;
    mbar_wait(&full[st], (it / kPfStages) & 1, a.status);
    const int rows = valid && !bad ? min(32, L - 32 * j) : 0;
    if (rows > 0) {
      const unsigned char* tile = ring + st * kPfTileBytes + (lane >> 3) * kTmaBoxBytes;
      const float* p = sc + 32 * j;
#pragma unroll 8
      for (int r = 0; r < rows; ++r) {
        const float4 v = *reinterpret_cast<const float4*>(tile + r * 128 + (((lane & 7) ^ (r & 7)) << 4));
        const float pr = p[r];
        acc.x = __fadd_rn(acc.x, __fmul_rn(pr, v.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(pr, v.y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(pr, v.z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(pr, v.w));
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (valid && !bad)
    *reinterpret_cast<float4*>(a.out + static_cast<long long>(i) * a.ld_out +
                               static_cast<long long>(h) * 128 + 4 * lane) = acc;
}

bool attention_prefill_ok(const AttnArgs& a) {
  return a.tiled && a.dim == 128 && a.causal && a.tokens > 0 &&
         attn_prefill_smem(a.tokens) <= 227 * 1024 && a.ld_q % 4 == 0 && a.ld_out % 4 == 0 &&
         reinterpret_cast<uintptr_t>(a.q) % 16 == 0 && reinterpret_cast<uintptr_t>(a.out) % 16 == 0;
}

cudaError_t launch_attention_prefill(const AttnMaps& m, const AttnArgs& a, cudaStream_t st) {
  if (!attention_prefill_ok(a) || a.heads <= 0 || a.heads > 65535) return cudaErrorInvalidValue;
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         227 * 1024);
  });
  const int blocks = (a.tokens + kPfRows - 1) / kPfRows;
  attn_prefill_kernel<<<dim3(blocks, a.heads), kPfThreads, attn_prefill_smem(a.tokens), st>>>(
      *reinterpret_cast<const CUtensorMap*>(m.k), *reinterpret_cast<const CUtensorMap*>(m.v), a);
  return cudaGetLastError();
}

}  // namespace uocr
