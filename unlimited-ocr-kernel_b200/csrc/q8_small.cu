// q8_small.cu — grouped projections for groups of at most 16 rows.
//
// A MoE layer at decode batch sizes gives each expert a handful of rows
// (config 4: 64 tokens x top-6 over 64 experts, about 6 rows per expert).
// For such groups the work is streaming the expert's weights once; the
// tcgen05 GEMMs pay a fixed cost per MMA instruction whatever N is (75-210
// cycles for M = 128, K = 16 measured, N <= 256), issued by one thread, so a
// 16-row tile costs them as much as a 256-row one.  Here every warp issues
// its own warp-level MMAs over the group's rows, so the instruction cost is
// spread over the SM and the weights stream at memory speed.
//
// Layout: a CTA of 4 warps owns 128 weight rows of one group's matrix; a warp
// owns 32 of them as four n8 tiles; the group's rows (<= 16, the MMA's M) are
// the A operand.  Within each 32-wide q8 block K is permuted consistently for
// A and B (a product over K does not depend on the order) so that lane
// (g = lane / 4, q = lane % 4) needs only bytes [8q, 8q + 8) of its rows:
//   bf16 m16n8k16, step j in {0, 1}: logical k in {2q, 2q+1} <- physical
//     8q + 4j + {0, 1}; {2q+8, 2q+9} <- 8q + 4j + {2, 3};
//   s8 m16n8k32 (one step): logical 4q + i <- physical 8q + i, 4q + 16 + i <-
//     8q + 4 + i.
//
// FP32 activations (Int8Matrix::linear, FP32 tolerance): the rows come as the
// exact three-way bf16 split of the row scaled by 2^e (launch_split_rows); a
// block's sum over the three pieces accumulates in the MMA's fp32 registers,
// then acc = fma(sum, ws, acc), and the row's total is multiplied by 2^-e.
// int8 activations (linear_dynamic_int8, bit-exact): the s8 MMA gives the
// exact int32 block sum S; then acc = acc + ((float)S * ws) * xs block by
// block from -0.0, one IEEE rounding per operation, as the reference.
#include "common.cuh"
#include "kernels.h"

namespace uocr {

namespace {

constexpr int kSmallWarps = 4;
constexpr int kSmallCtaRows = 32 * kSmallWarps;  // weight rows per CTA

struct SmallArgs {
  const FfnView* ffns;  // grouped: device [groups]; nullptr: `single`
  Q8View single;
  int proj;  // 0 gate, 1 up, 2 down
  const int* counts;
  const int* offsets;
  int groups;
  int lo, hi;  // groups with lo <= count <= hi
  int N, K;
  const uint16_t* pieces;  // FP32 mode: [3][piece_rows][K] bf16
  long long piece_elems;
  const float* rinv;
  const int8_t* xq;  // int8 mode: [rows][K], scales [rows][K / 32]
  const float* xs;
  float* y;
  long long ldy;
};

__device__ __forceinline__ void mma_bf16_m16n8k16(float (&d)[4], uint32_t a0, uint32_t a1,
                                                  uint32_t a2, uint32_t a3, uint32_t b0,
                                                  uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8_m16n8k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four int8 (one word) -> four bf16 (two words), exact (see q8_tc.cu).
__device__ __forceinline__ uint2 i8x4_bf16(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;
  const float magic = 8388736.0f;  // 2^23 + 128
  const float f0 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)), magic);
  const float f1 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)), magic);
  const float f2 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)), magic);
  const float f3 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)), magic);
  return make_uint2(__byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632),
                    __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632));
}

__device__ __forceinline__ const Q8View& small_matrix(const SmallArgs& a, int g) {
  if (!a.ffns) return a.single;
  const FfnView& f = a.ffns[g];
  return a.proj == 0 ? f.gate : a.proj == 1 ? f.up : f.down;
}

template <bool INT8>
__global__ void __launch_bounds__(32 * kSmallWarps) small_rows_kernel(const __grid_constant__ SmallArgs a) {
  const int g = blockIdx.y;
  const int count = a.counts ? a.counts[g] : a.hi;
  if (count < a.lo || count > a.hi || count < 1) return;
  const int off = a.counts ? a.offsets[g] : 0;
  const Q8View m = small_matrix(a, g);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, q = lane & 3;
  const int n0 = blockIdx.x * kSmallCtaRows + 32 * warp;
  if (n0 >= a.N) return;
  const int K = a.K, nb = K >> 5;
  // this lane's weight rows (B columns) for the four n8 tiles, clamped for loads
  const int8_t* wrow[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int r = n0 + 8 * t + gq;
    wrow[t] = m.w + static_cast<long long>(r < a.N ? r : a.N - 1) * K + 8 * q;
  }
  // this lane's scale rows: output columns 2q, 2q + 1 of each tile (offsets
  // from m.s; tile t adds 8 * t rows)
  const int sr0 = n0 + 2 * q;
  // this lane's activation rows (A rows gq and gq + 8), clamped into the group
  const int i0 = gq < count ? gq : 0, i1 = gq + 8 < count ? gq + 8 : 0;
  const long long row0 = off + i0, row1 = off + i1;

  float acc[4][4];
#pragma unroll
  for (int t = 0; t < 4; ++t)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[t][c] = INT8 ? -0.0f : 0.0f;

  for (int b = 0; b < nb; ++b) {
    // the block's weight scales (rows past N clamp to the last row; their
    // outputs are not stored)
    float wsv[4][2];
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = sr0 + 8 * t + h;
        wsv[t][h] = __ldg(m.s + static_cast<long long>(r < a.N ? r : a.N - 1) * nb + b);
      }
    uint2 wv[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) wv[t] = __ldg(reinterpret_cast<const uint2*>(wrow[t] + 32 * b));
    if (INT8) {
      const uint2 x0 = __ldg(reinterpret_cast<const uint2*>(a.xq + row0 * K + 32 * b + 8 * q));
      const uint2 x1 = __ldg(reinterpret_cast<const uint2*>(a.xq + row1 * K + 32 * b + 8 * q));
      const float xs0 = __ldg(a.xs + row0 * nb + b), xs1 = __ldg(a.xs + row1 * nb + b);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        int d[4] = {0, 0, 0, 0};
        mma_s8_m16n8k32(d, x0.x, x1.x, x0.y, x1.y, wv[t].x, wv[t].y);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float wsb = wsv[t][h];
          // ((float)S * ws) * xs, then the running sum: |S| < 2^24, so the
          // conversion is exact; every operation rounded on its own
          acc[t][h] = __fadd_rn(acc[t][h], __fmul_rn(__fmul_rn(static_cast<float>(d[h]), wsb), xs0));
          acc[t][2 + h] =
              __fadd_rn(acc[t][2 + h], __fmul_rn(__fmul_rn(static_cast<float>(d[2 + h]), wsb), xs1));
        }
      }
    } else {
      float d[4][4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int c = 0; c < 4; ++c) d[t][c] = 0.0f;
      uint2 bw[4][2];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        bw[t][0] = i8x4_bf16(wv[t].x);  // step 0: physical 8q + 0..3
        bw[t][1] = i8x4_bf16(wv[t].y);  // step 1: physical 8q + 4..7
      }
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        const uint16_t* base = a.pieces + p * a.piece_elems + 32 * b + 8 * q;
        const uint4 r0 = __ldg(reinterpret_cast<const uint4*>(base + row0 * K));
        const uint4 r1 = __ldg(reinterpret_cast<const uint4*>(base + row1 * K));
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          mma_bf16_m16n8k16(d[t], r0.x, r1.x, r0.y, r1.y, bw[t][0].x, bw[t][0].y);
          mma_bf16_m16n8k16(d[t], r0.z, r1.z, r0.w, r1.w, bw[t][1].x, bw[t][1].y);
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          acc[t][h] = fmaf(d[t][h], wsv[t][h], acc[t][h]);
          acc[t][2 + h] = fmaf(d[t][2 + h], wsv[t][h], acc[t][2 + h]);
        }
    }
  }
  // C layout: c0, c1 -> row gq, columns 2q, 2q + 1; c2, c3 -> row gq + 8
  const float sc0 = INT8 ? 1.0f : __ldg(a.rinv + off + i0);
  const float sc1 = INT8 ? 1.0f : __ldg(a.rinv + off + i1);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int col = n0 + 8 * t + 2 * q;
    if (col >= a.N) continue;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int i = gq + 8 * hr;
      if (i >= count) continue;
      float v0 = acc[t][2 * hr], v1 = acc[t][2 * hr + 1];
      if (!INT8) {
        const float sc = hr ? sc1 : sc0;
        v0 = __fmul_rn(v0, sc);
        v1 = __fmul_rn(v1, sc);
      }
      float* yr = a.y + (off + i) * a.ldy + col;
      yr[0] = v0;
      if (col + 1 < a.N) yr[1] = v1;
    }
  }
}

}  // namespace

bool small_rows_supported(int N, int K) { return N > 0 && N % 8 == 0 && K > 0 && K % 128 == 0; }

cudaError_t launch_small_rows(bool int8, const FfnView* ffns, const Q8View* single, int proj,
                              const int* counts, const int* offsets, int groups, int lo, int hi,
                              int N, int K, const uint16_t* pieces, long long piece_rows,
                              const float* rinv, const int8_t* xq, const float* xs, float* y,
                              long long ldy, cudaStream_t st) {
  if (!small_rows_supported(N, K) || hi > kSmallRowsMax || groups < 1) return cudaErrorInvalidValue;
  SmallArgs a{};
  a.ffns = ffns;
  if (single) a.single = *single;
  a.proj = proj;
  a.counts = counts;
  a.offsets = offsets;
  a.groups = groups;
  a.lo = lo;
  a.hi = hi;
  a.N = N;
  a.K = K;
  a.pieces = pieces;
  a.piece_elems = piece_rows * K;
  a.rinv = rinv;
  a.xq = xq;
  a.xs = xs;
  a.y = y;
  a.ldy = ldy;
  const dim3 grid((N + kSmallCtaRows - 1) / kSmallCtaRows, groups);
  if (int8)
    small_rows_kernel<true><<<grid, 32 * kSmallWarps, 0, st>>>(a);
  else
    small_rows_kernel<false><<<grid, 32 * kSmallWarps, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace uocr
