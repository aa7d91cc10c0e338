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
// A CTA owns 128 weight rows of one group's matrix.  Its producer lane moves
// each 128-wide slice of K into a ring of shared-memory stages with TMA: the
// weights' int8 tile [128][128] (128-byte swizzle), their block scales
// [128][4], and the group's 16 activation rows (the three bf16 pieces
// [16][128] each, or int8 rows [16][128] and their scales [16][4]); rows past
// the group read as other rows or as zeros and are never stored.  Four warps
// compute: a warp owns 32 weight rows as four n8 tiles (eight warps of two
// tiles measured slower: the activation fragments, shared by every warp, are
// read from shared memory once per warp); the group's rows (the MMA's M) are
// the A operand.  Within each 32-wide q8 block K is permuted
// consistently for A and B (a product over K does not depend on the order) so
// that lane (g = lane / 4, q = lane % 4) needs only elements [8q, 8q + 8) of
// the block in its rows:
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
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_maps.cuh"

namespace uocr {

namespace {

constexpr int kSmWarps = 4;                         // consumer warps
constexpr int kSmTiles = 4;                         // n8 tiles of weight rows per warp
constexpr int kSmThreads = 32 * (kSmWarps + 1);     // + the producer warp
constexpr int kSmRows = 8 * kSmTiles * kSmWarps;    // weight rows per CTA (128)
constexpr int kSmK = 128;                           // K per stage (4 q8 blocks)
// Ring depth: three stages, so that two FP32 CTAs (or three int8 CTAs) share
// an SM and one computes while the other waits for its tiles.
constexpr int kSmStagesF = 3;
constexpr int kSmStagesI = 3;
constexpr int kSmW = kSmRows * kSmK;                // 16 KB int8 weights
constexpr int kSmWs = kSmRows * 4 * 4;              // 2 KB weight scales
constexpr int kSmXp = 16 * kSmK * 2;                // 4 KB per bf16 piece tile
constexpr int kSmXq = 16 * kSmK;                    // 2 KB int8 rows
constexpr int kSmXs = 16 * 4 * 4;                   // 256 B activation scales
constexpr int kSmStageF = kSmW + kSmWs + 3 * kSmXp;          // 30 KB
constexpr int kSmStageI = 21 * 1024;                         // 16 + 2 + 2 + 0.25 KB, padded
constexpr int kSmSmemF = kSmStagesF * kSmStageF + 1024 + 256;
constexpr int kSmSmemI = kSmStagesI * kSmStageI + 1024 + 256;
static_assert(kSmStageF % 1024 == 0 && kSmStageI % 1024 == 0, "swizzled tiles: 1024-byte stages");
static_assert(kSmW + kSmWs + kSmXq + kSmXs <= kSmStageI, "int8 stage layout");

struct SmallArgs {
  const TcMatrixMaps* maps;  // grouped: device [groups]; nullptr: the single maps
  const int* counts;         // grouped: rows per group; nullptr: total_rows in groups of 16
  const int* offsets;
  int groups, lo, hi, total_rows;
  int chunks;                // grouped: 16-row chunks per group (grid.y = groups * chunks)
  int N, K, piece_rows;
  const float* rinv;
  float* y;
  long long ldy;
  unsigned* status;
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

// Four int8 (one word) -> four bf16 (two words), exact: each byte, offset to
// u = v + 128, is placed under the exponent of 2^23; subtracting 2^23 + 128
// leaves v, whose bf16 is the float's high half.
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

template <bool INT8>
__global__ void __launch_bounds__(kSmThreads, 2)
    small_rows_kernel(const __grid_constant__ CUtensorMap tw,   // single: weights
                      const __grid_constant__ CUtensorMap tws,  // single: weight scales
                      const __grid_constant__ CUtensorMap tx,   // pieces, or int8 rows
                      const __grid_constant__ CUtensorMap txs,  // int8 row scales
                      const SmallArgs a) {
  constexpr int kStage = INT8 ? kSmStageI : kSmStageF;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int kSmStages = INT8 ? kSmStagesI : kSmStagesF;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSmStages * kStage);
  uint64_t* empty = full + kSmStages;

  int g = blockIdx.y;
  int count, off;
  if (a.counts) {
    // group g's rows [16c, 16c + 16) of chunk c; the group qualifies by its
    // whole row count
    const int c = g % a.chunks;
    g /= a.chunks;
    const int total = a.counts[g];
    if (total < a.lo || total > a.hi) return;
    off = a.offsets[g] + 16 * c;
    count = total - 16 * c < 16 ? total - 16 * c : 16;
  } else {
    off = 16 * g;
    count = a.total_rows - off < 16 ? a.total_rows - off : 16;
  }
  if (count < 1) return;
  const int n0 = blockIdx.x * kSmRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kstages = a.K / kSmK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSmWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ---- producer
    if (lane == 0) {
      const CUtensorMap* wmap = a.maps ? &a.maps[g].w_sw128 : &tw;
      const CUtensorMap* smap = a.maps ? &a.maps[g].ws : &tws;
      const uint32_t tx_bytes = INT8 ? kSmW + kSmWs + kSmXq + kSmXs : kSmW + kSmWs + 3 * kSmXp;
      for (int ks = 0; ks < kstages; ++ks) {
        const int s = ks % kSmStages;
        if (ks >= kSmStages && !mbar_wait_spin(&empty[s], ((ks / kSmStages) - 1) & 1, a.status))
          break;
        unsigned char* st = smem + s * kStage;
        mbar_arrive_expect_tx(&full[s], tx_bytes);
        tma_load_2d(st, wmap, ks * kSmK, n0, &full[s]);
        tma_load_2d(st + kSmW, smap, ks * 4, n0, &full[s]);
        if (INT8) {
          tma_load_2d(st + kSmW + kSmWs, &tx, ks * kSmK, off, &full[s]);
          tma_load_2d(st + kSmW + kSmWs + kSmXq, &txs, ks * 4, off, &full[s]);
        } else {
#pragma unroll
          for (int p = 0; p < 3; ++p)
            tma_load_2d(st + kSmW + kSmWs + p * kSmXp, &tx, ks * kSmK, p * a.piece_rows + off,
                        &full[s]);
        }
      }
    }
    return;
  }

  // ---- consumers: warp cw owns weight rows wr0 .. wr0 + 8 kSmTiles - 1 of the tile
  const int cw = warp - 1, gq = lane >> 2, q = lane & 3;
  const int wr0 = 8 * kSmTiles * cw;
  const int i0 = gq, i1 = gq + 8;  // A rows (the group's rows gq, gq + 8)
  float acc[kSmTiles][4];
#pragma unroll
  for (int t = 0; t < kSmTiles; ++t)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[t][c] = INT8 ? -0.0f : 0.0f;
  bool ok = true;
  for (int ks = 0; ks < kstages; ++ks) {
    const int s = ks % kSmStages;
    if (ok) ok = mbar_wait_spin(&full[s], (ks / kSmStages) & 1, a.status);
    const unsigned char* st = smem + s * kStage;
    const float* wsm = reinterpret_cast<const float*>(st + kSmW);  // [128][4]
    // this lane's weight scales for the stage's four blocks: rows wr0 + 8t + 2q + h
    float4 ws4[kSmTiles][2];
#pragma unroll
    for (int t = 0; t < kSmTiles; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        ws4[t][h] = *reinterpret_cast<const float4*>(wsm + 4 * (wr0 + 8 * t + 2 * q + h));
    float4 xs4[2];
    if (INT8) {
      const float* xsm = reinterpret_cast<const float*>(st + kSmW + kSmWs + kSmXq);  // [16][4]
      xs4[0] = *reinterpret_cast<const float4*>(xsm + 4 * i0);
      xs4[1] = *reinterpret_cast<const float4*>(xsm + 4 * i1);
    }
#pragma unroll
    for (int jb = 0; jb < 4; ++jb) {
      // weights: row r = 32 cw + 8 t + gq, bytes [32 jb + 8q, + 8) of the
      // 128-byte row; 16-byte unit (2 jb + q / 2) sits at unit ^ (r % 8)
      uint2 wv[kSmTiles];
#pragma unroll
      for (int t = 0; t < kSmTiles; ++t) {
        const int r = wr0 + 8 * t + gq;
        const int unit = (2 * jb + (q >> 1)) ^ gq;
        wv[t] = *reinterpret_cast<const uint2*>(st + r * 128 + (unit << 4) + ((q & 1) << 3));
      }
      if (INT8) {
        const unsigned char* xq = st + kSmW + kSmWs;  // [16][128]
        const uint2 x0 = *reinterpret_cast<const uint2*>(xq + i0 * 128 + 32 * jb + 8 * q);
        const uint2 x1 = *reinterpret_cast<const uint2*>(xq + i1 * 128 + 32 * jb + 8 * q);
        const float xs0 = jb == 0 ? xs4[0].x : jb == 1 ? xs4[0].y : jb == 2 ? xs4[0].z : xs4[0].w;
        const float xs1 = jb == 0 ? xs4[1].x : jb == 1 ? xs4[1].y : jb == 2 ? xs4[1].z : xs4[1].w;
#pragma unroll
        for (int t = 0; t < kSmTiles; ++t) {
          int d[4] = {0, 0, 0, 0};
          mma_s8_m16n8k32(d, x0.x, x1.x, x0.y, x1.y, wv[t].x, wv[t].y);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float4 w4 = ws4[t][h];
            const float wsb = jb == 0 ? w4.x : jb == 1 ? w4.y : jb == 2 ? w4.z : w4.w;
            // ((float)S * ws) * xs, then the running sum: |S| < 2^24, so the
            // conversion is exact; every operation rounded on its own
            acc[t][h] =
                __fadd_rn(acc[t][h], __fmul_rn(__fmul_rn(static_cast<float>(d[h]), wsb), xs0));
            acc[t][2 + h] = __fadd_rn(acc[t][2 + h],
                                      __fmul_rn(__fmul_rn(static_cast<float>(d[2 + h]), wsb), xs1));
          }
        }
      } else {
        float d[kSmTiles][4];
#pragma unroll
        for (int t = 0; t < kSmTiles; ++t)
#pragma unroll
          for (int c = 0; c < 4; ++c) d[t][c] = 0.0f;
        uint2 bw[kSmTiles][2];
#pragma unroll
        for (int t = 0; t < kSmTiles; ++t) {
          bw[t][0] = i8x4_bf16(wv[t].x);  // step 0: physical 8q + 0..3
          bw[t][1] = i8x4_bf16(wv[t].y);  // step 1: physical 8q + 4..7
        }
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          const unsigned char* xp = st + kSmW + kSmWs + p * kSmXp;  // [16][128] bf16
          const uint4 r0 = *reinterpret_cast<const uint4*>(xp + i0 * 256 + 2 * (32 * jb + 8 * q));
          const uint4 r1 = *reinterpret_cast<const uint4*>(xp + i1 * 256 + 2 * (32 * jb + 8 * q));
#pragma unroll
          for (int t = 0; t < kSmTiles; ++t) {
            mma_bf16_m16n8k16(d[t], r0.x, r1.x, r0.y, r1.y, bw[t][0].x, bw[t][0].y);
            mma_bf16_m16n8k16(d[t], r0.z, r1.z, r0.w, r1.w, bw[t][1].x, bw[t][1].y);
          }
        }
#pragma unroll
        for (int t = 0; t < kSmTiles; ++t)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float4 w4 = ws4[t][h];
            const float wsb = jb == 0 ? w4.x : jb == 1 ? w4.y : jb == 2 ? w4.z : w4.w;
            acc[t][h] = fmaf(d[t][h], wsb, acc[t][h]);
            acc[t][2 + h] = fmaf(d[t][2 + h], wsb, acc[t][2 + h]);
          }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // C layout: c0, c1 -> row gq, columns 2q, 2q + 1; c2, c3 -> row gq + 8
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int i = gq + 8 * hr;
    if (i >= count) continue;
    const float sc = INT8 ? 1.0f : __ldg(a.rinv + off + i);
#pragma unroll
    for (int t = 0; t < kSmTiles; ++t) {
      const int col = n0 + wr0 + 8 * t + 2 * q;
      float v0 = acc[t][2 * hr], v1 = acc[t][2 * hr + 1];
      if (!INT8) {
        v0 = __fmul_rn(v0, sc);
        v1 = __fmul_rn(v1, sc);
      }
      *reinterpret_cast<float2*>(a.y + (off + i) * a.ldy + col) = make_float2(v0, v1);
    }
  }
}

void configure_small() {
  static std::mutex mu;
  static unsigned long long done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && !(done & (1ull << dev))) {
    cudaFuncSetAttribute(small_rows_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmSmemF);
    cudaFuncSetAttribute(small_rows_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmSmemI);
    // all of the unified L1 as shared memory, so that two CTAs fit on an SM
    cudaFuncSetAttribute(small_rows_kernel<false>,
                         cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(small_rows_kernel<true>,
                         cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    done |= 1ull << dev;
  }
}

}  // namespace

bool small_rows_supported(int N, int K) {
  return N > 0 && N % kSmRows == 0 && K > 0 && K % kSmK == 0 && tma_encode_fn() != nullptr;
}

cudaError_t launch_small_rows(bool int8, const void* maps, const Q8View* single, const int* counts,
                              const int* offsets, int groups, int lo, int hi, int total_rows, int N,
                              int K, const uint16_t* pieces, int piece_rows, const float* rinv,
                              const int8_t* xq, const float* xs, int x_rows, float* y,
                              long long ldy, unsigned* status, cudaStream_t st) {
  if (!small_rows_supported(N, K) || hi > kSmallChunkedMax || lo < 1) return cudaErrorInvalidValue;
  if (!maps && !single) return cudaErrorInvalidValue;
  const int chunks = counts ? (hi + 15) / 16 : 1;
  if (!counts) groups = (total_rows + 15) / 16;
  if (groups < 1 || reinterpret_cast<uintptr_t>(y) % 8 || ldy % 2) return cudaErrorInvalidValue;
  CUtensorMap tw{}, tws{}, tx{}, txs{};
  if (single) {
    TcMatrixMaps mm;
    if (!q8_tc_weight_maps(&mm, *single)) return cudaErrorInvalidValue;
    tw = mm.w_sw128;
    tws = mm.ws;
  }
  if (int8) {
    if (!make_map_i8_plain(&tx, xq, x_rows, K, 16) || !make_map_f32(&txs, xs, x_rows, K / 32, 16))
      return cudaErrorInvalidValue;
  } else if (!make_map_pieces_plain(&tx, pieces, piece_rows, K, 16)) {
    return cudaErrorInvalidValue;
  }
  configure_small();
  SmallArgs a{};
  a.maps = static_cast<const TcMatrixMaps*>(maps);
  if (single) a.maps = nullptr;
  a.counts = counts;
  a.offsets = offsets;
  a.groups = groups;
  a.chunks = chunks;
  a.lo = lo;
  a.hi = hi;
  a.total_rows = total_rows;
  a.N = N;
  a.K = K;
  a.piece_rows = piece_rows;
  a.rinv = rinv;
  a.y = y;
  a.ldy = ldy;
  a.status = status;
  const dim3 grid(N / kSmRows, groups * chunks);
  if (int8)
    small_rows_kernel<true><<<grid, kSmThreads, kSmSmemI, st>>>(tw, tws, tx, txs, a);
  else
    small_rows_kernel<false><<<grid, kSmThreads, kSmSmemF, st>>>(tw, tws, tx, txs, a);
  return cudaGetLastError();
}

}  // namespace uocr
