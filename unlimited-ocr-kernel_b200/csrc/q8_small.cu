// q8_small.cu — grouped projections for groups of a few rows (up to 64).
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
// [128][4], and 8 of the group's rows (the three bf16 pieces [8][128] each,
// or int8 rows [8][128] and their scales [8][4]); a group of more than 8
// rows takes one CTA per 8-row chunk (the weight tiles of its other chunks
// mostly come from L2), and rows past the group read as other rows or as
// zeros and are never stored.  Four warps compute: a warp owns 32 weight rows
// as two m16 tiles, the MMA's A operand, and the chunk's rows are the n8 N
// operand.  (With the group's rows as M every MMA covers 16 rows however few
// the group has; at about 6 rows per expert the weights as M halve the MMAs
// and the int8 per-block epilogue, and the 8-row stages fit three CTAs on an
// SM.)
// Within each 32-wide q8 block K is permuted
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
#include "device_once.h"
#include "kernels.h"
#include "tc_maps.cuh"

namespace uocr {

namespace {

constexpr int kSmWarps = 4;                         // consumer warps
constexpr int kSmTiles = 4;                         // n8 tiles of weight rows per warp
constexpr int kSmThreads = 32 * (kSmWarps + 1);     // + the producer warp
constexpr int kSmRows = 8 * kSmTiles * kSmWarps;    // weight rows per CTA (128)
constexpr int kSmK = 128;                           // K per stage (4 q8 blocks)
constexpr int kSmChunk = 8;                         // group rows per CTA (the MMA's N)
// Ring depth: three stages, and three CTAs share an SM (registers <= 136 and
// <= 75 KB of shared memory each), so that one computes while the others wait
// for their tiles.
constexpr int kSmStagesF = 3;
constexpr int kSmStagesI = 3;
constexpr int kSmW = kSmRows * kSmK;                // 16 KB int8 weights
constexpr int kSmWs = kSmRows * 4 * 4;              // 2 KB weight scales
constexpr int kSmXp = kSmChunk * kSmK * 2;          // 2 KB per bf16 piece tile
constexpr int kSmXq = kSmChunk * kSmK;              // 1 KB int8 rows
constexpr int kSmXs = kSmChunk * 4 * 4;             // 128 B activation scales
constexpr int kSmStageF = kSmW + kSmWs + 3 * kSmXp;          // 24 KB
constexpr int kSmStageI = 20 * 1024;                         // 16 + 2 + 1 + 0.125 KB, padded
constexpr int kSmSmemF = kSmStagesF * kSmStageF + 1024 + 256;
constexpr int kSmSmemI = kSmStagesI * kSmStageI + 1024 + 256;
static_assert(kSmStageF % 1024 == 0 && kSmStageI % 1024 == 0, "swizzled tiles: 1024-byte stages");
static_assert(kSmW + kSmWs + kSmXq + kSmXs <= kSmStageI, "int8 stage layout");

struct SmallArgs {
  const TcMatrixMaps* maps;  // grouped: device [groups]; nullptr: the single maps
  const int* counts;         // grouped: rows per group; nullptr: total_rows in chunks of 8
  const int* offsets;
  int groups, lo, hi, total_rows;
  int chunks;                // grouped: 8-row chunks per group (grid.y = chunks * groups)
  const int* items;          // grouped, optional: [0] = n, [1 + i] = chunk << 8 | group
  const TcMatrixMaps* maps2;  // optional second matrix of the same shape (gate and up in one
  float* y2;                  // launch): CTAs x >= tiles compute it into y2
  int tiles;                  // N / kSmRows
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
// u = v + 128, is placed under the exponent of 2^23; adding -(2^23 + 128)
// (two lanes per packed add) leaves v, whose bf16 is the float's high half.
__device__ __forceinline__ uint2 i8x4_bf16(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;
  const float2 magic = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
  const float2 a = f2_add(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)),
                                      __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441))),
                          magic);
  const float2 b = f2_add(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)),
                                      __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443))),
                          magic);
  return make_uint2(__byte_perm(__float_as_uint(a.x), __float_as_uint(a.y), 0x7632),
                    __byte_perm(__float_as_uint(b.x), __float_as_uint(b.y), 0x7632));
}

template <bool INT8>
__global__ void __launch_bounds__(kSmThreads, 3)
    small_rows_kernel(const __grid_constant__ CUtensorMap tw,   // single: weights
                      const __grid_constant__ CUtensorMap tws,  // single: weight scales
                      const __grid_constant__ CUtensorMap tx,   // pieces, or int8 rows
                      const __grid_constant__ CUtensorMap txs,  // int8 row scales
                      const __grid_constant__ CUtensorMap tw2,  // single: second matrix
                      const __grid_constant__ CUtensorMap tws2,
                      const SmallArgs a) {
  pdl_launch_dependents();  // launched as a programmatic dependent (launch_dependent):
  pdl_wait_prior_grids();   // nothing is touched before the previous kernel completes
  constexpr int kStage = INT8 ? kSmStageI : kSmStageF;
  extern __shared__ unsigned char smem_raw[];
  // offset from the shared array itself: derived pointers stay shared-memory
  // pointers to the compiler (an integer-cast alignment makes them generic)
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  constexpr int kSmStages = INT8 ? kSmStagesI : kSmStagesF;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSmStages * kStage);
  uint64_t* empty = full + kSmStages;

  int g = blockIdx.y;
  int count, off;
  if (a.counts) {
    // group g's rows [8c, 8c + 8) of chunk c; the group qualifies by its whole
    // row count.  From the chunk list when there is one; otherwise
    // chunk-major, so that every group's first chunk is dispatched before the
    // (mostly empty) later ones.
    int c;
    if (a.items) {
      if (g >= a.items[0]) return;
      const int packed = a.items[1 + g];
      c = packed >> 8;
      g = packed & 255;
    } else {
      c = g / a.groups;
      g -= c * a.groups;
    }
    const int total = a.counts[g];
    if (total < a.lo || total > a.hi) return;
    off = a.offsets[g] + kSmChunk * c;
    count = total - kSmChunk * c < kSmChunk ? total - kSmChunk * c : kSmChunk;
  } else {
    off = kSmChunk * g;
    count = a.total_rows - off < kSmChunk ? a.total_rows - off : kSmChunk;
  }
  if (count < 1) return;
  const bool second = static_cast<int>(blockIdx.x) >= a.tiles;  // only with y2
  const int n0 = (second ? blockIdx.x - a.tiles : blockIdx.x) * kSmRows;
  float* const y = second ? a.y2 : a.y;
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
      const TcMatrixMaps* gm = second ? a.maps2 : a.maps;
      const CUtensorMap* wmap = gm ? &gm[g].w_sw128 : second ? &tw2 : &tw;
      const CUtensorMap* smap = gm ? &gm[g].ws : second ? &tws2 : &tws;
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

  // ---- consumers: warp cw owns weight rows wr0 .. wr0 + 31 of the tile as two
  // m16 tiles (the MMA's A operand); the chunk's (up to 8) rows are the N
  // operand.  Lane (gq, q) holds the outputs of weight rows wr0 + 16 m + 8 h +
  // gq (h = 0, 1) for chunk rows 2 q and 2 q + 1.
  const int cw = warp - 1, gq = lane >> 2, q = lane & 3;
  const int wr0 = 8 * kSmTiles * cw;
  float acc[2][4];
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[m][c] = INT8 ? -0.0f : 0.0f;
  bool ok = true;
  for (int ks = 0; ks < kstages; ++ks) {
    const int s = ks % kSmStages;
    if (ok) ok = mbar_wait_spin(&full[s], (ks / kSmStages) & 1, a.status);
    const unsigned char* st = smem + s * kStage;
    const float* wsm = reinterpret_cast<const float*>(st + kSmW);  // [128][4]
    // this lane's weight scales for the stage's four blocks
    float4 ws4[2][2];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        ws4[m][h] = *reinterpret_cast<const float4*>(wsm + 4 * (wr0 + 16 * m + 8 * h + gq));
    float4 xs4[2];
    if (INT8) {
      const float* xsm = reinterpret_cast<const float*>(st + kSmW + kSmWs + kSmXq);  // [8][4]
#pragma unroll
      for (int e = 0; e < 2; ++e) xs4[e] = *reinterpret_cast<const float4*>(xsm + 4 * (2 * q + e));
    }
#pragma unroll
    for (int jb = 0; jb < 4; ++jb) {
      // weights: row r = wr0 + 16 m + 8 h + gq, bytes [32 jb + 8q, + 8) of
      // the 128-byte row; 16-byte unit (2 jb + q / 2) sits at unit ^ (r % 8)
      uint2 wv[2][2];
      const int unit = (2 * jb + (q >> 1)) ^ gq;
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = wr0 + 16 * m + 8 * h + gq;
          wv[m][h] = *reinterpret_cast<const uint2*>(st + r * 128 + (unit << 4) + ((q & 1) << 3));
        }
      if (INT8) {
        const unsigned char* xq = st + kSmW + kSmWs;  // [8][128]
        const uint2 xv = *reinterpret_cast<const uint2*>(xq + gq * 128 + 32 * jb + 8 * q);
        const float2 xs2 = make_float2(jb == 0 ? xs4[0].x : jb == 1 ? xs4[0].y : jb == 2 ? xs4[0].z : xs4[0].w,
                                       jb == 0 ? xs4[1].x : jb == 1 ? xs4[1].y : jb == 2 ? xs4[1].z : xs4[1].w);
        const float2 magic = make_float2(-12582912.0f, -12582912.0f);
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          int d[4] = {0, 0, 0, 0};
          mma_s8_m16n8k32(d, wv[m][0].x, wv[m][1].x, wv[m][0].y, wv[m][1].y, xv.x, xv.y);
          // (c, c + 1) = one weight row and chunk rows 2q, 2q + 1: a packed pair
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float4 w4 = ws4[m][h];
            const float wsb = jb == 0 ? w4.x : jb == 1 ? w4.y : jb == 2 ? w4.z : w4.w;
            // exact int32 -> float: |S| < 2^22 (32 * 128 * 128), 2^23 + 2^22 + S
            // minus 2^23 + 2^22
            const float2 sf = f2_add(make_float2(__int_as_float(0x4B400000 + d[2 * h]),
                                                 __int_as_float(0x4B400000 + d[2 * h + 1])),
                                     magic);
            // ((float)S * ws) * xs (packed: each lane is the scalar IEEE
            // product), then the running sum, every operation rounded on its own
            const float2 t = f2_mul(f2_mul(sf, make_float2(wsb, wsb)), xs2);
            acc[m][2 * h] = __fadd_rn(acc[m][2 * h], t.x);  // scalar adds: see f2_mul
            acc[m][2 * h + 1] = __fadd_rn(acc[m][2 * h + 1], t.y);
          }
        }
      } else {
        float d[2][4];
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int c = 0; c < 4; ++c) d[m][c] = 0.0f;
        uint2 bw[2][2][2];  // [m][h][step]
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            bw[m][h][0] = i8x4_bf16(wv[m][h].x);  // step 0: physical 8q + 0..3
            bw[m][h][1] = i8x4_bf16(wv[m][h].y);  // step 1: physical 8q + 4..7
          }
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          const unsigned char* xp = st + kSmW + kSmWs + p * kSmXp;  // [8][128] bf16
          const uint4 rb = *reinterpret_cast<const uint4*>(xp + gq * 256 + 2 * (32 * jb + 8 * q));
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            mma_bf16_m16n8k16(d[m], bw[m][0][0].x, bw[m][1][0].x, bw[m][0][0].y, bw[m][1][0].y,
                              rb.x, rb.y);
            mma_bf16_m16n8k16(d[m], bw[m][0][1].x, bw[m][1][1].x, bw[m][0][1].y, bw[m][1][1].y,
                              rb.z, rb.w);
          }
        }
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float4 w4 = ws4[m][c >> 1];
            const float wsb = jb == 0 ? w4.x : jb == 1 ? w4.y : jb == 2 ? w4.z : w4.w;
            acc[m][c] = fmaf(d[m][c], wsb, acc[m][c]);
          }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // C layout: c0, c1 -> weight row gq, chunk rows 2q, 2q + 1; c2, c3 -> weight row gq + 8
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int i = 2 * q + e;
    if (i >= count) continue;
    const float sc = INT8 ? 1.0f : __ldg(a.rinv + off + i);
    float* yr = y + (off + i) * a.ldy + n0 + wr0 + gq;
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v = acc[m][2 * h + e];
        if (!INT8) v = __fmul_rn(v, sc);
        yr[16 * m + 8 * h] = v;
      }
  }
}

void configure_small() {
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(small_rows_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmSmemF);
    cudaFuncSetAttribute(small_rows_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmSmemI);
    // all of the unified L1 as shared memory, so that two CTAs fit on an SM
    cudaFuncSetAttribute(small_rows_kernel<false>,
                         cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(small_rows_kernel<true>,
                         cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  });
}

}  // namespace

bool small_rows_supported(int N, int K) {
  return N > 0 && N % kSmRows == 0 && K > 0 && K % kSmK == 0 && tma_encode_fn() != nullptr;
}

cudaError_t launch_small_rows(bool int8, const void* maps, const Q8View* single, const int* counts,
                              const int* offsets, int groups, int lo, int hi, int total_rows, int N,
                              int K, const uint16_t* pieces, int piece_rows, const float* rinv,
                              const int8_t* xq, const float* xs, int x_rows, float* y,
                              long long ldy, unsigned* status, cudaStream_t st,
                              const int* items, int max_items, const void* maps2,
                              const Q8View* single2, float* y2) {
  if (!small_rows_supported(N, K) || (!items && hi > kSmallChunkedMax) || lo < 1)
    return cudaErrorInvalidValue;
  if (items && (!counts || max_items < 1 || groups > 256)) return cudaErrorInvalidValue;
  if (!maps && !single) return cudaErrorInvalidValue;
  if (y2 && (single ? !single2 : !maps2)) return cudaErrorInvalidValue;
  if (y2 && reinterpret_cast<uintptr_t>(y2) % 8) return cudaErrorInvalidValue;
  const int chunks = counts ? (hi + kSmChunk - 1) / kSmChunk : 1;
  if (!counts) groups = (total_rows + kSmChunk - 1) / kSmChunk;
  if (groups < 1 || reinterpret_cast<uintptr_t>(y) % 8 || ldy % 2) return cudaErrorInvalidValue;
  CUtensorMap tw{}, tws{}, tx{}, txs{}, tw2{}, tws2{};
  if (single) {
    TcMatrixMaps mm;
    if (!q8_tc_weight_maps(&mm, *single)) return cudaErrorInvalidValue;
    tw = mm.w_sw128;
    tws = mm.ws;
    if (y2) {
      if (single2->rows != single->rows || single2->cols != single->cols ||
          !q8_tc_weight_maps(&mm, *single2))
        return cudaErrorInvalidValue;
      tw2 = mm.w_sw128;
      tws2 = mm.ws;
    }
  }
  if (int8) {
    if (!make_map_i8_plain(&tx, xq, x_rows, K, kSmChunk) ||
        !make_map_f32(&txs, xs, x_rows, K / 32, kSmChunk))
      return cudaErrorInvalidValue;
  } else if (!make_map_pieces_plain(&tx, pieces, piece_rows, K, kSmChunk)) {
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
  a.items = items;
  a.tiles = y2 ? N / kSmRows : 1 << 30;
  a.y2 = y2;
  a.maps2 = single ? nullptr : static_cast<const TcMatrixMaps*>(maps2);
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
  const dim3 grid((N / kSmRows) * (y2 ? 2 : 1), items ? max_items : chunks * groups);
  if (int8)
    return launch_dependent(small_rows_kernel<true>, grid, dim3(kSmThreads), kSmSmemI, st, tw, tws,
                            tx, txs, tw2, tws2, a);
  return launch_dependent(small_rows_kernel<false>, grid, dim3(kSmThreads), kSmSmemF, st, tw, tws,
                          tx, txs, tw2, tws2, a);
}

}  // namespace uocr
