// q8_tc.cu — Int8Matrix::linear_dynamic_int8 for many rows
// (src/cpu/quantized.rs:155-236, applied row by row) on the 5th-generation
// tensor cores.
//
// y[m][n] = sum over blocks b, in order, from -0.0:
//             ((float)S[m][n][b] * ws[n][b]) * xs[m][b]
// with S the exact int32 sum of one 32-wide block of int8 products.
//
// One tcgen05.mma of kind::i8 has K = 32: exactly one q8 block.  So every
// block gets its own MMA into its own TMEM buffer (no accumulation across
// blocks on the tensor core), and the epilogue warps apply the reference's
// float steps block by block, in order, each one an IEEE round-to-nearest
// operation — bit-identical to the scalar reference.
//
// Tile: 128 weight rows (MMA M, one TMEM lane each) x 64 activation rows
// (MMA N).  Each stage of a 6-stage shared-memory ring holds 128 bytes of K
// (4 blocks) of both operands (TMA, 128-byte swizzle, K-major as both
// matrices are stored) and the stage's block scales of both (TMA, 16-byte
// rows: [128][4] weight scales, [64][4] activation scales), all on one
// mbarrier.  Warp 0: TMA producer (one thread).  Warp 1: TMEM owner and MMA
// issuer (one thread).  Warps 2-17: epilogue, four per TMEM lane quarter, one
// weight row and 16 activation rows per thread, the TMEM load of the next
// block in flight while the current one is applied.  Eight 64-column TMEM
// buffers (all of TMEM) let the MMA run up to 7 blocks ahead of the epilogue,
// covering the MMA's completion latency; a ring slot is
// reused once its MMAs have completed and every epilogue warp has read its
// scales.
//
// A "group" launch serves the MoE prefill: group g owns activation rows
// [offsets[g], offsets[g] + counts[g]) and multiplies them by its own
// weights; the grid's y dimension enumerates 64-row tiles over the groups.
#include <cuda_bf16.h>

#include <mutex>

#include "common.cuh"
#include "device_once.h"
#include "kernels.h"
#include "tc_maps.cuh"
#include "tile_list.cuh"

namespace uocr {

namespace {

constexpr int kBN = 128;       // weight rows per tile (MMA M)
constexpr int kBM = 64;        // activation rows per tile (MMA N)
constexpr int kBK = 128;       // bytes of K per stage (4 blocks)
constexpr int kStages = 6;
constexpr int kAccBufs = 8;    // TMEM buffers of kBM columns: all of TMEM (one CTA per SM)
constexpr int kTmemCols = kAccBufs * kBM;  // 512
constexpr int kEpiWarps = 16;  // four per TMEM lane quarter, 16 columns each
constexpr int kEpiCols = kBM / (kEpiWarps / 4);
// warp 0 TMA, warp 1 MMA, warps 2 .. 2 + kEpiWarps - 1 epilogue, then one warp
// that writes each stage's activation-scale tile transposed ([block][row])
constexpr int kThreads = 64 + 32 * kEpiWarps + 32;
constexpr int kXposeWarp = 2 + kEpiWarps;
constexpr int kABytes = kBN * kBK;     // 16 KB weights
constexpr int kBBytes = kBM * kBK;     // 8 KB activations
constexpr int kWsBytes = kBN * 4 * 4;  // weight scales [128][4]
constexpr int kXsBytes = kBM * 4 * 4;  // activation scales [64][4]
constexpr int kStageBytes = kABytes + kBBytes + kWsBytes + kXsBytes;  // 27 KB (1024-multiple)
// Persistent CTAs: one per SM walks a list of tiles (at most kMaxCtaTiles,
// {group, first row, rows, first weight row} each, built once per CTA).
constexpr int kMaxCtaTiles = 128;
constexpr int kTileListBytes = kMaxCtaTiles * 16;
constexpr int kXsTBytes = kStages * kXsBytes;  // the transposed scale tiles, one per stage
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*alignment*/ + 512 /*barriers*/ +
                           kTileListBytes + kXsTBytes;
static_assert(kStageBytes % 1024 == 0, "swizzled tiles need 1024-byte alignment");


struct TcArgs {
  const TcMatrixMaps* maps;  // grouped: [groups]
  const int* counts;        // grouped: rows per group
  const int* offsets;       // grouped: first row of each group
  int groups;
  float* y;  // [rows][ldy]
  int M, N, K, ldy;
  unsigned* status;
};

// ---- PTX wrappers ----------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* holder, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(holder)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy ones (tensor-core reads, bulk copies into the same bytes).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] = A[smem] x B[smem]^T (accumulate = 0: overwrite), kind::i8, s32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(0)
      : "memory");
}

// Arrive on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Waits for this thread's TMEM loads.  The loaded registers are operands so
// that no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (tiles are 128 bytes of K wide).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* p) {
  const uint64_t addr = smem_addr(p);
  uint64_t d = (addr >> 4) & 0x3FFF;    // start address
  d |= static_cast<uint64_t>(1) << 16;  // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;          // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;          // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::i8, signed A and B, s32 D, both K-major,
// M = 128, N = 64.
constexpr uint32_t kIdescI8 = (2u << 4)               // D format: s32
                              | (1u << 7)             // A: signed 8-bit
                              | (1u << 10)            // B: signed 8-bit
                              | ((kBM >> 3) << 17)    // N
                              | ((kBN >> 4) << 24);   // M

// ---- the kernel --------------------------------------------------------------
// Persistent: CTA c takes the tiles c, c + gridDim.x, c + 2 gridDim.x, ... of
// the linear order L = (row tile) * (N / kBN) + (weight tile), so that the
// CTAs working at the same time share activation tiles and a group's weight
// tiles.  The TMA ring, the MMA's TMEM buffers and the epilogue's block
// sequence all run on across tile boundaries: a tile's first stages load while
// the previous tile's last blocks are applied, and the pipeline fills once per
// CTA instead of once per tile.
struct TileRef {
  int group, row0, rows, n0;
};

__global__ void __launch_bounds__(kThreads, 1)
    q8_tc_gemm_i8_kernel(const __grid_constant__ CUtensorMap tmap_w,
                         const __grid_constant__ CUtensorMap tmap_ws,
                         const __grid_constant__ CUtensorMap tmap_x,
                         const __grid_constant__ CUtensorMap tmap_xs, const TcArgs a) {
  extern __shared__ unsigned char smem_raw[];
  // offset from the shared array itself: derived pointers stay shared-memory
  // pointers to the compiler (an integer-cast alignment makes them generic)
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + kAccBufs;
  uint64_t* xsready = tempty + kAccBufs;  // stage's transposed scales written
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(xsready + kStages);
  int* ntiles_s = reinterpret_cast<int*>(tmem_holder + 1);
  TileRef* tiles = reinterpret_cast<TileRef*>(smem + kStages * kStageBytes + 512);
  float* xs_t = reinterpret_cast<float*>(smem + kStages * kStageBytes + 512 + kTileListBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntn = a.N / kBN;
  const int nbk = a.K >> 5, kstages = a.K / kBK;
  // The group counts are copied to shared memory by all threads first (one
  // thread walking them in global memory pays an L2 round trip per group),
  // into the ring, before any copy lands there.
  int* scount = reinterpret_cast<int*>(smem);
  if (a.counts)
    for (int g = threadIdx.x; g < a.groups; g += blockDim.x) scount[g] = a.counts[g];
  __syncthreads();
  if (threadIdx.x == 0)  // this CTA's tiles in order (tile_list.cuh)
    *ntiles_s = cta_tile_list(blockIdx.x, gridDim.x, ntn, a.M, a.counts ? scount : nullptr,
                              a.offsets, a.groups, kBM, kMaxCtaTiles,
                              [&](int i, const TileSpec& t) {
                                tiles[i].group = t.group;
                                tiles[i].row0 = t.row0;
                                tiles[i].rows = t.rows;
                                tiles[i].n0 = t.nx * kBN;
                              });
  fence_proxy_async_smem();  // the scratch reads come before the copies that overwrite it
  __syncthreads();
  const int ntiles = *ntiles_s;
  if (ntiles == 0) return;  // nothing for this CTA (the grid is an upper bound)

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + kEpiWarps);  // the MMAs' commit + every epilogue warp
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    for (int s = 0; s < kStages; ++s) mbar_init(&xsready[s], 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_holder, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // stages and blocks are counted over the CTA's whole tile sequence: stage
  // gs = i * kstages + ks of tile i, block gb = 4 gs + j
  const int total_stages = ntiles * kstages;

  if (warp == 0) {
    // ---- TMA producer: operands and their block scales, one barrier a stage
    if (lane == 0) {
      int i = 0, ks = 0;
      for (int gs = 0; gs < total_stages; ++gs) {
        const int s = gs % kStages;
        if (gs >= kStages && !mbar_wait_try(&empty[s], ((gs / kStages) - 1) & 1, a.status)) break;
        const TileRef t = tiles[i];
        const CUtensorMap* wmap = a.counts ? &a.maps[t.group].w_sw128 : &tmap_w;
        const CUtensorMap* smap = a.counts ? &a.maps[t.group].ws : &tmap_ws;
        unsigned char* st = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_2d(st, wmap, ks * kBK, t.n0, &full[s]);
        tma_load_2d(st + kABytes, &tmap_x, ks * kBK, t.row0, &full[s]);
        tma_load_2d(st + kABytes + kBBytes, smap, 4 * ks, t.n0, &full[s]);
        tma_load_2d(st + kABytes + kBBytes + kWsBytes, &tmap_xs, 4 * ks, t.row0, &full[s]);
        if (++ks == kstages) {
          ks = 0;
          ++i;
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: one MMA per q8 block, each into its own TMEM buffer
    if (lane == 0) {
      int blk = 0;
      bool ok = true;
      for (int gs = 0; gs < total_stages && ok; ++gs) {
        const int s = gs % kStages;
        ok = mbar_wait_try(&full[s], (gs / kStages) & 1, a.status);
        if (!ok) break;
        tc_fence_after();
        const unsigned char* st = smem + s * kStageBytes;
        for (int j = 0; j < kBK / 32; ++j, ++blk) {
          const int buf = blk % kAccBufs;
          if (blk >= kAccBufs) {
            ok = mbar_wait_try(&tempty[buf], ((blk / kAccBufs) - 1) & 1, a.status);
            if (!ok) break;
            tc_fence_after();
          }
          mma_i8(tmem + buf * kBM, smem_desc_sw128(st + 32 * j),
                 smem_desc_sw128(st + kABytes + 32 * j), kIdescI8);
        }
        if (!ok) break;
        // one commit for the stage's four blocks (a commit per block made
        // this thread, not the tensor core, the limit): stage gs arrives on
        // tfull[gs % 2]
        mma_commit(&tfull[gs & 1]);
        mma_commit(&empty[s]);  // one of the slot's arrivals: its MMAs are done
      }
    }
  } else if (warp == kXposeWarp) {
    // ---- the stage's activation scales [64 rows][4 blocks] rewritten as
    // [4 blocks][64 rows], so that an epilogue thread loads its 16 columns'
    // scales of a block with four 16-byte loads.  The slot's next refill waits
    // for the epilogue, which waits for this (xsready), so the tile is read
    // here before it is overwritten, and xs_t[s] before it is rewritten.
    bool ok = true;
    for (int gs = 0; gs < total_stages && ok; ++gs) {
      const int s = gs % kStages;
      ok = mbar_wait_try(&full[s], (gs / kStages) & 1, a.status);
      const float4* src =
          reinterpret_cast<const float4*>(smem + s * kStageBytes + kABytes + kBBytes + kWsBytes);
      float* dst = xs_t + s * (kXsBytes / 4);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = lane + 32 * h;
        const float4 v = src[r];
        dst[r] = v.x;
        dst[64 + r] = v.y;
        dst[128 + r] = v.z;
        dst[192 + r] = v.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&xsready[s]);
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32*(w % 4) .. + 31 (the rows it
    // may access) and kEpiCols of the 64 columns; one weight row per thread.
    // The TMEM load of block b + 1 is in flight while block b is applied.
    const int q = warp & 3, part = (warp - 2) / 4;
    const int rl = 32 * q + lane, c0 = kEpiCols * part;
    const uint32_t tlane = tmem + (static_cast<uint32_t>(32 * q) << 16) + c0;
    // running sums of two neighbouring columns per register pair: the
    // conversion and the two products run as packed f32x2 instructions (each
    // lane is the scalar IEEE operation), the adds as scalar ones, so each
    // column keeps the reference's rounding sequence
    float2 acc[kEpiCols / 2];
#pragma unroll
    for (int i = 0; i < kEpiCols / 2; ++i) acc[i] = make_float2(-0.0f, -0.0f);
    bool ok = true;
    const int total_blocks = ntiles * nbk;
    int rows = 0;  // the current tile's activation rows
    float4 ws4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // this row's scales of the stage's blocks
    // Block gb: its S values are in `now`; start loading block gb + 1 into
    // `next` (across a tile boundary too), apply block gb, then wait for the
    // load.  Called with the two register sets alternating, so no copies are
    // needed.
    // (jb = gb % 4 is passed as a literal, so that the scale selection and
    // the stage-boundary branches fold)
    auto step = [&](uint32_t (&now)[kEpiCols], uint32_t (&next)[kEpiCols], int gb, int jb) {
      const int buf = gb % kAccBufs, gks = gb >> 2, s = gks % kStages;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);  // block gb is in registers
      if (gb + 1 < total_blocks) {
        const int b1 = gb + 1, buf1 = b1 % kAccBufs, ks1 = b1 >> 2;
        if (jb == 3 && ok) ok = mbar_wait_try(&full[ks1 % kStages], (ks1 / kStages) & 1, a.status);
        if (jb == 3 && ok) ok = mbar_wait_try(&xsready[ks1 % kStages], (ks1 / kStages) & 1, a.status);
        // the four blocks of stage ks1 land together (one commit per stage,
        // alternating between two barriers)
        if (jb == 3 && ok) ok = mbar_wait_try(&tfull[ks1 & 1], (ks1 >> 1) & 1, a.status);
        tc_fence_after();
        tmem_ld16(tlane + buf1 * kBM, next);
      }
      const unsigned char* st = smem + s * kStageBytes;
      const float4* xs4 = reinterpret_cast<const float4*>(xs_t + s * (kXsBytes / 4) + 64 * jb + c0);
      if (jb == 0)  // the weight row's scales of the stage's four blocks, one load
        ws4 = *reinterpret_cast<const float4*>(st + kABytes + kBBytes + 16 * rl);
      const float wsb = jb == 0 ? ws4.x : jb == 1 ? ws4.y : jb == 2 ? ws4.z : ws4.w;
      const float2 ws2 = make_float2(wsb, wsb);
      const float2 magic = make_float2(-12582912.0f, -12582912.0f);
      // columns past the tile's last row are padding: nothing to apply
      // (the warp still takes part in every barrier)
      float4 xv[kEpiCols / 4];
      if (c0 < rows) {
#pragma unroll
        for (int u = 0; u < kEpiCols / 4; ++u) xv[u] = xs4[u];
      }
#pragma unroll
      for (int c = 0; c < kEpiCols && c0 < rows; c += 2) {
        const float4 x4 = xv[c / 4];
        const float2 xs2 = (c & 2) ? make_float2(x4.z, x4.w) : make_float2(x4.x, x4.y);
        // exact int32 -> float: |S| < 2^22 (32 * 127 * 127), 2^23 + 2^22 + S
        // minus 2^23 + 2^22
        const float2 sf =
            f2_add(make_float2(__int_as_float(0x4B400000 + static_cast<int>(now[c])),
                               __int_as_float(0x4B400000 + static_cast<int>(now[c + 1]))),
                   magic);
        // ((float)S * ws) * xs, then the running sum: each step rounded on
        // its own (the reference never contracts into an fma)
        const float2 t = f2_mul(f2_mul(sf, ws2), xs2);
        acc[c / 2].x = __fadd_rn(acc[c / 2].x, t.x);  // scalar adds: see f2_mul
        acc[c / 2].y = __fadd_rn(acc[c / 2].y, t.y);
      }
      if (jb == 3) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the slot's scales
      }
      if (gb + 1 < total_blocks) tmem_ld_wait(next);
    };
    uint32_t ra[kEpiCols], rb[kEpiCols];
    // block 0: its stage and its TMEM buffer
    ok = mbar_wait_try(&full[0], 0, a.status) && mbar_wait_try(&xsready[0], 0, a.status) &&
         mbar_wait_try(&tfull[0], 0, a.status);
    tc_fence_after();
    tmem_ld16(tlane, ra);
    tmem_ld_wait(ra);
    for (int ti = 0, gb0 = 0; ti < ntiles; ++ti, gb0 += nbk) {
      const TileRef t = tiles[ti];
      rows = t.rows;
      // nbk is a multiple of 4: every tile starts with its first block in ra
      for (int b = 0; b < nbk; b += 4) {
        step(ra, rb, gb0 + b, 0);
        step(rb, ra, gb0 + b + 1, 1);
        step(ra, rb, gb0 + b + 2, 2);
        step(rb, ra, gb0 + b + 3, 3);
      }
      // the tile's outputs, then the next tile's sums from -0.0
      const int n = t.n0 + rl;
      if (n < a.N) {
#pragma unroll
        for (int i = 0; i < kEpiCols; ++i)
          if (c0 + i < t.rows)
            a.y[static_cast<long long>(t.row0 + c0 + i) * a.ldy + n] =
                (i & 1) ? acc[i / 2].y : acc[i / 2].x;
      }
#pragma unroll
      for (int i = 0; i < kEpiCols / 2; ++i) acc[i] = make_float2(-0.0f, -0.0f);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- FP32 activations ------------------------------------------------------------
// Int8Matrix::linear for many rows (src/cpu/quantized.rs:101-153; for a batch
// the reference multiplies the dequantized weights by the activations with an
// SGEMM, src/cpu/ops.rs:62-133):
//   y[m][n] = sum over blocks b of ws[n][b] * (sum over the block of w[n][k] * x[m][k])
// The int8 weights are exact in bf16.  Every activation row is first scaled
// by a power of two 2^e that brings its largest magnitude into [1, 2) (so no
// piece or product lands in the subnormal range the tensor cores flush, and
// none can overflow), then split exactly into three bf16 pieces
// x' = x1 + x2 + x3 (x1 = x' truncated to bf16, x2 = the rest truncated,
// x3 = what remains: 8 significant bits each, fp32's 24 in all).  So every
// product on the tensor core is exact and only the FP32 accumulation differs
// from the reference's order.  One kind::f16 MMA per 16 elements of K, with
// the three pieces stacked as one B operand, puts a block's three partial sums
// in a TMEM buffer; the epilogue adds them (smallest first), adds ws * sum
// block by block with one fma and multiplies the row's total by 2^-e (exact
// unless the result is subnormal, then rounded once).
//
// A stage is 64 elements of K (two q8 blocks): the weights' int8 tile
// [128][64] (TMA, unswizzled), converted by four warps into bf16 in the UMMA
// layout (K-major, 128-byte swizzle) inside the same stage, and the three
// activation pieces [box][64] bf16 (TMA, 128-byte swizzle; box = the tile's
// rows rounded up to 16, 32 or 64).  Warp 0: TMA.  Warp 1: TMEM owner and MMA issuer.
// Warps 2-5: conversion.  Warps 6-21: epilogue, laid out as in the int8
// kernel.  The MMA's N is the tile's row count rounded up to 16, so small
// expert groups cost few tensor-core cycles.  The single-thread roles and the
// conversion warps poll their barriers (they are on the critical path and a
// suspended waiter wakes late); the epilogue warps wait suspended, leaving
// their issue slots to the conversion.  The conversion uses integer and
// FP32 operations only (the int -> float conversion instructions have a
// quarter of their throughput and made the conversion the bottleneck).
constexpr int kFK = 64;
constexpr int kFConvWarps = 4;
constexpr int kFThreads = 96 + 32 * (kFConvWarps + kEpiWarps);  // 736
constexpr int kFWi8 = kBN * kFK;                                // 8 KB int8 weights
constexpr int kFW8Slots = 8;                                    // int8 weight ring: 64 KB
constexpr int kFWbf = kBN * kFK * 2;                            // 16 KB bf16 weights
constexpr int kFSRing = 160 * 1024;                             // MMA-stage ring
constexpr int kFMaxS = 8;
constexpr int kFSmemBytes = kFW8Slots * kFWi8 + kFSRing + 1024 + 512 + 512 /*tile list*/;

// kind::f16 with bf16 A and B, f32 D, both K-major, M = 128 (N is added at run time).
constexpr uint32_t kIdescBf16 = (1u << 4)              // D format: f32
                                | (1u << 7)            // A: bf16
                                | (1u << 10)           // B: bf16
                                | ((kBN >> 4) << 24);  // M

struct TcF32Args {
  const TcMatrixMaps* maps;  // grouped: [groups]
  const int* counts;
  const int* offsets;
  int groups;
  const float* s;     // single: weight scales [N][K / 32]
  const float* rinv;  // 2^-e of each activation row
  float* y;
  int M, N, K, ldy;
  int piece_rows;  // rows of each activation piece tensor
  unsigned* status;
};

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}


// Four int8 (one word, lowest byte first) -> four bf16, exact.  Each byte,
// offset to u = v + 128, is placed under the exponent of 2^23 (the float
// 2^23 + u); subtracting 2^23 + 128 leaves v exactly.  |v| <= 128 has at
// most 8 significant bits, so its bf16 is the float's high half.
__device__ __forceinline__ uint2 i8x4_to_bf16x4(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;
  const float2 magic = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128), two lanes per add
  const float2 lo = f2_add(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)),
                                       __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441))),
                           magic);
  const float2 hi = f2_add(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)),
                                       __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443))),
                           magic);
  return make_uint2(__byte_perm(__float_as_uint(lo.x), __float_as_uint(lo.y), 0x7632),
                    __byte_perm(__float_as_uint(hi.x), __float_as_uint(hi.y), 0x7632));
}

// Persistent, like the int8 kernel: CTA c takes the tiles c, c + gridDim.x,
// ... of the same linear order, listed once per CTA ({first row, group | rows
// << 8 | weight tile << 16}, 8 bytes each: shared memory is nearly full).
// The activation box is the largest its tiles need, fixed for the CTA, so the
// stage-slot layout never changes; every ring, the TMEM buffers and the
// epilogue run on across tile boundaries.
struct FTile {
  int row0, packed;
};
constexpr int kFMaxCtaTiles = 64;

__global__ void __launch_bounds__(kFThreads, 1)
    q8_tc_gemm_f32_kernel(const __grid_constant__ CUtensorMap tmap_w,
                          const __grid_constant__ CUtensorMap tmap_xp,
                          const __grid_constant__ CUtensorMap tmap_xp16,
                          const __grid_constant__ CUtensorMap tmap_xp32, const TcF32Args a) {
  extern __shared__ unsigned char smem_raw[];
  // offset from the shared array itself: derived pointers stay shared-memory
  // pointers to the compiler (an integer-cast alignment makes them generic)
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  unsigned char* w8ring = smem;                        // [kFW8Slots][128][64] int8
  unsigned char* sring = smem + kFW8Slots * kFWi8;     // [nS][bf16 weights | pieces]
  uint64_t* full8 = reinterpret_cast<uint64_t*>(sring + kFSRing);
  uint64_t* empty8 = full8 + kFW8Slots;
  uint64_t* fullx = empty8 + kFW8Slots;
  uint64_t* conv = fullx + kFMaxS;
  uint64_t* empty = conv + kFMaxS;
  uint64_t* tempty = empty + kFMaxS;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + kAccBufs);
  int* tile = reinterpret_cast<int*>(tmem_holder + 1);  // tile count, box
  FTile* ftiles = reinterpret_cast<FTile*>(sring + kFSRing + 512);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntn = a.N / kBN;
  const int nbk = a.K >> 5, kstages = a.K / kFK;
  // the tile list, over group counts staged in shared memory (as in the int8 kernel)
  int* scount = reinterpret_cast<int*>(sring);
  if (a.counts)
    for (int g = threadIdx.x; g < a.groups; g += blockDim.x) scount[g] = a.counts[g];
  __syncthreads();
  if (threadIdx.x == 0) {  // this CTA's tiles in order (tile_list.cuh) and the rows of its largest
    int maxrows = 0;
    tile[0] = cta_tile_list(blockIdx.x, gridDim.x, ntn, a.M, a.counts ? scount : nullptr, a.offsets,
                            a.groups, kBM, kFMaxCtaTiles, [&](int i, const TileSpec& t) {
                              ftiles[i].row0 = t.row0;
                              ftiles[i].packed = t.group | (t.rows << 8) | (t.nx << 16);
                              maxrows = t.rows > maxrows ? t.rows : maxrows;
                            });
    tile[1] = maxrows <= 16 ? 16 : maxrows <= 32 ? 32 : 64;
  }
  fence_proxy_async_smem();  // the scratch reads come before the copies that overwrite it
  __syncthreads();
  const int ntiles = tile[0];
  if (ntiles == 0) return;  // nothing for this CTA (the grid is an upper bound)
  // The activation box: the CTA's largest tile rounded up to 16, 32 or 64.
  // The three pieces sit one above the other as one B operand of 3 * box
  // rows, so one MMA per 16 elements of K covers all three (the MMA
  // instruction, not the tensor-core arithmetic, is what a stage pays for
  // with small tiles); a block's sums take 3 * box TMEM columns and the
  // epilogue adds the pieces.
  const int box = tile[1];
  const int bufcols = 3 * box;
  const int nbuf = kTmemCols / bufcols < kAccBufs ? kTmemCols / bufcols : kAccBufs;  // 8, 5 or 2
  // MMA-stage slots: bf16 weights then the pieces; 7, 5 or 4 of them
  const int sbytes = kFWbf + 3 * box * 128;
  const int ns_raw = kFSRing / sbytes;
  const int nS = ns_raw < kFMaxS ? ns_raw : kFMaxS;
  const int total_stages = ntiles * kstages;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kFW8Slots; ++i) {
      mbar_init(&full8[i], 1);
      mbar_init(&empty8[i], kFConvWarps);
    }
    for (int i = 0; i < kFMaxS; ++i) {
      mbar_init(&fullx[i], 1);
      mbar_init(&conv[i], kFConvWarps);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) mbar_init(&tempty[b], kEpiWarps);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_holder, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---- int8 weights: a deep ring whose slots free as soon as they are converted
    if (lane == 0) {
      int i = 0, ks = 0;
      for (int gs = 0; gs < total_stages; ++gs) {
        const int w = gs % kFW8Slots;
        if (gs >= kFW8Slots &&
            !mbar_wait_spin(&empty8[w], ((gs / kFW8Slots) - 1) & 1, a.status))
          break;
        const int packed = ftiles[i].packed;
        const CUtensorMap* wmap = a.counts ? &a.maps[packed & 255].w_rows64 : &tmap_w;
        mbar_arrive_expect_tx(&full8[w], kFWi8);
        tma_load_2d(w8ring + w * kFWi8, wmap, ks * kFK, (packed >> 16) * kBN, &full8[w]);
        if (++ks == kstages) {
          ks = 0;
          ++i;
        }
      }
    }
  } else if (warp == 2) {
    // ---- activation pieces into the MMA-stage slots
    if (lane == 0) {
      const CUtensorMap* xmap = box == 16 ? &tmap_xp16 : box == 32 ? &tmap_xp32 : &tmap_xp;
      const uint32_t tx = 3 * box * 128;
      int sl = 0, lap = 0, i = 0, ks = 0;
      for (int gs = 0; gs < total_stages; ++gs) {
        if (lap > 0 && !mbar_wait_spin(&empty[sl], (lap - 1) & 1, a.status)) break;
        unsigned char* st = sring + sl * sbytes;
        const int row0 = ftiles[i].row0;
        mbar_arrive_expect_tx(&fullx[sl], tx);
#pragma unroll
        for (int p = 0; p < 3; ++p)
          tma_load_2d(st + kFWbf + p * box * 128, xmap, ks * kFK, p * a.piece_rows + row0,
                      &fullx[sl]);
        if (++sl == nS) {
          sl = 0;
          ++lap;
        }
        if (++ks == kstages) {
          ks = 0;
          ++i;
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: per q8 block, one MMA per 16 elements of K into the
    // block's buffer (N = 3 * box: all pieces at once); one commit per stage.
    // Buffer and slot indices are kept incrementally (a division by a
    // run-time count costs the issuing thread more than an MMA).
    if (lane == 0) {
      const uint32_t idesc = kIdescBf16 | (static_cast<uint32_t>(bufcols >> 3) << 17);
      int buf = 0, blap = 0, sl = 0, lap = 0;
      bool ok = true;
      for (int gs = 0; gs < total_stages && ok; ++gs) {
        ok = mbar_wait_spin(&fullx[sl], lap & 1, a.status) &&
             mbar_wait_spin(&conv[sl], lap & 1, a.status);
        if (!ok) break;
        tc_fence_after();
        const unsigned char* st = sring + sl * sbytes;
        for (int j = 0; j < kFK / 32; ++j) {
          if (blap > 0) {
            ok = mbar_wait_spin(&tempty[buf], (blap - 1) & 1, a.status);
            if (!ok) break;
            tc_fence_after();
          }
#pragma unroll
          for (int h = 0; h < 2; ++h)
            mma_bf16(tmem + buf * bufcols, smem_desc_sw128(st + 64 * j + 32 * h),
                     smem_desc_sw128(st + kFWbf + 64 * j + 32 * h), idesc,
                     static_cast<uint32_t>(h));
          if (++buf == nbuf) {
            buf = 0;
            ++blap;
          }
        }
        // frees the slot and publishes both blocks (commits cost more than MMAs)
        mma_commit(&empty[sl]);
        if (++sl == nS) {
          sl = 0;
          ++lap;
        }
      }
    }
  } else if (warp < 3 + kFConvWarps) {
    // ---- int8 -> bf16 weights, from the int8 ring into the stage slot: thread
    // ct converts 16-byte chunks ct, ct + 32 * kFConvWarps, ... (row c / 4,
    // elements 16 * (c % 4) ..) into the swizzled layout: row r's 16-byte unit
    // j sits at (r / 8) * 1024 + (r % 8) * 128 + ((j ^ (r % 8)) * 16).
    const int ct = threadIdx.x - 96;
    int sl = 0, lap = 0;
    for (int gs = 0; gs < total_stages; ++gs) {
      const int w = gs % kFW8Slots;
      if (!mbar_wait_spin(&full8[w], (gs / kFW8Slots) & 1, a.status)) break;
      if (lap > 0 && !mbar_wait_spin(&empty[sl], (lap - 1) & 1, a.status)) break;
      unsigned char* st = sring + sl * sbytes;
      const unsigned char* wi8 = w8ring + w * kFWi8;
#pragma unroll
      for (int i = 0; i < (kBN * kFK / 16) / (32 * kFConvWarps); ++i) {
        const int c = ct + 32 * kFConvWarps * i, r = c >> 2, q = c & 3;
        const uint4 v = *reinterpret_cast<const uint4*>(wi8 + r * kFK + q * 16);
        const uint2 a0 = i8x4_to_bf16x4(v.x), a1 = i8x4_to_bf16x4(v.y);
        const uint2 a2 = i8x4_to_bf16x4(v.z), a3 = i8x4_to_bf16x4(v.w);
        unsigned char* rowp = st + (r >> 3) * 1024 + (r & 7) * 128;
        *reinterpret_cast<uint4*>(rowp + (((2 * q) ^ (r & 7)) << 4)) = make_uint4(a0.x, a0.y, a1.x, a1.y);
        *reinterpret_cast<uint4*>(rowp + (((2 * q + 1) ^ (r & 7)) << 4)) = make_uint4(a2.x, a2.y, a3.x, a3.y);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty8[w]);  // the int8 slot is read
        mbar_arrive(&conv[sl]);
      }
      if (++sl == nS) {
        sl = 0;
        ++lap;
      }
    }
  } else {
    // ---- epilogue: one weight row and 16 activation rows per thread; per
    // block, the three pieces' sums (smallest first) times the block scale
    const int ew = warp - 3 - kFConvWarps;
    const int q = warp & 3, part = ew / 4;
    const int rl = 32 * q + lane, c0 = kEpiCols * part;
    const uint32_t tlane = tmem + (static_cast<uint32_t>(32 * q) << 16) + c0;
    bool ok = true;
    int buf = 0, sl = 0, lap = 0;
    for (int ti = 0; ti < ntiles; ++ti) {
      const FTile t = ftiles[ti];
      const int group = t.packed & 255, rows = (t.packed >> 8) & 255;
      const int n = (t.packed >> 16) * kBN + rl;
      const bool active = c0 < rows;  // warp-uniform
      const float* srow = (a.counts ? a.maps[group].s : a.s) + static_cast<long long>(n) * nbk;
      // two neighbouring columns per register pair: the piece sums and the
      // scale fma run as packed f32x2 instructions, each lane rounded as the
      // scalar operation
      float2 acc[kEpiCols / 2];
#pragma unroll
      for (int i = 0; i < kEpiCols / 2; ++i) acc[i] = make_float2(0.0f, 0.0f);
      for (int b = 0; b < nbk; ++b) {
        const float sc = __ldg(srow + b);  // its latency hides behind the wait
        // the stage's commit (its slot's `empty` phase): the MMA cannot
        // complete this slot's next stage before this warp has released the
        // stage's TMEM buffers, so the phase waited for is the latest one
        if (ok) ok = mbar_wait_try(&empty[sl], lap & 1, a.status);
        tc_fence_after();
        // the two small pieces' sums first, then the leading piece's (two
        // rounds of loads keep the epilogue within the register budget)
        uint32_t ra[kEpiCols], rb[kEpiCols];
        if (active) {
          const uint32_t tb = tlane + buf * bufcols;
          tmem_ld16(tb + 2 * box, ra);
          tmem_ld16(tb + box, rb);
          tmem_ld_wait(ra);
          tmem_ld_wait(rb);
#pragma unroll
          for (int c = 0; c < kEpiCols; c += 2) {
            const float2 s2 = f2_add(make_float2(__uint_as_float(ra[c]), __uint_as_float(ra[c + 1])),
                                     make_float2(__uint_as_float(rb[c]), __uint_as_float(rb[c + 1])));
            ra[c] = __float_as_uint(s2.x);
            ra[c + 1] = __float_as_uint(s2.y);
          }
          tmem_ld16(tb, rb);
          tmem_ld_wait(rb);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        if (active) {
          const float2 sc2 = make_float2(sc, sc);
#pragma unroll
          for (int c = 0; c < kEpiCols; c += 2)
            acc[c / 2] = f2_fma(f2_add(make_float2(__uint_as_float(ra[c]), __uint_as_float(ra[c + 1])),
                                       make_float2(__uint_as_float(rb[c]), __uint_as_float(rb[c + 1]))),
                                sc2, acc[c / 2]);
        }
        if (++buf == nbuf) buf = 0;
        if (b & 1) {
          if (++sl == nS) {
            sl = 0;
            ++lap;
          }
        }
      }
      if (active) {
#pragma unroll
        for (int i = 0; i < kEpiCols; ++i)
          if (c0 + i < rows)
            a.y[static_cast<long long>(t.row0 + c0 + i) * a.ldy + n] =
                __fmul_rn((i & 1) ? acc[i / 2].y : acc[i / 2].x, __ldg(a.rinv + t.row0 + c0 + i));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Power-of-two exponent e with max * 2^e in [1, 2); 0 for a zero row or one
// holding a non-finite value (whose pieces then carry the inf or NaN).
__device__ __forceinline__ int row_norm_exp(float mx) {
  if (!(mx > 0.0f) || !isfinite(mx)) return 0;
  return -ilogbf(mx);
}

// v * 2^e in two exact steps (each factor a normal float for e in [-149, 149]).
__device__ __forceinline__ float4 scale_pow2(float4 v, int e) {
  const float f1 = __int_as_float((127 + e / 2) << 23), f2 = __int_as_float((127 + e - e / 2) << 23);
  return make_float4(__fmul_rn(__fmul_rn(v.x, f1), f2), __fmul_rn(__fmul_rn(v.y, f1), f2),
                     __fmul_rn(__fmul_rn(v.z, f1), f2), __fmul_rn(__fmul_rn(v.w, f1), f2));
}

__device__ __forceinline__ float max_abs4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// The exact three-way bf16 split of one fp32 value (see above): the first two
// pieces truncate (so no piece can round up past the value), the last holds
// at most 8 significant bits and is exact.
__device__ __forceinline__ void split3(float v, uint32_t& p0, uint32_t& p1, uint32_t& p2) {
  const uint32_t b0 = __float_as_uint(v) & 0xFFFF0000u;
  const float r1 = v - __uint_as_float(b0);
  const uint32_t b1 = __float_as_uint(r1) & 0xFFFF0000u;
  const float r2 = r1 - __uint_as_float(b1);
  p0 = b0 >> 16;
  p1 = b1 >> 16;
  p2 = __float_as_uint(r2) >> 16;
}

__device__ __forceinline__ void store_split4(float4 v, uint16_t* pieces, long long off,
                                             long long piece_elems) {
  uint32_t a[4], b[4], c[4];
  split3(v.x, a[0], b[0], c[0]);
  split3(v.y, a[1], b[1], c[1]);
  split3(v.z, a[2], b[2], c[2]);
  split3(v.w, a[3], b[3], c[3]);
  *reinterpret_cast<uint2*>(pieces + off) = make_uint2(a[0] | (a[1] << 16), a[2] | (a[3] << 16));
  *reinterpret_cast<uint2*>(pieces + piece_elems + off) =
      make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
  *reinterpret_cast<uint2*>(pieces + 2 * piece_elems + off) =
      make_uint2(c[0] | (c[1] << 16), c[2] | (c[3] << 16));
}

// One warp per row: pieces[p][r][k] = the split of x[src ? src[r] : r][k] * 2^e
// and rinv[r] = 2^-e.
__global__ void split_rows_kernel(const float* __restrict__ x, long long ld_x,
                                  const int* __restrict__ src, int rows, int cols,
                                  uint16_t* __restrict__ pieces, float* __restrict__ rinv,
                                  long long piece_elems, const int* __restrict__ live) {
  const int lane = threadIdx.x & 31, c4 = cols / 4;
  if (live) rows = min(rows, *live);
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + (src ? src[r] : r) * ld_x);
    float mx = 0.0f;
    for (int c = lane; c < c4; c += 32) mx = fmaxf(mx, max_abs4(xr[c]));
    const int e = row_norm_exp(warp_max(mx));
    for (int c = lane; c < c4; c += 32)
      store_split4(scale_pow2(xr[c], e), pieces, r * cols + 4 * c, piece_elems);
    if (lane == 0) rinv[r] = ldexpf(1.0f, -e);
  }
}

__device__ __forceinline__ float4 swiglu4(float4 g, float4 u) {
  return make_float4(__fmul_rn(silu_ref(g.x), u.x), __fmul_rn(silu_ref(g.y), u.y),
                     __fmul_rn(silu_ref(g.z), u.z), __fmul_rn(silu_ref(g.w), u.w));
}

// h = silu(gate) * up (src/decoder/mod.rs:114-122), one warp per row, split
// into pieces as split_rows_kernel does.
__global__ void swiglu_split_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                    int rows, int cols, uint16_t* __restrict__ pieces,
                                    float* __restrict__ rinv, long long piece_elems,
                                    const int* __restrict__ live) {
  const int lane = threadIdx.x & 31, c4 = cols / 4;
  if (live) rows = min(rows, *live);
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps) {
    const float4* gr = reinterpret_cast<const float4*>(g + r * cols);
    const float4* ur = reinterpret_cast<const float4*>(u + r * cols);
    float mx = 0.0f;
    for (int c = lane; c < c4; c += 32) mx = fmaxf(mx, max_abs4(swiglu4(gr[c], ur[c])));
    const int e = row_norm_exp(warp_max(mx));
    for (int c = lane; c < c4; c += 32)
      store_split4(scale_pow2(swiglu4(gr[c], ur[c]), e), pieces, r * cols + 4 * c, piece_elems);
    if (lane == 0) rinv[r] = ldexpf(1.0f, -e);
  }
}

// The same two splits with one CTA per row and the row held in registers: one
// pass over memory and a CTA-wide maximum (a warp per row walks the row twice
// with one warp's worth of loads in flight, which made these passes
// latency-bound when the rows are few).
constexpr int kSplitThreads = 256;
constexpr int kSplitMaxV = 8;  // float4 per thread: cols <= 8192

template <bool SWIGLU>
__global__ void __launch_bounds__(kSplitThreads) split_rows_cta_kernel(
    const float* __restrict__ x, long long ld_x, const int* __restrict__ src,
    const float* __restrict__ u, int rows, int cols, uint16_t* __restrict__ pieces,
    float* __restrict__ rinv, long long piece_elems, const int* __restrict__ live) {
  pdl_launch_dependents();  // launched as a programmatic dependent (launch_dependent):
  pdl_wait_prior_grids();   // nothing is touched before the previous kernel completes
  __shared__ float wmax[kSplitThreads / 32];
  const int r = blockIdx.x;
  if (r >= rows || (live && r >= *live)) return;
  const int c4 = cols / 4, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float4* xr = reinterpret_cast<const float4*>(
      SWIGLU ? x + static_cast<long long>(r) * cols : x + (src ? src[r] : r) * ld_x);
  const float4* ur = reinterpret_cast<const float4*>(u + static_cast<long long>(r) * cols);
  float4 v[kSplitMaxV];
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < kSplitMaxV; ++i) {
    const int c = threadIdx.x + i * kSplitThreads;
    if (c < c4) {
      v[i] = SWIGLU ? swiglu4(xr[c], ur[c]) : xr[c];
      mx = fmaxf(mx, max_abs4(v[i]));
    }
  }
  mx = warp_max(mx);
  if (lane == 0) wmax[warp] = mx;
  __syncthreads();
  if (warp == 0) {
    mx = lane < kSplitThreads / 32 ? wmax[lane] : 0.0f;
    mx = warp_max(mx);
    if (lane == 0) wmax[0] = mx;
  }
  __syncthreads();
  const int e = row_norm_exp(wmax[0]);
#pragma unroll
  for (int i = 0; i < kSplitMaxV; ++i) {
    const int c = threadIdx.x + i * kSplitThreads;
    if (c < c4)
      store_split4(scale_pow2(v[i], e), pieces, static_cast<long long>(r) * cols + 4 * c,
                   piece_elems);
  }
  if (threadIdx.x == 0) rinv[r] = ldexpf(1.0f, -e);
}

// ---- prefill helpers ---------------------------------------------------------
// Rows of the block-quantized activations gathered in pair order:
// xq_p[p] = xq[src[p]], xs_p[p] = xs[src[p]].
__global__ void gather_rows_kernel(const int8_t* __restrict__ xq, const float* __restrict__ xs,
                                   const int* __restrict__ src, int rows, int cols,
                                   int8_t* __restrict__ xq_p, float* __restrict__ xs_p,
                                   const int* __restrict__ live) {
  const int nb = cols / 32, c16 = cols / 16;
  if (live) rows = min(rows, *live);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       i < static_cast<long long>(rows) * c16; i += stride) {
    const int p = static_cast<int>(i / c16), c = static_cast<int>(i % c16);
    reinterpret_cast<uint4*>(xq_p)[i] =
        reinterpret_cast<const uint4*>(xq)[static_cast<long long>(src[p]) * c16 + c];
  }
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       i < static_cast<long long>(rows) * nb; i += stride) {
    const int p = static_cast<int>(i / nb), b = static_cast<int>(i % nb);
    xs_p[i] = xs[static_cast<long long>(src[p]) * nb + b];
  }
}

// h = silu(gate) * up (Decoder::feed_forward, src/decoder/mod.rs:114-122),
// block-quantized per row for the down projection in int8 mode
// (src/cpu/quantized.rs:43-74): one warp per 32-wide block.
__global__ void swiglu_quantize_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                       int rows, int cols, int8_t* __restrict__ hq,
                                       float* __restrict__ hs, unsigned* status,
                                       const int* __restrict__ live) {
  const int lane = threadIdx.x & 31, nb = cols / 32;
  if (live) rows = min(rows, *live);
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long w = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       w < static_cast<long long>(rows) * nb; w += warps) {
    const long long k = w * 32 + lane;  // rows are cols = 32 * nb wide
    const float h = __fmul_rn(silu_ref(g[k]), u[k]);
    if (__any_sync(0xffffffffu, !isfinite(h)) && lane == 0) flag(status, DEV_NONFINITE);
    const float mx = warp_max(fabsf(h));
    const float scale = __fdiv_rn(mx, 127.0f);
    if (lane == 0) {
      if (mx > 0.0f && scale == 0.0f) flag(status, DEV_UNDERFLOW);
      hs[w] = scale;
    }
    hq[k] = quantize_elem(h, scale);
  }
}

int grid_for(long long work, int sms) {
  const long long g = (work + 255) / 256;
  return static_cast<int>(g < 1 ? 1 : (g > 8LL * sms ? 8LL * sms : g));
}

// ---- host: tensor maps ------------------------------------------------------
// The dynamic shared-memory opt-in, once per device.
void configure() {
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(q8_tc_gemm_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemBytes);
    cudaFuncSetAttribute(q8_tc_gemm_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kFSmemBytes);
  });
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// Grid of a persistent GEMM for `tiles` (an upper bound on the tiles):
// persistent_ctas (tile_list.cuh) with this device's SM count.
int persistent_grid(long long tiles, int max_per_cta) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) {
    cudaGetLastError();
    sms = 148;
  }
  return persistent_ctas(tiles, sms, max_per_cta);
}

// ---- BF16 weights, FP32 activations (ops::linear_weight, BF16 branch) ---------
// y[m][n] = sum_k x[m][k] * w[n][k] for a large BF16 weight (the lm_head,
// 129,280 x 1280 at a decode batch of 64).  The weights need no conversion:
// a TMA box of 128 rows x 64 bf16 with the 128-byte swizzle is already the
// MMA's K-major operand layout.  The activations come as the exact three
// bf16 pieces of each row scaled by a power of two (launch_split_rows), stacked
// as one B operand of 3 * box rows, so every product is exact and one TMEM
// accumulator takes the whole of K (no per-block scale here): the epilogue
// runs once per tile, adds the three pieces' sums (smallest first) and
// rescales the row.  Persistent: each CTA takes tiles (128 weight rows x 64
// activation rows) in turn through one ring of stages, with two TMEM
// accumulators so that a tile's epilogue overlaps the next tile's MMAs.
// Warp 0: TMA.  Warp 1: TMEM owner and MMA issuer.  Warps 2-5: epilogue.
constexpr int kHK = 64;                           // K elements per stage (128 bytes of bf16)
constexpr int kHStages = 5;
constexpr int kHWBytes = kBN * kHK * 2;           // 16 KB weight tile
constexpr int kHStageBytes = kHWBytes + 3 * kBM * kHK * 2;  // + pieces of up to 64 rows: 40 KB
constexpr int kHEpiWarps = 4;
constexpr int kHThreads = 64 + 32 * kHEpiWarps;   // 192
constexpr int kHAccCols = 256;                    // TMEM columns per accumulator (3 * 64 used)
constexpr int kHTmemCols = 2 * kHAccCols;
constexpr int kHSmemBytes = kHStages * kHStageBytes + 1024 + 256;
static_assert(kHStageBytes % 1024 == 0, "swizzled tiles need 1024-byte alignment");

struct HeadArgs {
  const float* rinv;  // 2^-e of each activation row
  float* y;           // [batch][ldy]
  int n, k, batch, ldy;
  int piece_rows;     // rows of each piece tensor (batch)
  int box;            // activation rows per tile as loaded: 16, 32 or 64
  int n_tiles, row_tiles;
  unsigned* status;
};

__global__ void __launch_bounds__(kHThreads, 1)
    bf16_head_kernel(const __grid_constant__ CUtensorMap tmap_w,
                     const __grid_constant__ CUtensorMap tmap_x, const HeadArgs a) {
  extern __shared__ unsigned char smem_raw[];
  // offset from the shared array itself: derived pointers stay shared-memory
  // pointers to the compiler (an integer-cast alignment makes them generic)
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kHStages * kHStageBytes);
  uint64_t* empty = full + kHStages;
  uint64_t* tfull = empty + kHStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int box = a.box, ncols = 3 * box;
  const int kstages = a.k / kHK;
  const int total = a.n_tiles * a.row_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kHStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kHEpiWarps);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_holder, kHTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---- TMA: the weight tile and the three piece tiles of each stage
    if (lane == 0) {
      const uint32_t tx = kHWBytes + 3 * box * kHK * 2;
      int g = 0;  // stages issued
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const int n0 = (t % a.n_tiles) * kBN, r0 = (t / a.n_tiles) * kBM;
        for (int ks = 0; ks < kstages; ++ks, ++g) {
          const int s = g % kHStages;
          if (g >= kHStages && !(ok = mbar_wait_spin(&empty[s], ((g / kHStages) - 1) & 1, a.status)))
            break;
          unsigned char* st = smem + s * kHStageBytes;
          mbar_arrive_expect_tx(&full[s], tx);
          tma_load_2d(st, &tmap_w, ks * kHK, n0, &full[s]);
#pragma unroll
          for (int p = 0; p < 3; ++p)
            tma_load_2d(st + kHWBytes + p * box * kHK * 2, &tmap_x, ks * kHK,
                        p * a.piece_rows + r0, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA: four K = 16 steps per stage into the tile's accumulator
    if (lane == 0) {
      const uint32_t idesc = kIdescBf16 | (static_cast<uint32_t>(ncols >> 3) << 17);
      int g = 0, i = 0;  // stages consumed, tiles begun
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (i >= 2) {
          if (!(ok = mbar_wait_spin(&tempty[buf], ((i >> 1) - 1) & 1, a.status))) break;
          tc_fence_after();
        }
        const uint32_t d = tmem + buf * kHAccCols;
        for (int ks = 0; ks < kstages; ++ks, ++g) {
          const int s = g % kHStages;
          if (!(ok = mbar_wait_spin(&full[s], (g / kHStages) & 1, a.status))) break;
          tc_fence_after();
          const unsigned char* st = smem + s * kHStageBytes;
#pragma unroll
          for (int j = 0; j < kHK / 16; ++j)
            mma_bf16(d, smem_desc_sw128(st + 32 * j), smem_desc_sw128(st + kHWBytes + 32 * j), idesc,
                     (ks | j) ? 1u : 0u);
          mma_commit(&empty[s]);  // the slot is free once these MMAs are done
        }
        mma_commit(&tfull[buf]);  // the tile's accumulator is complete
      }
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31, one weight
    // row per thread; for every activation row, (p2 + p1) + p0, times 2^-e
    const int q = warp & 3;
    int i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
      const int buf = i & 1;
      const int n0 = (t % a.n_tiles) * kBN, r0 = (t / a.n_tiles) * kBM;
      if (ok) ok = mbar_wait_try(&tfull[buf], (i >> 1) & 1, a.status);
      tc_fence_after();
      const int n = n0 + 32 * q + lane;
      const int rows = a.batch - r0 < kBM ? a.batch - r0 : kBM;
      const uint32_t tl = tmem + (static_cast<uint32_t>(32 * q) << 16) + buf * kHAccCols;
      for (int c = 0; c < box; c += 16) {
        uint32_t p0[16], p1[16], p2[16];
        tmem_ld16(tl + c, p0);
        tmem_ld16(tl + box + c, p1);
        tmem_ld16(tl + 2 * box + c, p2);
        tmem_ld_wait(p0);
        tmem_ld_wait(p1);
        tmem_ld_wait(p2);
        if (ok && n < a.n) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c + e < rows) {
              const float v = __fadd_rn(__fadd_rn(__uint_as_float(p2[e]), __uint_as_float(p1[e])),
                                        __uint_as_float(p0[e]));
              a.y[static_cast<long long>(r0 + c + e) * a.ldy + n] =
                  __fmul_rn(v, __ldg(a.rinv + r0 + c + e));
            }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kHTmemCols);
  }
}

}  // namespace

bool q8_tc_supported(int rows, int cols) {
  return rows > 0 && cols > 0 && rows % kBN == 0 && cols % kBK == 0 && tma_encode_fn() != nullptr;
}

size_t q8_tc_maps_bytes() { return sizeof(TcMatrixMaps); }

bool q8_tc_weight_maps(void* maps, const Q8View& m) {
  TcMatrixMaps* mp = static_cast<TcMatrixMaps*>(maps);
  if (!q8_tc_supported(static_cast<int>(m.rows), static_cast<int>(m.cols)) || !aligned16(m.w) ||
      !aligned16(m.s))
    return false;
  mp->s = m.s;
  mp->nb = m.cols / 32;
  return make_map_i8(&mp->w_sw128, m.w, m.rows, m.cols, kBN) &&
         make_map_f32(&mp->ws, m.s, m.rows, m.cols / 32, kBN) &&
         make_map_w_rows64(&mp->w_rows64, m.w, m.rows, m.cols);
}

cudaError_t launch_q8_tc_single_i8(const Q8View& m, const int8_t* xq, const float* xs, int batch,
                                   float* y, long long ldy, unsigned* status, cudaStream_t st) {
  if (!q8_tc_supported(static_cast<int>(m.rows), static_cast<int>(m.cols)) || batch < 1)
    return cudaErrorInvalidValue;
  if (!aligned16(m.w) || !aligned16(m.s) || !aligned16(xq) || !aligned16(xs))
    return cudaErrorMisalignedAddress;
  const int N = static_cast<int>(m.rows), K = static_cast<int>(m.cols);
  TcMatrixMaps mm;
  CUtensorMap tx, txs;
  if (!q8_tc_weight_maps(&mm, m) || !make_map_i8(&tx, xq, batch, K, kBM) ||
      !make_map_f32(&txs, xs, batch, K / 32, kBM))
    return cudaErrorInvalidValue;
  configure();
  TcArgs a{};
  a.groups = 1;
  a.y = y;
  a.M = batch;
  a.N = N;
  a.K = K;
  a.ldy = static_cast<int>(ldy);
  a.status = status;
  q8_tc_gemm_i8_kernel<<<persistent_grid(static_cast<long long>(N / kBN) * ((batch + kBM - 1) / kBM), kMaxCtaTiles),
                         kThreads, kSmemBytes, st>>>(mm.w_sw128, mm.ws, tx, txs, a);
  return cudaGetLastError();
}

cudaError_t launch_q8_tc_grouped_i8(const void* maps, int groups, const int* counts,
                                    const int* offsets, int max_tiles, int N, int K,
                                    const int8_t* xq, const float* xs, int total_rows, float* y,
                                    long long ldy, unsigned* status, cudaStream_t st) {
  if (N % kBN || K % kBK || total_rows < 1 || max_tiles < 1) return cudaErrorInvalidValue;
  if (!aligned16(xq) || !aligned16(xs) || reinterpret_cast<uintptr_t>(maps) % 64)
    return cudaErrorMisalignedAddress;
  CUtensorMap tx, txs;
  if (!make_map_i8(&tx, xq, total_rows, K, kBM) || !make_map_f32(&txs, xs, total_rows, K / 32, kBM))
    return cudaErrorInvalidValue;
  configure();
  TcArgs a{};
  a.maps = static_cast<const TcMatrixMaps*>(maps);
  a.counts = counts;
  a.offsets = offsets;
  a.groups = groups;
  a.y = y;
  a.M = total_rows;
  a.N = N;
  a.K = K;
  a.ldy = static_cast<int>(ldy);
  a.status = status;
  // the weight-map parameters are unused when grouped (the maps array is)
  q8_tc_gemm_i8_kernel<<<persistent_grid(static_cast<long long>(N / kBN) * max_tiles, kMaxCtaTiles), kThreads,
                         kSmemBytes, st>>>(tx, txs, tx, txs, a);
  return cudaGetLastError();
}

cudaError_t launch_q8_tc_single_f32(const Q8View& m, const uint16_t* pieces, const float* rinv,
                                    int batch, float* y, long long ldy, unsigned* status,
                                    cudaStream_t st) {
  if (!q8_tc_supported(static_cast<int>(m.rows), static_cast<int>(m.cols)) || batch < 1)
    return cudaErrorInvalidValue;
  if (!aligned16(m.w) || !aligned16(m.s) || !aligned16(pieces)) return cudaErrorMisalignedAddress;
  const int N = static_cast<int>(m.rows), K = static_cast<int>(m.cols);
  if (N / kBN > 32767) return cudaErrorInvalidValue;  // the tile list packs the weight tile in 15 bits
  CUtensorMap tw, tp, tp16, tp32;
  if (!make_map_w_rows64(&tw, m.w, N, K) || !make_map_pieces(&tp, pieces, batch, K, kBM) ||
      !make_map_pieces(&tp16, pieces, batch, K, 16) || !make_map_pieces(&tp32, pieces, batch, K, 32))
    return cudaErrorInvalidValue;
  configure();
  TcF32Args a{};
  a.groups = 1;
  a.s = m.s;
  a.rinv = rinv;
  a.y = y;
  a.M = batch;
  a.N = N;
  a.K = K;
  a.ldy = static_cast<int>(ldy);
  a.piece_rows = batch;
  a.status = status;
  q8_tc_gemm_f32_kernel<<<persistent_grid(static_cast<long long>(N / kBN) * ((batch + kBM - 1) / kBM),
                                           kFMaxCtaTiles),
                          kFThreads, kFSmemBytes, st>>>(tw, tp, tp16, tp32, a);
  return cudaGetLastError();
}

cudaError_t launch_q8_tc_grouped_f32(const void* maps, int groups, const int* counts,
                                     const int* offsets, int max_tiles, int N, int K,
                                     const uint16_t* pieces, const float* rinv, int total_rows,
                                     float* y, long long ldy, unsigned* status, cudaStream_t st) {
  if (N % kBN || K % kBK || total_rows < 1 || max_tiles < 1 || N / kBN > 32767 || groups > 256)
    return cudaErrorInvalidValue;
  if (!aligned16(pieces) || reinterpret_cast<uintptr_t>(maps) % 64) return cudaErrorMisalignedAddress;
  CUtensorMap tp, tp16, tp32;
  if (!make_map_pieces(&tp, pieces, total_rows, K, kBM) ||
      !make_map_pieces(&tp16, pieces, total_rows, K, 16) ||
      !make_map_pieces(&tp32, pieces, total_rows, K, 32))
    return cudaErrorInvalidValue;
  configure();
  TcF32Args a{};
  a.maps = static_cast<const TcMatrixMaps*>(maps);
  a.counts = counts;
  a.offsets = offsets;
  a.groups = groups;
  a.rinv = rinv;
  a.y = y;
  a.M = total_rows;
  a.N = N;
  a.K = K;
  a.ldy = static_cast<int>(ldy);
  a.piece_rows = total_rows;
  a.status = status;
  // the weight-map parameter is unused when grouped (the maps array is)
  q8_tc_gemm_f32_kernel<<<persistent_grid(static_cast<long long>(N / kBN) * max_tiles, kFMaxCtaTiles),
                          kFThreads, kFSmemBytes, st>>>(tp, tp, tp16, tp32, a);
  return cudaGetLastError();
}

void launch_split_rows(const float* x, long long ld_x, const int* src, int rows, int cols,
                       uint16_t* pieces, float* rinv, int sms, cudaStream_t st, const int* live) {
  if (rows <= 0) return;
  if (cols <= 4 * kSplitThreads * kSplitMaxV)
    launch_dependent(split_rows_cta_kernel<false>, dim3(rows), dim3(kSplitThreads), 0, st, x, ld_x,
                     src, static_cast<const float*>(nullptr), rows, cols, pieces, rinv,
                     static_cast<long long>(rows) * cols, live);
  else
    split_rows_kernel<<<grid_for(static_cast<long long>(rows) * 32, sms), 256, 0, st>>>(
        x, ld_x, src, rows, cols, pieces, rinv, static_cast<long long>(rows) * cols, live);
}

void launch_swiglu_split(const float* g, const float* u, int rows, int cols, uint16_t* pieces,
                         float* rinv, int sms, cudaStream_t st, const int* live) {
  if (rows <= 0) return;
  if (cols <= 4 * kSplitThreads * kSplitMaxV)
    launch_dependent(split_rows_cta_kernel<true>, dim3(rows), dim3(kSplitThreads), 0, st, g,
                     static_cast<long long>(cols), static_cast<const int*>(nullptr), u, rows, cols,
                     pieces, rinv, static_cast<long long>(rows) * cols, live);
  else
    swiglu_split_kernel<<<grid_for(static_cast<long long>(rows) * 32, sms), 256, 0, st>>>(
        g, u, rows, cols, pieces, rinv, static_cast<long long>(rows) * cols, live);
}

void launch_gather_rows(const int8_t* xq, const float* xs, const int* src, int rows, int cols,
                        int8_t* xq_p, float* xs_p, int sms, cudaStream_t st, const int* live) {
  gather_rows_kernel<<<grid_for(static_cast<long long>(rows) * (cols / 16), sms), 256, 0, st>>>(
      xq, xs, src, rows, cols, xq_p, xs_p, live);
}

void launch_swiglu_quantize(const float* g, const float* u, int rows, int cols, int8_t* hq,
                            float* hs, unsigned* status, int sms, cudaStream_t st,
                            const int* live) {
  const long long warps = static_cast<long long>(rows) * (cols / 32);
  swiglu_quantize_kernel<<<grid_for(warps * 32, sms), 256, 0, st>>>(g, u, rows, cols, hq, hs,
                                                                     status, live);
}

bool linear_bf16_tc_supported(int n, int k) { return n > 0 && k > 0 && k % kHK == 0; }

cudaError_t launch_linear_bf16_tc(const uint16_t* w, int n, int k, const uint16_t* pieces,
                                  const float* rinv, int batch, float* y, long long ldy,
                                  unsigned* status, int sms, cudaStream_t st) {
  if (!linear_bf16_tc_supported(n, k) || batch < 1) return cudaErrorInvalidValue;
  if (!aligned16(w) || !aligned16(pieces)) return cudaErrorMisalignedAddress;
  const int box = batch <= 16 ? 16 : batch <= 32 ? 32 : kBM;
  CUtensorMap tw, tx;
  if (!make_map_bf16_sw128(&tw, w, n, k) || !make_map_pieces(&tx, pieces, batch, k, box))
    return cudaErrorInvalidValue;
  static PerDeviceOnce configured;
  configured.run([] {
    cudaFuncSetAttribute(bf16_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kHSmemBytes);
  });
  HeadArgs a{};
  a.rinv = rinv;
  a.y = y;
  a.n = n;
  a.k = k;
  a.batch = batch;
  a.ldy = static_cast<int>(ldy);
  a.piece_rows = batch;
  a.box = box;
  a.n_tiles = (n + kBN - 1) / kBN;
  a.row_tiles = (batch + kBM - 1) / kBM;
  a.status = status;
  const int total = a.n_tiles * a.row_tiles;
  const int grid = total < sms ? total : sms;
  bf16_head_kernel<<<grid, kHThreads, kHSmemBytes, st>>>(tw, tx, a);
  return cudaGetLastError();
}

}  // namespace uocr
