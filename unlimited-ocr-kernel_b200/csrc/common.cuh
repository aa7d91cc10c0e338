// common.cuh — shared device helpers for the q8-block32 kernels (sm_100a).
//
// Conventions used by every kernel in this library:
//  * A matrix is row-major int8 weights [rows x cols] plus one float32 scale
//    per 32-column block, [rows x ceil(cols/32)]; the last block of a row may
//    be short (src/cpu/quantized.rs:9-16 of the reference).
//  * Bit-exact arithmetic uses the _rn intrinsics, which the compiler never
//    contracts into an FMA, and this library is built without fast-math, so
//    denormals are kept (the reference runs with IEEE semantics throughout).
//  * Device-detected input errors never trap: a kernel ORs a bit into the
//    context's status word, the host maps it to a status code at a sync point.
//  * Every spin-wait is bounded; on expiry it records UOCR_DEV_TIMEOUT and
//    the kernel returns.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace uocr {

constexpr int kBlock = 32;

// Bits of the device status word (mapped to uocr_status by the host).
enum DevStatus : unsigned {
  DEV_NONFINITE = 1u << 0,      // quantize / dynamic input held NaN or Inf
  DEV_UNDERFLOW = 1u << 1,      // nonzero block whose scale underflowed to 0
  DEV_BAD_SCALE = 1u << 2,      // scale NaN, Inf or negative
  DEV_RANGE = 1u << 3,          // weight byte -128 in an overlay matrix
  DEV_SOFTMAX = 1u << 4,        // router row with NaN/+inf or no finite max
  DEV_TIMEOUT = 1u << 5,        // a bounded wait expired
  DEV_BAD_ROUTE = 1u << 6,      // expert id outside the layer
  DEV_CAPACITY = 1u << 7,       // more pairs for one rank than the dispatch capacity
  DEV_NORM = 1u << 8,           // normalization row or weight held NaN or Inf
  DEV_POSITION = 1u << 9,       // rotary position outside the table (context exceeded)
  DEV_CACHE = 1u << 10,         // KV cache used before its prefill
};

__device__ __forceinline__ void flag(unsigned* status, unsigned bits) {
  if (status) atomicOr(status, bits);
}

__host__ __device__ __forceinline__ int blocks_of(int cols) { return (cols + kBlock - 1) / kBlock; }

// exp evaluated in double and rounded once to float.  The reference's
// softmax and silu call the platform libm expf (glibc on Linux), whose result
// is the correctly rounded value in all but rare cases; one rounding of a
// double-precision exp reproduces that value except when the exact result
// lies within ~1 double ulp of a float rounding boundary.
__device__ __forceinline__ float exp_f32_via_f64(float v) {
  return __double2float_rn(exp(static_cast<double>(v)));
}

// silu(v) = v / (1 + exp(-v)) with the reference's rounding sequence
// (src/cpu/ops.rs:225-229): one exp, one add, one IEEE division.
__device__ __forceinline__ float silu_ref(float v) {
  return __fdiv_rn(v, __fadd_rn(1.0f, exp_f32_via_f64(-v)));
}

// ---- int8 -> float conversion without the quarter-rate I2F path ----------
// Byte b (two's complement) is flipped to offset binary u = b ^ 0x80 and
// placed in the mantissa of 2^23: float(0x4B000000 | u) = 8388608 + u, so
// subtracting 8388736 = 2^23 + 128 gives b exactly (a published trick for
// small-integer conversion via the float mantissa).  The byte_perm selector
// 0x744N builds the word [byte N of the input, 0x00, 0x00, 0x4B] (bytes 4..7
// address the constant 0x4B000000).
__device__ __forceinline__ float byte_as_float(uint32_t flipped_word, uint32_t sel) {
  return __uint_as_float(__byte_perm(flipped_word, 0x4B000000u, sel)) - 8388736.0f;
}

// Dot of 4 int8 weights (packed in w) with 4 floats, accumulated in fp32.
__device__ __forceinline__ float dot4_i8_f32(uint32_t w, float4 x) {
  const uint32_t f = w ^ 0x80808080u;
  float d = byte_as_float(f, 0x7440) * x.x;
  d = fmaf(byte_as_float(f, 0x7441), x.y, d);
  d = fmaf(byte_as_float(f, 0x7442), x.z, d);
  d = fmaf(byte_as_float(f, 0x7443), x.w, d);
  return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- packed f32x2 arithmetic (sm_100: two fp32 lanes per instruction) -----
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Two IEEE products, each rounded on its own; lane for lane bit-identical to
// __fmul_rn, subnormals included (checked on ten million pairs of arbitrary
// bit patterns).  Its result must not feed a packed add (f2_add) where the
// two roundings matter: the PTX assembler (CUDA 12.9) fuses a mul.rn.f32x2
// whose result feeds an add.rn.f32x2 into one fused multiply-add despite the
// rounding modifiers (about 23% of 2 million random pairs differed from the
// separately rounded operations, every one equal to the fused result, with or
// without -fmad=false, and in a running sum even with the product moved
// through another register first; also when the add is written as a packed
// fma(product, 1, acc)).  Add such a product with __fadd_rn per lane: that
// pairing stays separately rounded (measured over running sums of 40 blocks),
// and the bit-exact int8 tests hold it.
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mov.b64 rc, {%6, %7};\n fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// Dot of 16 int8 weights (one 16-byte chunk, inside one 32-column block) with
// 16 floats: two packed accumulators, magic-number conversion (above).
__device__ __forceinline__ float chunk16_dot(uint4 w, const float4 (&x)[4]) {
  const float2 C = make_float2(-8388736.0f, -8388736.0f);
  float2 a0 = make_float2(0.0f, 0.0f), a1 = make_float2(0.0f, 0.0f);
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t f = words[q] ^ 0x80808080u;
    float2 lo = make_float2(__uint_as_float(__byte_perm(f, 0x4B000000u, 0x7440)),
                            __uint_as_float(__byte_perm(f, 0x4B000000u, 0x7441)));
    float2 hi = make_float2(__uint_as_float(__byte_perm(f, 0x4B000000u, 0x7442)),
                            __uint_as_float(__byte_perm(f, 0x4B000000u, 0x7443)));
    lo = f2_add(lo, C);
    hi = f2_add(hi, C);
    a0 = f2_fma(lo, make_float2(x[q].x, x[q].y), a0);
    a1 = f2_fma(hi, make_float2(x[q].z, x[q].w), a1);
  }
  const float2 s = f2_add(a0, a1);
  return s.x + s.y;
}

// Barrier among `threads` threads (whole warps) of the CTA, id 1..15.
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// x staged in shared memory in "chunk-transposed" order: float4 q (q = 0..3)
// of 16-float chunk c is stored at index q*C + c (C = n/16 chunks), so when
// lane l reads part q of chunk l, consecutive lanes read consecutive 16-byte
// words (no bank conflicts).  n % 16 == 0.
__device__ __forceinline__ void stage_x_transposed(float* dst, const float* __restrict__ src, int n,
                                                   int tid, int nthreads) {
  const int C = n >> 4;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  int i = tid;
  for (; i + 3 * nthreads < 4 * C; i += 4 * nthreads) {  // 4 loads in flight per thread
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldg(s4 + i + u * nthreads);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = i + u * nthreads;
      d4[(k & 3) * C + (k >> 2)] = v[u];
    }
  }
  for (; i < 4 * C; i += nthreads) d4[(i & 3) * C + (i >> 2)] = __ldg(s4 + i);
}

// FP32-mode dots of 4 rows of width K (K % 16 == 0) against one x vector
// staged chunk-transposed in shared memory (xT).  Lane l walks the 16-byte
// weight chunks l, l+32, ...; each x chunk is loaded once and used by all 4
// rows (4 independent accumulation chains).  The 4 warp sums are formed by a
// transposed butterfly (6 shuffles instead of 20): afterwards lane l holds the
// sum of row 2*bit4(l) + bit3(l), i.e. row 0 in lanes 0-7, row 1 in lanes
// 8-15, row 2 in lanes 16-23, row 3 in lanes 24-31.
__device__ __forceinline__ float rows4_dot_xsmem(const int8_t* r0, const int8_t* r1,
                                                 const int8_t* r2, const int8_t* r3,
                                                 const float* s0, const float* s1,
                                                 const float* s2, const float* s3,
                                                 const float* xT, int K, int lane) {
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  const int chunks = K >> 4;
  const float4* x4 = reinterpret_cast<const float4*>(xT);
#pragma unroll 1
  for (int c = lane; c < chunks; c += 32) {
    float4 xv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) xv[q] = x4[q * chunks + c];
    const uint4 w0 = *reinterpret_cast<const uint4*>(r0 + 16 * c);
    const uint4 w1 = *reinterpret_cast<const uint4*>(r1 + 16 * c);
    const uint4 w2 = *reinterpret_cast<const uint4*>(r2 + 16 * c);
    const uint4 w3 = *reinterpret_cast<const uint4*>(r3 + 16 * c);
    const int b = c >> 1;
    a0 = fmaf(s0[b], chunk16_dot(w0, xv), a0);
    a1 = fmaf(s1[b], chunk16_dot(w1, xv), a1);
    a2 = fmaf(s2[b], chunk16_dot(w2, xv), a2);
    a3 = fmaf(s3[b], chunk16_dot(w3, xv), a3);
  }
  const bool hi16 = lane & 16;
  float k0 = hi16 ? a2 : a0, k1 = hi16 ? a3 : a1;
  k0 += __shfl_xor_sync(0xffffffffu, hi16 ? a0 : a2, 16);
  k1 += __shfl_xor_sync(0xffffffffu, hi16 ? a1 : a3, 16);
  const bool hi8 = lane & 8;
  float k = hi8 ? k1 : k0;
  k += __shfl_xor_sync(0xffffffffu, hi8 ? k0 : k1, 8);
  k += __shfl_xor_sync(0xffffffffu, k, 4);
  k += __shfl_xor_sync(0xffffffffu, k, 2);
  k += __shfl_xor_sync(0xffffffffu, k, 1);
  return k;
}

// linear_dynamic_int8's ordered row dot (src/cpu/quantized.rs:155-236) for
// four rows at once, one warp: lane l owns bytes [4l, 4l + 4) of every
// 128-byte window (block = window * 4 + l / 8); per window and row the exact
// int32 block sums S (dp4a, then a reduction over the block's 8 lanes), then
// acc = acc + ((float)S * ws) * xs block by block from -0.0.  The four rows'
// chains are interleaved so that their shuffles and ordered sums overlap;
// each row's result is that of the row on its own.
__device__ __forceinline__ void rows4_dot_int8(const int8_t* const (&wr)[4],
                                               const float* const (&sr)[4], const int8_t* xq,
                                               const float* xs, int cols, int lane,
                                               float (&out)[4]) {
  float acc[4] = {-0.0f, -0.0f, -0.0f, -0.0f};
  for (int k0 = lane * 4; k0 < cols; k0 += 128) {
    const int b = k0 >> 5;
    const int xv = *reinterpret_cast<const int*>(xq + k0);
    const float xsb = xs[b];
    int p[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) p[r] = __dp4a(*reinterpret_cast<const int*>(wr[r] + k0), xv, 0);
#pragma unroll
    for (int m = 1; m <= 4; m <<= 1)
#pragma unroll
      for (int r = 0; r < 4; ++r) p[r] += __shfl_xor_sync(0xffffffffu, p[r], m);
    float t[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) t[r] = __fmul_rn(__fmul_rn(static_cast<float>(p[r]), sr[r][b]), xsb);
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[r] = __fadd_rn(acc[r], __shfl_sync(0xffffffffu, t[r], 8 * q));
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) out[r] = acc[r];
}

// ---- mbarrier / bulk-copy PTX wrappers --------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait limits.  Bounds are measured with the SM's cycle counter (clock64 is
// a cheap register read; the global nanosecond timer is a slow
// memory-mapped read that would delay every retry).  4e9 cycles is about
// 2 s at the 1.965 GHz maximum clock and longer at lower clocks.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // for global_ns() users
constexpr long long kWaitLimitCycles = 4000000000ll;

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or the hint (ns) expires, instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(100000u)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase: gives up after kWaitLimitCycles, flags
// DEV_TIMEOUT and returns false.  Every phase a kernel waits on is completed
// by its own bulk copies or by its own warps, so the limit is a safety net.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (clock64() - t0 > kWaitLimitCycles) break;
  }
  flag(status, DEV_TIMEOUT);
  return false;
}

// Latency-critical bounded wait: polls with test_wait (never suspends the
// thread), for hand-offs where a suspended waiter would wake late.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, unsigned* status) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_test_wait(bar, parity)) {
    if (clock64() - t0 > kWaitLimitCycles) {
      flag(status, DEV_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Bounded wait through mbarrier.try_wait without a time hint: between polls
// the hardware may suspend the thread until the phase completes, so warps
// that wait leave their issue slots to the warps doing the work (a test_wait
// spin by many warps starves the workers of the same scheduler).
__device__ __forceinline__ bool mbar_wait_try(uint64_t* bar, uint32_t parity, unsigned* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitLimitCycles) {
      flag(status, DEV_TIMEOUT);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared, completion signalled on `bar` as tx bytes.
// Both addresses 16-byte aligned, bytes a multiple of 16 (checked by callers).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Launch on `st` as a programmatic dependent of the previous kernel in the
// stream (cudaLaunchAttributeProgrammaticStreamSerialization), so that its
// launch overlaps the previous kernel's end.  The kernel must call
// pdl_wait_prior_grids() before it reads or writes anything the previous
// kernel touches (the chain kernels below call it first thing).  Falls back
// to ordinary stream order when the attribute is refused.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t st, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    cfg.numAttrs = 0;
    e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  }
  return e;
}

// Programmatic dependent launch controls (no-ops when launched without PDL).
__device__ __forceinline__ void pdl_wait_prior_grids() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes a
// multiple of 16).  Issued before pdl_wait_prior_grids() by kernels whose
// first tiles are weights or cached keys: the fetch overlaps the previous
// kernel's tail.  It is safe even when the previous kernel writes those
// bytes: L2 is where every store of the GPU lands, so a line fetched early is
// updated by such a store, and the kernel reads it only after the wait.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Reference quantizer element (src/cpu/quantized.rs:64-69): 0 for a zero
// scale, else clamp(round_half_even(v / scale), -127, 127).
__device__ __forceinline__ int8_t quantize_elem(float v, float scale) {
  if (scale == 0.0f) return 0;
  int q = __float2int_rn(__fdiv_rn(v, scale));
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  return static_cast<int8_t>(q);
}

// Block quantization of v[0, n) in shared memory (16-byte aligned) into q and
// s (shared memory), the activation step of linear_dynamic_int8
// (src/cpu/quantized.rs:43-74 applied at :169), by the `nt` threads
// tid in [0, nt) of a named barrier `bar`.  Two short steps: one thread per
// 32-element block takes the block's max |v| (the reference folds from 0
// with f32::max, which ignores NaN like fmaxf; a max does not depend on the
// order) and the scale max / 127; then every element is divided by its
// block's scale on its own.  (One warp per block instead chains a block's
// shuffles and two dependent divisions, block after block.)  Lane-rotated
// 16-byte reads keep the per-block scans free of bank conflicts.
__device__ __forceinline__ void quantize_blocks_smem(const float* v, int n, int8_t* q, float* s,
                                                     int tid, int nt, int bar, unsigned* status) {
  const int nb = blocks_of(n);
  for (int b = tid; b < nb; b += nt) {
    const int k0 = b * kBlock;
    float mx = 0.0f;
    bool bad = false;
    if (k0 + kBlock <= n) {
      const float4* v4 = reinterpret_cast<const float4*>(v + k0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 c = v4[(j + b) & 7];
        bad |= !isfinite(c.x) || !isfinite(c.y) || !isfinite(c.z) || !isfinite(c.w);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(c.x), fabsf(c.y)), fmaxf(fabsf(c.z), fabsf(c.w))));
      }
    } else {
      for (int k = k0; k < n; ++k) {
        bad |= !isfinite(v[k]);
        mx = fmaxf(mx, fabsf(v[k]));
      }
    }
    const float scale = __fdiv_rn(mx, 127.0f);
    if (bad) flag(status, DEV_NONFINITE);
    if (mx > 0.0f && scale == 0.0f) flag(status, DEV_UNDERFLOW);
    s[b] = scale;
  }
  named_barrier(bar, nt);
#pragma unroll 4
  for (int k = tid; k < n; k += nt) q[k] = quantize_elem(v[k], s[k / kBlock]);
}

}  // namespace uocr
