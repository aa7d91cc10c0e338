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

// Two rows of the same width K (K % 256 == 0) treated as one 2K-byte vector of
// 16-byte chunks; lane l owns chunks l, l+32, ... (CPL = K/256 of them), so a
// lane always meets the same x positions and keeps them in registers.
template <int CPL>
__device__ __forceinline__ void load_pair_x(const float* xsm, int K, int lane, float4 (&xr)[CPL][4]) {
  const int per_row = K >> 4;
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c = lane + 32 * j;
    const int kc = c < per_row ? c : c - per_row;
#pragma unroll
    for (int q = 0; q < 4; ++q) xr[j][q] = *reinterpret_cast<const float4*>(xsm + 16 * kc + 4 * q);
  }
}

// FP32-mode dots of two rows sharing x (gate/up rows of one index, or two
// rows of one matrix).  Returns the warp-reduced sums in o0 / o1.
template <int CPL>
__device__ __forceinline__ void pair_dot_xregs(const int8_t* r0, const float* s0, const int8_t* r1,
                                               const float* s1, int K, const float4 (&xr)[CPL][4],
                                               int lane, float& o0, float& o1) {
  const int per_row = K >> 4;
  float a0 = 0.0f, a1 = 0.0f;
  uint4 w[CPL];
  float s[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c = lane + 32 * j;
    const bool second = c >= per_row;
    const int kc = second ? c - per_row : c;
    w[j] = *reinterpret_cast<const uint4*>((second ? r1 : r0) + 16 * kc);
    s[j] = (second ? s1 : s0)[kc >> 1];
  }
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c = lane + 32 * j;
    const float v = chunk16_dot(w[j], xr[j]);
    if (c >= per_row)
      a1 = fmaf(s[j], v, a1);
    else
      a0 = fmaf(s[j], v, a0);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a0 += __shfl_xor_sync(0xffffffffu, a0, o);
    a1 += __shfl_xor_sync(0xffffffffu, a1, o);
  }
  o0 = a0;
  o1 = a1;
}

// FP32-mode dot of one row against x in shared memory (any K % 16 == 0).
__device__ __forceinline__ float row_dot_xsmem(const int8_t* wrow, const float* srow,
                                               const float* xsm, int K, int lane) {
  float acc0 = 0.0f, acc1 = 0.0f;
  const int chunks = K >> 4;
  int c = lane;
  for (; c + 32 < chunks; c += 64) {
    const uint4 wa = *reinterpret_cast<const uint4*>(wrow + 16 * c);
    const uint4 wb = *reinterpret_cast<const uint4*>(wrow + 16 * (c + 32));
    float4 xa[4], xb[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      xa[q] = *reinterpret_cast<const float4*>(xsm + 16 * c + 4 * q);
      xb[q] = *reinterpret_cast<const float4*>(xsm + 16 * (c + 32) + 4 * q);
    }
    acc0 = fmaf(srow[c >> 1], chunk16_dot(wa, xa), acc0);
    acc1 = fmaf(srow[(c + 32) >> 1], chunk16_dot(wb, xb), acc1);
  }
  if (c < chunks) {
    const uint4 wa = *reinterpret_cast<const uint4*>(wrow + 16 * c);
    float4 xa[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) xa[q] = *reinterpret_cast<const float4*>(xsm + 16 * c + 4 * q);
    acc0 = fmaf(srow[c >> 1], chunk16_dot(wa, xa), acc0);
  }
  return warp_sum(acc0 + acc1);
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

// Bounded wait on an mbarrier phase: gives up after kWaitLimitNs of wall
// time (measured on the global nanosecond timer), flags DEV_TIMEOUT and
// returns false.  Every phase a kernel waits on is completed by its own
// bulk copies or by its own warps, so the limit is only a safety net.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  flag(status, DEV_TIMEOUT);
  return false;
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

// Programmatic dependent launch controls (no-ops when launched without PDL).
__device__ __forceinline__ void pdl_wait_prior_grids() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Reference quantizer element (src/cpu/quantized.rs:64-69): 0 for a zero
// scale, else clamp(round_half_even(v / scale), -127, 127).
__device__ __forceinline__ int8_t quantize_elem(float v, float scale) {
  if (scale == 0.0f) return 0;
  int q = __float2int_rn(__fdiv_rn(v, scale));
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  return static_cast<int8_t>(q);
}

}  // namespace uocr
