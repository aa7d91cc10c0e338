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
// small-integer conversion via the float mantissa).
__device__ __forceinline__ float byte_as_float(uint32_t flipped_word, uint32_t sel) {
  return __uint_as_float(__byte_perm(flipped_word, 0x4B000000u, sel)) - 8388736.0f;
}

// Dot of 4 int8 weights (packed in w) with 4 floats, accumulated in fp32.
__device__ __forceinline__ float dot4_i8_f32(uint32_t w, float4 x) {
  const uint32_t f = w ^ 0x80808080u;
  float d = byte_as_float(f, 0x7770) * x.x;
  d = fmaf(byte_as_float(f, 0x7771), x.y, d);
  d = fmaf(byte_as_float(f, 0x7772), x.z, d);
  d = fmaf(byte_as_float(f, 0x7773), x.w, d);
  return d;
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

// Reference quantizer element (src/cpu/quantized.rs:64-69): 0 for a zero
// scale, else clamp(round_half_even(v / scale), -127, 127).
__device__ __forceinline__ int8_t quantize_elem(float v, float scale) {
  if (scale == 0.0f) return 0;
  int q = __float2int_rn(__fdiv_rn(v, scale));
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  return static_cast<int8_t>(q);
}

}  // namespace uocr
