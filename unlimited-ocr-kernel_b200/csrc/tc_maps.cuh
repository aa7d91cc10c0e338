// tc_maps.cuh — TMA tensor maps shared by the tensor-core kernels (q8_tc.cu,
// q8_small.cu): the per-matrix map set and the builders of each layout.
#pragma once

#include <cuda.h>  // CUtensorMap and its enums (types only)
#include <cudaTypedefs.h>
#include <stdint.h>

#include "common.cuh"

namespace uocr {

// Everything the tensor-core kernels need of one weight matrix, built once
// per matrix on the host (q8_tc_weight_maps) and read by the kernels from
// device memory in grouped launches.
struct alignas(64) TcMatrixMaps {
  CUtensorMap w_sw128;   // int8 weights, 128-byte K boxes x 128 rows, 128-byte swizzle
  CUtensorMap ws;        // weight scales, 4-block boxes x 128 rows
  CUtensorMap w_rows64;  // int8 weights, 64-byte K boxes x 128 rows, unswizzled
  const float* s;        // weight scales [rows][nb] (FP32-activation epilogue)
  int nb;                // scale blocks per row
};

// 2-D TMA tile load into shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (null when
// the driver lacks it).
PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn();
// int8 [rows][cols], box 128 bytes x box_rows, 128-byte swizzle.
bool make_map_i8(CUtensorMap* map, const void* base, long long rows, long long cols, int box_rows);
// int8 [rows][cols], box 128 bytes x box_rows, unswizzled.
bool make_map_i8_plain(CUtensorMap* map, const void* base, long long rows, long long cols,
                       int box_rows);
// float [rows][nb] block scales, box 4 blocks x box_rows.
bool make_map_f32(CUtensorMap* map, const float* base, long long rows, long long nb, int box_rows);
// float [rows][cols], box 32 floats (128 bytes) x 32 rows, 128-byte swizzle
// (token-major KV rows for the decode attention kernel).
bool make_map_f32_sw128(CUtensorMap* map, const float* base, long long rows, long long cols,
                        int box_rows = 32);
// int8 weights [rows][cols], box 64 bytes x 128 rows, unswizzled.
bool make_map_w_rows64(CUtensorMap* map, const void* base, long long rows, long long cols);
// bf16 pieces [3 * piece_rows][cols], box 64 elements x box_rows, 128-byte swizzle.
bool make_map_pieces(CUtensorMap* map, const uint16_t* base, long long piece_rows, long long cols,
                     int box_rows);
// bf16 weights [rows][cols], box 64 elements x 128 rows, 128-byte swizzle.
bool make_map_bf16_sw128(CUtensorMap* map, const uint16_t* base, long long rows, long long cols);
// bf16 pieces [3 * piece_rows][cols], box 128 elements x box_rows, unswizzled.
bool make_map_pieces_plain(CUtensorMap* map, const uint16_t* base, long long piece_rows,
                           long long cols, int box_rows);

}  // namespace uocr
