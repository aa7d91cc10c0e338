// moe_route.cu — batched moe::route: one warp per token.
#include "kernels.h"
#include "route.cuh"

namespace uocr {

constexpr int kRouteWarps = 4;

__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(
    const float* __restrict__ logits, int tokens, int n_experts, int top_k, int normalize,
    float scale, int32_t* __restrict__ ids, float* __restrict__ weights, unsigned* status) {
  extern __shared__ float route_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // up to 64 experts and 8 kept: the warp-collective form (route_row_warp64,
  // the same IEEE sequence on the warp's reductions); otherwise the general one
  const bool warp64 = n_experts <= 64 && top_k <= 8;
  __shared__ __align__(16) float r64p[kRouteWarps][64];
  __shared__ int r64ids[kRouteWarps][8], r64sorted[kRouteWarps][8];
  __shared__ float r64wts[kRouteWarps][8], r64sorted_w[kRouteWarps][8];
  float* p = route_smem + warp * (n_experts + 2 * top_k);
  int* sel = warp64 ? r64ids[warp] : reinterpret_cast<int*>(p + n_experts);
  float* wts = warp64 ? r64wts[warp] : p + n_experts + top_k;
  for (int t = blockIdx.x * kRouteWarps + warp; t < tokens; t += gridDim.x * kRouteWarps) {
    const float* lrow = logits + static_cast<long long>(t) * n_experts;
    if (warp64 ? route_row_warp64(lrow, n_experts, top_k, normalize, scale, r64p[warp], sel, wts,
                                  r64sorted[warp], r64sorted_w[warp], status)
               : route_row_warp(lrow, n_experts, top_k, normalize, scale, p, sel, wts, status)) {
      for (int r = lane; r < top_k; r += 32) {
        ids[static_cast<long long>(t) * top_k + r] = sel[r];
        weights[static_cast<long long>(t) * top_k + r] = wts[r];
      }
    } else {
      for (int r = lane; r < top_k; r += 32) {
        ids[static_cast<long long>(t) * top_k + r] = -1;
        weights[static_cast<long long>(t) * top_k + r] = 0.0f;
      }
    }
    __syncwarp();
  }
}

void launch_route(const float* logits, int tokens, int n_experts, int top_k, int normalize,
                  float scale, int32_t* ids, float* weights, unsigned* status, int sms,
                  cudaStream_t st) {
  int grid = (tokens + kRouteWarps - 1) / kRouteWarps;
  grid = grid < 1 ? 1 : (grid > sms * 8 ? sms * 8 : grid);
  const size_t smem = sizeof(float) * kRouteWarps * (n_experts + 2 * top_k);
  route_kernel<<<grid, kRouteWarps * 32, smem, st>>>(logits, tokens, n_experts, top_k, normalize,
                                                     scale, ids, weights, status);
}

}  // namespace uocr
