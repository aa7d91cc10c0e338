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
  float* p = route_smem + warp * (n_experts + 2 * top_k);
  int* sel = reinterpret_cast<int*>(p + n_experts);
  float* wts = p + n_experts + top_k;
  for (int t = blockIdx.x * kRouteWarps + warp; t < tokens; t += gridDim.x * kRouteWarps) {
    if (route_row_warp(logits + static_cast<long long>(t) * n_experts, n_experts, top_k,
                       normalize, scale, p, sel, wts, status)) {
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
