// Deterministic reduction of the attention kernel's per-CTA importance partials.
//
//   tok_out[z, n]  = tok_in[z, n] + sum_{h, tile} tok_partial[z, h, tile, n]
//   head_out[h]    = sum_{z, tile} head_partial[z, h, tile]
//
// Token importance is the reference's attention_probs.sum(dim=(1, 2)) and
// the cumulative `+=` (spatten_bert.py:136-142); head importance is the sum
// behind context_layer.abs().mean(dim=(0, 2, 3)) (spatten_bert.py:120-121).
// Every output element is summed in fp64 in a fixed order (four fixed row
// ranges, then their four sums), so the result does not depend on
// scheduling and the rounding error of the sum stays far below the gaps that
// the top-k decisions depend on.
#include "common.cuh"
#include "kernels.h"

namespace spatten {

// A block covers 64 key columns of one batch row; its 4 row groups (64
// threads each) sum consecutive quarters of the H * mtiles partial rows of a
// column, each in fp64 in a fixed order, and the four quarter sums are added
// in a fixed order: deterministic, with 4x the loads in flight of one thread
// per column.
constexpr int kTokCols = 64, kTokGroups = 4;

__global__ void __launch_bounds__(kTokCols * kTokGroups)
    tok_reduce_kernel(const float* __restrict__ part, int Z, int H, int mtiles, int N,
                      const float* __restrict__ tok_in, float* __restrict__ tok_out) {
  __shared__ double qs[kTokGroups][kTokCols];
  const int c = threadIdx.x % kTokCols, rg = threadIdx.x / kTokCols;
  const int n = blockIdx.x * kTokCols + c;
  const int z = blockIdx.y;
  const int64_t stride = N;
  const int cnt = H * mtiles;
  const int r0 = (int)((int64_t)cnt * rg / kTokGroups), r1 = (int)((int64_t)cnt * (rg + 1) / kTokGroups);
  double acc = 0.0;
  if (n < N) {
    const float* p = part + (int64_t)z * cnt * stride + n;
    int i = r0;
    for (; i + 8 <= r1; i += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __ldg(p + (int64_t)(i + j) * stride);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc += (double)v[j];
    }
    for (; i < r1; ++i) acc += (double)__ldg(p + (int64_t)i * stride);
  }
  qs[rg][c] = acc;
  __syncthreads();
  if (rg == 0 && n < N) {
    float r = (float)(((qs[0][c] + qs[1][c]) + qs[2][c]) + qs[3][c]);
    if (tok_in) r = tok_in[(int64_t)z * N + n] + r;
    tok_out[(int64_t)z * N + n] = r;
  }
}

__global__ void head_reduce_kernel(const float* __restrict__ part, int Z, int H, int mtiles,
                                   float* __restrict__ head_out) {
  __shared__ double sh[256];
  const int h = blockIdx.x;
  double acc = 0.0;
  const int cnt = Z * mtiles;
  for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
    const int z = i / mtiles, t = i % mtiles;
    acc += (double)part[((int64_t)z * H + h) * mtiles + t];
  }
  sh[threadIdx.x] = acc;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) head_out[h] = (float)sh[0];
}

cudaError_t launch_importance_reduce(const float* tok_partial, const float* head_partial, int Z,
                                     int H, int mtiles, int N, const float* tok_in,
                                     float* tok_out, float* head_out, cudaStream_t st) {
  if (tok_out) {
    dim3 grid((N + kTokCols - 1) / kTokCols, Z);
    tok_reduce_kernel<<<grid, kTokCols * kTokGroups, 0, st>>>(tok_partial, Z, H, mtiles, N, tok_in, tok_out);
  }
  if (head_out) head_reduce_kernel<<<H, 256, 0, st>>>(head_partial, Z, H, mtiles, head_out);
  return cudaGetLastError();
}

}  // namespace spatten
