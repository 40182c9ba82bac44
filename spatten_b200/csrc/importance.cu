// Deterministic reduction of the attention kernel's per-CTA importance partials.
//
//   tok_out[z, n]  = tok_in[z, n] + sum_{h, tile} tok_partial[z, h, tile, n]
//   head_out[h]    = sum_{z, tile} head_partial[z, h, tile]
//
// Token importance is the reference's attention_probs.sum(dim=(1, 2)) and
// the cumulative `+=` (spatten_bert.py:136-142); head importance is the sum
// behind context_layer.abs().mean(dim=(0, 2, 3)) (spatten_bert.py:120-121).
// Every output element is summed by one thread in a fixed order, in fp64, so
// the result does not depend on scheduling and the rounding error of the sum
// stays far below the gaps that the top-k decisions depend on.
#include "common.cuh"
#include "kernels.h"

namespace spatten {

__global__ void tok_reduce_kernel(const float* __restrict__ part, int Z, int H, int mtiles, int N,
                                  const float* __restrict__ tok_in, float* __restrict__ tok_out) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int z = blockIdx.y;
  if (n >= N) return;
  const int64_t stride = N;
  const float* p = part + (int64_t)z * H * mtiles * stride + n;
  double acc = 0.0;
  const int cnt = H * mtiles;
  // batches of 16 loads in flight, summed in the same fixed order
  int i = 0;
  for (; i + 16 <= cnt; i += 16) {
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __ldg(p + (int64_t)(i + j) * stride);
#pragma unroll
    for (int j = 0; j < 16; ++j) acc += (double)v[j];
  }
  for (; i < cnt; ++i) acc += (double)__ldg(p + (int64_t)i * stride);
  float r = (float)acc;
  if (tok_in) r = tok_in[(int64_t)z * N + n] + r;
  tok_out[(int64_t)z * N + n] = r;
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
    dim3 grid((N + 255) / 256, Z);
    tok_reduce_kernel<<<grid, 256, 0, st>>>(tok_partial, Z, H, mtiles, N, tok_in, tok_out);
  }
  if (head_out) head_reduce_kernel<<<H, 256, 0, st>>>(head_partial, Z, H, mtiles, head_out);
  return cudaGetLastError();
}

}  // namespace spatten
