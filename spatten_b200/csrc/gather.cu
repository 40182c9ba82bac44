// Stream-compaction row gather.
//
// Replaces torch.gather of the kept tokens' hidden states and cumulative
// scores (module.py:53-54, 62-63) and torch.index_select of the kept heads'
// rows of the Q/K/V weights and biases (module.py:22-28):
//   dst[b, i*rpi + j, :] = src[b, idx[b, i]*idx_scale + j, :],  j < rpi
// on raw bytes. HBM-bound copy: each thread moves one vector of the widest
// width (16/8/4/1 bytes) that divides every address and stride, grid-stride
// over all destination vectors, grid sized to the SM count. An index outside
// [0, src_rows) zero-fills its destination rows instead of reading.
#include "common.cuh"
#include "kernels.h"

namespace spatten {

template <typename V>
__global__ void __launch_bounds__(256) gather_kernel(
    const uint8_t* __restrict__ src, int64_t src_b, int64_t src_r, int64_t src_rows,
    const int64_t* __restrict__ idx, int64_t idx_b, int B, int K, int rpi, int64_t idx_scale,
    int64_t row_bytes, uint8_t* __restrict__ dst, int64_t dst_b, int64_t dst_r) {
  const int64_t vpr = row_bytes / (int64_t)sizeof(V);  // vectors per row
  const int64_t rows = (int64_t)K * rpi;
  const int64_t total = (int64_t)B * rows * vpr;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t v = e % vpr;
    const int64_t rj = (e / vpr) % rows;
    const int64_t b = e / (vpr * rows);
    const int64_t i = rj / rpi, j = rj % rpi;
    const int64_t sr = __ldg(idx + b * idx_b + i) * idx_scale + j;
    V val;
    if (sr >= 0 && sr < src_rows)
      val = *reinterpret_cast<const V*>(src + b * src_b + sr * src_r + v * (int64_t)sizeof(V));
    else
      memset(&val, 0, sizeof(V));
    *reinterpret_cast<V*>(dst + b * dst_b + rj * dst_r + v * (int64_t)sizeof(V)) = val;
  }
}

static int vec_width(uint64_t a) {
  if (a % 16 == 0) return 16;
  if (a % 8 == 0) return 8;
  if (a % 4 == 0) return 4;
  return 1;
}

cudaError_t launch_gather(const void* src, int64_t src_b, int64_t src_r, const int64_t* idx,
                          int64_t idx_b, int B, int K, int rows_per_idx, int64_t idx_scale,
                          int64_t row_bytes, void* dst, int64_t dst_b, int64_t dst_r,
                          cudaStream_t st, int n_sm, int64_t src_rows) {
  uint64_t a = (uint64_t)row_bytes | (uint64_t)src_b | (uint64_t)src_r | (uint64_t)dst_b |
               (uint64_t)dst_r | (uint64_t)(uintptr_t)src | (uint64_t)(uintptr_t)dst;
  const int w = vec_width(a == 0 ? 16 : (a & (~a + 1)));
  const int64_t total = (int64_t)B * K * rows_per_idx * (row_bytes / w);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)n_sm * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const uint8_t* s = static_cast<const uint8_t*>(src);
  uint8_t* d = static_cast<uint8_t*>(dst);
#define SPATTEN_GL(V)                                                                        \
  gather_kernel<V><<<(unsigned)blocks, 256, 0, st>>>(s, src_b, src_r, src_rows, idx, idx_b, B, K, \
                                                     rows_per_idx, idx_scale, row_bytes, d,  \
                                                     dst_b, dst_r)
  switch (w) {
    case 16: SPATTEN_GL(uint4); break;
    case 8: SPATTEN_GL(uint2); break;
    case 4: SPATTEN_GL(uint32_t); break;
    default: SPATTEN_GL(uint8_t); break;
  }
#undef SPATTEN_GL
  return cudaGetLastError();
}

}  // namespace spatten
