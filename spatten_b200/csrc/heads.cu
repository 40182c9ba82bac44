// Head selection of the cascade in one small launch: the head importance
// (the per-head mean |context|, spatten_bert.py:120-121), its top-`keep`
// heads in ascending position (ties at the k-th value to the smaller
// position, as spatten_topk_indices orders them), and those positions mapped
// through the layer's active head list (module.py:89: the next layer's
// active heads). Replaces a division, a top-k and an index gather per layer,
// and emits the int32 copy of the next heads that the attention kernel's
// head-slot map reads.
//
// One CTA of up to 1024 threads, a thread per head: a head's rank is the
// number of heads ahead of it in (value descending, position ascending).
#include "common.cuh"
#include "kernels.h"

namespace spatten {

namespace {

// imp_out may be imp_in (each thread reads its value before any write)
__global__ void __launch_bounds__(1024) select_heads_kernel(const float* imp_in, float scale,
                                                             const int64_t* __restrict__ heads, int cur,
                                                             int keep, float* imp_out,
                                                             int64_t* __restrict__ next_heads,
                                                             int32_t* __restrict__ next_heads32) {
  __shared__ uint32_t key[1024];
  __shared__ int sel[1024];
  const int i = threadIdx.x;
  float v = 0.f;
  if (i < cur) {
    v = imp_in[i] * scale;
    key[i] = float_order_key(v);
  }
  __syncthreads();
  int in = 0;
  if (i < cur) {
    const uint32_t ki = key[i];
    int rank = 0;
    for (int j = 0; j < cur; ++j) {
      const uint32_t kj = key[j];
      rank += (kj > ki || (kj == ki && j < i)) ? 1 : 0;
    }
    in = rank < keep;
    sel[i] = in;
  }
  __syncthreads();
  if (i < cur) {
    if (imp_out) imp_out[i] = v;
    if (in) {
      int slot = 0;  // selected positions before i: ascending order
      for (int j = 0; j < i; ++j) slot += sel[j];
      const int64_t h = heads ? heads[i] : (int64_t)i;
      next_heads[slot] = h;
      if (next_heads32) next_heads32[slot] = (int32_t)h;
    }
  }
}

}  // namespace

cudaError_t launch_select_heads(const float* imp_in, float scale, const int64_t* heads, int cur, int keep,
                                float* imp_out, int64_t* next_heads, int32_t* next_heads32, cudaStream_t st) {
  const int threads = ((cur + 31) / 32) * 32;
  select_heads_kernel<<<1, threads, 0, st>>>(imp_in, scale, heads, cur, keep, imp_out, next_heads,
                                              next_heads32);
  return cudaGetLastError();
}

}  // namespace spatten
