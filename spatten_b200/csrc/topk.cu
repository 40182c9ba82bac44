// Radix-select top-k with ordered compaction: the cascade pruning decision.
//
// Replaces sort(topk(x, k).indices) on the head importance [H]
// (spatten_bert.py:123-128) and on the cumulative token importance [B, S]
// (spatten_bert.py:143-148). One CTA per row:
//   1. map every float to an order-preserving 32-bit key;
//   2. four rounds of an 8-bit radix histogram (shared-memory atomics) walk
//      down from the most significant digit to the exact key T of the k-th
//      largest value and the number r of entries equal to T that are kept;
//   3. one ordered stream compaction over the row writes the indices with
//      key > T, plus the first r indices with key == T, in ascending order --
//      no sort is needed. Ties at the k-th value thus go to smaller indices.
// Rows up to kCacheN entries keep their keys in shared memory; longer rows
// re-read the row (L2 resident) on every round.
#include "common.cuh"
#include "kernels.h"

namespace spatten {

namespace {
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kCacheN = 8192;
}  // namespace

__global__ void __launch_bounds__(kThreads) topk_kernel(const float* __restrict__ x, int n,
                                                        int64_t stride, int k,
                                                        int64_t* __restrict__ out) {
  __shared__ uint32_t cache[kCacheN];
  __shared__ int hist[256];
  __shared__ int wsum[kWarps][2];
  __shared__ int s_digit, s_krem;
  const int row = blockIdx.x;
  const float* xr = x + (int64_t)row * stride;
  int64_t* outr = out + (int64_t)row * k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool cached = n <= kCacheN;
  if (cached)
    for (int i = tid; i < n; i += kThreads) cache[i] = float_order_key(xr[i]);
  __syncthreads();
  auto key_at = [&](int i) -> uint32_t { return cached ? cache[i] : float_order_key(xr[i]); };

  uint32_t prefix = 0, mask = 0;
  int krem = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kThreads) {
      const uint32_t u = key_at(i);
      if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns digits [255 - 8l - 7, 255 - 8l], scanned from the top
      int c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - 8 * lane - j];
        tot += c[j];
      }
      int incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int excl = incl - tot;
      if (excl < krem && krem <= incl) {
        int above = excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (above < krem && krem <= above + c[j]) {
            s_digit = 255 - 8 * lane - j;
            s_krem = krem - above;
          }
          above += c[j];
        }
      }
    }
    __syncthreads();
    prefix |= (uint32_t)s_digit << shift;
    mask |= 255u << shift;
    krem = s_krem;
    __syncthreads();
  }
  const uint32_t T = prefix;
  // ordered compaction
  int base_sel = 0, base_eq = 0;
  for (int c0 = 0; c0 < n; c0 += kThreads) {
    const int i = c0 + tid;
    const uint32_t u = i < n ? key_at(i) : 0u;
    const bool gt = i < n && u > T;
    const bool eq = i < n && u == T;
    const uint32_t beq = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) wsum[warp][0] = __popc(beq);
    __syncthreads();
    int eq_before = base_eq, eq_total = 0;
    for (int w = 0; w < kWarps; ++w) {
      if (w < warp) eq_before += wsum[w][0];
      eq_total += wsum[w][0];
    }
    eq_before += __popc(beq & ((1u << lane) - 1u));
    const bool sel = gt || (eq && eq_before < krem);
    const uint32_t bsel = __ballot_sync(0xffffffffu, sel);
    if (lane == 0) wsum[warp][1] = __popc(bsel);
    __syncthreads();
    int pos = base_sel, sel_total = 0;
    for (int w = 0; w < kWarps; ++w) {
      if (w < warp) pos += wsum[w][1];
      sel_total += wsum[w][1];
    }
    pos += __popc(bsel & ((1u << lane) - 1u));
    if (sel && pos < k) outr[pos] = i;
    base_sel += sel_total;
    base_eq += eq_total;
    __syncthreads();
  }
}

cudaError_t launch_topk(const float* x, int rows, int n, int64_t row_stride, int k,
                        int64_t* out, cudaStream_t st) {
  topk_kernel<<<rows, kThreads, 0, st>>>(x, n, row_stride, k, out);
  return cudaGetLastError();
}

}  // namespace spatten
