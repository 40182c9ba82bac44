// Radix-select top-k with ordered compaction: the cascade pruning decision.
//
// Replaces sort(topk(x, k).indices) on the head importance [H]
// (spatten_bert.py:123-128) and on the cumulative token importance [B, S]
// (spatten_bert.py:143-148); the decode path uses it for its top-2048 of
// 32768 cached tokens. One CTA per row:
//   1. map every float to an order-preserving 32-bit key (kept in dynamic
//      shared memory for rows up to kCacheMax entries; longer rows re-read
//      the row, L2 resident, when they are walked), and take the row's
//      smallest and largest key;
//   2. radix rounds of up to 8 bits walk down from the highest bit in which
//      the smallest and largest key differ (the bits above it are common to
//      the row) to the exact key T of the k-th largest value and the number r
//      of entries equal to T that are kept. Starting at the first differing
//      bit spreads the first round over many histogram bins (importance
//      values share their sign and leading exponent bits, which would
//      otherwise serialise the shared atomics on one bin). After the first
//      round the entries still in play are appended (unordered) to a
//      candidate list, and the later rounds walk only that list;
//   3. one ordered stream compaction writes the indices with key > T, plus
//      the first r indices with key == T, in ascending order -- no sort is
//      needed. Ties at the k-th value thus go to smaller indices.
// Warp w owns the contiguous segment [w*seg, (w+1)*seg) of the row, read
// 32 consecutive entries per step, so the compaction needs one block-wide
// scan of per-warp counts and no barrier inside its loops.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace spatten {

namespace {
constexpr int kCacheMax = 32768;  // keys cached in shared memory (128 KB)
constexpr int kCandMax = 16384;   // candidates after the first round (64 KB)

template <int NT>
__global__ void __launch_bounds__(NT, 1) topk_kernel(const float* __restrict__ x, int n, int64_t stride,
                                                  int k, int64_t* __restrict__ out, int cache_n,
                                                  int cand_cap) {
  constexpr int NW = NT / 32;
  extern __shared__ uint32_t dyn[];
  uint32_t* cache = dyn;           // [cache_n] keys
  uint32_t* cand = dyn + cache_n;  // [cand_cap] keys still in play after round 1
  __shared__ int hist[256];
  __shared__ int wgt[NW], weq[NW];
  __shared__ uint32_t wmin[NW], wmax[NW];
  __shared__ int s_digit, s_krem, s_fill;
  const int row = blockIdx.x;
  const float* xr = x + (int64_t)row * stride;
  int64_t* outr = out + (int64_t)row * k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool cached = n <= cache_n;
  const int seg = ((n + NW - 1) / NW + 31) & ~31;
  const int w0 = min(warp * seg, n), w1 = min(w0 + seg, n);
  auto key_at = [&](int i) -> uint32_t { return cached ? cache[i] : float_order_key(__ldg(xr + i)); };

  // 1. keys, smallest and largest key
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  int i_rest = 0;
  if (cached && (reinterpret_cast<uintptr_t>(xr) & 15) == 0) {
    const int n4 = n / 4;
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    uint4* c4 = reinterpret_cast<uint4*>(cache);
#pragma unroll 8
    for (int i = tid; i < n4; i += NT) {
      const float4 v = __ldg(x4 + i);
      const uint4 u = make_uint4(float_order_key(v.x), float_order_key(v.y), float_order_key(v.z),
                                 float_order_key(v.w));
      c4[i] = u;
      kmin = min(kmin, min(min(u.x, u.y), min(u.z, u.w)));
      kmax = max(kmax, max(max(u.x, u.y), max(u.z, u.w)));
    }
    i_rest = 4 * n4;
  }
  for (int i = i_rest + tid; i < n; i += NT) {
    const uint32_t u = float_order_key(__ldg(xr + i));
    if (cached) cache[i] = u;
    kmin = min(kmin, u);
    kmax = max(kmax, u);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
    kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
  }
  if (lane == 0) {
    wmin[warp] = kmin;
    wmax[warp] = kmax;
  }
  if (tid == 0) s_fill = 0;
  __syncthreads();
  for (int w = 0; w < NW; ++w) {
    kmin = min(kmin, wmin[w]);
    kmax = max(kmax, wmax[w]);
  }

  // 2. radix rounds from the highest differing bit down
  int hi = 32 - __clz(kmin ^ kmax);  // bits [hi, 32) are common to the row
  uint32_t mask = hi >= 32 ? 0u : ~((1u << hi) - 1u);
  uint32_t prefix = kmin & mask;
  int krem = k;
  bool use_cand = false;
  int ncand = 0;
  while (hi > 0) {
    const int lo = max(hi - 8, 0);
    const uint32_t dmask = (1u << (hi - lo)) - 1u;
    for (int i = tid; i < 256; i += NT) hist[i] = 0;
    __syncthreads();
    if (use_cand) {
      for (int i = tid; i < ncand; i += NT) {
        const uint32_t u = cand[i];
        if ((u & mask) == prefix) atomicAdd(&hist[(u >> lo) & dmask], 1);
      }
    } else {
      for (int i = tid; i < n; i += NT) {
        const uint32_t u = key_at(i);
        if ((u & mask) == prefix) atomicAdd(&hist[(u >> lo) & dmask], 1);
      }
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
    const int digit = s_digit;
    prefix |= (uint32_t)digit << lo;
    mask |= dmask << lo;
    krem = s_krem;
    hi = lo;
    if (!use_cand && hi > 0 && hist[digit] <= cand_cap) {
      // entries still in play -> candidate list (order does not matter)
      const uint32_t lt = (1u << lane) - 1u;
      for (int i0 = w0; i0 < w1; i0 += 32) {
        const int i = i0 + lane;
        const uint32_t u = i < w1 ? key_at(i) : 0u;
        const bool in = i < w1 && (u & mask) == prefix;
        const uint32_t m = __ballot_sync(0xffffffffu, in);
        int base = 0;
        if (lane == 0 && m) base = atomicAdd(&s_fill, __popc(m));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (in) cand[base + __popc(m & lt)] = u;
      }
      ncand = hist[digit];
      use_cand = true;
    }
    __syncthreads();
  }
  const uint32_t T = prefix;
  // ordered compaction: counts of key > T and key == T per warp segment
  int ngt = 0, neq = 0;
  for (int i0 = w0; i0 < w1; i0 += 32) {
    const int i = i0 + lane;
    const uint32_t u = i < w1 ? key_at(i) : 0u;
    ngt += __popc(__ballot_sync(0xffffffffu, i < w1 && u > T));
    neq += __popc(__ballot_sync(0xffffffffu, i < w1 && u == T));
  }
  if (lane == 0) {
    wgt[warp] = ngt;
    weq[warp] = neq;
  }
  __syncthreads();
  int gt_before = 0, eq_before = 0;
  for (int w = 0; w < warp; ++w) {
    gt_before += wgt[w];
    eq_before += weq[w];
  }
  const uint32_t lt = (1u << lane) - 1u;
  for (int i0 = w0; i0 < w1; i0 += 32) {
    const int i = i0 + lane;
    const uint32_t u = i < w1 ? key_at(i) : 0u;
    const bool gt = i < w1 && u > T, eq = i < w1 && u == T;
    const uint32_t bgt = __ballot_sync(0xffffffffu, gt), beq = __ballot_sync(0xffffffffu, eq);
    const int g_me = gt_before + __popc(bgt & lt), e_me = eq_before + __popc(beq & lt);
    // entries before this one that are kept: all larger ones, the first krem equal ones
    const int pos = g_me + min(e_me, krem);
    if ((gt || (eq && e_me < krem)) && pos < k) outr[pos] = i;
    gt_before += __popc(bgt);
    eq_before += __popc(beq);
  }
}

// Rows of 8192 entries or more: a cluster of kClu CTAs per row, CTA c owning
// the contiguous segment c of the row (its keys cached in its own shared
// memory). The radix rounds sum the CTAs' histograms through distributed
// shared memory, so every CTA takes the same digit; the ordered compaction
// offsets each CTA's output by the counts of the CTAs before it. Same
// selection and order as topk_kernel.
namespace cg = cooperative_groups;
constexpr int kClu = 4;
constexpr int kCluThreads = 512;
constexpr int kCluSegMax = 16384;  // entries per CTA (64 KB of keys)

__global__ void __cluster_dims__(kClu, 1, 1) __launch_bounds__(kCluThreads)
    topk_cluster_kernel(const float* __restrict__ x, int n, int64_t stride, int k, int64_t* __restrict__ out) {
  constexpr int NT = kCluThreads, NW = NT / 32;
  cg::cluster_group cl = cg::this_cluster();
  const int cr = (int)cl.block_rank();
  extern __shared__ uint32_t cache[];
  __shared__ int hist[256];
  __shared__ int ctot[256];
  __shared__ int wgt[NW], weq[NW];
  __shared__ uint32_t wmin[NW], wmax[NW];
  __shared__ uint32_t xmm[2];  // this CTA's smallest / largest key
  __shared__ int xcnt[2];      // this CTA's count of keys > T / == T
  __shared__ int s_digit, s_krem;
  const int row = blockIdx.x / kClu;
  const float* xr = x + (int64_t)row * stride;
  int64_t* outr = out + (int64_t)row * k;
  const int seg = (n + kClu - 1) / kClu;
  const int s0 = min(cr * seg, n), sn = min(s0 + seg, n) - s0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wseg = ((sn + NW - 1) / NW + 31) & ~31;
  const int w0 = min(warp * wseg, sn), w1 = min(w0 + wseg, sn);

  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  for (int i = tid; i < sn; i += NT) {
    const uint32_t u = float_order_key(__ldg(xr + s0 + i));
    cache[i] = u;
    kmin = min(kmin, u);
    kmax = max(kmax, u);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
    kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
  }
  if (lane == 0) {
    wmin[warp] = kmin;
    wmax[warp] = kmax;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 0; w < NW; ++w) {
      kmin = min(kmin, wmin[w]);
      kmax = max(kmax, wmax[w]);
    }
    xmm[0] = kmin;
    xmm[1] = kmax;
  }
  cl.sync();
  kmin = 0xFFFFFFFFu;
  kmax = 0u;
  for (int r = 0; r < kClu; ++r) {
    const uint32_t* pm = cl.map_shared_rank(xmm, r);
    kmin = min(kmin, pm[0]);
    kmax = max(kmax, pm[1]);
  }

  int hi = 32 - __clz(kmin ^ kmax);
  uint32_t mask = hi >= 32 ? 0u : ~((1u << hi) - 1u);
  uint32_t prefix = kmin & mask;
  int krem = k;
  while (hi > 0) {
    const int lo = max(hi - 8, 0);
    const uint32_t dmask = (1u << (hi - lo)) - 1u;
    for (int i = tid; i < 256; i += NT) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < sn; i += NT) {
      const uint32_t u = cache[i];
      if ((u & mask) == prefix) atomicAdd(&hist[(u >> lo) & dmask], 1);
    }
    cl.sync();  // every CTA's histogram is complete
    for (int d = tid; d < 256; d += NT) {  // the cluster's histogram, one bin per thread
      int v = 0;
#pragma unroll
      for (int r = 0; r < kClu; ++r) v += cl.map_shared_rank(hist, r)[d];
      ctot[d] = v;
    }
    cl.sync();  // the peers have read this CTA's histogram; ctot is complete
    if (warp == 0) {
      int c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = ctot[255 - 8 * lane - j];
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
    prefix |= (uint32_t)s_digit << lo;
    mask |= dmask << lo;
    krem = s_krem;
    hi = lo;
  }
  const uint32_t T = prefix;
  int ngt = 0, neq = 0;
  for (int i0 = w0; i0 < w1; i0 += 32) {
    const int i = i0 + lane;
    const uint32_t u = i < w1 ? cache[i] : 0u;
    ngt += __popc(__ballot_sync(0xffffffffu, i < w1 && u > T));
    neq += __popc(__ballot_sync(0xffffffffu, i < w1 && u == T));
  }
  if (lane == 0) {
    wgt[warp] = ngt;
    weq[warp] = neq;
  }
  __syncthreads();
  if (tid == 0) {
    int a = 0, b = 0;
    for (int w = 0; w < NW; ++w) {
      a += wgt[w];
      b += weq[w];
    }
    xcnt[0] = a;
    xcnt[1] = b;
  }
  cl.sync();
  int gt_before = 0, eq_before = 0;
  for (int r = 0; r < cr; ++r) {
    const int* pc = cl.map_shared_rank(xcnt, r);
    gt_before += pc[0];
    eq_before += pc[1];
  }
  cl.sync();  // no CTA leaves while a peer may still read its counts
  for (int w = 0; w < warp; ++w) {
    gt_before += wgt[w];
    eq_before += weq[w];
  }
  const uint32_t lt = (1u << lane) - 1u;
  for (int i0 = w0; i0 < w1; i0 += 32) {
    const int i = i0 + lane;
    const uint32_t u = i < w1 ? cache[i] : 0u;
    const bool gt = i < w1 && u > T, eq = i < w1 && u == T;
    const uint32_t bgt = __ballot_sync(0xffffffffu, gt), beq = __ballot_sync(0xffffffffu, eq);
    const int g_me = gt_before + __popc(bgt & lt), e_me = eq_before + __popc(beq & lt);
    const int pos = g_me + min(e_me, krem);
    if ((gt || (eq && e_me < krem)) && pos < k) outr[pos] = s0 + i;
    gt_before += __popc(bgt);
    eq_before += __popc(beq);
  }
}

template <int NT>
cudaError_t launch_nt(const float* x, int rows, int n, int64_t row_stride, int k, int64_t* out,
                      cudaStream_t st) {
  const int cache_n = n <= kCacheMax ? n : 0;
  const int cand_cap = n < kCandMax ? n : kCandMax;
  const size_t smem = ((size_t)cache_n + cand_cap) * sizeof(uint32_t);
  if (smem > 40 * 1024) {  // with the static shared memory, past the 48 KB default
    cudaError_t e = cudaFuncSetAttribute(topk_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)((kCacheMax + kCandMax) * sizeof(uint32_t)));
    if (e != cudaSuccess) return e;
  }
  topk_kernel<NT><<<rows, NT, smem, st>>>(x, n, row_stride, k, out, cache_n, cand_cap);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_topk(const float* x, int rows, int n, int64_t row_stride, int k,
                        int64_t* out, cudaStream_t st) {
  if (n <= 1024) return launch_nt<128>(x, rows, n, row_stride, k, out, st);
  if (n < 8192) return launch_nt<512>(x, rows, n, row_stride, k, out, st);
  if (n <= kClu * kCluSegMax) {
    const size_t smem = (size_t)((n + kClu - 1) / kClu) * sizeof(uint32_t);
    // static shared memory counts against the 48 KB default too: always raise the limit
    cudaError_t e = cudaFuncSetAttribute(topk_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(kCluSegMax * sizeof(uint32_t)));
    if (e != cudaSuccess) return e;
    topk_cluster_kernel<<<(unsigned)rows * kClu, kCluThreads, smem, st>>>(x, n, row_stride, k, out);
    return cudaGetLastError();
  }
  return launch_nt<1024>(x, rows, n, row_stride, k, out, st);
}

}  // namespace spatten
