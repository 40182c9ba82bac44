// Decode attention over a progressive-quantised KV cache with top-k token
// selection (one new query per sequence, GQA).
//
// The cache holds K as packed 4-bit MSB / LSB planes (the prefill format:
// [B, G, N, D/2] uint8, split at D/2, plus a per-key fp32 scale) and V in
// fp16/bf16. A decode step per layer:
//   1. importance: the MSB score s = (q8 . 16*msb) * q_scale * k_scale *
//      sm_scale of every cached key for every query head, the softmax of
//      each head over the keys, and the token importance = the sum over the
//      heads of those probabilities (decode_scores + decode_importance). Only
//      the 4-bit MSB plane of the whole cache is read.
//   2. top-k over the importance (topk.cu), all-reduced first when the KV
//      heads are split over ranks.
//   3. exact attention over the kept keys only: full int8 scores q8 . k8
//      (the LSB plane is fetched for the kept keys only), softmax, P.V, in
//      token splits whose partial (max, sum, output) are combined at the end
//      (decode_attend + decode_combine).
// All of it is byte / integer work bound by HBM: CUDA cores with dp4a,
// coalesced 16-byte loads, no tensor cores.
#include <climits>

#include "common.cuh"
#include "decode.h"
#include "kernels.h"

namespace spatten {
namespace {

constexpr int kTok = 256;   // keys per CTA in the score and attend kernels
constexpr int kMaxR = 8;    // query heads per KV head (GQA group)

SPATTEN_DEV int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// two consecutive 16-bit values as floats (4-byte aligned)
template <typename T>
SPATTEN_DEV float2 load2(const T* p);
template <>
SPATTEN_DEV float2 load2<__half>(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
template <>
SPATTEN_DEV float2 load2<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

// Exact int scores of K keys for R heads. w[k] holds key k's packed plane
// words (D/8 words of the MSB plane; byte p = dim p | dim p+D/2 << 4); with
// `lw` the LSB plane's, for the full int8 key k8 = 16*msb + lsb. The query
// words of head r sit at qs[r*D/4 ..] in shared memory, read 16 bytes at a
// time and shared by the K keys.
template <int D, int R, int K>
SPATTEN_DEV void key_dots(const uint32_t (&w)[K][D / 8], const uint32_t (*lw)[D / 8], const uint32_t* qs,
                          int (&acc)[K][R]) {
  const uint4* q4 = reinterpret_cast<const uint4*>(qs);
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int k = 0; k < K; ++k) acc[k][r] = 0;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      const uint4 ql = q4[r * (D / 16) + j];           // query words 4j..4j+3 (dims 16j..)
      const uint4 qh = q4[r * (D / 16) + D / 32 + j];  // words D/8+4j.. (dims D/2+16j..)
      const uint32_t qlw[4] = {ql.x, ql.y, ql.z, ql.w}, qhw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
      for (int k = 0; k < K; ++k) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int i = 4 * j + t;
          uint32_t lo = (w[k][i] << 4) & 0xF0F0F0F0u;  // 16*msb of dims 4i..4i+3
          uint32_t hi = w[k][i] & 0xF0F0F0F0u;         // 16*msb of dims D/2+4i..
          if (lw) {
            lo |= lw[k][i] & 0x0F0F0F0Fu;
            hi |= (lw[k][i] >> 4) & 0x0F0F0F0Fu;
          }
          acc[k][r] = dp4a(lo, qlw[t], acc[k][r]);
          acc[k][r] = dp4a(hi, qhw[t], acc[k][r]);
        }
      }
    }
  }
}

template <int D, int K>
SPATTEN_DEV void load_rows(const uint8_t* base, const int64_t (&key)[K], const bool (&ok)[K],
                           uint32_t (&w)[K][D / 8]) {
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const uint4* src = reinterpret_cast<const uint4*>(base + (ok[k] ? key[k] : 0) * (D / 2));
#pragma unroll
    for (int i = 0; i < D / 32; ++i) {
      const uint4 v = ok[k] ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
      w[k][4 * i] = v.x; w[k][4 * i + 1] = v.y; w[k][4 * i + 2] = v.z; w[k][4 * i + 3] = v.w;
    }
  }
}

// Block-wide softmax statistics of K values per thread and head (-inf for
// no key): the block max m_r, e[k][r] = exp2(s[k][r] - m_r) for the caller
// and the sum l_r of the e; threads r < R write (m_r, l_r) to out[r*stride].
// Max first, then one exp2 per value, then a sum: fixed reduction order.
template <int R, int K>
SPATTEN_DEV void block_softmax(const float (&s)[K][R], float* sh, float* out, int64_t stride,
                               float (&e)[K][R]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float* smax = sh;
  float* ssum = sh + R * nw;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float mm = s[0][r];
#pragma unroll
    for (int k = 1; k < K; ++k) mm = fmaxf(mm, s[k][r]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
    if (lane == 0) smax[r * nw + warp] = mm;
  }
  __syncthreads();
  float mc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float m = -INFINITY;
    for (int w = 0; w < nw; ++w) m = fmaxf(m, smax[r * nw + w]);
    mc[r] = m;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      e[k][r] = (m == -INFINITY) ? 0.f : fast_exp2(s[k][r] - m);
      sum += e[k][r];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) ssum[r * nw + warp] = sum;
  }
  __syncthreads();
  if (threadIdx.x < R) {
    const int r = threadIdx.x;
    float l = 0.f;
    for (int w = 0; w < nw; ++w) l += ssum[r * nw + w];
    out[r * stride] = mc[r];
    out[r * stride + 1] = l;
  }
}

// 1. MSB scores of every valid key for the R query heads of one KV head:
// grid (chunks of kScoreKeys, G, B), kKeysPerThread keys per thread (keys t
// and t + kTok of the chunk: consecutive threads read consecutive rows).
// scores [B, H, N] (log2 domain), chunk statistics [B, H, chunks, 2].
constexpr int kKeysPerThread = 2;
constexpr int kScoreKeys = kTok * kKeysPerThread;

template <int D, int R>
__global__ void __launch_bounds__(kTok) decode_scores_kernel(const DecodeParams p, float* scores,
                                                             float* part) {
  constexpr int K = kKeysPerThread;
  __shared__ __align__(16) uint32_t qs[R * D / 4];
  __shared__ float cq[R];
  __shared__ float sh[R * (kTok / 32) * 2];
  const int b = blockIdx.z, g = blockIdx.y, chunk = blockIdx.x;
  for (int i = threadIdx.x; i < R * D / 4; i += blockDim.x)
    qs[i] = reinterpret_cast<const uint32_t*>(p.q8 + ((int64_t)b * p.H + g * R) * D)[i];
  if (threadIdx.x < R) cq[threadIdx.x] = p.q_scale[(int64_t)b * p.H + g * R + threadIdx.x] * p.sm_scale * kLog2e;
  int n[K];
  int64_t key[K];
  bool ok[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    n[k] = chunk * kScoreKeys + k * kTok + threadIdx.x;
    ok[k] = n[k] < p.n_valid;
    key[k] = ((int64_t)b * p.G + g) * p.N + n[k];
  }
  uint32_t w[K][D / 8];
  load_rows<D, K>(p.k_msb, key, ok, w);  // in flight while the query lands in smem
  float ks[K];
#pragma unroll
  for (int k = 0; k < K; ++k) ks[k] = ok[k] ? __ldg(p.k_scale + key[k]) : 0.f;
  __syncthreads();
  int acc[K][R];
  key_dots<D, R, K>(w, nullptr, qs, acc);
  float sv[K][R];
#pragma unroll
  for (int k = 0; k < K; ++k)
#pragma unroll
    for (int r = 0; r < R; ++r) {
      sv[k][r] = ok[k] ? (float)acc[k][r] * (cq[r] * ks[k]) : -INFINITY;
      if (ok[k]) scores[((int64_t)b * p.H + g * R + r) * p.N + n[k]] = sv[k][r];
    }
  const int chunks = gridDim.x;
  float e[K][R];
  block_softmax<R, K>(sv, sh, part + (((int64_t)b * p.H + g * R) * chunks + chunk) * 2, (int64_t)chunks * 2, e);
}

// 1b. global softmax statistics per (b, h) from the chunk statistics: a warp
// per head; st [B, H, 2] = (max, 1 / sum).
__global__ void __launch_bounds__(256) decode_stats_kernel(const DecodeParams p, const float* part, int chunks,
                                                           float* st) {
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (bh >= p.B * p.H) return;
  const float* pp = part + (int64_t)bh * chunks * 2;
  float mm = -INFINITY;
  for (int c = lane; c < chunks; c += 32) mm = fmaxf(mm, pp[2 * c]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
  float ll = 0.f;
  if (mm != -INFINITY)
    for (int c = lane; c < chunks; c += 32) ll += pp[2 * c + 1] * fast_exp2(pp[2 * c] - mm);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ll += __shfl_xor_sync(0xffffffffu, ll, o);
  if (lane == 0) {
    st[2 * bh] = mm;
    st[2 * bh + 1] = ll > 0.f ? 1.f / ll : 0.f;
  }
}

// 2. token importance = sum over the H heads of exp2(s - m_h) / l_h:
// grid (ceil(N / 256), B).
__global__ void __launch_bounds__(256) decode_importance_kernel(const DecodeParams p, const float* scores,
                                                                const float* stg) {
  extern __shared__ float st[];  // [H][2]: m, 1/l
  const int b = blockIdx.y;
  for (int i = threadIdx.x; i < 2 * p.H; i += blockDim.x) st[i] = stg[(int64_t)b * p.H * 2 + i];
  __syncthreads();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= p.N) return;
  float imp = 0.f;
  if (n < p.n_valid) {
    for (int h = 0; h < p.H; ++h)
      imp += fast_exp2(scores[((int64_t)b * p.H + h) * p.N + n] - st[2 * h]) * st[2 * h + 1];
  }
  p.importance[(int64_t)b * p.N + n] = imp;
}

// 3. exact attention over the kept keys, in splits of kTok keys: grid
// (splits, G, B). Phase 1: one kept key per thread, full int8 scores for
// the R heads -> smem; split max / sum per head. Phase 2: P.V with 64
// dim-pairs x 4 key groups per CTA.
template <int D, int R, typename T>
__global__ void __launch_bounds__(kTok) decode_attend_kernel(const DecodeParams p, float* part_ml,
                                                             float* part_o) {
  __shared__ __align__(16) uint32_t qs[R * D / 4];
  __shared__ float cq[R];
  __shared__ float ps[R * kTok];  // exp2(s - m_split) per head and key
  __shared__ float sh[R * (kTok / 32) * 2];
  __shared__ float red[(kTok / (D / 2)) * R * D];  // phase 2: partial outputs per key group
  __shared__ int kidx[kTok];
  const int b = blockIdx.z, g = blockIdx.y, split = blockIdx.x, splits = gridDim.x;
  for (int i = threadIdx.x; i < R * D / 4; i += blockDim.x)
    qs[i] = reinterpret_cast<const uint32_t*>(p.q8 + ((int64_t)b * p.H + g * R) * D)[i];
  if (threadIdx.x < R) cq[threadIdx.x] = p.q_scale[(int64_t)b * p.H + g * R + threadIdx.x] * p.sm_scale * kLog2e;
  const int j = split * kTok + threadIdx.x;  // position in the kept list
  const bool have = j < p.top_k;
  const int n = have ? (int)p.kept[(int64_t)b * p.top_k + j] : -1;
  kidx[threadIdx.x] = n;
  __syncthreads();
  float s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) s[r] = -INFINITY;
  {
    const bool okk[1] = {have && n >= 0 && n < p.n_valid};
    const int64_t key[1] = {((int64_t)b * p.G + g) * p.N + (okk[0] ? n : 0)};
    uint32_t w[1][D / 8], lw[1][D / 8];
    load_rows<D, 1>(p.k_msb, key, okk, w);
    load_rows<D, 1>(p.k_lsb, key, okk, lw);
    const float ks = okk[0] ? __ldg(p.k_scale + key[0]) : 0.f;
    int acc[1][R];
    key_dots<D, R, 1>(w, lw, qs, acc);
    if (okk[0]) {
#pragma unroll
      for (int r = 0; r < R; ++r) s[r] = (float)acc[0][r] * (cq[r] * ks);
    }
  }
  // split statistics (max, sum) per head -> part_ml; exp2(s - max) -> ps
  float* ml = part_ml + (((int64_t)b * p.H + g * R) * splits + split) * 2;
  float sk[1][R], e[1][R];
#pragma unroll
  for (int r = 0; r < R; ++r) sk[0][r] = s[r];
  block_softmax<R, 1>(sk, sh, ml, (int64_t)splits * 2, e);
#pragma unroll
  for (int r = 0; r < R; ++r) ps[r * kTok + threadIdx.x] = e[0][r];
  __syncthreads();
  // phase 2: thread = (key group kg of 4, dim pair dp of D/2)
  const int dp = threadIdx.x % (D / 2), kg = threadIdx.x / (D / 2);
  constexpr int kGroups = kTok / (D / 2);
  float o[R][2];
#pragma unroll
  for (int r = 0; r < R; ++r) o[r][0] = o[r][1] = 0.f;
  const T* vb = static_cast<const T*>(p.v) + ((int64_t)b * p.G + g) * p.N * D;
  const int cnt = min(kTok, p.top_k - split * kTok);
#pragma unroll 4
  for (int t = kg; t < cnt; t += kGroups) {
    const int nn = kidx[t];
    const bool okv = nn >= 0 && nn < p.n_valid;
    const float2 vv = okv ? load2<T>(vb + (int64_t)nn * D + 2 * dp) : make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float pr = ps[r * kTok + t];
      o[r][0] = fmaf(pr, vv.x, o[r][0]);
      o[r][1] = fmaf(pr, vv.y, o[r][1]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    red[((kg * R) + r) * D + 2 * dp] = o[r][0];
    red[((kg * R) + r) * D + 2 * dp + 1] = o[r][1];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R * D; i += blockDim.x) {
    float a = 0.f;
    for (int k = 0; k < kGroups; ++k) a += red[k * R * D + i];
    const int r = i / D, d = i % D;
    part_o[((((int64_t)b * p.H + g * R + r) * splits) + split) * D + d] = a;
  }
}

// 4. combine the splits: grid (H, B), D threads.
template <typename T>
__global__ void decode_combine_kernel(const DecodeParams p, const float* part_ml, const float* part_o,
                                      int splits) {
  const int b = blockIdx.y, h = blockIdx.x, d = threadIdx.x;
  const float* ml = part_ml + ((int64_t)b * p.H + h) * splits * 2;
  float mm = -INFINITY;
  for (int s = 0; s < splits; ++s) mm = fmaxf(mm, ml[2 * s]);
  float l = 0.f, o = 0.f;
  if (mm != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float f = (ml[2 * s] == -INFINITY) ? 0.f : exp2f(ml[2 * s] - mm);
      l += ml[2 * s + 1] * f;
      o += part_o[(((int64_t)b * p.H + h) * splits + s) * p.D + d] * f;
    }
  }
  static_cast<T*>(p.out)[((int64_t)b * p.H + h) * p.D + d] = from_f32<T>(l > 0.f ? o / l : 0.f);
}

template <int D, int R>
cudaError_t importance_d(const DecodeParams& p, const DecodeWorkspace& w, cudaStream_t st) {
  const int chunks = (p.n_valid + kScoreKeys - 1) / kScoreKeys;
  decode_scores_kernel<D, R><<<dim3(chunks, p.G, p.B), kTok, 0, st>>>(p, w.scores, w.part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  decode_stats_kernel<<<(p.B * p.H + 7) / 8, 256, 0, st>>>(p, w.part, chunks, w.st);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  decode_importance_kernel<<<dim3((p.N + 255) / 256, p.B), 256, p.H * 2 * sizeof(float), st>>>(p, w.scores,
                                                                                               w.st);
  return cudaGetLastError();
}

template <int D, int R, typename T>
cudaError_t attend_dt(const DecodeParams& p, const DecodeWorkspace& w, cudaStream_t st) {
  const int splits = (p.top_k + kTok - 1) / kTok;
  decode_attend_kernel<D, R, T><<<dim3(splits, p.G, p.B), kTok, 0, st>>>(p, w.ml, w.o);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  decode_combine_kernel<T><<<dim3(p.H, p.B), D, 0, st>>>(p, w.ml, w.o, splits);
  return cudaGetLastError();
}

}  // namespace

DecodeWorkspaceSizes decode_workspace_sizes(const DecodeParams& p) {
  DecodeWorkspaceSizes s;
  const int chunks = (p.n_valid + kScoreKeys - 1) / kScoreKeys;
  const int splits = (p.top_k + kTok - 1) / kTok;
  s.scores = (size_t)p.B * p.H * p.N * sizeof(float);
  s.part = (size_t)p.B * p.H * (chunks > 0 ? chunks : 1) * 2 * sizeof(float);
  s.st = (size_t)p.B * p.H * 2 * sizeof(float);
  s.ml = (size_t)p.B * p.H * (splits > 0 ? splits : 1) * 2 * sizeof(float);
  s.o = (size_t)p.B * p.H * (splits > 0 ? splits : 1) * p.D * sizeof(float);
  return s;
}

template <int D>
cudaError_t importance_r(const DecodeParams& p, const DecodeWorkspace& w, cudaStream_t st) {
  switch (p.H / p.G) {
    case 1: return importance_d<D, 1>(p, w, st);
    case 2: return importance_d<D, 2>(p, w, st);
    case 4: return importance_d<D, 4>(p, w, st);
    case 8: return importance_d<D, 8>(p, w, st);
    default: return cudaErrorInvalidValue;
  }
}

template <int D, typename T>
cudaError_t attend_r(const DecodeParams& p, const DecodeWorkspace& w, cudaStream_t st) {
  switch (p.H / p.G) {
    case 1: return attend_dt<D, 1, T>(p, w, st);
    case 2: return attend_dt<D, 2, T>(p, w, st);
    case 4: return attend_dt<D, 4, T>(p, w, st);
    case 8: return attend_dt<D, 8, T>(p, w, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_decode_importance(const DecodeParams& p, const DecodeWorkspace& w, cudaStream_t st) {
  if (p.D == 128) return importance_r<128>(p, w, st);
  if (p.D == 64) return importance_r<64>(p, w, st);
  return cudaErrorInvalidValue;
}

cudaError_t launch_decode_attend(const DecodeParams& p, const DecodeWorkspace& w, cudaStream_t st) {
  const bool f16 = p.dtype == kF16;
  if (p.D == 128) return f16 ? attend_r<128, __half>(p, w, st) : attend_r<128, __nv_bfloat16>(p, w, st);
  if (p.D == 64) return f16 ? attend_r<64, __half>(p, w, st) : attend_r<64, __nv_bfloat16>(p, w, st);
  return cudaErrorInvalidValue;
}

}  // namespace spatten
