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

// Fused scores of one key for R heads: `w` holds the key's packed MSB plane
// (D/2 bytes as D/8 words; byte p = dim p | dim p+D/2 << 4). With `lsb`, the
// full int8 key k8 = 16*msb + lsb. q8 words of head r at qs[r*D/4 + ...].
template <int D, int R>
SPATTEN_DEV void key_dots(const uint32_t (&w)[D / 8], const uint32_t* lw, const uint32_t* qs,
                          int (&acc)[R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    int a = 0;
    const uint32_t* q = qs + r * (D / 4);
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      uint32_t lo = (w[i] << 4) & 0xF0F0F0F0u;  // 16*msb of dims 4i..4i+3
      uint32_t hi = w[i] & 0xF0F0F0F0u;         // 16*msb of dims D/2+4i..
      if (lw) {
        lo |= lw[i] & 0x0F0F0F0Fu;
        hi |= (lw[i] >> 4) & 0x0F0F0F0Fu;
      }
      a = dp4a(lo, q[i], a);
      a = dp4a(hi, q[D / 8 + i], a);
    }
    acc[r] = a;
  }
}

// Block-wide (max, sum of exp2) of per-thread values for R heads, written
// by thread 0 of the block to out[r*stride].
template <int R>
SPATTEN_DEV void block_stats(const float (&m)[R], const float (&l)[R], float* sh, float* out,
                             int64_t stride) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float mm = m[r], ll = l[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, mm, o);
      const float lo = __shfl_xor_sync(0xffffffffu, ll, o);
      const float mn = fmaxf(mm, mo);
      ll = (mn == -INFINITY) ? 0.f : ll * exp2f(mm - mn) + lo * exp2f(mo - mn);
      mm = mn;
    }
    if (lane == 0) {
      sh[(r * nw + warp) * 2] = mm;
      sh[(r * nw + warp) * 2 + 1] = ll;
    }
  }
  __syncthreads();
  if (threadIdx.x < R) {
    const int r = threadIdx.x;
    float mm = -INFINITY, ll = 0.f;
    for (int w = 0; w < nw; ++w) {
      const float mo = sh[(r * nw + w) * 2], lo = sh[(r * nw + w) * 2 + 1];
      const float mn = fmaxf(mm, mo);
      ll = (mn == -INFINITY) ? 0.f : ll * exp2f(mm - mn) + lo * exp2f(mo - mn);
      mm = mn;
    }
    out[r * stride] = mm;
    out[r * stride + 1] = ll;
  }
}

// 1. MSB scores of every valid key for the R query heads of one KV head:
// grid (chunks, G, B), one key per thread. scores [B, H, N] (log2 domain),
// chunk statistics [B, H, chunks, 2].
template <int D, int R>
__global__ void __launch_bounds__(kTok) decode_scores_kernel(const DecodeParams p, float* scores,
                                                             float* part) {
  __shared__ uint32_t qs[R * D / 4];
  __shared__ float cq[R];
  __shared__ float sh[R * (kTok / 32) * 2];
  const int b = blockIdx.z, g = blockIdx.y, chunk = blockIdx.x;
  for (int i = threadIdx.x; i < R * D / 4; i += blockDim.x)
    qs[i] = reinterpret_cast<const uint32_t*>(p.q8 + ((int64_t)b * p.H + g * R) * D)[i];
  if (threadIdx.x < R) cq[threadIdx.x] = p.q_scale[(int64_t)b * p.H + g * R + threadIdx.x] * p.sm_scale * kLog2e;
  __syncthreads();
  const int n = chunk * kTok + threadIdx.x;
  float m[R], l[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
  }
  if (n < p.n_valid) {
    const int64_t key = ((int64_t)b * p.G + g) * p.N + n;
    uint32_t w[D / 8];
    const uint4* src = reinterpret_cast<const uint4*>(p.k_msb + key * (D / 2));
#pragma unroll
    for (int i = 0; i < D / 32; ++i) {
      const uint4 v = __ldg(src + i);
      w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
    const float ks = __ldg(p.k_scale + key);
    int acc[R];
    key_dots<D, R>(w, nullptr, qs, acc);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float s = (float)acc[r] * (cq[r] * ks);
      scores[((int64_t)b * p.H + g * R + r) * p.N + n] = s;
      m[r] = s;
      l[r] = 1.f;
    }
  }
  const int chunks = gridDim.x;
  block_stats<R>(m, l, sh, part + (((int64_t)b * p.H + g * R) * chunks + chunk) * 2, (int64_t)chunks * 2);
}

// 2. token importance = sum over the H heads of exp2(s - m_h) / l_h:
// grid (ceil(N / 256), B); each CTA first reduces the chunk statistics.
__global__ void __launch_bounds__(256) decode_importance_kernel(const DecodeParams p, const float* scores,
                                                                const float* part, int chunks) {
  extern __shared__ float st[];  // [H][2]: m, 1/l
  const int b = blockIdx.y;
  for (int h = threadIdx.x; h < p.H; h += blockDim.x) {
    const float* pp = part + ((int64_t)b * p.H + h) * chunks * 2;
    float mm = -INFINITY, ll = 0.f;
    for (int c = 0; c < chunks; ++c) {
      const float mo = pp[2 * c], lo = pp[2 * c + 1];
      const float mn = fmaxf(mm, mo);
      ll = (mn == -INFINITY) ? 0.f : ll * exp2f(mm - mn) + lo * exp2f(mo - mn);
      mm = mn;
    }
    st[2 * h] = mm;
    st[2 * h + 1] = ll > 0.f ? 1.f / ll : 0.f;
  }
  __syncthreads();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= p.N) return;
  float imp = 0.f;
  if (n < p.n_valid) {
    for (int h = 0; h < p.H; ++h)
      imp += exp2f(scores[((int64_t)b * p.H + h) * p.N + n] - st[2 * h]) * st[2 * h + 1];
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
  __shared__ uint32_t qs[R * D / 4];
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
  float m[R], l[R], s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
    s[r] = -INFINITY;
  }
  if (have && n >= 0 && n < p.n_valid) {
    const int64_t key = ((int64_t)b * p.G + g) * p.N + n;
    uint32_t w[D / 8], lw[D / 8];
    const uint4* ms = reinterpret_cast<const uint4*>(p.k_msb + key * (D / 2));
    const uint4* ls = reinterpret_cast<const uint4*>(p.k_lsb + key * (D / 2));
#pragma unroll
    for (int i = 0; i < D / 32; ++i) {
      const uint4 a = __ldg(ms + i), c = __ldg(ls + i);
      w[4 * i] = a.x; w[4 * i + 1] = a.y; w[4 * i + 2] = a.z; w[4 * i + 3] = a.w;
      lw[4 * i] = c.x; lw[4 * i + 1] = c.y; lw[4 * i + 2] = c.z; lw[4 * i + 3] = c.w;
    }
    const float ks = __ldg(p.k_scale + key);
    int acc[R];
    key_dots<D, R>(w, lw, qs, acc);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      s[r] = (float)acc[r] * (cq[r] * ks);
      m[r] = s[r];
      l[r] = 1.f;
    }
  }
  // split statistics -> sh_ml (thread 0 .. R-1 write them to part_ml)
  float* ml = part_ml + (((int64_t)b * p.H + g * R) * splits + split) * 2;
  block_stats<R>(m, l, sh, ml, (int64_t)splits * 2);
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float mr = ml[r * (int64_t)splits * 2];
    ps[r * kTok + threadIdx.x] = (s[r] == -INFINITY) ? 0.f : exp2f(s[r] - mr);
  }
  __syncthreads();
  // phase 2: thread = (key group kg of 4, dim pair dp of D/2)
  const int dp = threadIdx.x % (D / 2), kg = threadIdx.x / (D / 2);
  constexpr int kGroups = kTok / (D / 2);
  float o[R][2];
#pragma unroll
  for (int r = 0; r < R; ++r) o[r][0] = o[r][1] = 0.f;
  const T* vb = static_cast<const T*>(p.v) + ((int64_t)b * p.G + g) * p.N * D;
  const int cnt = min(kTok, p.top_k - split * kTok);
  for (int t = kg; t < cnt; t += kGroups) {
    const int nn = kidx[t];
    if (nn < 0 || nn >= p.n_valid) continue;
    const float2 vv = load2<T>(vb + (int64_t)nn * D + 2 * dp);
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
  const int chunks = (p.n_valid + kTok - 1) / kTok;
  decode_scores_kernel<D, R><<<dim3(chunks, p.G, p.B), kTok, 0, st>>>(p, w.scores, w.part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  decode_importance_kernel<<<dim3((p.N + 255) / 256, p.B), 256, p.H * 2 * sizeof(float), st>>>(p, w.scores,
                                                                                               w.part, chunks);
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
  const int chunks = (p.n_valid + kTok - 1) / kTok;
  const int splits = (p.top_k + kTok - 1) / kTok;
  s.scores = (size_t)p.B * p.H * p.N * sizeof(float);
  s.part = (size_t)p.B * p.H * (chunks > 0 ? chunks : 1) * 2 * sizeof(float);
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
