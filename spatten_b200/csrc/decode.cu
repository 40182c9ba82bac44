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
// All of it is bound by HBM: the only contraction is q (R <= 8 heads of a
// GQA group) against the keys, done as int8 mma.m16n8k32 tiles with the
// operands expanded in registers from the packed nibbles; the gathers and
// the plane stream are cp.async copies into shared memory.
#include <climits>

#include "common.cuh"
#include "decode.h"
#include "kernels.h"

namespace spatten {
namespace {

constexpr int kTok = 256;  // threads of the score kernel, keys per ring stage

// eight consecutive 16-bit values (one 16-byte load) as floats
template <typename T>
SPATTEN_DEV void unpack8(const uint4& u, float (&f)[8]);
template <>
SPATTEN_DEV void unpack8<__half>(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
template <>
SPATTEN_DEV void unpack8<__nv_bfloat16>(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
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
    float l = 0.f, m = -INFINITY;
    for (int w = 0; w < nw; ++w) {
      l += ssum[r * nw + w];
      m = fmaxf(m, smax[r * nw + w]);
    }
    out[r * stride] = m;
    out[r * stride + 1] = l;
  }
}

// 1. MSB scores of every valid key for the R query heads of one KV head.
// Grid (ceil(n_valid / kCtaKeys), G, B), kTok threads. A CTA streams its
// kCtaKeys keys through a kStages-deep ring of cp.async stages (kStageKeys
// packed MSB rows + their scales per stage; rows XOR-swizzled by 16-byte
// chunk so that the fragment reads below are free of bank conflicts). Warp w
// contracts keys 32w .. 32w+31 of each stage on the tensor cores, as two
// mma.m16n8k32 s8 tiles: A = 16 keys x 32 dims of the int8 operand 16*msb,
// expanded in registers straight from the packed words (one packed word
// holds 4 dims of the low half of the row and the same 4 dims of the high
// half), B = the group's R query heads padded to 8 (registers, loaded once),
// exact int32 accumulators. The epilogue scales the scores, stores them and
// keeps an online (max, sum of exp2) per head; the CTA combines them once:
// chunk statistics [B, H, chunks, 2]. scores [B, H, N] (log2 domain).
// The contraction is tiny (N = R heads); the kernel is bound by the HBM read
// of the MSB plane, and the tensor cores keep the integer work off the issue
// slots that dp4a would fill.
constexpr int kStageKeys = kTok;
constexpr int kStages = 4;
constexpr int kCtaKeys = 2048;

template <int D>
__host__ __device__ constexpr size_t scores_smem_bytes() {
  return (size_t)kStages * kStageKeys * (D / 2 + sizeof(float));
}

template <int D>
SPATTEN_DEV int row_swizzle(int row) {
  constexpr int RB = D / 2, CH = RB / 16, L = 128 / RB;  // chunks per row, rows per 128 B
  return (row / L) % CH;
}

// Online combination of two (max, sum of exp2) pairs.
SPATTEN_DEV void ml_combine(float& m, float& l, float mo, float lo) {
  const float mn = fmaxf(m, mo);
  if (mn == -INFINITY) return;
  l = l * fast_exp2(m - mn) + lo * fast_exp2(mo - mn);
  m = mn;
}

SPATTEN_DEV void ml_push(float& m, float& l, float s) {
  if (s > m) {
    l = l * fast_exp2(m - s) + 1.f;
    m = s;
  } else {
    l += fast_exp2(s - m);
  }
}

template <int D, int R>
__global__ void __launch_bounds__(kTok) decode_scores_kernel(const DecodeParams p, float* scores,
                                                             float* part) {
  static_assert(R <= 8, "one n8 tile of query heads");
  constexpr int RB = D / 2, CH = RB / 16, NWD = D / 32;  // packed words per lane and key; = k-steps
  constexpr int NW = kTok / 32;
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* rows = dsm;                                                    // [kStages][kStageKeys][RB]
  float* scl = reinterpret_cast<float*>(dsm + kStages * kStageKeys * RB);  // [kStages][kStageKeys]
  __shared__ float cq[8];
  __shared__ float sh[8 * NW * 2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gq = lane >> 2, tq = lane & 3;
  const int b = blockIdx.z, g = blockIdx.y, cta = blockIdx.x;
  const int n0 = cta * kCtaKeys;
  const int nend = min(n0 + kCtaKeys, p.n_valid);
  const int nst = (nend - n0 + kStageKeys - 1) / kStageKeys;
  const int64_t bg = (int64_t)b * p.G + g;
  const uint8_t* plane = p.k_msb + bg * p.N * RB;
  const float* ksc = p.k_scale + bg * p.N;
  if (tid < 8) cq[tid] = tid < R ? p.q_scale[(int64_t)b * p.H + g * R + tid] * p.sm_scale * kLog2e : 0.f;

  // stage s of this CTA -> ring slot s % kStages (an empty group past the end)
  auto issue = [&](int s) {
    if (s < nst) {
      const int slot = s % kStages, kb = n0 + s * kStageKeys;
      uint8_t* dst = rows + slot * kStageKeys * RB;
#pragma unroll
      for (int c = tid; c < kStageKeys * CH; c += kTok) {
        const int row = c / CH, col = c % CH, n = kb + row;
        const bool v = n < nend;
        cp_async16(dst + row * RB + ((col ^ row_swizzle<D>(row)) * 16), plane + (int64_t)(v ? n : n0) * RB + col * 16, v);
      }
      const int n = kb + tid;
      cp_async4(scl + slot * kStageKeys + tid, ksc + (n < nend ? n : n0), n < nend);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) issue(s);

  // B fragments: head gq (zero beyond R), dims 32kk + 4tq .. and 32kk + 16 + 4tq ..
  uint32_t qb[NWD][2];
  {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(p.q8 + ((int64_t)b * p.H + g * R + (gq < R ? gq : 0)) * D);
#pragma unroll
    for (int kk = 0; kk < NWD; ++kk) {
      qb[kk][0] = gq < R ? __ldg(qw + 8 * kk + tq) : 0u;
      qb[kk][1] = gq < R ? __ldg(qw + 8 * kk + 4 + tq) : 0u;
    }
  }
  // this lane's heads 2tq, 2tq + 1
  const int h0 = 2 * tq, h1 = 2 * tq + 1;
  float m0 = -INFINITY, l0 = 0.f, m1 = -INFINITY, l1 = 0.f;
  float* sc0 = scores + ((int64_t)b * p.H + g * R + (h0 < R ? h0 : 0)) * p.N;
  float* sc1 = scores + ((int64_t)b * p.H + g * R + (h1 < R ? h1 : 0)) * p.N;
  for (int s = 0; s < nst; ++s) {
    cp_async_wait<kStages - 2>();
    __syncthreads();  // stage s landed for every thread; slot (s - 1) % kStages is free
    issue(s + kStages - 1);
    const int slot = s % kStages;
    const uint8_t* st = rows + slot * kStageKeys * RB;
    const float cq0 = cq[h0 < 8 ? h0 : 0], cq1 = cq[h1 < 8 ? h1 : 0];
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
      const int r0 = warp * 32 + grp * 16 + gq, r1 = r0 + 8;  // key rows of this lane in the stage
      uint32_t w0[NWD], w1[NWD];
#pragma unroll
      for (int j = 0; j < NWD; ++j) {
        w0[j] = *reinterpret_cast<const uint32_t*>(st + r0 * RB + ((j ^ row_swizzle<D>(r0)) << 4) + 4 * tq);
        w1[j] = *reinterpret_cast<const uint32_t*>(st + r1 * RB + ((j ^ row_swizzle<D>(r1)) << 4) + 4 * tq);
      }
      int acc[4] = {0, 0, 0, 0};
#pragma unroll
      for (int kk = 0; kk < NWD; ++kk) {
        // k-step kk covers dims 32kk .. 32kk+31: the low nibbles of words 2kk, 2kk+1
        // for the first D/2 dims, the high nibbles of words 2kk - NWD, .. after
        const bool hi = kk >= NWD / 2;
        const int j = 2 * (hi ? kk - NWD / 2 : kk);
        uint32_t a[4];
        a[0] = hi ? (w0[j] & 0xF0F0F0F0u) : ((w0[j] << 4) & 0xF0F0F0F0u);
        a[1] = hi ? (w1[j] & 0xF0F0F0F0u) : ((w1[j] << 4) & 0xF0F0F0F0u);
        a[2] = hi ? (w0[j + 1] & 0xF0F0F0F0u) : ((w0[j + 1] << 4) & 0xF0F0F0F0u);
        a[3] = hi ? (w1[j + 1] & 0xF0F0F0F0u) : ((w1[j + 1] << 4) & 0xF0F0F0F0u);
        mma_s8_16832(acc, a, qb[kk][0], qb[kk][1]);
      }
      // acc: (key r0, head h0), (r0, h1), (r1, h0), (r1, h1)
      const int na = n0 + s * kStageKeys + r0, nb = na + 8;
      const float ka = scl[slot * kStageKeys + r0], kb = scl[slot * kStageKeys + r1];
      if (h0 < R) {
        if (na < nend) {
          const float v = (float)acc[0] * (cq0 * ka);
          sc0[na] = v;
          ml_push(m0, l0, v);
        }
        if (nb < nend) {
          const float v = (float)acc[2] * (cq0 * kb);
          sc0[nb] = v;
          ml_push(m0, l0, v);
        }
      }
      if (h1 < R) {
        if (na < nend) {
          const float v = (float)acc[1] * (cq1 * ka);
          sc1[na] = v;
          ml_push(m1, l1, v);
        }
        if (nb < nend) {
          const float v = (float)acc[3] * (cq1 * kb);
          sc1[nb] = v;
          ml_push(m1, l1, v);
        }
      }
    }
  }
  cp_async_wait<0>();
  // CTA statistics per head: lanes of the same tq hold the same heads
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    ml_combine(m0, l0, __shfl_xor_sync(0xffffffffu, m0, o), __shfl_xor_sync(0xffffffffu, l0, o));
    ml_combine(m1, l1, __shfl_xor_sync(0xffffffffu, m1, o), __shfl_xor_sync(0xffffffffu, l1, o));
  }
  if (gq == 0) {
    sh[(h0 * NW + warp) * 2] = m0;
    sh[(h0 * NW + warp) * 2 + 1] = l0;
    sh[(h1 * NW + warp) * 2] = m1;
    sh[(h1 * NW + warp) * 2 + 1] = l1;
  }
  __syncthreads();
  if (tid < R) {
    const int r = tid;
    float mm = -INFINITY, ll = 0.f;
    for (int w = 0; w < NW; ++w) ml_combine(mm, ll, sh[(r * NW + w) * 2], sh[(r * NW + w) * 2 + 1]);
    float* out = part + (((int64_t)b * p.H + g * R + r) * gridDim.x + cta) * 2;
    out[0] = mm;
    out[1] = ll;
  }
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

// 3. exact attention over the kept keys, in splits of kAttKeys keys: grid
// (splits, G, B), kAttKeys threads. The split's kept rows are gathered with
// cp.async into shared memory at once: both K planes and the scales (first
// group) and the V rows (second group, in flight during phase 1).
// Phase 1: exact int8 scores q8 . k8 on the tensor cores (mma.m16n8k32 s8,
// A = k8 = 16*msb + lsb expanded in registers from the two packed planes,
// B = the R query heads padded to 8), then the split's softmax per head
// (max, sum -> part_ml; exp2(s - max) -> ps). Phase 2: P.V out of shared
// memory, a lane per 8 dims of a row; the per-warp partial outputs are then
// summed in the (by then free) V buffer.
constexpr int kAttKeys = 128;

template <int D>
struct AttendLayout {
  static constexpr int RB = D / 2;
  static constexpr int oMsb = 0;                          // [kAttKeys][RB], 16-byte chunks swizzled
  static constexpr int oLsb = oMsb + kAttKeys * RB;       // same
  static constexpr int oV = oLsb + kAttKeys * RB;         // [kAttKeys][D] 16-bit
  static constexpr int oScale = oV + kAttKeys * D * 2;    // [kAttKeys]
  static constexpr int kBytes = oScale + kAttKeys * 4;
};

// R consecutive floats from shared memory (16-byte aligned for R >= 4)
template <int R>
SPATTEN_DEV void load_heads(const float* src, float (&f)[R]) {
  if constexpr (R >= 4) {
#pragma unroll
    for (int i = 0; i < R / 4; ++i) {
      const float4 v = reinterpret_cast<const float4*>(src)[i];
      f[4 * i] = v.x; f[4 * i + 1] = v.y; f[4 * i + 2] = v.z; f[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < R; ++i) f[i] = src[i];
  }
}

template <int D, int R, typename T>
__global__ void __launch_bounds__(kAttKeys) decode_attend_kernel(const DecodeParams p, float* part_ml,
                                                                 float* part_o) {
  static_assert(R <= 8, "one n8 tile of query heads");
  using L = AttendLayout<D>;
  constexpr int RB = L::RB, CH = RB / 16, NWD = D / 32, NW = kAttKeys / 32;
  constexpr int LPR = D / 8, RPW = 32 / LPR;  // 16-byte chunks per V row, V rows per warp step
  static_assert(NW * R * D * sizeof(float) <= (size_t)kAttKeys * D * 2, "partial outputs fit the V buffer");
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* msb = dsm + L::oMsb;
  uint8_t* lsb = dsm + L::oLsb;
  uint4* vs = reinterpret_cast<uint4*>(dsm + L::oV);
  float* ksm = reinterpret_cast<float*>(dsm + L::oScale);
  __shared__ __align__(16) float ps[kAttKeys * R];  // [key][head]: scores, then exp2(s - m_split)
  __shared__ float cq[8];
  __shared__ float sh[R * NW * 2];
  __shared__ int kidx[kAttKeys];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gq = lane >> 2, tq = lane & 3;
  const int b = blockIdx.z, g = blockIdx.y, split = blockIdx.x, splits = gridDim.x;
  if (tid < 8) cq[tid] = tid < R ? p.q_scale[(int64_t)b * p.H + g * R + tid] * p.sm_scale * kLog2e : 0.f;
  const int j = split * kAttKeys + tid;  // position in the kept list
  const int64_t nk = j < p.top_k ? p.kept[(int64_t)b * p.top_k + j] : -1;
  const int n = (nk >= 0 && nk < p.n_valid) ? (int)nk : -1;  // -1: no key
  kidx[tid] = n;
  __syncthreads();
  const int64_t bgN = ((int64_t)b * p.G + g) * p.N;
  const int cnt = min(kAttKeys, p.top_k - split * kAttKeys);
  for (int c = tid; c < kAttKeys * CH; c += kAttKeys) {
    const int t = c / CH, col = c % CH, nn = kidx[t];
    const int64_t row = bgN + (nn >= 0 ? nn : 0);
    const int off = t * RB + ((col ^ row_swizzle<D>(t)) << 4);
    cp_async16(msb + off, p.k_msb + row * RB + col * 16, nn >= 0);
    cp_async16(lsb + off, p.k_lsb + row * RB + col * 16, nn >= 0);
  }
  cp_async4(ksm + tid, p.k_scale + bgN + (n >= 0 ? n : 0), n >= 0);
  cp_async_commit();
  const T* vb = static_cast<const T*>(p.v) + bgN * D;
  for (int c = tid; c < cnt * LPR; c += kAttKeys) {
    const int t = c / LPR, dc = c % LPR, nn = kidx[t];
    cp_async16(vs + c, vb + (int64_t)(nn >= 0 ? nn : 0) * D + dc * 8, nn >= 0);
  }
  cp_async_commit();
  // B fragments: head gq (zero beyond R), dims 32kk + 4tq .. and 32kk + 16 + 4tq ..
  uint32_t qb[NWD][2];
  {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(p.q8 + ((int64_t)b * p.H + g * R + (gq < R ? gq : 0)) * D);
#pragma unroll
    for (int kk = 0; kk < NWD; ++kk) {
      qb[kk][0] = gq < R ? __ldg(qw + 8 * kk + tq) : 0u;
      qb[kk][1] = gq < R ? __ldg(qw + 8 * kk + 4 + tq) : 0u;
    }
  }
  cp_async_wait<1>();
  __syncthreads();
  // phase 1: warp w scores keys 32w .. 32w+31 of the split (two 16-key tiles)
  const int h0 = 2 * tq, h1 = 2 * tq + 1;
#pragma unroll
  for (int grp = 0; grp < 2; ++grp) {
    const int r0 = warp * 32 + grp * 16 + gq, r1 = r0 + 8;
    uint32_t m0[NWD], l0[NWD], m1[NWD], l1[NWD];
#pragma unroll
    for (int jj = 0; jj < NWD; ++jj) {
      const int o0 = r0 * RB + ((jj ^ row_swizzle<D>(r0)) << 4) + 4 * tq;
      const int o1 = r1 * RB + ((jj ^ row_swizzle<D>(r1)) << 4) + 4 * tq;
      m0[jj] = *reinterpret_cast<const uint32_t*>(msb + o0);
      l0[jj] = *reinterpret_cast<const uint32_t*>(lsb + o0);
      m1[jj] = *reinterpret_cast<const uint32_t*>(msb + o1);
      l1[jj] = *reinterpret_cast<const uint32_t*>(lsb + o1);
    }
    // k8 = 16*msb + lsb of 4 dims: low nibbles for the first D/2 dims, high after
    auto full = [](uint32_t mw, uint32_t lw, bool hi) -> uint32_t {
      return hi ? ((mw & 0xF0F0F0F0u) | ((lw >> 4) & 0x0F0F0F0Fu))
                : (((mw << 4) & 0xF0F0F0F0u) | (lw & 0x0F0F0F0Fu));
    };
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int kk = 0; kk < NWD; ++kk) {
      const bool hi = kk >= NWD / 2;
      const int jj = 2 * (hi ? kk - NWD / 2 : kk);
      const uint32_t a[4] = {full(m0[jj], l0[jj], hi), full(m1[jj], l1[jj], hi), full(m0[jj + 1], l0[jj + 1], hi),
                             full(m1[jj + 1], l1[jj + 1], hi)};
      mma_s8_16832(acc, a, qb[kk][0], qb[kk][1]);
    }
    const float ka = ksm[r0], kb = ksm[r1];
    const bool va = kidx[r0] >= 0, vb2 = kidx[r1] >= 0;
    if (h0 < R) {
      ps[r0 * R + h0] = va ? (float)acc[0] * (cq[h0] * ka) : -INFINITY;
      ps[r1 * R + h0] = vb2 ? (float)acc[2] * (cq[h0] * kb) : -INFINITY;
    }
    if (h1 < R) {
      ps[r0 * R + h1] = va ? (float)acc[1] * (cq[h1] * ka) : -INFINITY;
      ps[r1 * R + h1] = vb2 ? (float)acc[3] * (cq[h1] * kb) : -INFINITY;
    }
  }
  __syncthreads();
  // the split's statistics (max, sum) per head -> part_ml; exp2(s - max) -> ps
  {
    float* ml = part_ml + (((int64_t)b * p.H + g * R) * splits + split) * 2;
    float sk[1][R], e[1][R];
    load_heads<R>(ps + tid * R, sk[0]);
    block_softmax<R, 1>(sk, sh, ml, (int64_t)splits * 2, e);
#pragma unroll
    for (int r = 0; r < R; ++r) ps[tid * R + r] = e[0][r];
  }
  cp_async_wait<0>();
  __syncthreads();
  // phase 2: lane = (key row slot rs, 8-dim chunk dc)
  const int dc = lane % LPR, rs = lane / LPR;
  float o[R][8];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) o[r][jj] = 0.f;
#pragma unroll 4
  for (int t = warp * RPW + rs; t < cnt; t += NW * RPW) {
    float vv[8], pr[R];
    unpack8<T>(vs[t * LPR + dc], vv);
    load_heads<R>(ps + t * R, pr);
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) o[r][jj] = fmaf(pr[r], vv[jj], o[r][jj]);
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
      for (int off = LPR; off < 32; off <<= 1) o[r][jj] += __shfl_xor_sync(0xffffffffu, o[r][jj], off);
    }
  __syncthreads();  // every warp is done with the V rows
  float* red = reinterpret_cast<float*>(dsm + L::oV);  // [NW][R][D]
  if (rs == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) red[(warp * R + r) * D + dc * 8 + jj] = o[r][jj];
  }
  __syncthreads();
  for (int i = tid; i < R * D; i += blockDim.x) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) a += red[w * R * D + i];
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
  const int chunks = (p.n_valid + kCtaKeys - 1) / kCtaKeys;
  constexpr size_t smem = scores_smem_bytes<D>();
  cudaError_t e = cudaFuncSetAttribute(decode_scores_kernel<D, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  decode_scores_kernel<D, R><<<dim3(chunks, p.G, p.B), kTok, smem, st>>>(p, w.scores, w.part);
  e = cudaGetLastError();
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
  const int splits = (p.top_k + kAttKeys - 1) / kAttKeys;
  constexpr size_t smem = AttendLayout<D>::kBytes;
  cudaError_t e = cudaFuncSetAttribute(decode_attend_kernel<D, R, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  decode_attend_kernel<D, R, T><<<dim3(splits, p.G, p.B), kAttKeys, smem, st>>>(p, w.ml, w.o);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  decode_combine_kernel<T><<<dim3(p.H, p.B), D, 0, st>>>(p, w.ml, w.o, splits);
  return cudaGetLastError();
}

}  // namespace

DecodeWorkspaceSizes decode_workspace_sizes(const DecodeParams& p) {
  DecodeWorkspaceSizes s;
  const int chunks = (p.n_valid + kCtaKeys - 1) / kCtaKeys;
  const int splits = (p.top_k + kAttKeys - 1) / kAttKeys;
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
