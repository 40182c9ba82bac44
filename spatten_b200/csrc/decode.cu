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

// 3. exact attention over the kept keys, in splits of kTok keys: grid
// (splits, G, B). The V rows of the split's kept keys are requested first
// (cp.async into shared memory) so that their gather overlaps phase 1.
// Phase 1: one kept key per thread, full int8 scores for the R heads ->
// smem; split max / sum per head. Phase 2: P.V out of shared memory, a lane
// per 8 dims of a row; the per-warp partial outputs are then summed in the
// (by then free) V buffer.
template <int D>
__host__ __device__ constexpr size_t attend_smem_bytes() {
  return (size_t)kTok * D * 2;  // V rows, 16-bit
}

template <int D, int R, typename T>
__global__ void __launch_bounds__(kTok) decode_attend_kernel(const DecodeParams p, float* part_ml,
                                                             float* part_o) {
  constexpr int LPR = D / 8, RPW = 32 / LPR, NW = kTok / 32;  // 16-byte chunks per V row
  static_assert(NW * R * D * sizeof(float) <= attend_smem_bytes<D>(), "partial outputs fit the V buffer");
  extern __shared__ __align__(128) uint8_t dsm[];
  uint4* vs = reinterpret_cast<uint4*>(dsm);  // [kTok][LPR]
  __shared__ __align__(16) uint32_t qs[R * D / 4];
  __shared__ float cq[R];
  __shared__ float ps[R * kTok];  // exp2(s - m_split) per head and key
  __shared__ float sh[R * (kTok / 32) * 2];
  __shared__ int kidx[kTok];
  const int b = blockIdx.z, g = blockIdx.y, split = blockIdx.x, splits = gridDim.x;
  for (int i = threadIdx.x; i < R * D / 4; i += blockDim.x)
    qs[i] = reinterpret_cast<const uint32_t*>(p.q8 + ((int64_t)b * p.H + g * R) * D)[i];
  if (threadIdx.x < R) cq[threadIdx.x] = p.q_scale[(int64_t)b * p.H + g * R + threadIdx.x] * p.sm_scale * kLog2e;
  const int j = split * kTok + threadIdx.x;  // position in the kept list
  const int64_t nk = j < p.top_k ? p.kept[(int64_t)b * p.top_k + j] : -1;
  const int n = (nk >= 0 && nk < p.n_valid) ? (int)nk : -1;  // -1: no key
  kidx[threadIdx.x] = n;
  __syncthreads();
  const T* vb = static_cast<const T*>(p.v) + ((int64_t)b * p.G + g) * p.N * D;
  const int cnt = min(kTok, p.top_k - split * kTok);
  for (int c = threadIdx.x; c < cnt * LPR; c += kTok) {
    const int t = c / LPR, dc = c % LPR, nn = kidx[t];
    cp_async16(vs + c, vb + (int64_t)(nn >= 0 ? nn : 0) * D + dc * 8, nn >= 0);
  }
  cp_async_commit();
  float s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) s[r] = -INFINITY;
  {
    const bool okk[1] = {n >= 0};
    const int64_t key[1] = {((int64_t)b * p.G + g) * p.N + (n >= 0 ? n : 0)};
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
  cp_async_wait<0>();
  __syncthreads();
  // phase 2: lane = (key row slot rs, 8-dim chunk dc)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int dc = lane % LPR, rs = lane / LPR;
  float o[R][8];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) o[r][jj] = 0.f;
#pragma unroll 4
  for (int t = warp * RPW + rs; t < cnt; t += NW * RPW) {
    float vv[8];
    unpack8<T>(vs[t * LPR + dc], vv);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float pr = ps[r * kTok + t];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) o[r][jj] = fmaf(pr, vv[jj], o[r][jj]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
      for (int off = LPR; off < 32; off <<= 1) o[r][jj] += __shfl_xor_sync(0xffffffffu, o[r][jj], off);
    }
  __syncthreads();  // every warp is done with the V rows
  float* red = reinterpret_cast<float*>(dsm);  // [NW][R][D]
  if (rs == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) red[(warp * R + r) * D + dc * 8 + jj] = o[r][jj];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R * D; i += blockDim.x) {
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
  const int splits = (p.top_k + kTok - 1) / kTok;
  constexpr size_t smem = attend_smem_bytes<D>();
  cudaError_t e = cudaFuncSetAttribute(decode_attend_kernel<D, R, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  decode_attend_kernel<D, R, T><<<dim3(splits, p.G, p.B), kTok, smem, st>>>(p, w.ml, w.o);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  decode_combine_kernel<T><<<dim3(p.H, p.B), D, 0, st>>>(p, w.ml, w.o, splits);
  return cudaGetLastError();
}

}  // namespace

DecodeWorkspaceSizes decode_workspace_sizes(const DecodeParams& p) {
  DecodeWorkspaceSizes s;
  const int chunks = (p.n_valid + kCtaKeys - 1) / kCtaKeys;
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
