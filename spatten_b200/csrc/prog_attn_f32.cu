// Progressive sparse attention for fp32 tensors (QUANT and DENSE modes).
//
// The reference's CPU configuration runs BERT in fp32; on the GPU those
// shapes are small (batch 1, seq 128), so this path favours exactness over
// throughput: plain fp32 FMA dot products (QUANT: exact int32 dot products
// of the unpacked 4-bit planes), accurate exp2f, the same pass structure and
// decision rules as the tensor-core kernel. One warp per CTA handles 8
// query rows in turn; lane j owns keys j, j+32, ...; the per-CTA column sums
// of P' live in shared memory (N <= kMaxN) and are written as the CTA's
// token-importance partial.
#include <climits>

#include "common.cuh"
#include "kernels.h"

namespace spatten {
namespace {

constexpr int kRows = 8;      // query rows per CTA
constexpr int kMaxN = 8192;   // keys (shared-memory column sums)
enum Mode : int { kQuant = 0, kDense = 1 };

template <int MODE, int D>
struct F32Attn {
  const AttnParams& p;
  float* colsum;  // [N]
  float* qs;      // [D] query row (QUANT: int values)
  float* pc;      // [32] probabilities of the current key chunk
  int lane, z, h, kvh, mt;

  // integer (QUANT) or fp32 (DENSE) score of key n for the query row in qs,
  // in the log2 domain; full = include the LSB plane
  SPATTEN_DEV float score(int n, float c2, bool full) const {
    float acc = 0.f;
    if (MODE == kQuant) {
      const uint8_t* mp = static_cast<const uint8_t*>(p.k0) + (int64_t)z * p.k_sz + (int64_t)kvh * p.k_sh + (int64_t)n * p.k_sn;
      const uint8_t* lp = static_cast<const uint8_t*>(p.k1) + (int64_t)z * p.k_sz + (int64_t)kvh * p.k_sh + (int64_t)n * p.k_sn;
      int a = 0;
#pragma unroll 8
      for (int b = 0; b < D / 2; ++b) {
        const int mb = mp[b], lb = lp[b];
        int m0 = mb & 15, m1 = mb >> 4;
        m0 = m0 >= 8 ? m0 - 16 : m0;
        m1 = m1 >= 8 ? m1 - 16 : m1;
        int k0 = 16 * m0, k1 = 16 * m1;
        if (full) {
          k0 += lb & 15;
          k1 += lb >> 4;
        }
        a += (int)qs[b] * k0 + (int)qs[b + D / 2] * k1;
      }
      const float ks = p.k_scale[((int64_t)z * p.Hkv + kvh) * p.N + n];
      acc = (float)a * (c2 * ks);
    } else {
      const float* kp = static_cast<const float*>(p.k0) + (int64_t)z * p.k_sz + (int64_t)kvh * p.k_sh + (int64_t)n * p.k_sn;
#pragma unroll 8
      for (int d = 0; d < D; ++d) acc = fmaf(qs[d], kp[d], acc);
      acc *= c2;
    }
    return acc;
  }

  SPATTEN_DEV float biased(float s, int row, int n) const {
    if (p.bias)
      s += p.bias[(int64_t)z * p.b_sz + (int64_t)h * p.b_sh + (int64_t)row * p.b_sm + (int64_t)n * p.b_sn] * kLog2e;
    if (p.causal && n > row + (p.N - p.M)) s = -INFINITY;
    if (p.key_limit && n >= p.key_limit[(int64_t)z * p.M + row]) s = -INFINITY;
    return s;
  }

  // row statistics (max, sum of exp2) of the score over all keys
  SPATTEN_DEV void stats(int row, float c2, bool full, float& m, float& l) const {
    float lm = -INFINITY, ll = 0.f;
    for (int n = lane; n < p.N; n += 32) {
      const float s = biased(score(n, c2, full), row, n);
      const float mn = fmaxf(lm, s);
      if (mn == -INFINITY) continue;
      ll = ll * exp2f(lm - mn) + exp2f(s - mn);
      lm = mn;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, lm, o);
      const float lo = __shfl_xor_sync(0xffffffffu, ll, o);
      const float mn = fmaxf(lm, mo);
      if (mn != -INFINITY) {
        ll = ll * exp2f(lm - mn) + lo * exp2f(mo - mn);
        lm = mn;
      }
    }
    m = lm;
    l = ll;
  }

  // Count V prune: the row's v_count-th smallest (score, key) pair over its
  // keys, ties to the smaller key (each lane keeps its kMaxVPruneCount
  // smallest pairs, then v_count rounds of a warp arg-min over the lists).
  SPATTEN_DEV void count_threshold(int row, float c2, bool full, float& kvs, int& kvn) const {
    float cv[kMaxVPruneCount];
    int cn[kMaxVPruneCount];
#pragma unroll
    for (int q = 0; q < kMaxVPruneCount; ++q) {
      cv[q] = INFINITY;
      cn[q] = INT_MAX;
    }
    for (int n = lane; n < p.N; n += 32) {
      float x = biased(score(n, c2, full), row, n);
      int xn = n;
      if (!(x < cv[kMaxVPruneCount - 1])) continue;
#pragma unroll
      for (int q = 0; q < kMaxVPruneCount; ++q) {
        if (x < cv[q] || (x == cv[q] && xn < cn[q])) {
          const float tv = cv[q];
          const int tn = cn[q];
          cv[q] = x;
          cn[q] = xn;
          x = tv;
          xn = tn;
        }
      }
    }
    int head = 0;
    for (int t = 0; t < p.v_count; ++t) {
      float hv = INFINITY;
      int hn = INT_MAX;
#pragma unroll
      for (int q = 0; q < kMaxVPruneCount; ++q)
        if (q == head) {
          hv = cv[q];
          hn = cn[q];
        }
      float bv = hv;
      int bn = hn;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int on = __shfl_xor_sync(0xffffffffu, bn, o);
        if (ov < bv || (ov == bv && on < bn)) {
          bv = ov;
          bn = on;
        }
      }
      kvs = bv;
      kvn = bn;
      if (hv == bv && hn == bn) ++head;  // keys are unique: the owning lane pops
    }
  }

  SPATTEN_DEV void run() {
    for (int i = lane; i < p.N; i += 32) colsum[i] = 0.f;
    __syncwarp();
    float hsum = 0.f;
    const int hslot = p.out_head_map ? p.out_head_map[h] : h;
    const bool out_ok = hslot >= 0 && hslot < p.out_head_slots;
    for (int r = 0; r < kRows; ++r) {
      const int row = mt * kRows + r;
      if (row >= p.M) break;
      // query row -> shared memory
      for (int d = lane; d < D; d += 32) {
        if (MODE == kQuant) {
          const int8_t* q8 = static_cast<const int8_t*>(p.q) + (int64_t)z * p.q_sz + (int64_t)h * p.q_sh + (int64_t)row * p.q_sm;
          qs[d] = (float)q8[d];
        } else {
          const float* qf = static_cast<const float*>(p.q) + (int64_t)z * p.q_sz + (int64_t)h * p.q_sh + (int64_t)row * p.q_sm;
          qs[d] = qf[d];
        }
      }
      __syncwarp();
      const float c2 = (MODE == kQuant)
                           ? p.q_scale[((int64_t)z * p.H + h) * p.M + row] * p.sm_scale * kLog2e
                           : p.sm_scale * kLog2e;
      float m, l;
      stats(row, c2, false, m, l);
      bool full = false;
      if (MODE == kQuant) {
        full = __frcp_rn(l) < p.refetch_thr;
        if (full) stats(row, c2, true, m, l);
        if (p.refetch_out && lane == 0) p.refetch_out[((int64_t)z * p.H + h) * p.M + row] = full;
      }
      float kvs = -INFINITY;
      int kvn = -1;
      if (p.v_count > 0) count_threshold(row, c2, full, kvs, kvn);
      const float inv_l = (m == -INFINITY || l <= 0.f) ? 0.f : 1.f / l;
      const float mm = m == -INFINITY ? 0.f : m;
      float o[D / 32];
#pragma unroll
      for (int i = 0; i < D / 32; ++i) o[i] = 0.f;
      const float* vb = static_cast<const float*>(p.v) + (int64_t)z * p.v_sz + (int64_t)kvh * p.v_sh;
      for (int n0 = 0; n0 < p.N; n0 += 32) {
        const int n = n0 + lane;
        float pr = 0.f;
        if (n < p.N) {
          const float s = biased(score(n, c2, full), row, n);
          pr = exp2f(s - mm) * inv_l;
          if (pr < p.v_thr) pr = 0.f;
          if (p.v_count > 0 && (s < kvs || (s == kvs && n <= kvn))) pr = 0.f;
          colsum[n] += pr;
        }
        pc[lane] = pr;
        __syncwarp();
        const int cnt = min(32, p.N - n0);
        for (int j = 0; j < cnt; ++j) {
          const float pj = pc[j];
          const float* vr = vb + (int64_t)(n0 + j) * p.v_sn;
#pragma unroll
          for (int i = 0; i < D / 32; ++i) o[i] = fmaf(pj, vr[lane + 32 * i], o[i]);
        }
        __syncwarp();
      }
      float* orow = static_cast<float*>(p.out) + (int64_t)z * p.o_sz + (int64_t)hslot * p.o_sh + (int64_t)row * p.o_sm;
#pragma unroll
      for (int i = 0; i < D / 32; ++i) {
        if (out_ok) orow[lane + 32 * i] = o[i];
        hsum += fabsf(o[i]);
      }
      __syncwarp();
    }
    if (p.tok_partial) {
      float* tp = p.tok_partial + (((int64_t)z * p.H + h) * p.mtiles + mt) * p.N;
      for (int i = lane; i < p.N; i += 32) tp[i] = colsum[i];
    }
    if (p.head_partial) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) hsum += __shfl_xor_sync(0xffffffffu, hsum, o);
      if (lane == 0) p.head_partial[((int64_t)z * p.H + h) * p.mtiles + mt] = hsum;
    }
  }
};

template <int MODE, int D>
__global__ void __launch_bounds__(32) prog_attn_f32_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ float smf[];
  F32Attn<MODE, D> a{p, smf, smf + p.N, smf + p.N + D, (int)threadIdx.x, (int)blockIdx.z,
                     (int)blockIdx.y, (int)(blockIdx.y / (p.H / p.Hkv)), (int)blockIdx.x};
  a.run();
}

template <int MODE, int D>
cudaError_t launch_f32_t(const AttnParams& p, cudaStream_t st) {
  const size_t smem = (size_t)(p.N + D + 32) * sizeof(float);
  auto kern = prog_attn_f32_kernel<MODE, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)p.mtiles, (unsigned)p.H, (unsigned)p.Z);
  kern<<<grid, 32, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

int f32_tile_rows() { return kRows; }
int f32_max_keys() { return kMaxN; }

cudaError_t launch_prog_attn_f32(const AttnParams& p, cudaStream_t st) {
  if (p.N > kMaxN) return cudaErrorInvalidValue;
  if (p.mode == kQuant) return p.D == 64 ? launch_f32_t<kQuant, 64>(p, st) : launch_f32_t<kQuant, 128>(p, st);
  if (p.mode == kDense) return p.D == 64 ? launch_f32_t<kDense, 64>(p, st) : launch_f32_t<kDense, 128>(p, st);
  return cudaErrorInvalidValue;
}

}  // namespace spatten
