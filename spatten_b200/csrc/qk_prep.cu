// Per-head RMSNorm (QK-norm) + rotary position embedding of Q and K, with the
// int8 quantisation of Q, in one pass over the projections.
//
// The Qwen3 attention (installed transformers/models/qwen3/modeling_qwen3.py,
// Qwen3Attention.forward) normalises every query / key head row with
// Qwen3RMSNorm, then applies apply_rotary_pos_emb; the progressive attention
// then needs Q as int8. Done by the HF modules that is a dozen elementwise
// launches per layer over the projections (fp32 copies, pow, mean, rsqrt,
// two multiplies, the rotate_half concatenation, negation, ...). This kernel
// reads each projection once and reproduces the HF arithmetic step for step,
// with each intermediate rounded where HF rounds it:
//   x   = float(row)                       (fp16 / bf16 -> fp32)
//   var = sum(x * x) / D                   (fp32; the summation order is this
//                                           kernel's own, a tree over lanes)
//   y   = T(x * rsqrtf(var + eps))         (rounded to the activation type)
//   n   = T(w * y)                         (the norm weight)
//   out = T(T(n * cos) + T(rot(n) * sin))  rot(n) = (-n[D/2:], n[:D/2])
// and then, for Q, the quantisation kernels' arithmetic (scale = max|out| /
// 127, q8 = rint(out / scale)). Outputs: K (and Q in the dense mode) in the
// activation type, token-major [B, S, H, D] like the HF tensors; Q int8
// head-major [B, H, S, D] + scale [B, H, S] in the quantised mode.
//
// One warp per token; D / 8 lanes per head row (one 16-byte load each), so a
// warp step covers 32 / (D / 8) head rows; the row sum is a shuffle tree over
// the row's lanes and the rotary partner of a lane's dims sits D/16 lanes
// away. HBM-bound: reads the projections and cos / sin once.
#include "common.cuh"
#include "kernels.h"

namespace spatten {

namespace {

// a and b rounded to T (nearest even) by one packed conversion, which halves
// the conversion-pipe work of rounding every intermediate to T; returns the
// packed pair
template <typename T>
SPATTEN_DEV uint32_t rnd2(float& a, float& b) {
  const uint32_t u = pack2<T>(a, b);
  const T* e = reinterpret_cast<const T*>(&u);
  a = to_f32<T>(e[0]);
  b = to_f32<T>(e[1]);
  return u;
}

template <typename T>
SPATTEN_DEV void load8(const T* p, float (&f)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32<T>(e[i]);
}

template <typename T, int D>
__global__ void __launch_bounds__(256) qk_prep_kernel(const QkPrepParams p) {
  constexpr int LPR = D / 8;     // lanes per head row
  constexpr int RPS = 32 / LPR;  // head rows per warp step
  const int lane = threadIdx.x & 31, sub = lane / LPR, li = lane % LPR;
  const int64_t tok = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t T_ = (int64_t)p.B * p.S;
  if (tok >= T_) return;  // warp-uniform
  const int b = (int)(tok / p.S), s = (int)(tok % p.S);
  float c[8], sn[8], wq[8], wk[8];
  load8<T>(static_cast<const T*>(p.cos) + (int64_t)b * p.cs_sb + (int64_t)s * p.cs_ss + li * 8, c);
  load8<T>(static_cast<const T*>(p.sin) + (int64_t)b * p.cs_sb + (int64_t)s * p.cs_ss + li * 8, sn);
  load8<T>(static_cast<const T*>(p.q_w) + li * 8, wq);
  load8<T>(static_cast<const T*>(p.k_w) + li * 8, wk);
  const int rows = p.Hq + p.Hk;
  for (int r0 = 0; r0 < rows; r0 += RPS) {
    const int hr = r0 + sub;  // head row: query heads first, then key heads
    const bool live = hr < rows;
    const bool isq = hr < p.Hq;
    const int h = isq ? hr : hr - p.Hq;
    const T* src = live ? (isq ? static_cast<const T*>(p.q) + tok * p.q_st + (int64_t)h * D
                               : static_cast<const T*>(p.k) + tok * p.k_st + (int64_t)h * D)
                        : static_cast<const T*>(p.q);
    float x[8];
    if (live) {
      load8<T>(src + li * 8, x);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = 0.f;
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss * (1.0f / (float)D) + p.eps);
    float n[8];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      float a = x[i] * inv, b = x[i + 1] * inv;
      rnd2<T>(a, b);
      n[i] = (isq ? wq[i] : wk[i]) * a;
      n[i + 1] = (isq ? wq[i + 1] : wk[i + 1]) * b;
      rnd2<T>(n[i], n[i + 1]);
    }
    // rotary partner: dims d +- D/2 live LPR/2 lanes away
    float pn[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) pn[i] = __shfl_xor_sync(0xffffffffu, n[i], LPR / 2);
    const bool first_half = li < LPR / 2;
    float o[8];
    uint4 packed;  // o as T, for the stores
    uint32_t* pw = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      float a0 = n[i] * c[i], a1 = n[i + 1] * c[i + 1];
      float b0 = (first_half ? -pn[i] : pn[i]) * sn[i], b1 = (first_half ? -pn[i + 1] : pn[i + 1]) * sn[i + 1];
      rnd2<T>(a0, a1);
      rnd2<T>(b0, b1);
      o[i] = a0 + b0;
      o[i + 1] = a1 + b1;
      pw[i >> 1] = rnd2<T>(o[i], o[i + 1]);
    }
    if (!isq) {
      if (live) *reinterpret_cast<uint4*>(static_cast<T*>(p.k_out) + tok * p.ko_st + (int64_t)h * D + li * 8) = packed;
      continue;
    }
    if (p.q_out && live)
      *reinterpret_cast<uint4*>(static_cast<T*>(p.q_out) + tok * p.qo_st + (int64_t)h * D + li * 8) = packed;
    if (p.q8) {
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(o[i]));
#pragma unroll
      for (int off = LPR / 2; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const float sc = div127_rn(amax);
      const float rc = rcp_approx(sc);
      uint32_t w[2] = {0u, 0u};
      if (sc != 0.f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i >> 2] |= ((uint32_t)quant_div_fadd(o[i], sc, rc) & 0xFFu) << (8 * (i & 3));
      }
      if (live) {
        const int64_t orow = ((int64_t)b * p.Hq + h) * p.S + s;
        *reinterpret_cast<uint2*>(p.q8 + orow * D + li * 8) = make_uint2(w[0], w[1]);
        if (li == 0) p.q_scale[orow] = sc;
      }
    }
  }
}

template <typename T>
cudaError_t launch_t(const QkPrepParams& p, cudaStream_t st) {
  const int64_t T_ = (int64_t)p.B * p.S;
  const unsigned blocks = (unsigned)((T_ + 7) / 8);
  if (p.D == 128) qk_prep_kernel<T, 128><<<blocks, 256, 0, st>>>(p);
  else if (p.D == 64) qk_prep_kernel<T, 64><<<blocks, 256, 0, st>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qk_prep(const QkPrepParams& p, cudaStream_t st) {
  if (p.dtype == kF16) return launch_t<__half>(p, st);
  if (p.dtype == kBF16) return launch_t<__nv_bfloat16>(p, st);
  return cudaErrorInvalidValue;
}

}  // namespace spatten
