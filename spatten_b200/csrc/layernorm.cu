// Residual add + LayerNorm over rows of n features:
//   h = round_T(x + res)            (res optional; the add of HF's BertOutput)
//   y = (h - mean) * rstd * gamma + beta,  rstd = 1 / sqrt(var + eps)
// mean and the biased variance in fp32, two passes over the row held in
// registers. This is the tail of the HF BertLayer that the reference's
// encoder loop runs for every layer (module.py:75): BertSelfOutput's
// LayerNorm (after the output projection and its residual) and BertOutput's
// residual add + LayerNorm, in one launch each instead of torch's add and
// layer-norm kernels.
//
// HBM-bound: reads 2 (or 4 with res) bytes and writes 2 bytes per element.
// A warp per row (a grid-stride loop over rows); lane l holds the 16-byte vectors l, l + 32, ... of the
// row (consecutive lanes read consecutive 16 bytes); n = 256 * VPL.
#include "common.cuh"
#include "kernels.h"

namespace spatten {

namespace {

template <typename T>
SPATTEN_DEV void unpack8(const uint4& u, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32<T>(e[i]);
}

template <typename T, int VPL>
__global__ void __launch_bounds__(256) add_ln_kernel(const T* __restrict__ x, const T* __restrict__ res,
                                                     const T* __restrict__ gamma,
                                                     const T* __restrict__ beta, T* __restrict__ y,
                                                     int64_t rows, int64_t xs, int64_t rs, int64_t ys,
                                                     float eps) {
  constexpr int N = 256 * VPL;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  // one resident wave of CTAs; each warp walks rows warps apart
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    float h[VPL][8];
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * xs);
    uint4 raw[VPL];
#pragma unroll
    for (int k = 0; k < VPL; ++k) raw[k] = __ldg(xr + k * 32 + lane);
    if (res) {
      const uint4* rr = reinterpret_cast<const uint4*>(res + row * rs);
      uint4 rw[VPL];
#pragma unroll
      for (int k = 0; k < VPL; ++k) rw[k] = __ldg(rr + k * 32 + lane);
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        float a[8], b[8];
        unpack8<T>(raw[k], a);
        unpack8<T>(rw[k], b);
        // the residual sum is rounded to T, as the T-typed add before the
        // layer norm rounds it
#pragma unroll
        for (int i = 0; i < 8; ++i) h[k][i] = to_f32<T>(from_f32<T>(a[i] + b[i]));
      }
    } else {
#pragma unroll
      for (int k = 0; k < VPL; ++k) unpack8<T>(raw[k], h[k]);
    }
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k)
#pragma unroll
      for (int i = 0; i < 8; ++i) s += h[k][i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * (1.0f / (float)N);
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = h[k][i] - mean;
        q += d * d;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = rsqrtf(q * (1.0f / (float)N) + eps);
    const uint4* gr = reinterpret_cast<const uint4*>(gamma);
    const uint4* br = reinterpret_cast<const uint4*>(beta);
    uint4* yr = reinterpret_cast<uint4*>(y + row * ys);
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      float g[8], b[8];
      unpack8<T>(__ldg(gr + k * 32 + lane), g);
      unpack8<T>(__ldg(br + k * 32 + lane), b);
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 8; i += 2)
        ow[i >> 1] = pack2<T>((h[k][i] - mean) * rstd * g[i] + b[i],
                              (h[k][i + 1] - mean) * rstd * g[i + 1] + b[i + 1]);
      yr[k * 32 + lane] = o;
    }
  }
}

// CTAs of 256 threads resident per SM for add_ln_kernel<T, V> (occupancy
// calculator, once per instantiation)
template <typename T, int V>
int ln_blocks_per_sm() {
  static int per_sm = 0;
  if (per_sm == 0) {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, add_ln_kernel<T, V>, 256, 0) != cudaSuccess || b < 1) b = 1;
    per_sm = b;
  }
  return per_sm;
}

template <typename T>
cudaError_t launch_t(const void* x, const void* res, const void* gamma, const void* beta, void* y,
                     int64_t rows, int n, int64_t xs, int64_t rs, int64_t ys, float eps, int n_sm,
                     cudaStream_t st) {
  const int64_t want = (rows + 7) / 8;
  const T* xp = static_cast<const T*>(x);
  const T* rp = static_cast<const T*>(res);
  const T* gp = static_cast<const T*>(gamma);
  const T* bp = static_cast<const T*>(beta);
  T* yp = static_cast<T*>(y);
#define SPATTEN_LN(V)                                                                              \
  {                                                                                                \
    const int64_t wave = (int64_t)ln_blocks_per_sm<T, V>() * (n_sm > 0 ? n_sm : 1);                 \
    const unsigned blocks = (unsigned)(want < wave ? want : wave);                                  \
    add_ln_kernel<T, V><<<blocks, 256, 0, st>>>(xp, rp, gp, bp, yp, rows, xs, rs, ys, eps);        \
  }
  switch (n) {
    case 256: SPATTEN_LN(1); break;
    case 512: SPATTEN_LN(2); break;
    case 768: SPATTEN_LN(3); break;
    case 1024: SPATTEN_LN(4); break;
    case 1536: SPATTEN_LN(6); break;
    case 2048: SPATTEN_LN(8); break;
    default: return cudaErrorInvalidValue;
  }
#undef SPATTEN_LN
  return cudaGetLastError();
}

}  // namespace

bool add_layer_norm_supported(int n) {
  return n == 256 || n == 512 || n == 768 || n == 1024 || n == 1536 || n == 2048;
}

cudaError_t launch_add_layer_norm(const void* x, const void* res, const void* gamma, const void* beta,
                                  void* y, int64_t rows, int n, int64_t xs, int64_t rs, int64_t ys,
                                  int dtype, float eps, int n_sm, cudaStream_t st) {
  if (dtype == kF16) return launch_t<__half>(x, res, gamma, beta, y, rows, n, xs, rs, ys, eps, n_sm, st);
  if (dtype == kBF16)
    return launch_t<__nv_bfloat16>(x, res, gamma, beta, y, rows, n, xs, rs, ys, eps, n_sm, st);
  return cudaErrorInvalidValue;
}

}  // namespace spatten
