// Per-row symmetric int8 quantisation of Q and of K into 4-bit MSB/LSB planes.
//
// Replaces the reference's float split of K (k_msb = 0.8*K, k_lsb = 0.2*K,
// spatten_bert_ultimate.py:184-185) with an integer one:
//   scale = max|x| / 127, x8 = clamp(rint(x / scale), -127, 127)
//   msb = x8 >> 4 (signed nibble), lsb = x8 & 15, x8 == 16*msb + lsb.
// Packing: byte p of a row holds dim p (low nibble) and dim p + D/2 (high).
//
// HBM-bound: one warp per row, each lane owns D/32 consecutive dims; the row
// max is a warp reduction. Reads 2*D (fp16) bytes and writes D (+4) bytes per
// row; the grid is a grid-stride loop sized to the SM count.
#include "common.cuh"
#include "kernels.h"

namespace spatten {

template <typename T, int E>
SPATTEN_DEV void load_row(const T* p, float (&v)[E]) {
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = to_f32<T>(p[e]);
}

template <typename T, int E, bool PLANES>
__global__ void __launch_bounds__(256) quant_rows_kernel(const T* __restrict__ x, int Z, int H,
                                                         int M, int64_t sz, int64_t sh,
                                                         int64_t sm, int8_t* __restrict__ q8,
                                                         uint8_t* __restrict__ msb,
                                                         uint8_t* __restrict__ lsb,
                                                         float* __restrict__ scale) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)Z * H * M;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += warps) {
    const int64_t m = r % M;
    const int64_t zh = r / M;
    const int64_t h = zh % H, z = zh / H;
    const T* src = x + z * sz + h * sh + m * sm + lane * E;
    float v[E];
    load_row<T, E>(src, v);
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) amax = fmaxf(amax, fabsf(v[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = __fdiv_rn(amax, 127.0f);
    int qv[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      int t = 0;
      if (s != 0.f) {
        t = __float2int_rn(__fdiv_rn(v[e], s));
        t = max(-127, min(127, t));
      }
      qv[e] = t;
    }
    if (lane == 0) scale[r] = s;
    if (!PLANES) {
      int8_t* dst = q8 + r * D + lane * E;
#pragma unroll
      for (int e = 0; e < E; ++e) dst[e] = (int8_t)qv[e];
    } else {
      // lane l < 16 owns dims [l*E, l*E+E) = the low nibbles of bytes
      // [l*E, l*E+E); lane l+16 owns the dims D/2 above them (high nibbles).
      int hi[E];
#pragma unroll
      for (int e = 0; e < E; ++e) hi[e] = __shfl_down_sync(0xffffffffu, qv[e], 16);
      if (lane < 16) {
        uint8_t* pm = msb + r * (D / 2) + lane * E;
        uint8_t* pl = lsb + r * (D / 2) + lane * E;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int lo8 = qv[e], hi8 = hi[e];
          pm[e] = (uint8_t)(((lo8 >> 4) & 15) | (((hi8 >> 4) & 15) << 4));
          pl[e] = (uint8_t)((lo8 & 15) | ((hi8 & 15) << 4));
        }
      }
    }
  }
}

template <typename T, bool PLANES>
static cudaError_t launch_quant_t(const void* x, int Z, int H, int M, int D, int64_t sz,
                                  int64_t sh, int64_t sm, int8_t* q8, uint8_t* msb, uint8_t* lsb,
                                  float* scale, cudaStream_t st, int n_sm) {
  const int64_t rows = (int64_t)Z * H * M;
  const int threads = 256;
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)n_sm * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const T* xp = static_cast<const T*>(x);
#define SPATTEN_QL(E)                                                                        \
  quant_rows_kernel<T, E, PLANES><<<(unsigned)blocks, threads, 0, st>>>(xp, Z, H, M, sz, sh, \
                                                                        sm, q8, msb, lsb, scale)
  switch (D / 32) {
    case 1: SPATTEN_QL(1); break;
    case 2: SPATTEN_QL(2); break;
    case 4: SPATTEN_QL(4); break;
    case 8: SPATTEN_QL(8); break;
    default: return cudaErrorInvalidValue;
  }
#undef SPATTEN_QL
  return cudaGetLastError();
}

cudaError_t launch_quant(int dtype, bool planes, const void* x, int Z, int H, int M, int D,
                         int64_t sz, int64_t sh, int64_t sm, int8_t* q8, uint8_t* msb,
                         uint8_t* lsb, float* scale, cudaStream_t st, int n_sm) {
  if (planes) {
    switch (dtype) {
      case kF16: return launch_quant_t<__half, true>(x, Z, H, M, D, sz, sh, sm, q8, msb, lsb, scale, st, n_sm);
      case kBF16: return launch_quant_t<__nv_bfloat16, true>(x, Z, H, M, D, sz, sh, sm, q8, msb, lsb, scale, st, n_sm);
      case kF32: return launch_quant_t<float, true>(x, Z, H, M, D, sz, sh, sm, q8, msb, lsb, scale, st, n_sm);
    }
  } else {
    switch (dtype) {
      case kF16: return launch_quant_t<__half, false>(x, Z, H, M, D, sz, sh, sm, q8, msb, lsb, scale, st, n_sm);
      case kBF16: return launch_quant_t<__nv_bfloat16, false>(x, Z, H, M, D, sz, sh, sm, q8, msb, lsb, scale, st, n_sm);
      case kF32: return launch_quant_t<float, false>(x, Z, H, M, D, sz, sh, sm, q8, msb, lsb, scale, st, n_sm);
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace spatten
