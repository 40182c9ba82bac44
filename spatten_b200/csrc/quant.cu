// Per-row symmetric int8 quantisation of Q and of K into 4-bit MSB/LSB planes.
//
// Replaces the reference's float split of K (k_msb = 0.8*K, k_lsb = 0.2*K,
// spatten_bert_ultimate.py:184-185) with an integer one:
//   scale = max|x| / 127, x8 = clamp(rint(x / scale), -127, 127)
// (x / scale correctly rounded, as IEEE division gives it: quant_div)
//   msb = x8 >> 4 (signed nibble), lsb = x8 & 15, x8 == 16*msb + lsb.
// Packing: byte p of a row holds dim p (low nibble) and dim p + D/2 (high).
//
// HBM-bound. Rows whose start is 16-byte aligned (the usual case: contiguous
// tensors and the strided Q/K views of a fused QKV GEMM output) take the
// vector kernel, D / (16 / sizeof(T)) lanes per row with one 16-byte load
// each; others take a warp per row, each lane owning D/32 consecutive dims.
// Reads 2*D (fp16) bytes and writes D (+4) bytes per row; the grid is a
// grid-stride loop sized to the SM count.
#include "common.cuh"
#include "kernels.h"

namespace spatten {

// (z, h, m) of row r of a [Z, H, M] grid of rows; 32-bit divisions when the
// row count allows (a 64-bit division is a long instruction sequence).
SPATTEN_DEV void row_coords(int64_t r, int M, int H, int64_t& m, int64_t& h, int64_t& z) {
  if (r < 0x7FFFFFFF) {
    const uint32_t ru = (uint32_t)r, zh = ru / (uint32_t)M;
    m = ru - zh * (uint32_t)M;
    z = zh / (uint32_t)H;
    h = zh - (uint32_t)z * (uint32_t)H;
  } else {
    m = r % M;
    const int64_t zh = r / M;
    h = zh % H;
    z = zh / H;
  }
}

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
    int64_t m, h, z;
    row_coords(r, M, H, m, h, z);
    const T* src = x + z * sz + h * sh + m * sm + lane * E;
    float v[E];
    load_row<T, E>(src, v);
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) amax = fmaxf(amax, fabsf(v[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = __fdiv_rn(amax, 127.0f);
    const float rs = s != 0.f ? 1.0f / s : 0.f;
    int qv[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      int t = 0;
      if (s != 0.f) {
        t = quant_div(v[e], s, rs);
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

// Vector variant for rows whose start is 16-byte aligned (every row when the
// base and the strides are): LPR = D / (32 / sizeof(T)) lanes per row, each
// with two 16-byte loads of EPL consecutive elements, 32 / LPR rows per warp
// step; the row max is a reduction over the row's lanes, and the quantised
// bytes leave in one 8- or 16-byte store per lane. Same arithmetic as above.
template <typename T, int D, bool PLANES>
__global__ void __launch_bounds__(256) quant_rows_vec_kernel(const T* __restrict__ x, int Z, int H,
                                                             int M, int64_t sz, int64_t sh,
                                                             int64_t sm, int8_t* __restrict__ q8,
                                                             uint8_t* __restrict__ msb,
                                                             uint8_t* __restrict__ lsb,
                                                             float* __restrict__ scale) {
  constexpr int EPL = 32 / sizeof(T);  // elements per lane: two 16-byte loads
  constexpr int LPR = D / EPL;         // lanes per row
  constexpr int RPW = 32 / LPR;        // rows per warp step
  constexpr int NWORD = EPL / 4;       // packed int8 words per lane
  static_assert(LPR >= 2 && LPR <= 32 && 32 % LPR == 0, "row must span 2..32 lanes");
  const int lane = threadIdx.x & 31, sub = lane / LPR, li = lane % LPR;
  const int64_t rows = (int64_t)Z * H * M;
  const int64_t step = (int64_t)gridDim.x * (blockDim.x >> 5) * RPW;
  // this lane's two 16-byte chunks of row r (zeros past the end)
  auto load = [&](int64_t r, uint4 (&raw)[2]) {
    if (r < rows) {
      int64_t m, h, z;
      row_coords(r, M, H, m, h, z);
      const uint4* src = reinterpret_cast<const uint4*>(x + z * sz + h * sh + m * sm) + 2 * li;
      raw[0] = __ldg(src);
      raw[1] = __ldg(src + 1);
    } else {
      raw[0] = raw[1] = make_uint4(0, 0, 0, 0);
    }
  };
  const int64_t first = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW;
  uint4 nxt[2];
  load(first + sub, nxt);
  // the next step's rows are loaded before this step's are quantised: two
  // steps of loads in flight per lane
  for (int64_t r0 = first; r0 < rows; r0 += step) {
    const int64_t r = r0 + sub;
    const bool live = r < rows;
    const uint4 raw[2] = {nxt[0], nxt[1]};
    load(r0 + step + sub, nxt);
    float v[EPL];
    {
      const T* e = reinterpret_cast<const T*>(raw);
#pragma unroll
      for (int i = 0; i < EPL; ++i) v[i] = to_f32<T>(e[i]);
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = div127_rn(amax);
    const float rs = rcp_approx(s);
    // |x| <= amax and s = RN(amax / 127) keep |x / s| <= 127 * (1 + 2^-23):
    // the rounded quotient never leaves [-127, 127], no clamp needed
    // x / s as x * (1 / s); the exact division only for the lane's values
    // that land within 1e-4 of a rounding tie (quant_div's rule), decided
    // once per lane so that the common path has no branch per value
    int t[EPL];
    bool near_tie = false;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const float y = v[i] * rs;
      float ti;
      t[i] = rint_small(y, ti);
      near_tie |= !(fabsf(y - ti) <= 0.49990f);
    }
    if (s == 0.f) {
#pragma unroll
      for (int i = 0; i < EPL; ++i) t[i] = 0;
    } else if (near_tie) {
#pragma unroll
      for (int i = 0; i < EPL; ++i) t[i] = quant_div(v[i], s, rs);
    }
    uint32_t w[NWORD];
#pragma unroll
    for (int k = 0; k < NWORD; ++k)
      w[k] = ((uint32_t)t[4 * k] & 0xFFu) | (((uint32_t)t[4 * k + 1] & 0xFFu) << 8) |
             (((uint32_t)t[4 * k + 2] & 0xFFu) << 16) | ((uint32_t)t[4 * k + 3] << 24);
    if (live && li == 0) scale[r] = s;
    if (!PLANES) {
      if (live) {
        int8_t* dst = q8 + r * D + li * EPL;
        if constexpr (NWORD == 4) *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        else *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
      }
    } else {
      // lane li < LPR/2 holds dims [li*EPL, +EPL) = the low nibbles of those
      // bytes; lane li + LPR/2 holds the dims D/2 above (the high nibbles)
      uint32_t hw[NWORD];
#pragma unroll
      for (int k = 0; k < NWORD; ++k) hw[k] = __shfl_down_sync(0xffffffffu, w[k], LPR / 2);
      if (live && li < LPR / 2) {
        uint32_t pm[NWORD], pl[NWORD];
#pragma unroll
        for (int k = 0; k < NWORD; ++k) {
          pm[k] = ((w[k] >> 4) & 0x0F0F0F0Fu) | (hw[k] & 0xF0F0F0F0u);
          pl[k] = (w[k] & 0x0F0F0F0Fu) | ((hw[k] & 0x0F0F0F0Fu) << 4);
        }
        uint8_t* dm = msb + r * (D / 2) + li * EPL;
        uint8_t* dl = lsb + r * (D / 2) + li * EPL;
        if constexpr (NWORD == 4) {
          *reinterpret_cast<uint4*>(dm) = make_uint4(pm[0], pm[1], pm[2], pm[3]);
          *reinterpret_cast<uint4*>(dl) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
        } else {
          *reinterpret_cast<uint2*>(dm) = make_uint2(pm[0], pm[1]);
          *reinterpret_cast<uint2*>(dl) = make_uint2(pl[0], pl[1]);
        }
      }
    }
  }
}

template <typename T, int D, bool PLANES>
static cudaError_t launch_quant_vec(const T* x, int Z, int H, int M, int64_t sz, int64_t sh, int64_t sm,
                                    int8_t* q8, uint8_t* msb, uint8_t* lsb, float* scale, cudaStream_t st,
                                    int64_t blocks, int n_sm) {
  constexpr int LPR = D / (32 / (int)sizeof(T));
  if constexpr (LPR >= 2 && LPR <= 32) {
    // one wave: the grid-stride loop gives every resident block the same
    // share of rows (more blocks than fit would leave a partial last wave)
    static int per_sm = 0;
    if (per_sm == 0) {
      int n = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, quant_rows_vec_kernel<T, D, PLANES>, 256, 0) !=
              cudaSuccess ||
          n < 1)
        n = 1;
      per_sm = n;
    }
    const int64_t wave = (int64_t)per_sm * (n_sm > 0 ? n_sm : 1);
    if (blocks > wave) blocks = wave;
    quant_rows_vec_kernel<T, D, PLANES><<<(unsigned)blocks, 256, 0, st>>>(x, Z, H, M, sz, sh, sm, q8, msb,
                                                                          lsb, scale);
    return cudaGetLastError();
  } else {
    return cudaErrorInvalidValue;
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
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (sz * (int64_t)sizeof(T)) % 16 == 0 &&
                   (sh * (int64_t)sizeof(T)) % 16 == 0 && (sm * (int64_t)sizeof(T)) % 16 == 0;
  constexpr int EPL = 32 / sizeof(T);  // elements per lane of the vector kernel
  if (vec && D >= 2 * EPL && D <= 32 * EPL) {
    const int rpw = 32 / (D / EPL);
    int64_t vblocks = (rows + 8 * rpw - 1) / (8 * rpw);
    if (vblocks > cap) vblocks = cap;
    if (vblocks < 1) vblocks = 1;
    switch (D) {
      case 32: return launch_quant_vec<T, 32, PLANES>(xp, Z, H, M, sz, sh, sm, q8, msb, lsb, scale, st, vblocks, n_sm);
      case 64: return launch_quant_vec<T, 64, PLANES>(xp, Z, H, M, sz, sh, sm, q8, msb, lsb, scale, st, vblocks, n_sm);
      case 128: return launch_quant_vec<T, 128, PLANES>(xp, Z, H, M, sz, sh, sm, q8, msb, lsb, scale, st, vblocks, n_sm);
      case 256: return launch_quant_vec<T, 256, PLANES>(xp, Z, H, M, sz, sh, sm, q8, msb, lsb, scale, st, vblocks, n_sm);
      default: return cudaErrorInvalidValue;
    }
  }
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
