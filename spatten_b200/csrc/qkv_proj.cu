// Fused Q/K/V projection of the active heads on the 5th-generation tensor
// cores, with the progressive-quantisation step in its epilogue.
//
// Replaces, for one layer of the cascade, the head-row slicing of the
// concatenated Q/K/V weights (slice_linear_weights, module.py:12-34: three
// index_select copies), the projection (spatten_bert.py:72-78) and the
// quantisation of Q and K that the attention kernel needs (the reference's
// float plane split, spatten_bert_ultimate.py:184-185). No weight is copied:
// the weight tile of output columns [c, c + 64) of head slot hs is loaded by
// TMA straight from the rows which * Hall * Dh + heads[hs] * Dh + (c % Dh)
// of the full weight, so the head pruning only changes tile coordinates.
//
// Persistent, warp-specialised: one CTA per SM walks the output tiles
// (128 tokens x 128 columns of one of Q / K / V: two heads at Dh = 64, one at
// Dh = 128), 10 warps:
//   warp 0     TMA producer: x tile [128 x 64] and two weight tiles [64 x 64]
//              per K step, 128B-swizzled, into a kStages ring (no multicast);
//              it runs ahead into the next tile while the MMAs of this one run;
//   warp 1     MMA issuer + TMEM owner: kind::f16 into one of two fp32
//              accumulators of 128 columns (double-buffered in TMEM, so the
//              next tile's MMAs overlap this tile's epilogue);
//   warps 2-9  epilogue, two warps per TMEM lane quarter (one token row per
//              thread; warp half h takes head h of the tile at Dh = 64, or
//              half the columns at Dh = 128): + bias, round to the activation
//              type (the value the unfused projection would store), then per
//              (token, head): Q -> int8 + scale, K -> packed 4-bit MSB / LSB
//              planes + scale (the quant_rows arithmetic: scale = max|x| / 127,
//              x8 = rint(x / scale), IEEE division), V (and Q, K in mode 1) in
//              the activation type; all outputs head-major [B, cur, S, ...],
//              which the attention kernel reads.
// Every wait is bounded; a timeout records a code in this file's device error
// word, the CTA lets its copies and MMAs land and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "proj.h"
#include "sm100.cuh"

namespace spatten {

namespace {

using namespace sm100;

constexpr int PM = 128;  // tokens per tile (TMEM lanes)
constexpr int PN = 256;  // output columns per tile (TMEM columns of one accumulator)
constexpr int PK = 64;   // K step: 64 elements = one 128-byte swizzle atom
constexpr int kStages = 4;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 2 * PN;
constexpr unsigned kErrProj = 0x200;

struct ProjLayout {
  static constexpr int kABytes = PM * PK * 2;
  static constexpr int kBBytes = PN * PK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int oStage = 0;                           // [kStages][A | B]
  static constexpr int oBar = kStages * kStageBytes;         // full, empty, acc_full[2], acc_empty[2], drain
  static constexpr int kNumBars = 2 * kStages + 5;
  static constexpr int oTmem = oBar + kNumBars * 8;
  static constexpr int oAbort = oTmem + 4;
  static constexpr int oBias = oAbort + 12;                  // float [kEpiWarps][128] per-warp bias copy (one head)
  static constexpr int kBytes = oBias + kEpiWarps * 128 * 4;
  static constexpr int kAlloc = kBytes + 1024;
};

struct ProjKParams {
  ProjParams a;
  CUtensorMap tm_x;  // [T, Kdim], box {64, 128}
  CUtensorMap tm_w;  // [3 Hall Dh, Kdim], box {64, 64}
};

// tile t -> (token tile, which of Q / K / V, first output column within it)
struct Tile {
  int m0, which, col0;
};
SPATTEN_DEV Tile tile_of(int t, int mt, int tiles_per) {
  const int n = t / mt;
  return Tile{(t % mt) * PM, n / tiles_per, (n % tiles_per) * PN};
}

template <typename T>
SPATTEN_DEV float round_to(float x) {
  return to_f32<T>(from_f32<T>(x));
}

// weight head of active slot hs (clamped into the weight: the slot list is
// caller data)
SPATTEN_DEV int head_of(const ProjParams& p, int hs) {
  int h = p.heads ? (int)p.heads[hs] : hs;
  return (h >= 0 && h < p.Hall) ? h : 0;
}

// Epilogue of one head of a tile for one token row (TMEM lane r; `tl` is
// the accumulator's lane base): head hc of the tile, all Dh of its columns.
// Values are the rounded activations acc + bias; `sb` is this warp's
// shared-memory copy of the head's bias (Dh floats).
template <typename T>
SPATTEN_DEV void epilogue_head(const ProjParams& p, uint32_t tl, const Tile& tl_, int r, int hc, int T_,
                               float* sb) {
  const int Dh = p.Dh, lane = threadIdx.x & 31;
  const int tok = tl_.m0 + r;
  const bool valid = tok < T_;
  const int b = valid ? tok / p.S : 0, s = valid ? tok % p.S : 0;
  const int hs = (tl_.col0 + hc * Dh) / Dh;  // active slot
  if (hs >= p.cur) return;                   // padding of the last tile (warp-uniform)
  const int cb = hc * Dh;                    // first accumulator column of the head
  const int64_t orow = ((int64_t)b * p.cur + hs) * p.S + s;
  {
    const T* bias = static_cast<const T*>(p.bias);
    const int64_t bcol = (int64_t)tl_.which * p.Hall * Dh + (int64_t)head_of(p, hs) * Dh;
    __syncwarp();  // the previous head's reads of sb are done
    for (int c = lane; c < Dh; c += 32) sb[c] = bias ? to_f32<T>(__ldg(bias + bcol + c)) : 0.f;
    __syncwarp();
  }
  const bool quant = p.mode == 0 && tl_.which < 2;
  if (!quant) {
    T* dst = static_cast<T*>(tl_.which == 2 ? p.v : (tl_.which == 0 ? p.q : p.k)) + orow * Dh;
    for (int cc = 0; cc < Dh; cc += 32) {
      uint32_t a[32];
      tmem_ld32(tl + cb + cc, a);
      tmem_wait_ld();
      if (valid) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack2<T>(__uint_as_float(a[2 * i]) + sb[cc + 2 * i], __uint_as_float(a[2 * i + 1]) + sb[cc + 2 * i + 1]);
        uint4* d4 = reinterpret_cast<uint4*>(dst + cc);
#pragma unroll
        for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
    }
    return;
  }
  float amax = 0.f;
  for (int cc = 0; cc < Dh; cc += 32) {
    uint32_t a[32];
    tmem_ld32(tl + cb + cc, a);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(round_to<T>(__uint_as_float(a[i]) + sb[cc + i])));
  }
  const float sc = div127_rn(amax);
  const float rc = rcp_approx(sc);
  // four int8 of head columns c .. c+3 (a[i] .. a[i+3]), packed little-endian:
  // x * (1 / sc), and the exact division (quant_div) only when one of the
  // four lands within 1e-4 of a rounding tie
  auto q4 = [&](const uint32_t (&a)[32], int i, int c) -> uint32_t {
    if (sc == 0.f) return 0u;
    float x[4];
    int t[4];
    bool near_tie = false;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      x[e] = round_to<T>(__uint_as_float(a[i + e]) + sb[c + e]);
      const float y = x[e] * rc;
      float ti;
      t[e] = rint_small(y, ti);
      near_tie |= !(fabsf(y - ti) <= 0.49990f);
    }
    if (near_tie) {
#pragma unroll
      for (int e = 0; e < 4; ++e) t[e] = quant_div(x[e], sc, rc);
    }
    return ((uint32_t)t[0] & 0xFFu) | (((uint32_t)t[1] & 0xFFu) << 8) | (((uint32_t)t[2] & 0xFFu) << 16) |
           ((uint32_t)t[3] << 24);
  };
  if (tl_.which == 0) {
    int8_t* dst = p.q8 + orow * Dh;
    for (int cc = 0; cc < Dh; cc += 32) {
      uint32_t a[32];
      tmem_ld32(tl + cb + cc, a);
      tmem_wait_ld();
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = q4(a, 4 * j, cc + 4 * j);
      if (valid) {
        uint4* d4 = reinterpret_cast<uint4*>(dst + cc);
        d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
        d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
      }
    }
    if (valid) p.q_scale[orow] = sc;
  } else {
    // packed byte p = dim p (low nibble) | dim p + Dh/2 (high nibble)
    for (int pp = 0; pp < Dh / 2; pp += 32) {
      uint32_t lo[32], hi[32];
      tmem_ld32(tl + cb + pp, lo);
      tmem_ld32(tl + cb + Dh / 2 + pp, hi);
      tmem_wait_ld();
      uint32_t wm[8], wl[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t L = q4(lo, 4 * j, pp + 4 * j);
        const uint32_t H = q4(hi, 4 * j, Dh / 2 + pp + 4 * j);
        wm[j] = ((L >> 4) & 0x0F0F0F0Fu) | (H & 0xF0F0F0F0u);
        wl[j] = (L & 0x0F0F0F0Fu) | ((H & 0x0F0F0F0Fu) << 4);
      }
      if (valid) {
        uint4* m4 = reinterpret_cast<uint4*>(p.k_msb + orow * (Dh / 2) + pp);
        uint4* l4 = reinterpret_cast<uint4*>(p.k_lsb + orow * (Dh / 2) + pp);
        m4[0] = make_uint4(wm[0], wm[1], wm[2], wm[3]);
        m4[1] = make_uint4(wm[4], wm[5], wm[6], wm[7]);
        l4[0] = make_uint4(wl[0], wl[1], wl[2], wl[3]);
        l4[1] = make_uint4(wl[4], wl[5], wl[6], wl[7]);
      }
    }
    if (valid) p.k_scale[orow] = sc;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) qkv_proj_kernel(const __grid_constant__ ProjKParams P) {
  using L = ProjLayout;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::oBar);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L::oTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(sm + L::oAbort);
  const ProjParams& p = P.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T_ = p.B * p.S;
  const int mt = (T_ + PM - 1) / PM;
  const int tiles_per = (p.cur * p.Dh + PN - 1) / PN;
  const int ntiles = mt * 3 * tiles_per;
  const int KT = (p.Kdim + PK - 1) / PK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    *abort = 0;
  }
  if (warp == 1) {
    tmem_alloc(tslot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&P.tm_x);
      prefetch_tmap(&P.tm_w);
      int g = 0;  // K steps issued over all tiles
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const Tile tile = tile_of(t, mt, tiles_per);
        int wrow[PN / 64];
#pragma unroll
        for (int u = 0; u < PN / 64; ++u) {
          const int c = tile.col0 + 64 * u;
          int hs = c / p.Dh, off = c % p.Dh;
          if (hs >= p.cur) {  // padding of the last tile: any valid rows
            hs = p.cur - 1;
            off = 0;
          }
          wrow[u] = tile.which * p.Hall * p.Dh + head_of(p, hs) * p.Dh + off;
        }
        for (int kb = 0; kb < KT; ++kb, ++g) {
          const int s = g % kStages;
          if (!mbar_wait(&empty[s], ((g / kStages) & 1) ^ 1, kErrProj | 1, abort)) { ok = false; break; }
          uint8_t* st = sm + L::oStage + s * L::kStageBytes;
          mbar_arrive_expect_tx(&full[s], L::kStageBytes);
          tma_load_2d(st, &P.tm_x, kb * PK, tile.m0, &full[s]);
#pragma unroll
          for (int u = 0; u < PN / 64; ++u)
            tma_load_2d(st + L::kABytes + u * 64 * 128, &P.tm_w, kb * PK, wrow[u], &full[s]);
        }
      }
      if (!ok) {  // let the copies in flight land before the CTA exits
        const long long t0 = clock64();
        for (int u = (g > kStages ? g - kStages : 0); u < g; ++u)
          while (!mbar_try_wait(&full[u % kStages], (u / kStages) & 1) && clock64() - t0 < 200000000LL) {
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ab = std::is_same<T, __half>::value ? 0 : 1;
      constexpr uint32_t idesc = instr_desc(1, ab, 0, 0, PM, PN);
      int g = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1, kErrProj | 4, abort)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * PN;
        for (int kb = 0; kb < KT; ++kb, ++g) {
          const int s = g % kStages;
          if (!mbar_wait(&full[s], (g / kStages) & 1, kErrProj | 2, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(sm + L::oStage + s * L::kStageBytes);
          const uint32_t bw = a + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < PK / 16; ++kk)
            mma_f16(acc, smem_desc_sw128(a + kk * 32, 16, 1024), smem_desc_sw128(bw + kk * 32, 16, 1024), idesc,
                    (kb | kk) != 0);
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[buf]);
      }
      // every MMA issued has completed before the TMEM is freed
      mma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < 400000000LL) {
      }
    }
  } else {
    const int e = warp - 2, half = e >> 2, qd = warp & 3;
    const int hpt = PN / p.Dh;  // heads per tile: warp half h takes heads [h * hpt / 2, (h + 1) * hpt / 2)
    const int r = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    int lt = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      bool ok = mbar_wait(&acc_full[buf], (lt >> 1) & 1, kErrProj | 3, abort);
      ok = __all_sync(0xffffffffu, ok && !*abort);
      if (!ok) break;
      tc_fence_after();
      const Tile tile = tile_of(t, mt, tiles_per);
      for (int hc = half * hpt / 2; hc < (half + 1) * hpt / 2; ++hc)
        epilogue_head<T>(p, tmem + lane_base + buf * PN, tile, r, hc, T_,
                         reinterpret_cast<float*>(sm + L::oBias) + e * 128);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 proj_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D map [rows, inner] (16-bit elements, row stride in bytes), box {64, box_rows}, 128B swizzle
cudaError_t make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, int inner, int rows,
                        int64_t row_bytes, int box_rows) {
  auto fn = proj_encode_fn();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)PK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

namespace {

template <typename T>
cudaError_t launch_proj_t(const ProjParams& a, cudaStream_t st) {
  ProjKParams P;
  memset(&P, 0, sizeof(P));
  P.a = a;
  const CUtensorMapDataType dt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int T_ = a.B * a.S;
  cudaError_t e = make_map_2d(&P.tm_x, dt, a.x, a.Kdim, T_, a.x_st * 2, PM);
  if (e != cudaSuccess) return e;
  e = make_map_2d(&P.tm_w, dt, a.w, a.Kdim, 3 * a.Hall * a.Dh, (int64_t)a.Kdim * 2, 64);
  if (e != cudaSuccess) return e;
  auto kern = qkv_proj_kernel<T>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, ProjLayout::kAlloc);
  if (e != cudaSuccess) return e;
  int dev = 0, n_sm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((T_ + PM - 1) / PM) * 3 * ((a.cur * a.Dh + PN - 1) / PN);
  kern<<<(unsigned)(tiles < n_sm ? tiles : n_sm), kThreads, ProjLayout::kAlloc, st>>>(P);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qkv_proj(const ProjParams& p, cudaStream_t st) {
  if (p.dtype == kF16) return launch_proj_t<__half>(p, st);
  if (p.dtype == kBF16) return launch_proj_t<__nv_bfloat16>(p, st);
  return cudaErrorInvalidValue;
}

cudaError_t read_proj_device_error(unsigned int* code, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(code, sm100::g_device_error, sizeof(unsigned int));
  if (e != cudaSuccess || !reset) return e;
  const unsigned int zero = 0;
  return cudaMemcpyToSymbol(sm100::g_device_error, &zero, sizeof(unsigned int));
}

}  // namespace spatten
