// Attention output projection of the kept tokens only, with the residual:
// the token gather of the cascade folded into a tensor-core GEMM.
//
// In the cascade encoder (module.py:49-63) layer i + 1 starts by gathering the
// hidden states of the tokens layer i's attention kept (torch.gather over the
// sequence); everything after layer i's attention (BertSelfOutput: dense +
// residual + LayerNorm, then the FFN) is row-wise, so the rows layer i + 1
// drops are computed and thrown away. This kernel computes the first step of
// that tail for the kept rows only, reading them through the kept positions:
//   out[b * L + j] = T(T(ctx[b * S + s] . W^T + bias) + res[b * S + s]),
//   s = kept[b, j]
// (T() = rounding to the activation type, where the unfused dense layer and
// the residual add round), so the LayerNorm and the FFN that follow run on
// the compacted sequence and no gather copy is made. The K dimension covers
// only the active heads' column blocks of the context row (the pruned heads'
// blocks are zeros, whose products add nothing), and the weight's matching
// column blocks are addressed in place.
//
// Persistent, warp-specialised: one CTA per SM walks the output tiles
// (128 kept rows x 256 features, n fastest so the CTAs on one row tile share
// its gathered rows in L2), 14 warps:
//   warp 0      TMA producer: weight tile [256 x 64] per K step (128B swizzle,
//               no multicast) into a kStages ring;
//   warp 1      MMA issuer + TMEM owner: kind::f16 into one of two fp32
//               accumulators of 256 columns (double-buffered: the next tile's
//               MMAs overlap this tile's epilogue);
//   warps 2-5   row gather: 32 tile rows per warp, eight lanes per row (one
//               16-byte cp.async each, so a warp instruction reads four whole
//               128-byte rows) per K step from the kept rows' context, written
//               in the 128-byte swizzled K-major layout the MMA reads; a stage
//               is released kLag K steps later, after cp.async.wait_group and
//               a proxy fence (generic writes -> async-proxy reads);
//   warps 6-13  epilogue, two warps per TMEM lane quarter (128 columns each):
//               + bias and rounding in the TMEM layout (a row per lane), then
//               through a per-warp shared-memory tile to a layout of four
//               lanes per 64-byte row segment, where the kept row's residual
//               is read and the sum stored with 16-byte accesses.
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

constexpr int OM = 128;  // kept rows per tile (TMEM lanes)
constexpr int ON = 256;  // output features per tile (TMEM columns of one accumulator)
constexpr int OK = 64;   // K step: 64 elements = one 128-byte swizzle atom
constexpr int kStages = 4;
constexpr int kLag = kStages - 2;  // K steps a gather thread keeps in flight before releasing one
constexpr int kGatherWarps = 4;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kGatherWarps + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 2 * ON;
constexpr unsigned kErrOut = 0x300;
constexpr int kMaxKT = 256;  // K steps whose first column is tabled in shared memory

struct OutLayout {
  static constexpr int kABytes = OM * OK * 2;
  static constexpr int kBBytes = ON * OK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int oStage = 0;                       // [kStages][A | B]
  static constexpr int oBar = kStages * kStageBytes;     // full, empty, acc_full[2], acc_empty[2], drain
  static constexpr int kNumBars = 2 * kStages + 5;
  static constexpr int oTmem = oBar + kNumBars * 8;
  static constexpr int oAbort = oTmem + 4;
  static constexpr int kEpiStride = 80;                  // bytes per staged row: 32 values + 16 pad
  static constexpr int oEpi = (oAbort + 12 + 15) & ~15;  // [kEpiWarps][32 rows][kEpiStride], 16-byte aligned
  static constexpr int oKcol = oEpi + kEpiWarps * 32 * kEpiStride;  // int [kMaxKT]: first column of each K step
  static constexpr int kBytes = oKcol + kMaxKT * 4;
  static constexpr int kAlloc = kBytes + 1024;
};
static_assert(OutLayout::kAlloc <= 227 * 1024, "shared memory");
static_assert(OutLayout::oEpi % 16 == 0 && OutLayout::kEpiStride % 16 == 0, "16-byte staging rows");
static_assert(OM == kGatherWarps * 32, "32 tile rows per gather warp");
static_assert(ON == 256, "epilogue: four 32-column chunks per warp half");

struct OutKParams {
  OutProjParams a;
  CUtensorMap tm_w;  // [N, H * Dh], box {64, 256}
};

// input row (b * S + s) of output row gr (< B * L); kept positions are caller
// data, clamped into the sequence
SPATTEN_DEV int64_t src_row(const OutProjParams& p, int gr) {
  const int b = gr / p.L;
  int64_t s = __ldg(p.kept + gr);
  s = s < 0 ? 0 : (s >= p.S ? p.S - 1 : s);
  return (int64_t)b * p.S + s;
}

// first context / weight column of K step kb (64 wide)
SPATTEN_DEV int k_col(const OutProjParams& p, int kb) {
  const int per = p.Dh / OK;
  const int hs = kb / per;
  int h = p.heads ? (int)__ldg(p.heads + hs) : hs;
  h = (h >= 0 && h < p.H) ? h : 0;
  return h * p.Dh + (kb % per) * OK;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) out_proj_kernel(const __grid_constant__ OutKParams P) {
  using Lay = OutLayout;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Lay::oBar);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + Lay::oTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(sm + Lay::oAbort);
  const OutProjParams& p = P.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = p.B * p.L;
  const int mt = (M + OM - 1) / OM, nt = (p.N + ON - 1) / ON;
  const int ntiles = mt * nt;
  const int KT = p.cur * (p.Dh / OK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], kGatherWarps + 1);  // the gather warps + the weight copy's expect_tx
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
  int* kcol_s = reinterpret_cast<int*>(sm + Lay::oKcol);
  for (int kb = threadIdx.x; kb < KT && kb < kMaxKT; kb += blockDim.x) kcol_s[kb] = k_col(p, kb);
  auto kcol = [&](int kb) { return kb < kMaxKT ? kcol_s[kb] : k_col(p, kb); };
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&P.tm_w);
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int n0 = (t % nt) * ON;
        for (int kb = 0; kb < KT; ++kb, ++g) {
          const int s = g % kStages;
          if (!mbar_wait(&empty[s], ((g / kStages) & 1) ^ 1, kErrOut | 1, abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], Lay::kBBytes);
          tma_load_2d(sm + Lay::oStage + s * Lay::kStageBytes + Lay::kABytes, &P.tm_w, kcol(kb), n0,
                      &full[s]);
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
      constexpr uint32_t idesc = instr_desc(1, ab, 0, 0, OM, ON);
      int g = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1, kErrOut | 4, abort)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * ON;
        for (int kb = 0; kb < KT; ++kb, ++g) {
          const int s = g % kStages;
          if (!mbar_wait(&full[s], (g / kStages) & 1, kErrOut | 2, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(sm + Lay::oStage + s * Lay::kStageBytes);
          const uint32_t bw = a + Lay::kABytes;
#pragma unroll
          for (int kk = 0; kk < OK / 16; ++kk)
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
  } else if (warp < 2 + kGatherWarps) {
    // row gather: warp gw fills tile rows gw*32 .. gw*32+31, lane = (row
    // sub-index, 16-byte chunk); one instruction covers rows i*4 .. i*4+3
    const int gw = warp - 2, sub = lane >> 3, ch = lane & 7;
    const T* ctx = static_cast<const T*>(p.ctx);
    // input rows of tile t's kept rows (rows past the end copy input row 0;
    // their results are not stored); the next tile's are loaded while this
    // tile's K steps run
    auto rows_of = [&](int t, int64_t (&src)[8]) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int gr = (t / nt) * OM + gw * 32 + i * 4 + sub;
        src[i] = (t < ntiles && gr < M) ? src_row(p, gr) : 0;
      }
    };
    int64_t src[8], nsrc[8];
    rows_of(blockIdx.x, src);
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const T* row[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) row[i] = ctx + src[i] * p.ctx_st + ch * 8;
      rows_of(t + gridDim.x, nsrc);
      for (int kb = 0; kb < KT; ++kb, ++g) {
        const int s = g % kStages;
        const bool w = mbar_wait(&empty[s], ((g / kStages) & 1) ^ 1, kErrOut | 5, abort);
        if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
        uint8_t* st = sm + Lay::oStage + s * Lay::kStageBytes;
        const int col = kcol(kb);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = gw * 32 + i * 4 + sub;
          cp_async16(st + r * 128 + ((ch ^ (r & 7)) << 4), row[i] + col, true);
        }
        cp_async_commit();
        if (g >= kLag) {
          cp_async_wait<kLag>();
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[(g - kLag) % kStages]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) src[i] = nsrc[i];
    }
    cp_async_wait<0>();
    fence_proxy_async_smem();
    __syncwarp();
    if (ok && lane == 0)
      for (int u = (g > kLag ? g - kLag : 0); u < g; ++u) mbar_arrive(&full[u % kStages]);
  } else {
    const int e = warp - 2 - kGatherWarps, half = e >> 2, qd = warp & 3;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const T* bias = static_cast<const T*>(p.bias);
    const T* res = static_cast<const T*>(p.res);
    T* out = static_cast<T*>(p.out);
    uint8_t* stg = sm + Lay::oEpi + e * 32 * Lay::kEpiStride;
    const int cq = lane & 3;  // 16-byte column chunk of the store layout
    int lt = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      // store layout: lane handles rows (lane >> 2) + 8 i of the warp's 32;
      // their residual segments are loaded before the accumulator is waited for
      const int m0 = (t / nt) * OM + qd * 32;
      int64_t rsrc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int gr = m0 + (lane >> 2) + 8 * i;
        rsrc[i] = gr < M ? src_row(p, gr) : -1;
      }
      uint4 rv[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int n = (t % nt) * ON + half * (ON / 2) + c * 32;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          rv[c][i] = (rsrc[i] >= 0 && n < p.N)
                         ? __ldg(reinterpret_cast<const uint4*>(res + rsrc[i] * p.res_st + n + cq * 8))
                         : make_uint4(0u, 0u, 0u, 0u);
      }
      bool ok = mbar_wait(&acc_full[buf], (lt >> 1) & 1, kErrOut | 3, abort);
      ok = __all_sync(0xffffffffu, ok && !*abort);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int cc = half * (ON / 2) + c * 32;
        const int n = (t % nt) * ON + cc;
        if (n >= p.N) break;  // warp-uniform: N is a multiple of 32
        uint32_t a[32];
        __syncwarp();
        tmem_ld32(tmem + lane_base + buf * ON + cc, a);
        tmem_wait_ld();
        // TMEM layout (lane = row): y = T(acc + bias), staged as 64 bytes of the row
        uint4 bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          bv[i] = bias ? __ldg(reinterpret_cast<const uint4*>(bias + n) + i) : make_uint4(0u, 0u, 0u, 0u);
        const T* be = reinterpret_cast<const T*>(bv);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack2<T>(__uint_as_float(a[2 * i]) + to_f32<T>(be[2 * i]),
                           __uint_as_float(a[2 * i + 1]) + to_f32<T>(be[2 * i + 1]));
        uint4* srow = reinterpret_cast<uint4*>(stg + lane * Lay::kEpiStride);
#pragma unroll
        for (int i = 0; i < 4; ++i) srow[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        __syncwarp();
        // store layout: out = T(y + residual), 16 bytes per lane
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (rsrc[i] < 0) continue;
          const int rr = (lane >> 2) + 8 * i;
          const uint4 yv = *reinterpret_cast<const uint4*>(stg + rr * Lay::kEpiStride + cq * 16);
          const T* ye = reinterpret_cast<const T*>(&yv);
          const T* re = reinterpret_cast<const T*>(&rv[c][i]);
          uint32_t o[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            o[k] = pack2<T>(to_f32<T>(ye[2 * k]) + to_f32<T>(re[2 * k]),
                            to_f32<T>(ye[2 * k + 1]) + to_f32<T>(re[2 * k + 1]));
          *reinterpret_cast<uint4*>(out + (int64_t)(m0 + rr) * p.N + n + cq * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
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

template <typename T>
cudaError_t launch_t(const OutProjParams& a, cudaStream_t st) {
  OutKParams P;
  memset(&P, 0, sizeof(P));
  P.a = a;
  const CUtensorMapDataType dt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int K = a.H * a.Dh;
  cudaError_t e = make_map_2d(&P.tm_w, dt, a.w, K, a.N, (int64_t)K * 2, ON);
  if (e != cudaSuccess) return e;
  auto kern = out_proj_kernel<T>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, OutLayout::kAlloc);
  if (e != cudaSuccess) return e;
  int dev = 0, n_sm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((a.B * a.L + OM - 1) / OM) * ((a.N + ON - 1) / ON);
  kern<<<(unsigned)(tiles < n_sm ? tiles : n_sm), kThreads, OutLayout::kAlloc, st>>>(P);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_out_proj(const OutProjParams& p, cudaStream_t st) {
  if (p.dtype == kF16) return launch_t<__half>(p, st);
  if (p.dtype == kBF16) return launch_t<__nv_bfloat16>(p, st);
  return cudaErrorInvalidValue;
}

cudaError_t read_out_proj_device_error(unsigned int* code, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(code, sm100::g_device_error, sizeof(unsigned int));
  if (e != cudaSuccess || !reset) return e;
  const unsigned int zero = 0;
  return cudaMemcpyToSymbol(sm100::g_device_error, &zero, sizeof(unsigned int));
}

}  // namespace spatten
