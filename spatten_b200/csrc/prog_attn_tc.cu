// Progressive sparse attention on the 5th-generation tensor cores (tcgen05).
//
// One CTA = 128 query rows of one (z, h), 8 warps, two CTAs per SM:
//   warps 0-3  softmax: one query row per thread (TMEM lane = row). Reads S
//              from TMEM, keeps the row statistics, decides the refetch,
//              writes P (fp16/bf16) to shared memory, sums P's columns
//              (token importance) and, at the end, reads O from TMEM.
//   warp 4     TMA producer: 4-bit K planes (QUANT) or K (DENSE) and V tiles
//              of 64 keys, straight into 128B-swizzled shared memory.
//   warp 5     MMA issuer (one thread) and TMEM owner:
//              S = Q' K'^T  (kind::i8, int32 accumulator, or kind::f16)
//              O += P V     (kind::f16, fp32 accumulator, V MN-major)
//   warps 6-7  expander (QUANT): one key per thread, unpacks the packed
//              MSB/LSB nibbles into the int8 operand K' = [16*msb | lsb] and
//              stages the per-key scale and mask bias for the softmax warps.
// Tensor memory: two S buffers of 64 columns (int32 / fp32) and O (D fp32
// columns). Every hand-off is an mbarrier; every wait is bounded (a timeout
// records an error word and unwinds instead of hanging).
//
// Passes over K (the integer scores are exact; what follows them is fp32):
//   pass 1   S = q8 . (16*msb)                     -> row max m, sum l
//   decide   refetch = 1/l < refetch_thr (the row's max probability)
//            Q' = [q8 | refetch ? q8 : 0]
//   pass 1b  (only if a row of the CTA refetches; only then are LSB planes
//            loaded) S = Q'.K' = q8.k8 for refetched rows -> their (m, l)
//   pass 2   S = Q'.K'; P = exp(S - m)/l; P' = P < v_thr ? 0 : P;
//            O += P'V; column sums of P' -> token-importance partials.
// DENSE runs pass 1 and pass 2 with S = q.k (fp16/bf16 operands).
// COMPAT (the reference op's float planes, spatten_bert_ultimate.py:58-74 and
// spatten_progressive_attention.py:38-60): one MMA of N = 128 per key tile
// gives S = [q.k_msb | q.k_lsb] (the K stage holds the tile's k_msb rows and
// then its k_lsb rows); for every criterion tile (32 or 64 rows x 32 or 64
// keys) whose largest q.k_msb * sm_scale is below tile_thr the scores become
// q.k_msb * sm_scale + q.k_lsb * sm_scale, else q.k_msb * sm_scale. The
// softmax warps covering one criterion tile vote through shared memory and
// an mbarrier (a warp vote for 32 x 32). Passes 1 and 2 as for DENSE.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <climits>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace spatten {

namespace {

using namespace sm100;

constexpr int BM = 128;        // query rows per CTA (= TMEM lanes)
constexpr int BN = 64;         // keys per tile
constexpr int kSoftWarps = 4;  // one thread per query row, all 64 columns of a tile
constexpr int kSoftThreads = kSoftWarps * 32;
// Expander warps (64 / 32 keys of a 64-key tile per thread).
#ifndef SPATTEN_TC_KS_CHUNK
#define SPATTEN_TC_KS_CHUNK 64
#endif
constexpr int kKsChunk = SPATTEN_TC_KS_CHUNK;  // key-scale columns read per fenced chunk
#ifndef SPATTEN_TC_EXP_WARPS
#define SPATTEN_TC_EXP_WARPS 2
#endif
constexpr int kExpWarps = SPATTEN_TC_EXP_WARPS;
constexpr int kThreads = (kSoftWarps + 2 + kExpWarps) * 32;
constexpr int kNStg = 3;       // packed-plane staging stages (QUANT)
constexpr int kNExp = 2;       // K operand stages
constexpr int kNV = 2;         // V stages
constexpr int kNP = 2;         // P buffers
constexpr int kCsCols = 16;    // N of the column-sum MMA (16 identical columns)
constexpr int kWarpTma = kSoftWarps, kWarpMma = kSoftWarps + 1, kWarpExp = kSoftWarps + 2;
// The two-CTA-per-SM instantiations (D = 64, no count prune) move registers
// from the producer warpgroup to the softmax warpgroup (setmaxnreg); the
// split adds up to the CTA's allocation only at kSplitLaunchRegs registers a
// thread, which the launcher checks before every first launch.
template <int D, bool VC>
constexpr bool kRegSplit = (D == 64 && !VC);
constexpr int kSplitLaunchRegs = 128;
static_assert(kSoftThreads * 160 + (kThreads - kSoftThreads) * 96 == kThreads * kSplitLaunchRegs,
              "register split must add up to the launch allocation");

enum Mode : int { kQuant = 0, kDense = 1, kCompat = 2 };

// error codes: 0x100 | role << 4 | site
enum : unsigned { kErrSoftmax = 0x110, kErrTma = 0x120, kErrMma = 0x130, kErrExp = 0x140 };

struct TcParams {
  AttnParams a;
  CUtensorMap tm_k0;  // QUANT: MSB plane (u8 [Z,Hkv,N,D/2]); DENSE: K ([Z,Hkv,N,D])
  CUtensorMap tm_k1;  // QUANT: LSB plane
  CUtensorMap tm_v;   // V ([Z,Hkv,N,D])
};

template <int MODE, typename T, int D, bool VC>
struct Layout {
  static constexpr int kAtoms = D / 64;                 // 128-byte K atoms of Q'/K' rows (2D bytes)
  static constexpr int kQBytes = kAtoms * BM * 128;     // Q' operand
  static constexpr int kKRows = (MODE == kCompat) ? 2 * BN : BN;  // K operand rows (COMPAT: msb | lsb)
  static constexpr int kKBytes = kAtoms * kKRows * 128;  // K' operand stage
  static constexpr int kSBuf = (MODE == kCompat) ? 1 : 2;  // S buffers in tensor memory
  static constexpr int kSW = (MODE == kCompat) ? 2 * BN : BN;  // S columns per buffer
  static constexpr int kStgBytes = (MODE == kQuant) ? BN * D : 0;  // msb + lsb packed
  static constexpr int kVBytes = (D / 64) * BN * 128;   // V stage (MN-major blocks of 64 dims)
  static constexpr int kPBytes = BM * 128;              // P stage (64 keys x 2 B per row)
  static constexpr int kOnesBytes = 2 * kCsCols * 128;  // ones [16][128] (B of the column sums)
  // tensor memory: S buffers [0, kSBuf*kSW), O (D columns), column sums after O
  static constexpr int kColO = kSBuf * kSW;
  static constexpr int kColCs = kColO + D;
  static constexpr uint32_t kTmemCols = (kColCs + 2 * kCsCols) <= 256 ? 256 : 512;
  static constexpr int oQ = 0;
  static constexpr int oK = oQ + kQBytes;
  static constexpr int oV = oK + kNExp * kKBytes;
  static constexpr int oP = oV + kNV * kVBytes;
  static constexpr int oStg = oP + kNP * kPBytes;       // 1024-aligned so far
  static constexpr int oOnes = oStg + kNStg * kStgBytes;  // 1024-aligned
  static constexpr int oKs = oOnes + kOnesBytes;        // float [kNExp][BN] key scale
  static constexpr int oKb = oKs + kNExp * BN * 4;      // float [kNExp][BN] key bias * log2e
  static constexpr int oHs = oKb + kNExp * BN * 4;      // float [kSoftWarps]
  static constexpr int oVote = oHs + 4 * kSoftWarps;    // int [2][kSoftWarps] COMPAT tile votes
  static constexpr int oBar = oVote + 2 * 4 * kSoftWarps;  // mbarriers
  static constexpr int kNumBars = 2 * kNStg + 2 * kNExp + 2 * 2 + 2 * kNP + 2 * kNV + 2 * 2 + 3 + 8;
  static constexpr int oTmem = oBar + kNumBars * 8;
  static constexpr int oFlag = oTmem + 4;  // int abort, int decision, int key tiles of the CTA
  static constexpr int kBytes = oFlag + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

struct Bars {
  SBarArr stg_full;
  SBarArr stg_empty;
  SBarArr k_full;
  SBarArr k_empty;
  SBarArr s_full;
  SBarArr s_empty;
  SBarArr p_full;
  SBarArr p_empty;
  SBarArr v_full;
  SBarArr v_empty;
  SBarArr cs_full;
  SBarArr cs_empty;
  SBar q_ready;
  SBar dec_ready;
  SBar o_full;
  SBarArr vote;  // [2 buffers][4 vote groups] (COMPAT)
};

// Pairs of fp32 values for the packed (f32x2) FP instructions of sm_100.
using f2 = uint64_t;
SPATTEN_DEV f2 pack_f2(float lo, float hi) {
  f2 d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
SPATTEN_DEV void unpack_f2(f2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
SPATTEN_DEV f2 fmul2(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
SPATTEN_DEV f2 fadd2(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// exact int32 -> fp32 for |x| < 2^22 without the conversion pipe:
// the bits of 1.5 * 2^23 + x, minus 1.5 * 2^23.
SPATTEN_DEV float i2f_exact(uint32_t x) { return __uint_as_float(x + 0x4B400000u); }
constexpr float kMagic = 12582912.0f;

template <int MODE, typename T, int D, bool VC>
struct Cta {
  using L = Layout<MODE, T, D, VC>;
  const TcParams& P;
  const AttnParams& p;
  uint8_t* sm;  // 1024-aligned base
  Bars b;
  volatile int* abort;
  int* decision;
  uint32_t tmem;
  int z, h, kvh, mt, m0, nt;

  SPATTEN_DEV Cta(const TcParams& pp, uint8_t* base) : P(pp), p(pp.a), sm(base) {
    uint32_t bar = smem_u32(sm + L::oBar);
    auto take = [&](int n) {
      const SBarArr r{bar};
      bar += 8u * (uint32_t)n;
      return r;
    };
    b.stg_full = take(kNStg);
    b.stg_empty = take(kNStg);
    b.k_full = take(kNExp);
    b.k_empty = take(kNExp);
    b.s_full = take(2);
    b.s_empty = take(2);
    b.p_full = take(kNP);
    b.p_empty = take(kNP);
    b.v_full = take(kNV);
    b.v_empty = take(kNV);
    b.cs_full = take(2);
    b.cs_empty = take(2);
    b.q_ready = take(1)[0];
    b.dec_ready = take(1)[0];
    b.o_full = take(1)[0];
    b.vote = take(8);
    abort = reinterpret_cast<volatile int*>(sm + L::oFlag);
    decision = reinterpret_cast<int*>(sm + L::oFlag + 4);
    // With a causal mask or key limits the work grows with the row index:
    // the launch order runs each head's query tiles heaviest first, so the
    // last CTAs to start are short ones and the tail stays short.
    mt = (p.causal || p.key_limit) ? (int)(gridDim.x - 1 - blockIdx.x) : (int)blockIdx.x;
    h = blockIdx.y;
    z = blockIdx.z;
    kvh = h / (p.H / p.Hkv);
    m0 = mt * BM;
    nt = (p.N + BN - 1) / BN;
  }

  // Key tiles this CTA visits (warp 0, before the start barrier): with a
  // causal mask or key_limit, tiles past the largest limit of the CTA's rows
  // are masked for every row and are skipped. The count V prune visits them
  // all (masked keys take part in its count), and so does the verification
  // dump of the integer scores (it records every key's score).
  SPATTEN_DEV void count_key_tiles() {
    const int lane = threadIdx.x & 31;
    int lim = p.N;
    if (!VC && !p.score_out && (p.key_limit || p.causal)) {
      int mx = 0;
      const int rows = min(BM, p.M - m0);
      for (int i = lane; i < rows; i += 32) {
        const int row = m0 + i;
        const int kl = p.key_limit ? p.key_limit[(int64_t)z * p.M + row] : row + (p.N - p.M) + 1;
        mx = max(mx, kl);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      lim = min(p.N, max(mx, 1));
    }
    if (lane == 0) *reinterpret_cast<int*>(sm + L::oFlag + 8) = (lim + BN - 1) / BN;
  }

  SPATTEN_DEV void init_barriers() {
    for (int i = 0; i < kNStg; ++i) {
      mbar_init(b.stg_full[i], 1);
      mbar_init(b.stg_empty[i], kExpWarps);
    }
    for (int i = 0; i < kNExp; ++i) {
      mbar_init(b.k_full[i], MODE == kQuant ? kExpWarps : 1 + kExpWarps);
      mbar_init(b.k_empty[i], 1 + kSoftWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(b.s_full[i], 1);
      mbar_init(b.s_empty[i], kSoftWarps);
      mbar_init(b.cs_full[i], 1);
      mbar_init(b.cs_empty[i], 4);
    }
    for (int i = 0; i < kNP; ++i) {
      mbar_init(b.p_full[i], kSoftWarps);
      mbar_init(b.p_empty[i], 1);
    }
    for (int i = 0; i < kNV; ++i) {
      mbar_init(b.v_full[i], 1);
      mbar_init(b.v_empty[i], 1);
    }
    mbar_init(b.q_ready, kSoftWarps);
    mbar_init(b.dec_ready, kSoftWarps);
    mbar_init(b.o_full, 1);
    // COMPAT: one arrival per softmax warp of a 64-row criterion tile
    for (int i = 0; i < 8; ++i) mbar_init(b.vote[i], 2);
    *abort = 0;
    *decision = 0;
    fence_barrier_init();
  }

  // pass schedule: pass 0 = stats of the MSB score, pass 1 = stats of the
  // full score (QUANT with a refetched row only), pass 2 = output.
  SPATTEN_DEV static bool pass_uses_lsb(int pass, int any) {
    return MODE == kQuant && pass > 0 && any;
  }

  // ------------------------------------------------------------------ TMA
  SPATTEN_DEV void tma_role() {
    if ((threadIdx.x & 31) != 0) return;
    prefetch_tmap(&P.tm_k0);
    if (MODE != kDense) prefetch_tmap(&P.tm_k1);
    prefetch_tmap(&P.tm_v);
    uint32_t t = 0, tv = 0;  // global tile counter, V tile counter
    int any = 0;
    for (int pass = 0; pass < 3; ++pass) {
      if (pass == 1) {
        if (!mbar_wait(b.dec_ready, 0, kErrTma | 1, abort)) break;
        any = *reinterpret_cast<volatile int*>(decision);
        if (!(MODE == kQuant && any)) continue;
      }
      const bool lsb = pass_uses_lsb(pass, any);
      bool ok = true;
      for (int j = 0; j < nt && ok; ++j, ++t) {
        const int n0 = j * BN;
        if (MODE == kQuant) {
          const int s = t % kNStg;
          if (!mbar_wait(b.stg_empty[s], ((t / kNStg) & 1) ^ 1, kErrTma | 2, abort)) { ok = false; break; }
          uint8_t* dst = sm + L::oStg + s * L::kStgBytes;
          mbar_arrive_expect_tx(b.stg_full[s], BN * (D / 2) * (lsb ? 2 : 1));
          tma_load_4d(dst, &P.tm_k0, 0, n0, kvh, z, b.stg_full[s]);
          if (lsb) tma_load_4d(dst + BN * (D / 2), &P.tm_k1, 0, n0, kvh, z, b.stg_full[s]);
        } else {
          const int s = t % kNExp;
          if (!mbar_wait(b.k_empty[s], ((t / kNExp) & 1) ^ 1, kErrTma | 3, abort)) { ok = false; break; }
          uint8_t* dst = sm + L::oK + s * L::kKBytes;
          mbar_arrive_expect_tx(b.k_full[s], L::kKRows * D * 2);
#pragma unroll
          for (int a = 0; a < D / 64; ++a) {
            tma_load_4d(dst + a * L::kKRows * 128, &P.tm_k0, 64 * a, n0, kvh, z, b.k_full[s]);
            if (MODE == kCompat)  // the tile's k_lsb rows after its k_msb rows
              tma_load_4d(dst + a * L::kKRows * 128 + BN * 128, &P.tm_k1, 64 * a, n0, kvh, z, b.k_full[s]);
          }
        }
        if (pass == 2) {
          const int s = tv % kNV;
          if (!mbar_wait(b.v_empty[s], ((tv / kNV) & 1) ^ 1, kErrTma | 4, abort)) { ok = false; break; }
          uint8_t* dst = sm + L::oV + s * L::kVBytes;
          mbar_arrive_expect_tx(b.v_full[s], BN * D * 2);
#pragma unroll
          for (int a = 0; a < D / 64; ++a)
            tma_load_4d(dst + a * BN * 128, &P.tm_v, 64 * a, n0, kvh, z, b.v_full[s]);
          ++tv;
        }
      }
      if (!ok) break;
    }
    if (*abort) drain_tma(t, tv);
  }

  // After an abort: let the copies this thread issued land before the CTA exits.
  SPATTEN_DEV void drain_tma(uint32_t t, uint32_t tv) {
    const long long t0 = clock64();
    auto spin = [&](SBar bar, uint32_t par) {
      while (!mbar_try_wait(bar, par) && clock64() - t0 < 200000000LL) {
      }
    };
    constexpr uint32_t ring = (MODE == kQuant) ? kNStg : kNExp;
    for (uint32_t u = (t > ring ? t - ring : 0); u < t; ++u) {
      if (MODE == kQuant) spin(b.stg_full[u % kNStg], (u / kNStg) & 1);
      else spin(b.k_full[u % kNExp], (u / kNExp) & 1);
    }
    for (uint32_t u = (tv > (uint32_t)kNV ? tv - kNV : 0); u < tv; ++u)
      spin(b.v_full[u % kNV], (u / kNV) & 1);
  }

  // ------------------------------------------------------------- expander
  SPATTEN_DEV void expand_role() {
    constexpr int KPT = BN / (kExpWarps * 32);  // keys of a tile per expander thread
    const int e0 = threadIdx.x - kWarpExp * 32;  // this thread's first key within the tile
    const float* ksrc = (MODE == kQuant) ? p.k_scale + ((int64_t)z * p.Hkv + kvh) * p.N : nullptr;
    const bool key_bias = p.bias != nullptr && p.b_sm == 0;
    const float* bsrc = key_bias ? p.bias + (int64_t)z * p.b_sz + (int64_t)h * p.b_sh : nullptr;
    uint32_t t = 0;
    int any = 0;
    for (int pass = 0; pass < 3; ++pass) {
      if (pass == 1) {
        if (!mbar_wait(b.dec_ready, 0, kErrExp | 1, abort)) return;
        any = *reinterpret_cast<volatile int*>(decision);
        if (!(MODE == kQuant && any)) continue;
      }
      const bool lsb = pass_uses_lsb(pass, any);
      // key scale / bias of tile j, loaded one tile ahead to hide the latency
      auto fetch = [&](int j, float (&ks)[KPT], float (&kb)[KPT]) {
#pragma unroll
        for (int k = 0; k < KPT; ++k) {
          const int n = j * BN + e0 + k * kExpWarps * 32;
          ks[k] = 0.f;
          kb[k] = 0.f;
          if (j < nt && n < p.N) {
            if (MODE == kQuant) ks[k] = __ldg(ksrc + n);
            if (key_bias) kb[k] = __ldg(bsrc + (int64_t)n * p.b_sn) * kLog2e;
          }
        }
      };
      float ks_next[KPT], kb_next[KPT];
      fetch(0, ks_next, kb_next);
      for (int j = 0; j < nt; ++j, ++t) {
        float ks[KPT], kb[KPT];
#pragma unroll
        for (int k = 0; k < KPT; ++k) {
          ks[k] = ks_next[k];
          kb[k] = kb_next[k];
        }
        fetch(j + 1, ks_next, kb_next);
        const int es = t % kNExp, s = t % kNStg;
        if (MODE == kQuant && !mbar_wait(b.stg_full[s], (t / kNStg) & 1, kErrExp | 2, abort)) return;
        if (!mbar_wait(b.k_empty[es], ((t / kNExp) & 1) ^ 1, kErrExp | 3, abort)) return;
#pragma unroll
        for (int k = 0; k < KPT; ++k) {
          const int e = e0 + k * kExpWarps * 32;
          if (MODE == kQuant) {
            uint32_t X[D / 8], Y[D / 8];
            // staging rows of D/2 bytes land with the TMA's 32-byte (D=64) or
            // 64-byte (D=128) swizzle: 16-byte chunk c of row e sits at c ^ sw
            const int sws = (D == 64) ? ((e >> 2) & 1) : ((e >> 1) & 3);
            const uint4* src = reinterpret_cast<const uint4*>(sm + L::oStg + s * L::kStgBytes + e * (D / 2));
#pragma unroll
            for (int i = 0; i < D / 32; ++i) {
              const uint4 v = src[i ^ sws];
              X[4 * i] = v.x; X[4 * i + 1] = v.y; X[4 * i + 2] = v.z; X[4 * i + 3] = v.w;
            }
            if (lsb) {
              const uint4* srcl = reinterpret_cast<const uint4*>(sm + L::oStg + s * L::kStgBytes +
                                                                 BN * (D / 2) + e * (D / 2));
#pragma unroll
              for (int i = 0; i < D / 32; ++i) {
                const uint4 v = srcl[i ^ sws];
                Y[4 * i] = v.x; Y[4 * i + 1] = v.y; Y[4 * i + 2] = v.z; Y[4 * i + 3] = v.w;
              }
            }
            // K' row = [16*msb (D bytes) | lsb (D bytes)], K-major, 128B swizzle
            uint8_t* row = sm + L::oK + es * L::kKBytes;
            const int sw = e & 7;
            auto put = [&](int byte_off, uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
              const int atom = byte_off >> 7, chunk = (byte_off >> 4) & 7;
              *reinterpret_cast<uint4*>(row + atom * (BN * 128) + e * 128 + ((chunk ^ sw) << 4)) =
                  make_uint4(w0, w1, w2, w3);
            };
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {  // 16 packed bytes -> 16 dims lo + 16 dims hi
              const uint32_t* x = X + 4 * c;
              put(16 * c, (x[0] << 4) & 0xF0F0F0F0u, (x[1] << 4) & 0xF0F0F0F0u,
                  (x[2] << 4) & 0xF0F0F0F0u, (x[3] << 4) & 0xF0F0F0F0u);
              put(D / 2 + 16 * c, x[0] & 0xF0F0F0F0u, x[1] & 0xF0F0F0F0u, x[2] & 0xF0F0F0F0u,
                  x[3] & 0xF0F0F0F0u);
              if (lsb) {
                const uint32_t* y = Y + 4 * c;
                put(D + 16 * c, y[0] & 0x0F0F0F0Fu, y[1] & 0x0F0F0F0Fu, y[2] & 0x0F0F0F0Fu,
                    y[3] & 0x0F0F0F0Fu);
                put(D + D / 2 + 16 * c, (y[0] >> 4) & 0x0F0F0F0Fu, (y[1] >> 4) & 0x0F0F0F0Fu,
                    (y[2] >> 4) & 0x0F0F0F0Fu, (y[3] >> 4) & 0x0F0F0F0Fu);
              }
            }
            reinterpret_cast<float*>(sm + L::oKs)[es * BN + e] = ks[k];
          }
          reinterpret_cast<float*>(sm + L::oKb)[es * BN + e] = kb[k];
        }
        // One proxy fence covers both hand-offs: the staging stage, read
        // through the generic proxy, is refilled by the TMA (async proxy) as
        // soon as it is released -- without the fence the next tile's bytes
        // could land before these reads were performed (seen with two CTAs
        // per SM) -- and the K' rows written here are read by the MMA.
        fence_proxy_async_smem();
        __syncwarp();
        if (MODE == kQuant) mbar_arrive_elect(b.stg_empty[s]);
        mbar_arrive_elect(b.k_full[es]);
      }
    }
  }

  // ------------------------------------------------------------------ MMA
  SPATTEN_DEV void mma_role() {
    if ((threadIdx.x & 31) != 0) return;
    constexpr uint32_t ab16 = std::is_same<T, __half>::value ? 0 : 1;
    constexpr uint32_t idesc_s = (MODE == kQuant) ? instr_desc(2, 1, 0, 0, BM, BN)
                                                  : instr_desc(1, ab16, 0, 0, BM, L::kSW);
    constexpr uint32_t idesc_pv = instr_desc(1, ab16, 0, 1, BM, D);
    constexpr uint32_t idesc_cs = instr_desc(1, ab16, 1, 0, BM, kCsCols);
    const bool want_tok = p.tok_partial != nullptr;
    const uint32_t qaddr = smem_u32(sm + L::oQ);
    if (!mbar_wait(b.q_ready, 0, kErrMma | 1, abort)) return;
    tc_fence_after();
    uint32_t t = 0, tv = 0;
    int any = 0;
    bool first_pv = true;
    for (int pass = 0; pass < 3; ++pass) {
      if (pass == 1) {
        if (!mbar_wait(b.dec_ready, 0, kErrMma | 2, abort)) break;
        tc_fence_after();
        any = *reinterpret_cast<volatile int*>(decision);
        if (!(MODE == kQuant && any)) continue;
      }
      // K steps of 32 bytes: QUANT uses D bytes (q8.16msb) or 2D bytes (Q'.K');
      // DENSE uses 2D bytes (D fp16/bf16 values).
      const int kbytes = (MODE == kQuant) ? (pass_uses_lsb(pass, any) ? 2 * D : D) : 2 * D;
      const int nk = kbytes / 32;
      bool ok = true;
      for (int j = 0; j <= nt; ++j) {
        if (j < nt) {
          const int es = t % kNExp, sb = t % L::kSBuf;
          if (!mbar_wait(b.k_full[es], (t / kNExp) & 1, kErrMma | 3, abort)) { ok = false; break; }
          if (!mbar_wait(b.s_empty[sb], ((t / L::kSBuf) & 1) ^ 1, kErrMma | 4, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t kaddr = smem_u32(sm + L::oK + es * L::kKBytes);
          for (int kk = 0; kk < nk; ++kk) {
            const int atom = kk >> 2, off = (kk & 3) * 32;
            const uint64_t ad = smem_desc_sw128(qaddr + atom * (BM * 128) + off, 16, 1024);
            const uint64_t bd = smem_desc_sw128(kaddr + atom * (L::kKRows * 128) + off, 16, 1024);
            if (MODE == kQuant) mma_i8(tmem + sb * L::kSW, ad, bd, idesc_s, kk > 0);
            else mma_f16(tmem + sb * L::kSW, ad, bd, idesc_s, kk > 0);
          }
          mma_commit(b.s_full[sb]);
          mma_commit(b.k_empty[es]);
          ++t;
        }
        if (pass == 2 && j >= 1) {  // O += P_jj V_jj, jj = j - 1
          const int jj = j - 1;
          const int pb = jj % kNP, vs = tv % kNV;
          if (!mbar_wait(b.p_full[pb], (jj / kNP) & 1, kErrMma | 5, abort)) { ok = false; break; }
          if (!mbar_wait(b.v_full[vs], (tv / kNV) & 1, kErrMma | 6, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t paddr = smem_u32(sm + L::oP + pb * L::kPBytes);
          const uint32_t vaddr = smem_u32(sm + L::oV + vs * L::kVBytes);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(paddr + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(vaddr + kk * 2048, BN * 128, 1024);
            mma_f16(tmem + L::kColO, ad, bd, idesc_pv, (first_pv && kk == 0) ? 0u : 1u);
          }
          first_pv = false;
          mma_commit(b.v_empty[vs]);
          ++tv;
          const bool pair_end = (jj & 1) || jj == nt - 1;
          if (!want_tok) {
            mma_commit(b.p_empty[pb]);
          } else if (pair_end) {
            // token importance of the pair's 128 keys: P'^T as an MN-major A
            // operand (the two P buffers are its two 64-key blocks, LBO apart)
            // times a [rows x 16] block of ones; K = the CTA's 128 query rows.
            const int pi = jj >> 1, cb = pi & 1;
            if (!mbar_wait(b.cs_empty[cb], ((pi >> 1) & 1) ^ 1, kErrMma | 7, abort)) { ok = false; break; }
            tc_fence_after();
            const uint32_t p0 = smem_u32(sm + L::oP);
            const uint32_t ones = smem_u32(sm + L::oOnes);
#pragma unroll
            for (int kk = 0; kk < BM / 16; ++kk) {
              const uint64_t ad = smem_desc_sw128(p0 + kk * 2048, L::kPBytes, 1024);
              const uint64_t bd = smem_desc_sw128(ones + (kk >> 2) * (kCsCols * 128) + (kk & 3) * 32, 16, 1024);
              mma_f16(tmem + L::kColCs + cb * kCsCols, ad, bd, idesc_cs, kk > 0 ? 1u : 0u);
            }
            mma_commit(b.cs_full[cb]);
            if (jj & 1) mma_commit(b.p_empty[0]);  // the pair's even tile
            mma_commit(b.p_empty[pb]);
          }
        }
        if (pass != 2 && j == nt - 1) break;
      }
      if (!ok) break;
    }
    // O is complete (or the CTA aborts): signal the epilogue either way, and
    // wait until every tcgen05 operation issued here has finished before the
    // CTA can free its tensor memory.
    mma_commit(b.o_full);
    const long long t0 = clock64();
    while (!mbar_try_wait(b.o_full, 0) && clock64() - t0 < kWaitLimitCycles) {
    }
  }

  // -------------------------------------------------------------- softmax
  SPATTEN_DEV void softmax_role();
  SPATTEN_DEV void load_q_row(int r, bool valid);
};

// Q row r -> Q' operand (first D bytes for QUANT, 2D bytes for DENSE and
// COMPAT), zeros if invalid.
template <int MODE, typename T, int D, bool VC>
SPATTEN_DEV void Cta<MODE, T, D, VC>::load_q_row(int r, bool valid) {
  const int row = m0 + r;
  uint8_t* base = sm + L::oQ;
  const int sw = r & 7;
  const int esz = (MODE == kQuant) ? 1 : (int)sizeof(T);
  constexpr int kChunks = D * ((MODE == kQuant) ? 1 : (int)sizeof(T)) / 16;
  const uint8_t* src = static_cast<const uint8_t*>(p.q) +
                       ((int64_t)z * p.q_sz + (int64_t)h * p.q_sh + (int64_t)row * p.q_sm) * esz;
  const bool al16 = ((reinterpret_cast<uintptr_t>(src)) & 15) == 0;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (valid) {
      if (al16) {
        v = __ldg(reinterpret_cast<const uint4*>(src) + c);
      } else {
        const uint32_t* s4 = reinterpret_cast<const uint32_t*>(src + 16 * c);
        v = make_uint4(__ldg(s4), __ldg(s4 + 1), __ldg(s4 + 2), __ldg(s4 + 3));
      }
    }
    const int off = 16 * c;
    const int atom = off >> 7, chunk = (off >> 4) & 7;
    *reinterpret_cast<uint4*>(base + atom * (BM * 128) + r * 128 + ((chunk ^ sw) << 4)) = v;
  }
}

// max(a, b, c) in one instruction
SPATTEN_DEV float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// 1.0f if a >= b, else 0.0f
SPATTEN_DEV float ge_one(float a, float b) {
  float d;
  asm("set.ge.f32.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// One softmax thread per query row (TMEM lane = row) owns all 64 columns of
// a key tile: the row statistics are thread-local. Scores are carried in the
// log2 domain, s = t * cs (+ a key bias) with one rounding (t: QUANT the
// exact integer score times the key scale, DENSE q.k, COMPAT the reference's
// tile-rule score; cs: the row scale, q scale * sm_scale * log2 e), so that a
// zero bias gives the same bits as none (HF materialises an all-zero mask
// where it cannot test the user's on the host, e.g. in graph capture).
template <int MODE, typename T, int D, bool VC>
SPATTEN_DEV void Cta<MODE, T, D, VC>::softmax_role() {
  const int tid = threadIdx.x;      // 0 .. kSoftThreads-1
  const int warp = tid >> 5, lane = tid & 31;
  const int r = tid;                // row within the tile = TMEM lane
  const int row = m0 + r;
  const bool valid = row < p.M;
  const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
  float cs = 0.f;
  if (valid) {
    cs = (MODE == kQuant) ? p.q_scale[((int64_t)z * p.H + h) * p.M + row] * p.sm_scale * kLog2e
         : (MODE == kCompat) ? kLog2e : p.sm_scale * kLog2e;
  }
  const bool key_bias = p.bias != nullptr && p.b_sm == 0;
  const bool gen_bias = p.bias != nullptr && p.b_sm != 0;
  {  // ones block: B operand of the column-sum MMA (every element 1.0)
    const uint32_t one2 = pack2<T>(1.f, 1.f);
    uint4* ob = reinterpret_cast<uint4*>(sm + L::oOnes);
    for (int i = tid; i < L::kOnesBytes / 16; i += kSoftThreads) ob[i] = make_uint4(one2, one2, one2, one2);
  }
  load_q_row(r, valid);
  fence_proxy_async_smem();
  __syncwarp();
  mbar_arrive_elect(b.q_ready);

  const float* brow = gen_bias ? p.bias + (int64_t)z * p.b_sz + (int64_t)h * p.b_sh + (int64_t)row * p.b_sm
                               : nullptr;
  const int shift = p.N - p.M;
  // keys this row sees: n < klim (key_limit, causal diagonal, or all)
  const int klim = p.key_limit ? (valid ? p.key_limit[(int64_t)z * p.M + row] : 0)
                               : (p.causal ? row + shift + 1 : p.N);
  const float* ksm = reinterpret_cast<const float*>(sm + L::oKs);
  const float* kbm = reinterpret_cast<const float*>(sm + L::oKb);

  uint32_t t = 0;
  bool alive = true;

  // COMPAT: OR over the criterion tile of "some q.k_msb * sm_scale >= thr",
  // separately for the tile's two 32-key halves. A warp covers 32 rows; a
  // 64-row criterion tile spans two warps, which vote through shared memory
  // and an mbarrier (double-buffered over the key tiles).
  auto compat_vote = [&](bool hlo, bool hhi, uint32_t tt, bool& any_lo, bool& any_hi) {
    bool wlo = __any_sync(0xffffffffu, hlo), whi = __any_sync(0xffffffffu, hhi);
    if (p.tile_n == 64) wlo = whi = (wlo || whi);
    if (p.tile_m == 64) {
      const int buf = tt & 1, grp = warp >> 1;
      int* votes = reinterpret_cast<int*>(sm + L::oVote) + buf * kSoftWarps;
      if (lane == 0) votes[warp] = (wlo ? 1 : 0) | (whi ? 2 : 0);
      __syncwarp();
      if (lane == 0) mbar_arrive(b.vote[buf * 4 + grp]);
      if (!mbar_wait(b.vote[buf * 4 + grp], (tt >> 1) & 1, kErrSoftmax | 6, abort)) {
        alive = false;
        wlo = whi = true;
      } else {
        const int v = votes[2 * grp] | votes[2 * grp + 1];
        wlo = (v & 1) != 0;
        whi = (v & 2) != 0;
      }
    }
    any_lo = wlo;
    any_hi = whi;
  };

  // This row's 64 scores of key tile j (see the function comment for their
  // scaling); keys past N and keys the row does not see are -inf. With
  // `dump`, the integer scores also go to score_out.
  auto scores = [&](int j, float (&s)[BN], int32_t* dump) {
    const int sb = t % L::kSBuf, es = t % kNExp;
    const uint32_t tt = t++;
    if (!alive) return;
    if (!mbar_wait(b.s_full[sb], (tt / L::kSBuf) & 1, kErrSoftmax | 1, abort)) { alive = false; return; }
    tc_fence_after();
    tmem_ld32f(tl + sb * L::kSW, s);
    tmem_ld32f(tl + sb * L::kSW + 32, s + 32);
    // the key scales / bias of this tile: waited for while the load is in flight
    const bool k_ok = mbar_wait(b.k_full[es], (tt / kNExp) & 1, kErrSoftmax | 2, abort);
    tmem_wait_ld();
    const int n0 = j * BN;
    if (MODE != kCompat) {
      tc_fence_before();
      __syncwarp();
      mbar_arrive_elect(b.s_empty[sb]);
    }
    if (MODE == kQuant && dump && valid && row % p.score_rs == 0) {
      int32_t* d = dump + (int64_t)(row / p.score_rs) * p.N + n0;
#pragma unroll
      for (int i = 0; i < BN; ++i)
        if (n0 + i < p.N) d[i] = (int32_t)__float_as_uint(s[i]);
    }
    if (!k_ok) { alive = false; return; }
    if (MODE == kQuant) {
      // exact int32 -> fp32 (|x| < 2^22): the bits of 1.5 * 2^23 + x, minus
      // 1.5 * 2^23; then times the key's scale. The key scales are read in
      // chunks of kKsChunk columns, fenced from each other, so that the
      // compiler does not hoist all 64 of them into registers at once.
      const float* ks = ksm + es * BN;
      const float2 nmag = make_float2(-kMagic, -kMagic);
#pragma unroll
      for (int i = 0; i < BN; i += 4) {
        if (kKsChunk < BN && i > 0 && i % kKsChunk == 0) asm volatile("" ::: "memory");
        const float4 k4 = *reinterpret_cast<const float4*>(ks + i);
        float2 a = __fadd2_rn(make_float2(i2f_exact(__float_as_uint(s[i])), i2f_exact(__float_as_uint(s[i + 1]))), nmag);
        float2 c = __fadd2_rn(make_float2(i2f_exact(__float_as_uint(s[i + 2])), i2f_exact(__float_as_uint(s[i + 3]))), nmag);
        a = __fmul2_rn(a, make_float2(k4.x, k4.y));
        c = __fmul2_rn(c, make_float2(k4.z, k4.w));
        s[i] = a.x;
        s[i + 1] = a.y;
        s[i + 2] = c.x;
        s[i + 3] = c.y;
      }
    } else if (MODE == kCompat) {
      // the reference's rule: q.k_msb * sm_scale, plus q.k_lsb * sm_scale
      // where the criterion tile's largest q.k_msb * sm_scale is below tile_thr
      const float sc = p.sm_scale, thr = p.tile_thr;
      const int lim_n = p.N - n0;
      bool hlo = false, hhi = false;
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        s[i] = s[i] * sc;
        const bool hot = (i < lim_n) && s[i] >= thr;
        if (i < 32) hlo |= hot;
        else hhi |= hot;
      }
      bool any_lo, any_hi;
      compat_vote(valid && hlo, valid && hhi, tt, any_lo, any_hi);
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf) {
        float lr[32];
        tmem_ld32f(tl + sb * L::kSW + BN + 32 * hlf, lr);
        tmem_wait_ld();
        if (!(hlf ? any_hi : any_lo)) {
#pragma unroll
          for (int i = 0; i < 32; ++i) s[32 * hlf + i] = s[32 * hlf + i] + lr[i] * sc;
        }
      }
      tc_fence_before();
      __syncwarp();
      mbar_arrive_elect(b.s_empty[sb]);
    }
    {
      const float2 cs2 = make_float2(cs, cs);
      if (key_bias) {  // s = t * cs + key bias * log2 e, one rounding
        const float* kb = kbm + es * BN;
#pragma unroll
        for (int i = 0; i < BN; i += 4) {
          const float4 k4 = *reinterpret_cast<const float4*>(kb + i);
          const float2 a = __ffma2_rn(make_float2(s[i], s[i + 1]), cs2, make_float2(k4.x, k4.y));
          const float2 c = __ffma2_rn(make_float2(s[i + 2], s[i + 3]), cs2, make_float2(k4.z, k4.w));
          s[i] = a.x;
          s[i + 1] = a.y;
          s[i + 2] = c.x;
          s[i + 3] = c.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < BN; i += 2) {
          const float2 a = __fmul2_rn(make_float2(s[i], s[i + 1]), cs2);
          s[i] = a.x;
          s[i + 1] = a.y;
        }
      }
    }
    __syncwarp();
    mbar_arrive_elect(b.k_empty[es]);
    if (gen_bias && valid) {
#pragma unroll
      for (int i = 0; i < BN; ++i)
        if (n0 + i < p.N) s[i] += __ldg(brow + (int64_t)(n0 + i) * p.b_sn) * kLog2e;
    }
    // keys past N and, with the causal mask, keys after the row's diagonal:
    // only tiles that reach them pay for the per-element test
    const int lim = min(p.N, klim) - n0;
    if (lim < BN) {
#pragma unroll
      for (int i = 0; i < BN; ++i)
        if (i >= lim) s[i] = -INFINITY;
    }
  };

  // Online statistics (log2 domain) of the row over one tile.
  auto stats = [&](const float (&s)[BN], float& m, float& l) {
    static_assert(BN % 8 == 0, "max tree over 8-column groups");
    float a0 = fmaxf(s[0], s[1]), a1 = fmaxf(s[2], s[3]), a2 = fmaxf(s[4], s[5]), a3 = fmaxf(s[6], s[7]);
#pragma unroll
    for (int i = 8; i < BN; i += 8) {
      a0 = fmax3(a0, s[i], s[i + 1]);
      a1 = fmax3(a1, s[i + 2], s[i + 3]);
      a2 = fmax3(a2, s[i + 4], s[i + 5]);
      a3 = fmax3(a3, s[i + 6], s[i + 7]);
    }
    const float mn = fmaxf(m, fmax3(fmaxf(a0, a1), a2, a3));
    if (mn == -INFINITY) return;
    const float2 nm = make_float2(-mn, -mn);
    float2 acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < BN; i += 8) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 x = __fadd2_rn(make_float2(s[i + 2 * k], s[i + 2 * k + 1]), nm);
        acc[k] = __fadd2_rn(acc[k], make_float2(fast_exp2(x.x), fast_exp2(x.y)));
      }
    }
    const float2 a = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
    l = l * fast_exp2(m - mn) + (a.x + a.y);
    m = mn;
  };

  const bool want_tok = p.tok_partial != nullptr;
  float* tokp = want_tok ? p.tok_partial + (((int64_t)z * p.H + h) * p.mtiles + mt) * p.N : nullptr;
  // column sums of tile pair pi (128 keys) from TMEM: lane = key
  auto read_pair = [&](int pi) {
    const int cb = pi & 1;
    if (!alive) return;
    if (!mbar_wait(b.cs_full[cb], (pi >> 1) & 1, kErrSoftmax | 5, abort)) { alive = false; return; }
    tc_fence_after();
    uint32_t v;
    tmem_ld1(tl + L::kColCs + cb * kCsCols, v);
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    mbar_arrive_elect(b.cs_empty[cb]);
    const int key = pi * 2 * BN + warp * 32 + lane;
    if (key < p.N && key < nt * BN) tokp[key] = __uint_as_float(v);
  };

  float s[BN];
  float m_run = -INFINITY, l_run = 0.f;  // statistics of the scores in use
  float mf = -INFINITY, lf = 0.f;        // statistics of the full score (pass 1b)
  bool flag = false, warp_any = false;
  int any = 0;
  const float vthr = p.v_thr;
  int32_t* dump = (MODE == kQuant && p.score_out)
                      ? p.score_out + ((int64_t)z * p.H + h) * ((p.M + p.score_rs - 1) / p.score_rs) * (int64_t)p.N
                      : nullptr;
  float mo = -INFINITY;  // pass 2: P = exp2(s + mo)
  // Count V prune (VC): this row's kMaxVPruneCount smallest (score, key)
  // pairs of the scores it ends up using, ascending in (score, key), in
  // registers (the count-prune instantiation runs one CTA per SM with the
  // register budget for it); the row's v_count-th smallest pair (kvs, kvn)
  // marks the keys to drop.
  constexpr int KC = VC ? kMaxVPruneCount : 1;
  float cv[KC];
  int cn[KC];
  float kvs = -INFINITY;
  int kvn = -1;
  auto track_reset = [&]() {
#pragma unroll
    for (int q = 0; q < KC; ++q) {
      cv[q] = INFINITY;
      cn[q] = INT_MAX;
    }
  };
  auto track = [&](int j) {
    const int n0 = j * BN;
    const int lim = p.N - n0;  // keys past N are not part of the row
#pragma unroll
    for (int i = 0; i < BN; ++i) {
      // keys arrive in increasing order, so an equal score ranks after the
      // entries already kept: only a smaller score enters the list, which
      // then bubbles into place
      float x = s[i];
      if (i < lim && x < cv[KC - 1]) {
        int xn = n0 + i;
#pragma unroll
        for (int q = 0; q < KC; ++q) {
          const bool lt = x < cv[q];
          const float tv = cv[q];
          const int tn = cn[q];
          cv[q] = lt ? x : tv;
          cn[q] = lt ? xn : tn;
          x = lt ? tv : x;
          xn = lt ? tn : xn;
        }
      }
    }
  };
  if (VC) track_reset();
  int pairs_read = 0;
  const int npairs = (nt + 1) / 2;
  // One loop over the passes keeps a single copy of the tile code:
  //   pass 0 statistics of the MSB (QUANT) / only (DENSE, COMPAT) score
  //   pass 1 statistics of the full score of refetched rows (QUANT, if any)
  //   pass 2 P, V prune, P -> shared memory (P.V and the column sums run on
  //          the tensor cores)
  for (int pass = 0; pass < 3; ++pass) {
    if (pass == 1) {
      // ---- decide the refetch, build Q'
      if (MODE == kQuant) {
        flag = alive && valid && __frcp_rn(l_run) < p.refetch_thr;
        if (VC && flag) track_reset();  // a refetched row ends up using its full scores
        // Q' bytes [D, 2D): q8 for a refetched row, zeros otherwise
        uint8_t* base = sm + L::oQ;
        const int sw = r & 7;
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          const int src_off = 16 * c, dst_off = D + 16 * c;
          const uint4 v = *reinterpret_cast<const uint4*>(base + (src_off >> 7) * (BM * 128) + r * 128 +
                                                          ((((src_off >> 4) & 7) ^ sw) << 4));
          *reinterpret_cast<uint4*>(base + (dst_off >> 7) * (BM * 128) + r * 128 +
                                    ((((dst_off >> 4) & 7) ^ sw) << 4)) =
              flag ? v : make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        uint32_t anyv;
        asm volatile(
            "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n barrier.cta.red.or.pred p, 1, %2, q;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(anyv)
            : "r"((uint32_t)flag), "n"(kSoftThreads)
            : "memory");
        any = (int)anyv;
        if (tid == 0) *decision = any;
        if (p.refetch_out && valid) p.refetch_out[((int64_t)z * p.H + h) * p.M + row] = flag;
      }
      __syncwarp();
      mbar_arrive_elect(b.dec_ready);
      if (!(MODE == kQuant && any)) continue;
      warp_any = __any_sync(0xffffffffu, flag);
    }
    if (pass == 2) {
      if (MODE == kQuant && any && flag) {
        m_run = mf;
        l_run = lf;
      }
      mo = (valid && m_run != -INFINITY && l_run > 0.f) ? -(m_run + __log2f(l_run)) : -INFINITY;
      if (VC && p.v_count > 0) {
        // the list is ascending: its v_count-th entry marks the keys to drop
#pragma unroll
        for (int q = 0; q < KC; ++q)
          if (q == p.v_count - 1) {
            kvs = cv[q];
            kvn = cn[q];
          }
      }
    }
    for (int j = 0; j < nt; ++j) {
      scores(j, s, pass == 2 ? dump : nullptr);
      if (pass < 2) {
        if (alive && (pass == 0 || warp_any)) {
          float m = pass == 0 ? m_run : mf;
          float l = pass == 0 ? l_run : lf;
          stats(s, m, l);
          if (VC && (pass == 0 || flag)) track(j);
          if (pass == 0) {
            m_run = m;
            l_run = l;
          } else {
            mf = m;
            lf = l;
          }
        }
        continue;
      }
      // ---- pass 2 tile
      const int pb = j % kNP;
      if (alive) {
        uint64_t drop = 0;  // count V prune: keys at or below (kvs, kvn)
        if (VC) {
          const int n0 = j * BN;
#pragma unroll
          for (int i = 0; i < BN; ++i)
            drop |= (uint64_t)(s[i] < kvs || (s[i] == kvs && n0 + i <= kvn)) << i;
        }
        const float2 mo2 = make_float2(mo, mo);
#pragma unroll
        for (int i = 0; i < BN; i += 2) {
          const float2 x = __fadd2_rn(make_float2(s[i], s[i + 1]), mo2);
          s[i] = fast_exp2(x.x);
          s[i + 1] = fast_exp2(x.y);
        }
        if (vthr > 0.f) {
#pragma unroll
          for (int i = 0; i < BN; i += 2) {
            const float2 k = make_float2(ge_one(s[i], vthr), ge_one(s[i + 1], vthr));
            const float2 q = __fmul2_rn(make_float2(s[i], s[i + 1]), k);
            s[i] = q.x;
            s[i + 1] = q.y;
          }
        }
        if (VC) {
#pragma unroll
          for (int i = 0; i < BN; ++i) s[i] = (drop >> i) & 1u ? 0.f : s[i];
        }
        // P -> shared memory: A operand of P.V (K-major) and, read as an
        // MN-major operand, of the column sums; 128B swizzle
        if (mbar_wait(b.p_empty[pb], ((j / kNP) & 1) ^ 1, kErrSoftmax | 3, abort)) {
          uint8_t* prow = sm + L::oP + pb * L::kPBytes + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4 v;
            v.x = pack2<T>(s[8 * c], s[8 * c + 1]);
            v.y = pack2<T>(s[8 * c + 2], s[8 * c + 3]);
            v.z = pack2<T>(s[8 * c + 4], s[8 * c + 5]);
            v.w = pack2<T>(s[8 * c + 6], s[8 * c + 7]);
            *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = v;
          }
          fence_proxy_async_smem();
          __syncwarp();
          mbar_arrive_elect(b.p_full[pb]);
        } else {
          alive = false;
        }
      }
      // column sums of the pair before last (its MMA had a pair's time to finish)
      if (want_tok && (j & 1) && j >= 3) read_pair(pairs_read++);
    }
  }
  if (want_tok)
    while (pairs_read < npairs) read_pair(pairs_read++);
  if (want_tok)  // skipped key tiles: no probability reached them
    for (int key = nt * BN + tid; key < p.N; key += kSoftThreads) tokp[key] = 0.f;

  // ---- epilogue: O (already normalised) from TMEM, this thread's row
  if (!mbar_wait(b.o_full, 0, kErrSoftmax | 4, abort)) alive = false;
  tc_fence_after();
  float asum = 0.f;
  const int hslot = p.out_head_map ? p.out_head_map[h] : h;
  const bool out_ok = hslot >= 0 && hslot < p.out_head_slots;
  T* orow = static_cast<T*>(p.out) + (int64_t)z * p.o_sz + (int64_t)hslot * p.o_sh + (int64_t)row * p.o_sm;
  const bool out16 = (reinterpret_cast<uintptr_t>(orow) & 15) == 0;
#pragma unroll
  for (int c = 0; c < D / 32; ++c) {
    float o[32];
    tmem_ld32f(tl + L::kColO + 32 * c, o);
    tmem_wait_ld();
    if (alive && valid) {
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        asum += fabsf(o[2 * i]) + fabsf(o[2 * i + 1]);
        pk[i] = pack2<T>(o[2 * i], o[2 * i + 1]);
      }
      if (out_ok) {
        if (out16) {
          uint4* dst = reinterpret_cast<uint4*>(orow + 32 * c);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        } else {
          uint32_t* dst = reinterpret_cast<uint32_t*>(orow + 32 * c);
#pragma unroll
          for (int i = 0; i < 16; ++i) dst[i] = pk[i];
        }
      }
    }
  }
  tc_fence_before();
  if (p.head_partial) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) asum += __shfl_xor_sync(0xffffffffu, asum, off);
    float* hs = reinterpret_cast<float*>(sm + L::oHs);
    if (lane == 0) hs[warp] = asum;
    named_sync(1, kSoftThreads);
    if (tid == 0 && alive) {
      float tot = 0.f;
      for (int w = 0; w < kSoftWarps; ++w) tot += hs[w];
      p.head_partial[((int64_t)z * p.H + h) * p.mtiles + mt] = tot;
    }
  }
}

template <int MODE, typename T, int D, bool VC>
__global__ void __launch_bounds__(kThreads, (D == 64 && !VC) ? 2 : 1)
    prog_attn_tc_kernel(const __grid_constant__ TcParams P) {
  extern __shared__ uint8_t smem_raw[];
  using L = Layout<MODE, T, D, VC>;
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  Cta<MODE, T, D, VC> c(P, base);
  const int warp = threadIdx.x >> 5;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + L::oTmem);
  if (threadIdx.x == 0) c.init_barriers();
  if (warp == 0) c.count_key_tiles();
  if (warp == kWarpMma) {
    tmem_alloc(tslot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  c.tmem = *tslot;
  c.nt = *reinterpret_cast<volatile int*>(base + L::oFlag + 8);
  // Two CTAs per SM launch at kSplitLaunchRegs registers a thread (the host
  // refuses the launch otherwise); the softmax warpgroup takes 160 of them
  // and the producer warpgroup (TMA, MMA, expanders) keeps 96:
  // 128 * 160 + 128 * 96 = 256 * 128, the CTA's launch allocation.
  if (warp < kSoftWarps) {
    if (kRegSplit<D, VC>) asm volatile("setmaxnreg.inc.sync.aligned.u32 160;\n" ::: "memory");
    c.softmax_role();
  } else {
    if (kRegSplit<D, VC>) asm volatile("setmaxnreg.dec.sync.aligned.u32 96;\n" ::: "memory");
    if (warp == kWarpTma) c.tma_role();
    else if (warp == kWarpMma) c.mma_role();
    else c.expand_role();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(c.tmem, L::kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 4-D map [Z, H, N, inner] with byte strides (sn, sh, sz); box {box_inner, 64, 1, 1}.
cudaError_t make_map(CUtensorMap* m, CUtensorMapDataType dt, int esz, const void* base, int inner,
                     int N, int H, int Z, int64_t sn, int64_t sh, int64_t sz, int box_inner,
                     CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  auto fix = [](int64_t s, int64_t minv) -> cuuint64_t { return (cuuint64_t)(s > 0 ? s : minv); };
  cuuint64_t dims[4] = {(cuuint64_t)inner, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)Z};
  cuuint64_t strides[3] = {fix(sn, 16), fix(sh, 16), fix(sz, 16)};
  cuuint32_t box[4] = {(cuuint32_t)box_inner, (cuuint32_t)BN, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  (void)esz;
  CUresult r = fn(m, dt, 4, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int MODE, typename T, int D, bool VC>
cudaError_t launch_tc_t(const AttnParams& a, cudaStream_t st) {
  using L = Layout<MODE, T, D, VC>;
  TcParams P;
  memset(&P, 0, sizeof(P));
  P.a = a;
  const CUtensorMapDataType vdt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cudaError_t e;
  if (MODE == kQuant) {
    const CUtensorMapSwizzle psw = (D == 64) ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
    e = make_map(&P.tm_k0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.k0, D / 2, a.N, a.Hkv, a.Z, a.k_sn,
                 a.k_sh, a.k_sz, D / 2, psw);
    if (e != cudaSuccess) return e;
    e = make_map(&P.tm_k1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.k1, D / 2, a.N, a.Hkv, a.Z, a.k_sn,
                 a.k_sh, a.k_sz, D / 2, psw);
    if (e != cudaSuccess) return e;
  } else {
    e = make_map(&P.tm_k0, vdt, 2, a.k0, D, a.N, a.Hkv, a.Z, a.k_sn * 2, a.k_sh * 2, a.k_sz * 2, 64,
                 CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
    if (MODE == kCompat) {  // k_lsb: the same layout as k_msb
      e = make_map(&P.tm_k1, vdt, 2, a.k1, D, a.N, a.Hkv, a.Z, a.k_sn * 2, a.k_sh * 2, a.k_sz * 2, 64,
                   CU_TENSOR_MAP_SWIZZLE_128B);
      if (e != cudaSuccess) return e;
    }
  }
  e = make_map(&P.tm_v, vdt, 2, a.v, D, a.N, a.Hkv, a.Z, a.v_sn * 2, a.v_sh * 2, a.v_sz * 2, 64,
               CU_TENSOR_MAP_SWIZZLE_128B);
  if (e != cudaSuccess) return e;
  auto kern = prog_attn_tc_kernel<MODE, T, D, VC>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return e;
  if (kRegSplit<D, VC>) {
    // the register split adds up only at this launch allocation; with any
    // other, setmaxnreg.inc would wait for registers the CTA does not hold
    static int regs = -1;  // one per instantiation
    if (regs < 0) {
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, kern);
      if (e != cudaSuccess) return e;
      regs = fa.numRegs;
    }
    if (regs != kSplitLaunchRegs) return cudaErrorInvalidConfiguration;
  }
  dim3 grid((unsigned)a.mtiles, (unsigned)a.H, (unsigned)a.Z);
  kern<<<grid, kThreads, L::kAlloc, st>>>(P);
  return cudaGetLastError();
}

template <int MODE, typename T>
cudaError_t launch_tc_d(const AttnParams& a, cudaStream_t st) {
  if (a.D == 64) return a.v_count > 0 ? launch_tc_t<MODE, T, 64, true>(a, st) : launch_tc_t<MODE, T, 64, false>(a, st);
  if (a.D == 128) return a.v_count > 0 ? launch_tc_t<MODE, T, 128, true>(a, st) : launch_tc_t<MODE, T, 128, false>(a, st);
  return cudaErrorInvalidValue;
}

}  // namespace

int tc_tile_rows() { return BM; }

cudaError_t launch_prog_attn_tc(const AttnParams& a, cudaStream_t st) {
  const bool f16 = a.dtype == kF16;
  if (a.mode == kQuant) return f16 ? launch_tc_d<kQuant, __half>(a, st) : launch_tc_d<kQuant, __nv_bfloat16>(a, st);
  if (a.mode == kDense) return f16 ? launch_tc_d<kDense, __half>(a, st) : launch_tc_d<kDense, __nv_bfloat16>(a, st);
  if (a.mode == kCompat) {
    if (a.v_count > 0) return cudaErrorInvalidValue;
    if (a.D == 64) return f16 ? launch_tc_t<kCompat, __half, 64, false>(a, st)
                              : launch_tc_t<kCompat, __nv_bfloat16, 64, false>(a, st);
    if (a.D == 128) return f16 ? launch_tc_t<kCompat, __half, 128, false>(a, st)
                               : launch_tc_t<kCompat, __nv_bfloat16, 128, false>(a, st);
  }
  return cudaErrorInvalidValue;
}

// fp16 / bf16 (every mode) on the tcgen05 kernel above, fp32 (QUANT, DENSE)
// on the SIMT kernel.
int attn_tile_rows(const AttnParams& p) { return p.dtype == kF32 ? f32_tile_rows() : tc_tile_rows(); }

cudaError_t launch_prog_attn(const AttnParams& p, cudaStream_t st, int) {
  if (p.dtype == kF32) return launch_prog_attn_f32(p, st);
  return launch_prog_attn_tc(p, st);
}

cudaError_t read_device_error(unsigned int* code, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(code, sm100::g_device_error, sizeof(unsigned int));
  if (e != cudaSuccess || !reset) return e;
  const unsigned int zero = 0;
  return cudaMemcpyToSymbol(sm100::g_device_error, &zero, sizeof(unsigned int));
}

}  // namespace spatten
