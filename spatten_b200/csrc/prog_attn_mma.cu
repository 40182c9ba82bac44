// Progressive sparse attention, warp-level tensor-core path (mma.sync).
//
// One CTA = 4 warps = 64 query rows of one (z, h); each warp owns 16 rows and
// keeps its S tile, P fragments and O accumulator in registers. K/V tiles of
// 64 keys stream through a 2-stage cp.async ring in shared memory, XOR
// swizzled so that every ldmatrix is conflict free.
//
// The row statistics that the refetch rule, the V-prune threshold and the
// token importance all need are those of the *final* softmax, so the kernel
// is multi-pass over K (the K re-reads hit L2):
//   QUANT : pass 1  S = q8 . (16*msb)           -> (m, l) per row
//           decide  refetch = 1/l < refetch_thr
//           pass 1b S = q8 . k8, k8 = 16*msb|lsb -> (m, l) of refetched rows
//                   (only when the CTA has a refetched row: the LSB plane is
//                    read only then -- the progressive fetch)
//           pass 2  S = q8.(16*msb) + [refetch] q8.lsb; P = exp(S-m)/l;
//                   P' = P < v_thr ? 0 : P; O = P'V; column sums of P'.
//   DENSE : pass 1 stats, pass 2 as above with S = q.k (fp16/bf16 MMA).
//   COMPAT: the reference's tile rule (spatten_bert_ultimate.py:67-74):
//           S = q.k_msb*sc; if max over the tm x tn tile < tile_thr then
//           S += q.k_lsb*sc. Pass 1 stats, pass 2 output.
// Integer scores are exact (int8 MMA into int32); everything after the
// scores is fp32 in the log2 domain, P is rounded to the V type for P.V.
//
// The 4-bit planes are expanded in registers: with the split-at-D/2 packing
// a 32-bit word of packed bytes gives, with one shift and one mask, the
// int8 B fragment of 4 consecutive dims (low nibbles) and of the 4 dims D/2
// above them (high nibbles); 16*msb is just the nibble in the high half of
// the byte, so it needs no sign extension.
#include "common.cuh"
#include "kernels.h"

namespace spatten {

namespace {

constexpr int BM = 64;  // query rows per CTA
constexpr int BN = 64;  // keys per tile
constexpr int NB = BN / 8;
constexpr int kThreads = 128;

enum Mode : int { kQuant = 0, kDense = 1, kCompat = 2 };
enum ScoreKind : int { kMsb = 0, kFull = 1, kMixed = 2 };

// physical 16-byte chunk of logical chunk c in row r (cpr chunks per row)
SPATTEN_DEV int swz(int r, int c, int cpr) {
  if (cpr >= 8) return c ^ (r & 7);
  return c ^ ((r / (8 / cpr)) & (cpr - 1));
}

template <int MODE, typename T, int D>
struct Cfg {
  static constexpr int kPlanes = (MODE == kDense) ? 1 : 2;
  static constexpr int kRowB = (MODE == kQuant) ? D / 2 : D * (int)sizeof(T);  // K row bytes
  static constexpr int kCpr = kRowB / 16;                                       // K chunks/row
  static constexpr int kVRowB = D * (int)sizeof(T);
  static constexpr int kVCpr = kVRowB / 16;
  static constexpr int kKStage = kPlanes * BN * kRowB;
  static constexpr int kVStage = BN * kVRowB;
  // byte offsets
  static constexpr int oK = 0;
  static constexpr int oV = oK + 2 * kKStage;
  static constexpr int oKs = oV + 2 * kVStage;       // float [2][BN] key scale * log2e-free
  static constexpr int oKb = oKs + 2 * BN * 4;       // float [2][BN] per-key bias * log2e
  static constexpr int oCs = oKb + 2 * BN * 4;       // float [2][4][BN] column sums
  static constexpr int oTm = oCs + 2 * 4 * BN * 4;   // float [2][4][2] tile maxima
  static constexpr int oHs = oTm + 2 * 4 * 2 * 4;    // float [4]
  static constexpr int kSmem = oHs + 4 * 4;
};

template <int MODE, typename T, int D>
struct Attn {
  using C = Cfg<MODE, T, D>;
  static constexpr int KS8 = D / 32;  // int8 k-steps
  static constexpr int KSF = D / 16;  // fp16 k-steps
  static constexpr int ND = D / 8;    // n8 blocks of the output

  const AttnParams& p;
  uint8_t* smem;
  int warp, lane, g, t, tid;
  int z, h, kvh, mt, hslot;
  bool out_ok;  // head slot inside [0, out_head_slots)
  int row_lo, row_hi;  // rows of this thread
  bool valid_lo, valid_hi;
  const uint8_t* k0b;  // base of (z, kvh) for plane 0 / k
  const uint8_t* k1b;
  const uint8_t* vb;
  float c2_lo, c2_hi;  // per-row score multiplier (log2 domain)
  bool per_key_bias;

  // query fragments
  uint32_t qa[(MODE == kQuant) ? KS8 : KSF][4];

  SPATTEN_DEV Attn(const AttnParams& pp, uint8_t* sm) : p(pp), smem(sm) {
    tid = threadIdx.x;
    warp = tid >> 5;
    lane = tid & 31;
    g = lane >> 2;
    t = lane & 3;
    mt = blockIdx.x;
    h = blockIdx.y;
    z = blockIdx.z;
    kvh = h / (p.H / p.Hkv);
    hslot = p.out_head_map ? p.out_head_map[h] : h;
    out_ok = hslot >= 0 && hslot < p.out_head_slots;
    row_lo = mt * BM + warp * 16 + g;
    row_hi = row_lo + 8;
    valid_lo = row_lo < p.M;
    valid_hi = row_hi < p.M;
    const int esz = (MODE == kQuant) ? 1 : (int)sizeof(T);
    k0b = static_cast<const uint8_t*>(p.k0) + ((int64_t)z * p.k_sz + (int64_t)kvh * p.k_sh) * esz;
    k1b = (MODE == kDense) ? nullptr
                           : static_cast<const uint8_t*>(p.k1) +
                                 ((int64_t)z * p.k_sz + (int64_t)kvh * p.k_sh) * esz;
    vb = static_cast<const uint8_t*>(p.v) + ((int64_t)z * p.v_sz + (int64_t)kvh * p.v_sh) * sizeof(T);
    per_key_bias = p.bias != nullptr && p.b_sm == 0;
    if (MODE == kQuant) {
      const float* qs = p.q_scale + ((int64_t)z * p.H + h) * p.M;
      c2_lo = valid_lo ? qs[row_lo] * p.sm_scale * kLog2e : 0.f;
      c2_hi = valid_hi ? qs[row_hi] * p.sm_scale * kLog2e : 0.f;
    } else {
      c2_lo = c2_hi = p.sm_scale * kLog2e;
    }
    load_q();
  }

  SPATTEN_DEV void load_q() {
    if (MODE == kQuant) {
      const int8_t* qb = static_cast<const int8_t*>(p.q) + (int64_t)z * p.q_sz + (int64_t)h * p.q_sh;
      const int8_t* rl = qb + (int64_t)row_lo * p.q_sm;
      const int8_t* rh = qb + (int64_t)row_hi * p.q_sm;
#pragma unroll
      for (int ks = 0; ks < KS8; ++ks) {
        const int c0 = ks * 32 + 4 * t;
        qa[ks][0] = valid_lo ? *reinterpret_cast<const uint32_t*>(rl + c0) : 0u;
        qa[ks][1] = valid_hi ? *reinterpret_cast<const uint32_t*>(rh + c0) : 0u;
        qa[ks][2] = valid_lo ? *reinterpret_cast<const uint32_t*>(rl + c0 + 16) : 0u;
        qa[ks][3] = valid_hi ? *reinterpret_cast<const uint32_t*>(rh + c0 + 16) : 0u;
      }
    } else {
      const T* qb = static_cast<const T*>(p.q) + (int64_t)z * p.q_sz + (int64_t)h * p.q_sh;
      const T* rl = qb + (int64_t)row_lo * p.q_sm;
      const T* rh = qb + (int64_t)row_hi * p.q_sm;
#pragma unroll
      for (int ks = 0; ks < KSF; ++ks) {
        const int c0 = ks * 16 + 2 * t;
        qa[ks][0] = valid_lo ? *reinterpret_cast<const uint32_t*>(rl + c0) : 0u;
        qa[ks][1] = valid_hi ? *reinterpret_cast<const uint32_t*>(rh + c0) : 0u;
        qa[ks][2] = valid_lo ? *reinterpret_cast<const uint32_t*>(rl + c0 + 8) : 0u;
        qa[ks][3] = valid_hi ? *reinterpret_cast<const uint32_t*>(rh + c0 + 8) : 0u;
      }
    }
  }

  SPATTEN_DEV uint8_t* kstage(int s, int plane) { return smem + C::oK + s * C::kKStage + plane * BN * C::kRowB; }
  SPATTEN_DEV uint8_t* vstage(int s) { return smem + C::oV + s * C::kVStage; }
  SPATTEN_DEV float* ks_s(int s) { return reinterpret_cast<float*>(smem + C::oKs) + s * BN; }
  SPATTEN_DEV float* kb_s(int s) { return reinterpret_cast<float*>(smem + C::oKb) + s * BN; }
  SPATTEN_DEV float* cs_s(int s) { return reinterpret_cast<float*>(smem + C::oCs) + s * 4 * BN; }
  SPATTEN_DEV float* tm_s(int s) { return reinterpret_cast<float*>(smem + C::oTm) + s * 8; }

  // Issue the cp.async loads of key tile [n0, n0+BN) into stage s.
  SPATTEN_DEV void load_tile(int s, int n0, bool plane1, bool with_v) {
    const int esz = (MODE == kQuant) ? 1 : (int)sizeof(T);
    const int nplanes = (MODE == kDense) ? 1 : (plane1 ? 2 : 1);
    for (int pl = 0; pl < nplanes; ++pl) {
      const uint8_t* base = pl == 0 ? k0b : k1b;
      uint8_t* dst = kstage(s, pl);
      for (int i = tid; i < BN * C::kCpr; i += kThreads) {
        const int r = i / C::kCpr, c = i % C::kCpr;
        const int n = n0 + r;
        const bool ok = n < p.N;
        const uint8_t* src = base + ((int64_t)(ok ? n : 0) * p.k_sn) * esz + c * 16;
        cp_async16(dst + r * C::kRowB + swz(r, c, C::kCpr) * 16, src, ok);
      }
    }
    if (with_v) {
      uint8_t* dst = vstage(s);
      for (int i = tid; i < BN * C::kVCpr; i += kThreads) {
        const int r = i / C::kVCpr, c = i % C::kVCpr;
        const int n = n0 + r;
        const bool ok = n < p.N;
        const uint8_t* src = vb + ((int64_t)(ok ? n : 0) * p.v_sn) * sizeof(T) + c * 16;
        cp_async16(dst + r * C::kVRowB + swz(r, c, C::kVCpr) * 16, src, ok);
      }
    }
    if (tid < BN) {
      const int n = n0 + tid;
      if (MODE == kQuant) {
        const float* ksc = p.k_scale + ((int64_t)z * p.Hkv + kvh) * p.N;
        ks_s(s)[tid] = n < p.N ? ksc[n] : 0.f;
      }
      if (per_key_bias) {
        kb_s(s)[tid] = n < p.N ? p.bias[(int64_t)z * p.b_sz + (int64_t)h * p.b_sh + (int64_t)n * p.b_sn] * kLog2e
                               : 0.f;
      }
    }
    cp_async_commit();
  }

  // ---- score tiles -------------------------------------------------------
  // s[nb][e]: row (e < 2 ? lo : hi), key n0 + nb*8 + 2t + (e & 1); log2 domain.

  // dump_n0 >= 0: also write the integer scores of key tile dump_n0 to score_out
  SPATTEN_DEV void quant_scores(int s, int kind, bool flag_lo, bool flag_hi, int dump_n0,
                                float (&sc)[NB][4]) {
    int acc[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nb][e] = 0;
    uint32_t qf[KS8][4];
    if (kind == kMixed) {
#pragma unroll
      for (int ks = 0; ks < KS8; ++ks) {
        qf[ks][0] = flag_lo ? qa[ks][0] : 0u;
        qf[ks][1] = flag_hi ? qa[ks][1] : 0u;
        qf[ks][2] = flag_lo ? qa[ks][2] : 0u;
        qf[ks][3] = flag_hi ? qa[ks][3] : 0u;
      }
    }
    const uint8_t* pm = kstage(s, 0);
    const uint8_t* pl = kstage(s, 1);
    const int mi = lane >> 3;
#pragma unroll
    for (int nb = 0; nb < NB; nb += 2) {
#pragma unroll
      for (int cp = 0; cp < KS8 / 2; ++cp) {
        // matrices: (nb, 2cp), (nb, 2cp+1), (nb+1, 2cp), (nb+1, 2cp+1)
        const int r = (nb + (mi >> 1)) * 8 + (lane & 7);
        const int c = 2 * cp + (mi & 1);
        const int off = r * C::kRowB + swz(r, c, C::kCpr) * 16;
        uint32_t x0a, x1a, x0b, x1b;
        ldmatrix_x4(x0a, x1a, x0b, x1b, pm + off);
        uint32_t y0a = 0, y1a = 0, y0b = 0, y1b = 0;
        if (kind != kMsb) ldmatrix_x4(y0a, y1a, y0b, y1b, pl + off);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t x0 = half ? x0b : x0a, x1 = half ? x1b : x1a;
          const uint32_t y0 = half ? y0b : y0a, y1 = half ? y1b : y1a;
          const int n = nb + half;
          // low nibbles -> k-step cp, high nibbles -> k-step cp + KS8/2
          const uint32_t mlo0 = (x0 << 4) & 0xF0F0F0F0u, mlo1 = (x1 << 4) & 0xF0F0F0F0u;
          const uint32_t mhi0 = x0 & 0xF0F0F0F0u, mhi1 = x1 & 0xF0F0F0F0u;
          if (kind == kMsb) {
            mma_s8_16832(acc[n], qa[cp], mlo0, mlo1);
            mma_s8_16832(acc[n], qa[cp + KS8 / 2], mhi0, mhi1);
          } else {
            const uint32_t llo0 = y0 & 0x0F0F0F0Fu, llo1 = y1 & 0x0F0F0F0Fu;
            const uint32_t lhi0 = (y0 >> 4) & 0x0F0F0F0Fu, lhi1 = (y1 >> 4) & 0x0F0F0F0Fu;
            if (kind == kFull) {
              mma_s8_16832(acc[n], qa[cp], mlo0 | llo0, mlo1 | llo1);
              mma_s8_16832(acc[n], qa[cp + KS8 / 2], mhi0 | lhi0, mhi1 | lhi1);
            } else {
              mma_s8_16832(acc[n], qa[cp], mlo0, mlo1);
              mma_s8_16832(acc[n], qa[cp + KS8 / 2], mhi0, mhi1);
              mma_s8_16832(acc[n], qf[cp], llo0, llo1);
              mma_s8_16832(acc[n], qf[cp + KS8 / 2], lhi0, lhi1);
            }
          }
        }
      }
    }
    if (dump_n0 >= 0) {
      int32_t* so = p.score_out + ((int64_t)z * p.H + h) * p.M * (int64_t)p.N;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = dump_n0 + nb * 8 + 2 * t + (e & 1);
          const int row = e < 2 ? row_lo : row_hi;
          if (row < p.M && key < p.N) so[(int64_t)row * p.N + key] = acc[nb][e];
        }
    }
    const float* ksc = ks_s(s);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int col = nb * 8 + 2 * t;
      const float k0 = ksc[col], k1 = ksc[col + 1];
      sc[nb][0] = (float)acc[nb][0] * (c2_lo * k0);
      sc[nb][1] = (float)acc[nb][1] * (c2_lo * k1);
      sc[nb][2] = (float)acc[nb][2] * (c2_hi * k0);
      sc[nb][3] = (float)acc[nb][3] * (c2_hi * k1);
    }
  }

  SPATTEN_DEV void float_mma(const uint8_t* kt, float (&acc)[NB][4]) {
    const int mi = lane >> 3;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nb][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KSF; ks += 2) {
        const int r = nb * 8 + (lane & 7);
        const int c = 2 * ks + mi;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3, kt + r * C::kRowB + swz(r, c, C::kCpr) * 16);
        mma_16816<T>(acc[nb], qa[ks], b0, b1);
        mma_16816<T>(acc[nb], qa[ks + 1], b2, b3);
      }
    }
  }

  SPATTEN_DEV void dense_scores(int s, float (&sc)[NB][4]) {
    float_mma(kstage(s, 0), sc);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      sc[nb][0] *= c2_lo;
      sc[nb][1] *= c2_lo;
      sc[nb][2] *= c2_hi;
      sc[nb][3] *= c2_hi;
    }
  }

  // Reference tile rule (spatten_bert_ultimate.py:67-74); the tile maxima of
  // the warps meet in the stage's scratch slot.
  SPATTEN_DEV void compat_scores(int s, int n0, float (&sc)[NB][4]) {
    float a1[NB][4], a2[NB][4];
    float_mma(kstage(s, 0), a1);
    float_mma(kstage(s, 1), a2);
    const float scl = p.sm_scale;
    // per key block (32 keys) maxima over this warp's valid entries
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        a1[nb][e] *= scl;
        const int key = n0 + nb * 8 + 2 * t + (e & 1);
        const bool ok = key < p.N && (e < 2 ? valid_lo : valid_hi);
        if (ok) mx[nb >> 2] = fmaxf(mx[nb >> 2], a1[nb][e]);
      }
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], o));
      mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], o));
    }
    float* tm = tm_s(s);
    if (lane == 0) {
      tm[warp * 2 + 0] = mx[0];
      tm[warp * 2 + 1] = mx[1];
    }
    __syncthreads();
    bool refetch[2];
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      float b;
      if (p.tile_m == 32) {
        const int w0 = warp & ~1;
        b = fmaxf(tm[w0 * 2 + kb], tm[(w0 + 1) * 2 + kb]);
        if (p.tile_n == 64) b = fmaxf(b, fmaxf(tm[w0 * 2 + (kb ^ 1)], tm[(w0 + 1) * 2 + (kb ^ 1)]));
      } else {
        b = fmaxf(fmaxf(tm[kb], tm[2 + kb]), fmaxf(tm[4 + kb], tm[6 + kb]));
        if (p.tile_n == 64)
          b = fmaxf(b, fmaxf(fmaxf(tm[kb ^ 1], tm[2 + (kb ^ 1)]), fmaxf(tm[4 + (kb ^ 1)], tm[6 + (kb ^ 1)])));
      }
      refetch[kb] = b < p.tile_thr;
    }
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = a1[nb][e];
        if (refetch[nb >> 2]) v = v + a2[nb][e] * scl;
        sc[nb][e] = v * kLog2e;
      }
  }

  // bias + masks (keys >= N, causal) applied to a score tile.
  SPATTEN_DEV void finish_scores(int s, int n0, float (&sc)[NB][4]) {
    const float* kb = kb_s(s);
    const bool gen_bias = p.bias != nullptr && !per_key_bias;
    const float* bz = gen_bias ? p.bias + (int64_t)z * p.b_sz + (int64_t)h * p.b_sh : nullptr;
    const int shift = p.N - p.M;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = nb * 8 + 2 * t + (e & 1);
        const int key = n0 + col;
        const int row = e < 2 ? row_lo : row_hi;
        float v = sc[nb][e];
        if (per_key_bias) v += kb[col];
        if (gen_bias && key < p.N && row < p.M)
          v += __ldg(bz + (int64_t)row * p.b_sm + (int64_t)key * p.b_sn) * kLog2e;
        if (key >= p.N || (p.causal && key > row + shift)) v = -INFINITY;
        sc[nb][e] = v;
      }
  }

  SPATTEN_DEV void scores(int s, int n0, int kind, bool flo, bool fhi, float (&sc)[NB][4],
                         bool dump = false) {
    if (MODE == kQuant) quant_scores(s, kind, flo, fhi, dump ? n0 : -1, sc);
    else if (MODE == kDense) dense_scores(s, sc);
    else compat_scores(s, n0, sc);
    finish_scores(s, n0, sc);
  }

  // ---- row statistics -------------------------------------------------------
  SPATTEN_DEV void accumulate_stats(const float (&sc)[NB][4], float (&m)[2], float (&l)[2]) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float tmax = -INFINITY;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) tmax = fmaxf(tmax, fmaxf(sc[nb][2 * r], sc[nb][2 * r + 1]));
      const float mn = fmaxf(m[r], tmax);
      if (mn == -INFINITY) continue;
      float sum = 0.f;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
        sum += fast_exp2(sc[nb][2 * r] - mn) + fast_exp2(sc[nb][2 * r + 1] - mn);
      l[r] = l[r] * fast_exp2(m[r] - mn) + sum;
      m[r] = mn;
    }
  }

  SPATTEN_DEV static void quad_combine(float (&m)[2], float (&l)[2]) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m[r], o);
        const float lo = __shfl_xor_sync(0xffffffffu, l[r], o);
        const float mn = fmaxf(m[r], mo);
        if (mn == -INFINITY) continue;
        l[r] = l[r] * fast_exp2(m[r] - mn) + lo * fast_exp2(mo - mn);
        m[r] = mn;
      }
    }
  }

  // One pass over all key tiles computing row statistics of `kind` scores.
  // `active` = this warp computes (warp-uniform); loads are CTA-wide.
  SPATTEN_DEV void stats_pass(int kind, bool plane1, bool active, bool flo, bool fhi, float (&m)[2],
                              float (&l)[2]) {
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
    const int nt = (p.N + BN - 1) / BN;
    load_tile(0, 0, plane1, false);
    for (int j = 0; j < nt; ++j) {
      if (j + 1 < nt) load_tile((j + 1) & 1, (j + 1) * BN, plane1, false);
      else cp_async_commit();
      cp_async_wait<1>();
      __syncthreads();
      if (active || MODE == kCompat) {
        float sc[NB][4];
        scores(j & 1, j * BN, kind, flo, fhi, sc);
        if (active) accumulate_stats(sc, m, l);
      }
      __syncthreads();
    }
    cp_async_wait<0>();
    quad_combine(m, l);
  }

  SPATTEN_DEV void run() {
    float m[2], l[2];
    bool flo = false, fhi = false;
    bool any_cta = false;
    stats_pass(kMsb, MODE == kCompat, true, false, false, m, l);
    if (MODE == kQuant) {
      flo = valid_lo && __frcp_rn(l[0]) < p.refetch_thr;
      fhi = valid_hi && __frcp_rn(l[1]) < p.refetch_thr;
      const bool any_w = __any_sync(0xffffffffu, flo || fhi);
      any_cta = __syncthreads_or(flo || fhi) != 0;
      if (any_cta) {
        float mf[2], lf[2];
        stats_pass(kFull, true, any_w, flo, fhi, mf, lf);
        if (flo) { m[0] = mf[0]; l[0] = lf[0]; }
        if (fhi) { m[1] = mf[1]; l[1] = lf[1]; }
      }
      if (p.refetch_out && t == 0) {
        uint8_t* rf = p.refetch_out + ((int64_t)z * p.H + h) * p.M;
        if (valid_lo) rf[row_lo] = flo;
        if (valid_hi) rf[row_hi] = fhi;
      }
    }
    // ---- pass 2: P, V prune, importance, P.V ----
    int kind = kMsb;
    if (MODE == kQuant) {
      const bool all_w = __all_sync(0xffffffffu, (flo || !valid_lo) && (fhi || !valid_hi));
      const bool any_w = __any_sync(0xffffffffu, flo || fhi);
      kind = all_w ? kFull : (any_w ? kMixed : kMsb);
    }
    const float inv_lo = (m[0] == -INFINITY || !valid_lo) ? 0.f : 1.f / l[0];
    const float inv_hi = (m[1] == -INFINITY || !valid_hi) ? 0.f : 1.f / l[1];
    const float mlo = m[0] == -INFINITY ? 0.f : m[0];
    const float mhi = m[1] == -INFINITY ? 0.f : m[1];
    float o[ND][4];
#pragma unroll
    for (int d = 0; d < ND; ++d)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[d][e] = 0.f;
    const bool want_tok = p.tok_partial != nullptr;
    const bool plane1 = (MODE == kCompat) || (MODE == kQuant && any_cta);
    const int nt = (p.N + BN - 1) / BN;
    float* tokp = want_tok ? p.tok_partial + (((int64_t)z * p.H + h) * p.mtiles + mt) * p.N : nullptr;
    load_tile(0, 0, plane1, true);
    for (int j = 0; j < nt; ++j) {
      const int s = j & 1;
      if (j + 1 < nt) load_tile((j + 1) & 1, (j + 1) * BN, plane1, true);
      else cp_async_commit();
      cp_async_wait<1>();
      __syncthreads();
      float sc[NB][4];
      scores(s, j * BN, kind, flo, fhi, sc, p.score_out != nullptr);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        sc[nb][0] = fast_exp2(sc[nb][0] - mlo) * inv_lo;
        sc[nb][1] = fast_exp2(sc[nb][1] - mlo) * inv_lo;
        sc[nb][2] = fast_exp2(sc[nb][2] - mhi) * inv_hi;
        sc[nb][3] = fast_exp2(sc[nb][3] - mhi) * inv_hi;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (sc[nb][e] < p.v_thr) sc[nb][e] = 0.f;
      }
      if (want_tok) {
        float v[16];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          v[2 * nb] = sc[nb][0] + sc[nb][2];
          v[2 * nb + 1] = sc[nb][1] + sc[nb][3];
        }
        const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float send = b4 ? v[i] : v[8 + i];
          const float keep = b4 ? v[8 + i] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float send = b3 ? v[i] : v[4 + i];
          const float keep = b3 ? v[4 + i] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float send = b2 ? v[i] : v[2 + i];
          const float keep = b2 ? v[2 + i] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        float* cs = cs_s(s) + warp * BN + g * 8 + 2 * t;
        cs[0] = v[0];
        cs[1] = v[1];
      }
      // P.V: A = P (rows x 16 keys), B = V tile via ldmatrix.trans
      const uint8_t* vt = vstage(s);
      const int mi = lane >> 3;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t a[4];
        a[0] = pack2<T>(sc[2 * kk][0], sc[2 * kk][1]);
        a[1] = pack2<T>(sc[2 * kk][2], sc[2 * kk][3]);
        a[2] = pack2<T>(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
        a[3] = pack2<T>(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
        for (int db = 0; db < ND; db += 2) {
          const int r = kk * 16 + (mi & 1) * 8 + (lane & 7);
          const int c = db + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(b0, b1, b2, b3, vt + r * C::kVRowB + swz(r, c, C::kVCpr) * 16);
          mma_16816<T>(o[db], a, b0, b1);
          mma_16816<T>(o[db + 1], a, b2, b3);
        }
      }
      __syncthreads();
      if (want_tok && tid < BN) {
        const int key = j * BN + tid;
        const float* cs = cs_s(s);
        if (key < p.N) tokp[key] = ((cs[tid] + cs[BN + tid]) + cs[2 * BN + tid]) + cs[3 * BN + tid];
      }
    }
    cp_async_wait<0>();
    // ---- epilogue ----
    T* ob = static_cast<T*>(p.out) + (int64_t)z * p.o_sz + (int64_t)hslot * p.o_sh;
    float asum = 0.f;
#pragma unroll
    for (int d = 0; d < ND; ++d) {
      const int col = d * 8 + 2 * t;
      if (valid_lo) {
        if (out_ok)
          *reinterpret_cast<uint32_t*>(ob + (int64_t)row_lo * p.o_sm + col) = pack2<T>(o[d][0], o[d][1]);
        asum += fabsf(o[d][0]) + fabsf(o[d][1]);
      }
      if (valid_hi) {
        if (out_ok)
          *reinterpret_cast<uint32_t*>(ob + (int64_t)row_hi * p.o_sm + col) = pack2<T>(o[d][2], o[d][3]);
        asum += fabsf(o[d][2]) + fabsf(o[d][3]);
      }
    }
    if (p.head_partial) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) asum += __shfl_xor_sync(0xffffffffu, asum, off);
      float* hs = reinterpret_cast<float*>(smem + C::oHs);
      if (lane == 0) hs[warp] = asum;
      __syncthreads();
      if (tid == 0)
        p.head_partial[((int64_t)z * p.H + h) * p.mtiles + mt] = ((hs[0] + hs[1]) + hs[2]) + hs[3];
    }
  }
};

template <int MODE, typename T, int D>
__global__ void __launch_bounds__(kThreads) prog_attn_mma_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  Attn<MODE, T, D> a(p, smem);
  a.run();
}

template <int MODE, typename T, int D>
cudaError_t launch_t(const AttnParams& p, cudaStream_t st) {
  constexpr int smem = Cfg<MODE, T, D>::kSmem;
  auto kern = prog_attn_mma_kernel<MODE, T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)p.mtiles, (unsigned)p.H, (unsigned)p.Z);
  kern<<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <int MODE, typename T>
cudaError_t launch_d(const AttnParams& p, cudaStream_t st) {
  if (p.D == 64) return launch_t<MODE, T, 64>(p, st);
  if (p.D == 128) return launch_t<MODE, T, 128>(p, st);
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t launch_m(const AttnParams& p, cudaStream_t st) {
  switch (p.mode) {
    case kQuant: return launch_d<kQuant, T>(p, st);
    case kDense: return launch_d<kDense, T>(p, st);
    case kCompat: return launch_d<kCompat, T>(p, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_prog_attn_mma(const AttnParams& p, cudaStream_t st) {
  if (p.dtype == kF16) return launch_m<__half>(p, st);
  if (p.dtype == kBF16) return launch_m<__nv_bfloat16>(p, st);
  return cudaErrorInvalidValue;
}

// QUANT and DENSE run on the tcgen05 kernel (fp16/bf16) or the fp32 kernel;
// the reference-compatible float planes (COMPAT) on the warp-level kernel above.
int attn_tile_rows(const AttnParams& p) {
  if (p.mode == kCompat) return BM;
  return p.dtype == kF32 ? f32_tile_rows() : tc_tile_rows();
}

cudaError_t launch_prog_attn(const AttnParams& p, cudaStream_t st, int) {
  if (p.mode == kCompat) return launch_prog_attn_mma(p, st);
  if (p.dtype == kF32) return launch_prog_attn_f32(p, st);
  return launch_prog_attn_tc(p, st);
}

}  // namespace spatten
