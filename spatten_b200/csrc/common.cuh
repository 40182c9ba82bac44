// Shared device helpers for the SpAtten B200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define SPATTEN_DEV __device__ __forceinline__

namespace spatten {

// dtype codes shared with include/spatten_b200.h
enum DType : int { kF16 = 0, kBF16 = 1, kF32 = 2 };

constexpr float kLog2e = 1.4426950408889634f;

SPATTEN_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte asynchronous global->shared copy; `valid` = false zero-fills.
SPATTEN_DEV void cp_async16(void* smem, const void* gmem, bool valid) {
  int src_bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(src_bytes));
}
// 4-byte asynchronous global->shared copy (through L1); `valid` = false zero-fills.
SPATTEN_DEV void cp_async4(void* smem, const void* gmem, bool valid) {
  int src_bytes = valid ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(src_bytes));
}
SPATTEN_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
SPATTEN_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

SPATTEN_DEV void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                             const void* smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(smem_row)));
}
SPATTEN_DEV void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                   const void* smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(smem_row)));
}

// D = A(16x32 s8) * B(32x8 s8) + C, int32 accumulate.
SPATTEN_DEV void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D = A(16x16) * B(16x8) + C, fp32 accumulate; T = half or bf16.
template <typename T>
SPATTEN_DEV void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
SPATTEN_DEV void mma_16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
SPATTEN_DEV void mma_16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
SPATTEN_DEV uint32_t pack2(float lo, float hi);
template <>
SPATTEN_DEV uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
SPATTEN_DEV uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
SPATTEN_DEV float to_f32(T x);
template <>
SPATTEN_DEV float to_f32<__half>(__half x) { return __half2float(x); }
template <>
SPATTEN_DEV float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
SPATTEN_DEV float to_f32<float>(float x) { return x; }

template <typename T>
SPATTEN_DEV T from_f32(float x);
template <>
SPATTEN_DEV __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
SPATTEN_DEV __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
SPATTEN_DEV float from_f32<float>(float x) { return x; }

SPATTEN_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// x / sc rounded to the nearest integer (ties to even), bit for bit what
// rint(__fdiv_rn(x, sc)) gives, for |x| <= 127 * sc: x * (1 / sc) is within
// 2 ulp of x / sc, so its rounding can only differ when it lies within a few
// ulp of a half-integer; those rare values take the exact division.
// y rounded to the nearest integer, ties to even, for |y| < 2^22 (other
// inputs give garbage, which the callers' tie test sends to the exact path):
// y + 1.5 * 2^23 lands in [2^23, 2^24), where the spacing of floats is 1,
// so the round-to-nearest addition leaves rint(y) in the low mantissa bits.
// FMA-pipe adds instead of the conversion pipe's round + float-to-int.
SPATTEN_DEV int rint_small(float y, float& ti) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const float f = __fadd_rn(y, kRound);
  ti = __fsub_rn(f, kRound);
  return __float_as_int(f) - 0x4B400000;
}

SPATTEN_DEV int quant_div(float x, float sc, float rc) {
  const float y = x * rc;
  const float t = rintf(y);
  if (!(fabsf(y - t) <= 0.49990f)) return __float2int_rn(__fdiv_rn(x, sc));  // also NaN / inf (denormal sc)
  return (int)t;
}

// The same result with the rounding on the FMA pipe (rint_small), for
// kernels that quantise every value through this call; it holds a few more
// registers, so the kernels that call quant_div only on the rare near-tie
// path keep the version above.
SPATTEN_DEV int quant_div_fadd(float x, float sc, float rc) {
  const float y = x * rc;
  float t;
  const int n = rint_small(y, t);
  if (!(fabsf(y - t) <= 0.49990f)) return __float2int_rn(__fdiv_rn(x, sc));  // also NaN / inf (denormal sc)
  return n;
}

// a / 127 rounded to nearest even (the quantisation scale max|x| / 127), for
// finite a >= 0, by Markstein's correction step (P. Markstein, "Computation
// of elementary functions on the IBM RISC System/6000 processor", 1990):
// with y = RN(1/127) and q = RN(a * y), the remainder a - 127 q is exact in
// one FMA and RN(q + remainder * y) is the correctly rounded quotient.
// Below 2^-100 (where q could be subnormal) the IEEE division is used.
SPATTEN_DEV float div127_rn(float a) {
  if (a < 7.8886091e-31f) return __fdiv_rn(a, 127.0f);
  constexpr float y = 1.0f / 127.0f;
  const float q = a * y;
  const float r = fmaf(-q, 127.0f, a);
  return fmaf(r, y, q);
}

// 1 / s to within an ulp (ex2-style approximation instruction); quant_div
// only needs its product with x within ~1e-4 of x / s.
SPATTEN_DEV float rcp_approx(float s) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(s));
  return r;
}

// Order-preserving map float -> uint32 (larger float -> larger key).
SPATTEN_DEV uint32_t float_order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace spatten
