// detmath.cuh -- deterministic arithmetic of the decode kernels, operation for operation the
// device twin of oracle/detmath.py (the CPU checker):
//   * BF16 <-> FP32/FP64 conversions with round-to-nearest-even done on the bit patterns;
//   * FP32 sums in specified orders: a product of two BF16 values is exact in FP32, so
//     fmaf(w, x, a) is the rounded a + w*x and a dot product is fixed by the order of its adds
//     alone; the orders (row dot, butterfly, block and lane sums) are written out in
//     oracle/detmath.py and followed here;
//   * det_exp (Cody-Waite reduction + degree-7 Taylor polynomial) and det_log (atanh series),
//     built only from __fmul_rn/__fadd_rn/__fsub_rn/__fdiv_rn, which are never contracted into
//     FMAs, so every intermediate is the IEEE-rounded value the CPU computes too.
// The methods are the published ones named in oracle/detmath.py; the constants are derived
// from the mathematics there (ln 2 split in a 16-bit head and a tail, 1/n!, 1/(2n+1)).
#pragma once
#include <cstdint>
#include <cuda_bf16.h>

namespace mk {

// ---- BF16 bits ----------------------------------------------------------------------------

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// FP32 -> BF16 bits, nearest even (the oracle's bf16(); NaN payloads are not preserved)
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return ((u >> 16) & 0x8000u) | 0x7FC0u;
  u = u + 0x7FFFu + ((u >> 16) & 1u);
  return u >> 16;
}
__device__ __forceinline__ float round_bf16(float x) { return bf16_bits_to_f32(f32_to_bf16_bits(x)); }

// FP64 -> BF16 bits with ONE rounding (nearest even): the oracle's bf16_from_f64
__device__ __forceinline__ uint32_t f64_to_bf16_bits(double x) {
  if (x != x) return 0x7FC0u;
  double ax = fabs(x);
  if (ax < 0x1p-126) {
    double q = rint(x * 0x1p133) * 0x1p-133;
    return __float_as_uint(__double2float_rn(q)) >> 16;
  }
  unsigned long long u = (unsigned long long)__double_as_longlong(x);
  unsigned long long lsb = (u >> 45) & 1ull;
  u = (u + 0xFFFFFFFFFFFull + lsb) & ~0x1FFFFFFFFFFFull;
  float f = __double2float_rn(__longlong_as_double((long long)u));   // exact, or +-inf
  return __float_as_uint(f) >> 16;
}

// ---- BF16 pairs as FP32 -------------------------------------------------------------------

// the BF16 value in the low / high 16 bits of u, as FP32 (exact)
__device__ __forceinline__ float lo_f32(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float hi_f32(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// a0 += lo(w) lo(x), a1 += hi(w) hi(x) for two BF16 pairs, each one FMA with FP32 accumulation
// and BF16 inputs (sm_100's mixed-precision fma): the product of two BF16 values is exact in FP32
// and the FMA rounds once, so each result equals fmaf(f32(w), f32(x), a) bit for bit, without the
// two unpacking instructions per product.
__device__ __forceinline__ void fma_bf16x2(float& a0, float& a1, uint32_t w, uint32_t x) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %2;\n\t"
      "mov.b32 {xl, xh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.bf16 %1, wh, xh, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(w), "r"(x));
}

// a += lo(w) lo(x), then a += hi(w) hi(x): one accumulator, the same mixed-precision FMAs
__device__ __forceinline__ float fma_bf16x2_seq(float a, uint32_t w, uint32_t x) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %1;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.bf16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.bf16 %0, wh, xh, %0;\n\t}"
      : "+f"(a)
      : "r"(w), "r"(x));
  return a;
}
// two rows of a column pair times their BF16 weights: s0 += lo(v0) p0, s1 += hi(v0) p0, then
// s0 += lo(v1) p1, s1 += hi(v1) p1 (p0 / p1 the low / high half of pw)
__device__ __forceinline__ void fma_pv2(float& s0, float& s1, uint32_t v0, uint32_t v1, uint32_t pw) {
  asm("{\n\t.reg .b16 al, ah, bl, bh, p0, p1;\n\t"
      "mov.b32 {al, ah}, %2;\n\t"
      "mov.b32 {bl, bh}, %3;\n\t"
      "mov.b32 {p0, p1}, %4;\n\t"
      "fma.rn.f32.bf16 %0, al, p0, %0;\n\t"
      "fma.rn.f32.bf16 %1, ah, p0, %1;\n\t"
      "fma.rn.f32.bf16 %0, bl, p1, %0;\n\t"
      "fma.rn.f32.bf16 %1, bh, p1, %1;\n\t}"
      : "+f"(s0), "+f"(s1)
      : "r"(v0), "r"(v1), "r"(pw));
}
// ---- FP8 (E4M3) weights -------------------------------------------------------------------
// The FP8 experts multiply E4M3 weights (4 significant bits) by FP16-rounded activations (11): the
// product is exact in FP32, so these FMAs, like the BF16 ones, round only the sums. A BF16
// activation is an FP16 exactly when its magnitude is in [2^-14, 65504]; smaller ones round to
// FP16 subnormals, larger ones saturate at +-65504. (Decoding the codes to BF16 with integer
// operations keeps the BF16 activations unrounded but costs four instructions per two weights
// where the conversion below costs one, and the expert units are issue-bound in this form.)
// two E4M3 codes (low byte: first value) -> FP16 pair (low half: first value), exact
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t q) {
  uint32_t d;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(q));
  return d;
}
// a BF16 pair -> FP16 pair, each rounded to the nearest FP16 (ties to even), finite values beyond
// the FP16 range saturated at +-65504
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
  uint32_t d;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;"
      : "=r"(d)
      : "f"(__uint_as_float(w & 0xFFFF0000u)), "f"(__uint_as_float(w << 16)));
  return d;
}
// a0 += lo(w) lo(x), a1 += hi(w) hi(x) for FP16 pairs, FP32 accumulation
__device__ __forceinline__ void fma_f16x2(float& a0, float& a1, uint32_t w, uint32_t x) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %2;\n\t"
      "mov.b32 {xl, xh}, %3;\n\t"
      "fma.rn.f32.f16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.f16 %1, wh, xh, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(w), "r"(x));
}
// eight E4M3 weights (w: bytes 0..7) against eight FP16 activations (x: halves 0..7): the row
// engine's lane value, even products into a0 and odd ones into a1, then a0 + a1
__device__ __forceinline__ float lane_fp8(uint2 w, uint4 x) {
  float a0 = 0.0f, a1 = 0.0f;
  fma_f16x2(a0, a1, e4m3x2_to_f16x2((uint16_t)(w.x & 0xFFFFu)), x.x);
  fma_f16x2(a0, a1, e4m3x2_to_f16x2((uint16_t)(w.x >> 16)), x.y);
  fma_f16x2(a0, a1, e4m3x2_to_f16x2((uint16_t)(w.y & 0xFFFFu)), x.z);
  fma_f16x2(a0, a1, e4m3x2_to_f16x2((uint16_t)(w.y >> 16)), x.w);
  return __fadd_rn(a0, a1);
}

// one row: s0 += lo(v) p, s1 += hi(v) p (p BF16 bits)
__device__ __forceinline__ void fma_pv1(float& s0, float& s1, uint32_t v, uint16_t p) {
  asm("{\n\t.reg .b16 al, ah;\n\t"
      "mov.b32 {al, ah}, %2;\n\t"
      "fma.rn.f32.bf16 %0, al, %3, %0;\n\t"
      "fma.rn.f32.bf16 %1, ah, %3, %1;\n\t}"
      : "+f"(s0), "+f"(s1)
      : "r"(v), "h"(p));
}

// FP32 butterfly over the warp: every lane ends with the sum, in the order
// a_l <- a_l + a_(l xor o), o = 16, 8, 4, 2, 1 (commutative, so both partners agree)
__device__ __forceinline__ float warp_butterfly(float a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
  return a;
}

// The same butterfly for 8 values per lane at once (one shuffle per pair of values and level
// instead of one per value): lane l ends with the full sum of value v(l) = 4 bit4(l) + 2 bit3(l)
// + bit2(l). Every level adds the same two partial sums as warp_butterfly, own value first, so
// each result is bit-identical to warp_butterfly of that value.
__device__ __forceinline__ float warp_butterfly8(const float (&a)[8], int lane) {
  const bool b4 = (lane & 16) != 0, b3 = (lane & 8) != 0, b2 = (lane & 4) != 0;
  float b[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    b[i] = __fadd_rn(b4 ? a[i + 4] : a[i], __shfl_xor_sync(0xffffffffu, b4 ? a[i] : a[i + 4], 16));
  float q[2];
#pragma unroll
  for (int i = 0; i < 2; ++i)
    q[i] = __fadd_rn(b3 ? b[i + 2] : b[i], __shfl_xor_sync(0xffffffffu, b3 ? b[i] : b[i + 2], 8));
  float d = __fadd_rn(b2 ? q[1] : q[0], __shfl_xor_sync(0xffffffffu, b2 ? q[0] : q[1], 4));
  d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 2));
  return __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 1));
}
__device__ __forceinline__ int butterfly8_value(int lane) { return ((lane >> 2) & 1) | ((lane >> 2) & 2) | ((lane >> 2) & 4); }

// ---- det_exp / det_log / silu -------------------------------------------------------------

// FP32 bit patterns of log2(e), of ln2 = LN2_HI + LN2_LO with LN2_HI = 45426/65536 (16 significant
// bits, so k * LN2_HI is exact for |k| < 256), of 1/n! and 1/(2n+1) and of sqrt(2), each the
// nearest FP32 to the mathematical value (the oracle derives the same values in Python).
#define MK_LOG2E __uint_as_float(1069066811u)
#define MK_LN2_HI __uint_as_float(1060205056u)
#define MK_LN2_LO __uint_as_float(901758606u)

__device__ __forceinline__ float det_exp(float x) {
  if (x != x) return x;
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) return __uint_as_float(0x7F800000u);
  const float k = rintf(__fmul_rn(x, MK_LOG2E));
  const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(k, MK_LN2_HI)), __fmul_rn(k, MK_LN2_LO));
  // Taylor coefficients 1/n!, n = 7..0, each rounded to FP32
  float p = __uint_as_float(961547521u);                                  // 1/5040
  p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(985008993u));   // 1/720
  p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(1007192201u));  // 1/120
  p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(1026206379u));  // 1/24
  p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(1042983595u));  // 1/6
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  const float scale = __int_as_float(((int)k + 127) << 23);
  return __fmul_rn(p, scale);
}

__device__ __forceinline__ float det_log(float x) {
  if (x != x || x < 0.0f) return __uint_as_float(0x7FC00000u);
  if (x == 0.0f) return __uint_as_float(0xFF800000u);
  if (x == __uint_as_float(0x7F800000u)) return x;
  int esub = 0;
  if (x < 0x1p-126f) { x = __fmul_rn(x, 0x1p24f); esub = 24; }
  const uint32_t bits = __float_as_uint(x);
  int e = (int)(bits >> 23) - 127 - esub;
  float m = __uint_as_float((bits & 0x7FFFFFu) | 0x3F800000u);
  if (m > __uint_as_float(1068827891u)) { m = __fmul_rn(m, 0.5f); e += 1; }   // FP32(sqrt 2)
  const float t = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  const float t2 = __fmul_rn(t, t);
  // atanh series coefficients 1/9, 1/7, 1/5, 1/3, 1, each rounded to FP32
  float s = __uint_as_float(1038323257u);                                 // 1/9
  s = __fadd_rn(__fmul_rn(s, t2), __uint_as_float(1041385765u));  // 1/7
  s = __fadd_rn(__fmul_rn(s, t2), __uint_as_float(1045220557u));  // 1/5
  s = __fadd_rn(__fmul_rn(s, t2), __uint_as_float(1051372203u));  // 1/3
  s = __fadd_rn(__fmul_rn(s, t2), 1.0f);
  const float logm = __fmul_rn(__fadd_rn(t, t), s);
  const float ef = (float)e;
  return __fadd_rn(__fmul_rn(ef, MK_LN2_HI), __fadd_rn(__fmul_rn(ef, MK_LN2_LO), logm));
}

__device__ __forceinline__ float det_silu(float x) {
  return __fdiv_rn(x, __fadd_rn(1.0f, det_exp(-x)));
}

}  // namespace mk
