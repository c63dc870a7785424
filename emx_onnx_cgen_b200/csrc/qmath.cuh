// Requantisation arithmetic of QLinearConv / QLinearAdd, bit-exact with the
// reference's generated C (templates/qlinear_conv_op.c.j2:34-38,
// qlinear_add_op.c.j2:11-17; gcc on x86-64: every float operation rounded on
// its own, no FMA contraction).
//
// Two forms of each:
//  * *_exact: the reference expression one rounding at a time
//    (__fmul_rn/__fadd_rn/__fdiv_rn, rintf, fmaxf/fminf).
//  * *_fast:  the same result with full-rate FP32 instructions only, used in
//    the tensor-core epilogue where conversion-pipe instructions (I2F/F2I/FRND
//    run at 1/8 of the FP32 rate) would otherwise bound the kernel:
//      - round-half-even to an integer: t = (v + 1.5*2^23) - 1.5*2^23 is
//        exactly rintf(v) for |v| < 2^22; beyond that the value saturates in
//        the clamp that follows (worked through in the comment of requant_fast);
//      - float -> byte: for an integer-valued r in [-128, 255], the low byte of
//        the bit pattern of (r + 1.5*2^23) is r (two's complement for r < 0);
//      - small int -> float: bits(k + 0x4B400000) - 1.5*2^23 is exactly k for
//        |k| < 2^22;
//      - QLinearAdd's division by the output scale: quotient q0 = s*(1/ys)
//        refined once with the exact remainder, e = fma(-q0, ys, s),
//        q = fma(e, 1/ys, q0) (Markstein's reciprocal refinement).  That
//        refinement is correctly rounded in almost all cases but not proven
//        for every operand, so the runtime checks it against __fdiv_rn for all
//        65536 operand pairs of each fused add when the plan is loaded and
//        keeps the exact division if a single pair differs.
#pragma once
#include <stdint.h>

namespace emx {

constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
constexpr int kMagicBits = 0x4B400000;

__device__ __forceinline__ int load_8bit(uint32_t byte, bool is_signed) {
  return is_signed ? (int)(int8_t)(uint8_t)byte : (int)(uint8_t)byte;
}

// ---------------------------------------------------------------- exact forms
__device__ __forceinline__ int requant_exact(int32_t acc, float scale, float zero, bool is_signed) {
  float v = __fmul_rn(__int2float_rn(acc), scale);
  float r = __fadd_rn(rintf(v), zero);
  r = fmaxf(r, is_signed ? -128.0f : 0.0f);
  r = fminf(r, is_signed ? 127.0f : 255.0f);
  return (int)r;
}

__device__ __forceinline__ int qadd_exact(int a, int za, float sa, int b, int zb, float sb, float ys, float yz,
                                          bool is_signed) {
  float ar = __fmul_rn(__int2float_rn(a - za), sa);
  float br = __fmul_rn(__int2float_rn(b - zb), sb);
  float s = __fadd_rn(__fdiv_rn(__fadd_rn(ar, br), ys), yz);
  float r = rintf(s);
  r = fmaxf(r, is_signed ? -128.0f : 0.0f);
  r = fminf(r, is_signed ? 127.0f : 255.0f);
  return (int)r;
}

// ---------------------------------------------------------------- fast forms
__device__ __forceinline__ float small_int_to_float(int k) {  // exact for |k| < 2^22
  return __fsub_rn(__int_as_float(k + kMagicBits), kMagic);
}

__device__ __forceinline__ uint32_t float_to_byte(float r) {  // r integer-valued in [-128, 255]
  return (uint32_t)__float_as_int(__fadd_rn(r, kMagic)) & 0xFFu;
}

// Returns the requantised value as an integer-valued float already clamped to
// the output range.  (v + M) - (M - zy) equals rint(v) + zy exactly when
// |v| < 2^22 (both steps exact: an integer below 2^24 minus an integer).  For
// |v| >= 2^22 the result stays within a few units of v + zy, so it is still
// far outside [-128, 255] and the clamp produces what the reference's clamp
// produces; NaN and +-inf go through fmaxf/fminf exactly like the reference's.
__device__ __forceinline__ float requant_fast(int32_t acc, float scale, float m_minus_zero, float lo, float hi) {
  const float v = __fmul_rn(__int2float_rn(acc), scale);
  float r = __fsub_rn(__fadd_rn(v, kMagic), m_minus_zero);
  r = fmaxf(r, lo);
  return fminf(r, hi);
}

// Integer form of requant_fast for |(float)acc * scale| < 2^21 (planner-proved,
// QC_RQ_INT): adding 1.5 * 2^23 rounds v half-to-even to an integer k exactly
// (the sum stays in [2^23, 2^24), where the float spacing is 1, and 1.5 * 2^23
// is even), and the bit pattern of that sum is kMagicBits + k; subtracting
// rq_sub = kMagicBits - zero leaves k + zero, the reference's rint(v) + zy, as
// an int32 that pack_sat_u8x4 clamps to the output range.
__device__ __forceinline__ int requant_int(int32_t acc, float scale, int rq_sub) {
  const float v = __fmul_rn(__int2float_rn(acc), scale);
  return __float_as_int(__fadd_rn(v, kMagic)) - rq_sub;
}

// Four int32 values saturated to [0, 255] and packed little-endian (y0 in the
// low byte): two cvt.pack.sat, each converting two values with saturation.
__device__ __forceinline__ uint32_t pack_sat_u8x4(int y0, int y1, int y2, int y3) {
  uint32_t hi, w;
  asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(y3), "r"(y2), "r"(0));
  asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(y1), "r"(y0), "r"(hi));
  return w;
}

// Stores with the state space stated: the output pointers come from a table
// indexed at run time, where the compiler cannot see that they are global.
__device__ __forceinline__ void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(__cvta_generic_to_global(p)), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ void st_global_v2(void* p, uint32_t a, uint32_t b) {
  asm volatile("st.global.v2.b32 [%0], {%1, %2};" ::"l"(__cvta_generic_to_global(p)), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void st_global_u8(void* p, uint32_t v) {
  asm volatile("st.global.u8 [%0], %1;" ::"l"(__cvta_generic_to_global(p)), "r"(v) : "memory");
}

__device__ __forceinline__ float div_refined(float s, float ys, float inv_ys) {
  const float q0 = __fmul_rn(s, inv_ys);
  const float e = __fmaf_rn(-q0, ys, s);
  return __fmaf_rn(e, inv_ys, q0);
}

template <bool FAST_DIV>
__device__ __forceinline__ float qadd_fast(float conv_val, float c_zero, float cs, int r, float r_zero_f, float rs,
                                           float ys, float inv_ys, float yz, float lo, float hi) {
  const float ar = __fmul_rn(__fsub_rn(conv_val, c_zero), cs);  // conv_val, c_zero: small integers, exact
  const float br = __fmul_rn(__fsub_rn(small_int_to_float(r), r_zero_f), rs);
  const float s = __fadd_rn(ar, br);
  const float q = FAST_DIV ? div_refined(s, ys, inv_ys) : __fdiv_rn(s, ys);
  float t = __fadd_rn(q, yz);
  t = __fsub_rn(__fadd_rn(t, kMagic), kMagic);  // rint, |t| < 2^22; beyond that the clamp decides
  t = fmaxf(t, lo);
  return fminf(t, hi);
}

}  // namespace emx
