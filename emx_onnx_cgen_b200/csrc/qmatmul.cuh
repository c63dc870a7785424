// QLinearMatMul / MatMulInteger arithmetic shared by the CUDA-core kernel
// (misc_ops.cu) and the tensor-core kernel (qgemm.cu); reference
// templates/qlinear_matmul_op.c.j2:1-81, matmul_integer_op.c.j2.
#pragma once
#include <stdint.h>

namespace emx {

struct QMatMulParams {
  const uint8_t* a;
  const uint8_t* b;
  void* y;
  int64_t m;
  int k, n, a_signed, b_signed, za, zb;
  // requantisation (QLinearMatMul only)
  int quantized, use_int, frac_bits, zy, y_signed;
  int64_t mult;
  float scale;
};

// The int32 sum sum_k (a - za)(b - zb) requantised to the output byte: the
// integer form (acc * multiplier, shift with round-half-even) when the host
// found the double multiplier exact in frac_bits fractional bits, else
// llrint((double)acc * (double)scale + zy); then the clamp.
__device__ __forceinline__ uint8_t qm_clamp_byte(int64_t q, const QMatMulParams& p) {
  const int64_t lo = p.y_signed ? -128 : 0, hi = p.y_signed ? 127 : 255;
  q = q < lo ? lo : (q > hi ? hi : q);
  return (uint8_t)q;
}

__device__ __forceinline__ uint8_t qm_requant_int(int32_t acc, const QMatMulParams& p) {
  int64_t r = (int64_t)acc * p.mult;
  if (p.frac_bits > 0) {
    const uint64_t mag = r < 0 ? (uint64_t)(-r) : (uint64_t)r;
    uint64_t quo = mag >> p.frac_bits;
    const uint64_t rem = mag & ((1ull << p.frac_bits) - 1ull), half = 1ull << (p.frac_bits - 1);
    if (rem > half || (rem == half && (quo & 1ull))) ++quo;
    r = r < 0 ? -(int64_t)quo : (int64_t)quo;
  }
  return qm_clamp_byte(r + (int64_t)p.zy, p);
}

__device__ __forceinline__ uint8_t qm_requant_double(int32_t acc, const QMatMulParams& p) {
  return qm_clamp_byte(__double2ll_rn(__dadd_rn(__dmul_rn((double)acc, (double)p.scale), (double)p.zy)), p);
}

__device__ __forceinline__ uint8_t qm_requant(int32_t acc, const QMatMulParams& p) {
  return p.use_int ? qm_requant_int(acc, p) : qm_requant_double(acc, p);
}

}  // namespace emx
