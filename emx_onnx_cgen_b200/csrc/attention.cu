// ONNX Attention (opset 23), fp16, in the reference's own arithmetic.
//
// Reference (src/emx_onnx_cgen/templates/attention_op.c.j2:47-188, c_type
// _Float16, gcc on x86-64: every _Float16 expression is evaluated in float
// and rounded to _Float16 when stored), per (b, h, qi):
//   score = 0; for d: score = r16(score + q*k)        (float add, then fp16)
//   score = r16(score * scale);  score_bias = r16(score + bias)
//   bias = -inf where is_causal and ki > qi + past, else 0
//   max = fmax chain from -inf
//   w[ki] = max != -inf ? r16(exp((double)r16(score_bias - max))) : 0
//   sum = r16(sum + w) over ki ascending;  inv = sum == 0 ? 0 : r16(1.0f / sum)
//   out[vd] = acc, acc = r16(acc + r16(w * inv) * v) over ki ascending
// where r16 rounds a float to fp16 (round to nearest even) and products of
// two fp16 values are exact in float.  This kernel repeats exactly these
// operations (float adds/multiplies with explicit rounding, cvt to fp16 and
// back), so its output is bit-identical to the reference's.  exp runs as a
// guarded float evaluation with a double fallback near fp16 rounding
// boundaries (see exp_f16_ref).
//
// Masked keys.  Under is_causal a masked score is -inf, its weight exp(-inf)
// = +0, and it leaves max, sum and (barring a -0 accumulator) every output
// unchanged -- provided no score is +inf or NaN and no V value is inf or NaN.
// A pre-pass checks Q, K, V for that (all finite, and D * max|q| * max|k|
// small enough that no partial score can overflow fp16); when it holds the
// kernel skips masked keys entirely (half the work), otherwise it evaluates
// every key with the mask arithmetic of the reference.
//
// Two kernels, the same arithmetic.  attention_exact2_kernel (head sizes D a
// multiple of 8 and DV a multiple of 4 up to 128, 16-byte aligned rows): one
// CTA of 256 threads per (q block of 16 rows, head, batch); each thread runs
// 8 chains at once (2 rows x 4 keys for the scores, 2 rows x 4 output
// channels for the outputs), its operands read from transposed tiles by one
// broadcast and one 8-byte shared-memory load per step; a step of a chain is
// a mixed-precision fma (fp16 operands, fp32 result -- the fp16 product is
// exact, so it equals the reference's float multiply and add) and half of a
// packed round to fp16.  attention_exact_kernel covers every other shape
// (64-key tiles, 8 chains per thread of 128, one fp16 operand load per step).
// Both: the row maxima, weights, per-row sequential sums and scaled weights in
// shared memory between the two phases; heaviest q blocks (last rows, most
// keys) first.
#include <cuda_fp16.h>

#include <algorithm>

#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

constexpr int AT_QB = 16;    // query rows per CTA
constexpr int AT_KT = 64;    // keys per K / V tile
constexpr int AT_THREADS = 128;

struct AttnParams {
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  uint16_t* o;
  int64_t q_sb, q_sh, q_st, k_sb, k_sh, k_st, v_sb, v_sh, v_st, o_sb, o_sh, o_st;
  int B, HQ, group, TQ, TK, past, D, DV, causal, scn;
  float scale;          // fp16 scale value
  const uint32_t* stats;  // [0] max|q| bits, [1] max|k| bits, [2] non-finite seen
  int* err;
};

__device__ __forceinline__ float h2f(uint16_t h) {
  float r;
  asm("cvt.f32.f16 %0, %1;" : "=f"(r) : "h"(h));
  return r;
}
__device__ __forceinline__ uint16_t f2h(float f) {
  uint16_t r;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(r) : "f"(f));
  return r;
}
__device__ __forceinline__ float r16(float f) { return h2f(f2h(f)); }
// RN32(a * b + c) for fp16 a, b (their product is exact in fp32)
__device__ __forceinline__ float fma_h(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
// RN16(a + b) for fp16 a, b, one rounding.  Equal to the reference's
// RN16(RN32(a + b)): when the exponents of a and b differ by at most 12 the
// sum has at most 24 significant bits and RN32 is exact; otherwise the smaller
// operand is below a quarter of the larger one's fp16 ulp, both roundings
// return the larger operand, and RN32 cannot land on an fp16 rounding
// midpoint (the largest such fp16 operand stays more than half an fp32 ulp
// away from it).
__device__ __forceinline__ uint16_t add_hh(uint16_t a, uint16_t b) {
  uint16_t d;
  asm("add.rn.f16 %0, %1, %2;" : "=h"(d) : "h"(a), "h"(b));
  return d;
}
// two floats rounded to fp16 (nearest even), packed: lo in bits 0-15
__device__ __forceinline__ uint32_t pack_r16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
constexpr uint16_t kHalfOne = 0x3C00u;
__device__ __forceinline__ uint16_t d2h(double v) {
  uint16_t r;
  asm("cvt.rn.f16.f64 %0, %1;" : "=h"(r) : "d"(v));
  return r;
}

// fp16(exp((double)a)) for an fp16 value a: float expf (documented <= 2 ulp)
// widened by a 2^-20 relative margin; if both ends round to the same fp16 it
// is the correctly rounded result, else the double evaluation decides.
__device__ __forceinline__ uint16_t exp_f16_ref(float a) {
  const float e = expf(a);
  const uint16_t lo = f2h(__fmul_rn(e, 1.0f - 0x1p-20f));
  const uint16_t hi = f2h(__fmul_rn(e, 1.0f + 0x1p-20f));
  if (lo == hi && !isnan(e)) return lo;
  return d2h(exp((double)a));
}

__global__ void attn_stats_reset_kernel(uint32_t* stats) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x < 4) stats[threadIdx.x] = 0;
}

// max |x| (as bits of a non-negative fp16) and a non-finite flag over n fp16 values
__global__ void attn_stats_kernel(const uint16_t* __restrict__ q, int64_t nq, const uint16_t* __restrict__ k,
                                  int64_t nk, const uint16_t* __restrict__ v, int64_t nv, uint32_t* stats) {
  pdl_wait();
  pdl_launch_dependents();
  uint32_t mq = 0, mk = 0, bad = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nq; i += stride) {
    const uint32_t a = q[i] & 0x7FFFu;
    mq = max(mq, a);
    bad |= a >= 0x7C00u;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nk; i += stride) {
    const uint32_t a = k[i] & 0x7FFFu;
    mk = max(mk, a);
    bad |= a >= 0x7C00u;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += stride)
    bad |= (v[i] & 0x7FFFu) >= 0x7C00u;
  for (int o = 16; o > 0; o >>= 1) {
    mq = max(mq, __shfl_xor_sync(0xffffffffu, mq, o));
    mk = max(mk, __shfl_xor_sync(0xffffffffu, mk, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if ((threadIdx.x & 31) == 0) {
    if (mq) atomicMax(&stats[0], mq);
    if (mk) atomicMax(&stats[1], mk);
    if (bad) atomicOr(&stats[2], 1u);
  }
}

__global__ void __launch_bounds__(AT_THREADS) attention_exact_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint8_t at_smem[];
  uint16_t* qs = reinterpret_cast<uint16_t*>(at_smem);        // [QB][D]
  uint16_t* kt = qs + AT_QB * p.D;                              // [D][KT]
  uint16_t* vt = kt + p.D * AT_KT;                              // [KT][DV]
  uint16_t* sc = vt + AT_KT * p.DV;                             // [QB][scn]
  float* rowmax = reinterpret_cast<float*>(sc + (size_t)AT_QB * p.scn);
  float* rowinv = rowmax + AT_QB;

  const int qblk = gridDim.x - 1 - blockIdx.x;  // heaviest (last) rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / p.group;
  const int q0 = qblk * AT_QB;
  const int tid = threadIdx.x;
  const uint16_t* qg = p.q + b * p.q_sb + h * p.q_sh;
  const uint16_t* kg = p.k + b * p.k_sb + kvh * p.k_sh;
  const uint16_t* vg = p.v + b * p.v_sb + kvh * p.v_sh;

  pdl_wait();
  pdl_launch_dependents();
  // masked keys may be skipped only when every score is finite (see header)
  bool fast = false;
  if (p.causal && p.stats[2] == 0) {
    const float mq = h2f((uint16_t)p.stats[0]), mk = h2f((uint16_t)p.stats[1]);
    fast = (float)p.D * mq * mk * 1.3f * fmaxf(1.0f, fabsf(p.scale)) < 60000.0f;
  }
  auto row_end = [&](int r) -> int {  // keys row r must visit
    const int qi = q0 + r;
    if (fast) return min(p.TK, qi + p.past + 1);
    return p.TK;
  };
  const int last_row = min(AT_QB, p.TQ - q0) - 1;
  const int kend_blk = row_end(last_row);

  for (int i = tid; i < AT_QB * p.D; i += AT_THREADS) {
    const int r = i / p.D, d = i - r * p.D;
    qs[i] = q0 + r < p.TQ ? qg[(int64_t)(q0 + r) * p.q_st + d] : 0;
  }

  // ---- phase 1: scores (8 chains per thread: key kk, rows rs, rs+2, ..., rs+14)
  const int kk = tid & (AT_KT - 1), rs = tid >> 6;
  for (int k0 = 0; k0 < kend_blk; k0 += AT_KT) {
    __syncthreads();
    // transpose into [d][key]: key fastest, so the shared-memory stores do not collide
    for (int i = tid; i < AT_KT * p.D; i += AT_THREADS) {
      const int key = i % AT_KT, d = i / AT_KT;
      kt[d * AT_KT + key] = k0 + key < p.TK ? kg[(int64_t)(k0 + key) * p.k_st + d] : 0;
    }
    __syncthreads();
    const int key = k0 + kk;
    float s[AT_QB / 2];
#pragma unroll
    for (int j = 0; j < AT_QB / 2; ++j) s[j] = 0.0f;
    for (int d = 0; d < p.D; ++d) {
      const float kf = h2f(kt[d * AT_KT + kk]);
#pragma unroll
      for (int j = 0; j < AT_QB / 2; ++j) s[j] = r16(__fadd_rn(s[j], __fmul_rn(h2f(qs[(rs + 2 * j) * p.D + d]), kf)));
    }
#pragma unroll
    for (int j = 0; j < AT_QB / 2; ++j) {
      const int r = rs + 2 * j;
      if (key >= row_end(r) || q0 + r >= p.TQ) continue;
      const float sv = r16(__fmul_rn(s[j], p.scale));
      const bool masked = p.causal && key > q0 + r + p.past;
      sc[r * p.scn + key] = f2h(__fadd_rn(sv, masked ? -INFINITY : 0.0f));
    }
  }
  __syncthreads();

  // ---- row maxima (fmax chain from -inf; NaN-ignoring and order-free)
  const int warp = tid >> 5, lane = tid & 31;
  for (int r = warp; r < AT_QB; r += AT_THREADS / 32) {
    float m = -INFINITY;
    if (q0 + r < p.TQ)
      for (int key = lane; key < row_end(r); key += 32) m = fmaxf(m, h2f(sc[r * p.scn + key]));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) rowmax[r] = m;
  }
  __syncthreads();
  // ---- weights
  for (int r = warp; r < AT_QB; r += AT_THREADS / 32) {
    if (q0 + r >= p.TQ) continue;
    const float m = rowmax[r];
    for (int key = lane; key < row_end(r); key += 32) {
      uint16_t w = 0;
      if (m != -INFINITY) w = exp_f16_ref(r16(__fsub_rn(h2f(sc[r * p.scn + key]), m)));
      sc[r * p.scn + key] = w;
    }
  }
  __syncthreads();
  // ---- sequential sums and reciprocals, one thread per row
  if (tid < AT_QB && q0 + tid < p.TQ) {
    uint16_t sum = 0;  // fp16 +0
    const int e = row_end(tid);
    for (int key = 0; key < e; ++key) sum = add_hh(sum, sc[tid * p.scn + key]);
    const float sf = h2f(sum);
    rowinv[tid] = sf == 0.0f ? 0.0f : r16(__fdiv_rn(1.0f, sf));
  }
  __syncthreads();
  // ---- scaled weights r16(w * inv)
  for (int r = warp; r < AT_QB; r += AT_THREADS / 32) {
    if (q0 + r >= p.TQ) continue;
    const float inv = rowinv[r];
    for (int key = lane; key < row_end(r); key += 32)
      sc[r * p.scn + key] = f2h(__fmul_rn(h2f(sc[r * p.scn + key]), inv));
  }

  // ---- phase 2: outputs (chains for vd pair vp, rows rs, rs+2, ...)
  const int vp = tid & 63;
  const bool vd_ok = 2 * vp < p.DV;
  float acc[AT_QB / 2][2];
#pragma unroll
  for (int j = 0; j < AT_QB / 2; ++j) acc[j][0] = acc[j][1] = 0.0f;
  for (int k0 = 0; k0 < kend_blk; k0 += AT_KT) {
    __syncthreads();
    for (int i = tid; i < AT_KT * p.DV; i += AT_THREADS) {
      const int key = i / p.DV, d = i - key * p.DV;
      vt[i] = k0 + key < p.TK ? vg[(int64_t)(k0 + key) * p.v_st + d] : 0;
    }
    __syncthreads();
    if (!vd_ok) continue;
    const int kn = min(AT_KT, kend_blk - k0);
    for (int kk2 = 0; kk2 < kn; ++kk2) {
      const int key = k0 + kk2;
      const uint32_t v2 = *reinterpret_cast<const uint32_t*>(&vt[kk2 * p.DV + 2 * vp]);
      const float v0 = h2f((uint16_t)v2), v1 = h2f((uint16_t)(v2 >> 16));
#pragma unroll
      for (int j = 0; j < AT_QB / 2; ++j) {
        const int r = rs + 2 * j;
        if (key >= row_end(r)) continue;
        const float w = h2f(sc[r * p.scn + key]);
        acc[j][0] = r16(__fadd_rn(acc[j][0], __fmul_rn(w, v0)));
        acc[j][1] = r16(__fadd_rn(acc[j][1], __fmul_rn(w, v1)));
      }
    }
  }
  if (!vd_ok) return;
#pragma unroll
  for (int j = 0; j < AT_QB / 2; ++j) {
    const int r = rs + 2 * j;
    const int qi = q0 + r;
    if (qi >= p.TQ) continue;
    if (fast) {
      // skipped keys each add r16(+0 * v) = +-0: it matters only to a -0 accumulator
      for (int c = 0; c < 2; ++c) {
        if (__float_as_uint(acc[j][c]) != 0x80000000u) continue;
        for (int key = row_end(r); key < p.TK; ++key)
          acc[j][c] = r16(__fadd_rn(acc[j][c], __fmul_rn(0.0f, h2f(vg[(int64_t)key * p.v_st + 2 * vp + c]))));
      }
    }
    uint16_t* og = p.o + b * p.o_sb + h * p.o_sh + (int64_t)qi * p.o_st + 2 * vp;
    og[0] = f2h(acc[j][0]);
    if (2 * vp + 1 < p.DV) og[1] = f2h(acc[j][1]);
  }
}


// ------------------------------------------------------------------ exact2
constexpr int AE_QB = 16;      // query rows per CTA
constexpr int AE_KT = 128;     // keys per K / V tile
constexpr int AE_THREADS = 256;

__global__ void __launch_bounds__(AE_THREADS, 2) attention_exact2_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint8_t ae_smem[];
  uint16_t* qT = reinterpret_cast<uint16_t*>(ae_smem);       // [D][QB]
  uint16_t* kv = qT + p.D * AE_QB;                            // K tile [D][KT], later V tile [KT][DV]
  uint16_t* sc = kv + max(p.D * AE_KT, AE_KT * p.DV);         // [scn][QB]: key-major
  float* rowmax = reinterpret_cast<float*>(sc + (size_t)p.scn * AE_QB);
  float* rowinv = rowmax + AE_QB;
  float* red = rowinv + AE_QB;  // [AE_THREADS / 32][QB] partial maxima

  const int qblk = gridDim.x - 1 - blockIdx.x;  // heaviest (last) rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / p.group;
  const int q0 = qblk * AE_QB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint16_t* qg = p.q + b * p.q_sb + h * p.q_sh;
  const uint16_t* kg = p.k + b * p.k_sb + kvh * p.k_sh;
  const uint16_t* vg = p.v + b * p.v_sb + kvh * p.v_sh;

  pdl_wait();
  pdl_launch_dependents();
  // masked keys may be skipped only when every score is finite (see header)
  bool fast = false;
  if (p.causal && p.stats[2] == 0) {
    const float mq = h2f((uint16_t)p.stats[0]), mk = h2f((uint16_t)p.stats[1]);
    fast = (float)p.D * mq * mk * 1.3f * fmaxf(1.0f, fabsf(p.scale)) < 60000.0f;
  }
  auto row_end = [&](int r) -> int {  // keys row r must visit
    if (fast) return min(p.TK, q0 + r + p.past + 1);
    return p.TK;
  };
  const int rows = min(AE_QB, p.TQ - q0);
  const int kend_blk = row_end(rows - 1);

  for (int i = tid; i < AE_QB * p.D; i += AE_THREADS) {  // Q block transposed: [d][row]
    const int r = i % AE_QB, d = i / AE_QB;
    qT[i] = r < rows ? qg[(int64_t)(q0 + r) * p.q_st + d] : 0;
  }

  // ---- scores: thread = (row pair rp, key quad kq); chains (rows 2rp, 2rp+1) x (keys 4kq .. 4kq+3)
  const int rp = tid >> 5, kq = lane;
  const int r0 = 2 * rp;
  for (int k0 = 0; k0 < kend_blk; k0 += AE_KT) {
    __syncthreads();
    // K tile transposed into [d][key]: a thread takes 8 consecutive d of one key
    // (one 16-byte load); for each d the warp writes 32 consecutive keys
    for (int i = tid; i < AE_KT * (p.D / 8); i += AE_THREADS) {
      const int key = i % AE_KT, d8 = i / AE_KT;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (k0 + key < p.TK) w = *reinterpret_cast<const uint4*>(kg + (int64_t)(k0 + key) * p.k_st + 8 * d8);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kv[(8 * d8 + 2 * j) * AE_KT + key] = (uint16_t)ww[j];
        kv[(8 * d8 + 2 * j + 1) * AE_KT + key] = (uint16_t)(ww[j] >> 16);
      }
    }
    __syncthreads();
    if (k0 + 4 * kq >= kend_blk) continue;  // every chain of this thread is past the block's last key
    uint32_t s2[2][2];  // [row][key pair]: the 4 chains of a row as two packed fp16 pairs
#pragma unroll
    for (int i = 0; i < 2; ++i) s2[i][0] = s2[i][1] = 0u;
    for (int d = 0; d < p.D; ++d) {
      const uint32_t qq = *reinterpret_cast<const uint32_t*>(&qT[d * AE_QB + r0]);        // rows r0, r0+1
      const uint2 kk = *reinterpret_cast<const uint2*>(&kv[d * AE_KT + 4 * kq]);          // keys 4kq .. 4kq+3
      const uint16_t kh[4] = {(uint16_t)kk.x, (uint16_t)(kk.x >> 16), (uint16_t)kk.y, (uint16_t)(kk.y >> 16)};
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint16_t qh = (uint16_t)(qq >> (16 * i));
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
          // s = r16(s + q*k): the product (exact) plus the fp16 accumulator, rounded to fp32, then to fp16
          const float a = fma_h((uint16_t)s2[i][jp], kHalfOne, fma_h(qh, kh[2 * jp], -0.0f));
          const float c = fma_h((uint16_t)(s2[i][jp] >> 16), kHalfOne, fma_h(qh, kh[2 * jp + 1], -0.0f));
          s2[i][jp] = pack_r16(a, c);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = r0 + i;
      if (r >= rows) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = k0 + 4 * kq + j;
        if (key >= row_end(r)) continue;
        const float sv = r16(__fmul_rn(h2f((uint16_t)(s2[i][j >> 1] >> (16 * (j & 1)))), p.scale));
        const bool masked = p.causal && key > q0 + r + p.past;
        sc[key * AE_QB + r] = f2h(__fadd_rn(sv, masked ? -INFINITY : 0.0f));
      }
    }
  }
  __syncthreads();

  // ---- row maxima (fmax is order-free): thread = (row t % 16, keys t / 16 + 16 i)
  {
    const int r = tid % AE_QB;
    float m = -INFINITY;
    if (r < rows)
      for (int key = tid / AE_QB; key < row_end(r); key += AE_THREADS / AE_QB) m = fmaxf(m, h2f(sc[key * AE_QB + r]));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
    if (lane < 16) red[warp * AE_QB + lane] = m;
    __syncthreads();
    if (tid < AE_QB) {
      float mm = -INFINITY;
      for (int w = 0; w < AE_THREADS / 32; ++w) mm = fmaxf(mm, red[w * AE_QB + tid]);
      rowmax[tid] = mm;
    }
    __syncthreads();
  }
  // ---- weights, element-wise
  for (int i = tid; i < kend_blk * AE_QB; i += AE_THREADS) {
    const int key = i / AE_QB, r = i % AE_QB;
    if (r >= rows || key >= row_end(r)) continue;
    const float m = rowmax[r];
    uint16_t w = 0;
    if (m != -INFINITY) w = exp_f16_ref(r16(__fsub_rn(h2f(sc[i]), m)));
    sc[i] = w;
  }
  __syncthreads();
  // ---- sequential sums and reciprocals, one thread per row
  if (tid < rows) {
    uint16_t sum = 0;  // fp16 +0
    const int e = row_end(tid);
    for (int key = 0; key < e; ++key) sum = add_hh(sum, sc[key * AE_QB + tid]);
    const float sf = h2f(sum);
    rowinv[tid] = sf == 0.0f ? 0.0f : r16(__fdiv_rn(1.0f, sf));
  }
  __syncthreads();
  // ---- scaled weights r16(w * inv), element-wise
  for (int i = tid; i < kend_blk * AE_QB; i += AE_THREADS) {
    const int key = i / AE_QB, r = i % AE_QB;
    if (r >= rows || key >= row_end(r)) continue;
    sc[i] = f2h(__fmul_rn(h2f(sc[i]), rowinv[r]));
  }

  // ---- outputs: thread = (row pair rp, channel quad vq); chains (rows r0, r0+1) x (channels 4vq .. 4vq+3)
  const int vq = lane;
  const bool vd_ok = 4 * vq < p.DV;
  const int e0 = row_end(r0), e1 = r0 + 1 < rows ? row_end(r0 + 1) : 0;
  uint32_t acc[2][2];  // [row][channel pair], packed fp16
#pragma unroll
  for (int i = 0; i < 2; ++i) acc[i][0] = acc[i][1] = 0u;
  for (int k0 = 0; k0 < kend_blk; k0 += AE_KT) {
    __syncthreads();
    const int kn = min(AE_KT, kend_blk - k0);
    for (int i = tid; i < kn * (p.DV / 4); i += AE_THREADS) {  // V tile [key][DV], 8-byte pieces
      const int key = i / (p.DV / 4), c4 = i % (p.DV / 4);
      *reinterpret_cast<uint2*>(&kv[key * p.DV + 4 * c4]) =
          *reinterpret_cast<const uint2*>(vg + (int64_t)(k0 + key) * p.v_st + 4 * c4);
    }
    __syncthreads();
    if (!vd_ok || r0 >= rows) continue;
    // acc = r16(acc + w * v) for key k0 + kk2 on the rows selected (w already the scaled fp16 weight)
    auto accumulate = [&](int kk2, bool row0, bool row1) {
      const int key = k0 + kk2;
      const uint32_t ww = *reinterpret_cast<const uint32_t*>(&sc[key * AE_QB + r0]);  // rows r0, r0+1
      const uint2 vv = *reinterpret_cast<const uint2*>(&kv[kk2 * p.DV + 4 * vq]);
      const uint16_t vh[4] = {(uint16_t)vv.x, (uint16_t)(vv.x >> 16), (uint16_t)vv.y, (uint16_t)(vv.y >> 16)};
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if (!(i ? row1 : row0)) continue;
        const uint16_t wh = (uint16_t)(ww >> (16 * i));
#pragma unroll
        for (int cp2 = 0; cp2 < 2; ++cp2) {
          const float a = fma_h((uint16_t)acc[i][cp2], kHalfOne, fma_h(wh, vh[2 * cp2], -0.0f));
          const float c = fma_h((uint16_t)(acc[i][cp2] >> 16), kHalfOne, fma_h(wh, vh[2 * cp2 + 1], -0.0f));
          acc[i][cp2] = pack_r16(a, c);
        }
      }
    };
    // keys both rows visit need no per-key bound test; the longer row's few extra keys follow
    const int both = max(0, min(kn, min(e0, e1) - k0));
    const int tail = max(0, min(kn, max(e0, e1) - k0));
    for (int kk2 = 0; kk2 < both; ++kk2) accumulate(kk2, true, true);
    for (int kk2 = both; kk2 < tail; ++kk2) accumulate(kk2, e0 > e1, e1 > e0);
  }
  if (!vd_ok) return;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = r0 + i;
    const int qi = q0 + r;
    if (r >= rows) continue;
    uint16_t o[4] = {(uint16_t)acc[i][0], (uint16_t)(acc[i][0] >> 16), (uint16_t)acc[i][1], (uint16_t)(acc[i][1] >> 16)};
    if (fast) {
      // skipped keys each add r16(+0 * v) = +-0: it matters only to a -0 accumulator
      for (int c = 0; c < 4; ++c) {
        if (o[c] != 0x8000u) continue;
        float a = h2f(o[c]);
        for (int key = row_end(r); key < p.TK; ++key)
          a = r16(__fadd_rn(a, __fmul_rn(0.0f, h2f(vg[(int64_t)key * p.v_st + 4 * vq + c]))));
        o[c] = f2h(a);
      }
    }
    uint16_t* og = p.o + b * p.o_sb + h * p.o_sh + (int64_t)qi * p.o_st + 4 * vq;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (4 * vq + c < p.DV) og[c] = o[c];
  }
}

// ------------------------------------------------------------------ host side
struct AttnState {
  size_t smem;
  int scn;
  int exact2;  // attention_exact2_kernel applies
};
static_assert(sizeof(AttnState) <= sizeof(OpState), "state fits");

static size_t attn_smem(int d, int dv, int scn) {
  return (size_t)2 * (AT_QB * d + d * AT_KT + AT_KT * dv + (size_t)AT_QB * scn) + 2 * AT_QB * 4 + 16;
}

static size_t attn2_smem(int d, int dv, int scn) {
  return (size_t)2 * (AE_QB * d + std::max(d * AE_KT, AE_KT * dv) + (size_t)AE_QB * scn) + 4 * (2 * AE_QB) +
         4 * (AE_THREADS / 32) * AE_QB + 16;
}

int prepare_attention(const PlanOp& op, void* const*, OpState* st_, int, char* msg, size_t n) {
  AttnState* st = reinterpret_cast<AttnState*>(st_);
  const int d = (int)op.ip[AT_D], dv = (int)op.ip[AT_DV], tk = (int)op.ip[AT_TK];
  if (d <= 0 || dv <= 0 || dv > 128 || (dv & 1)) return fail(msg, n, 5, "Attention: head sizes D=%d DV=%d", d, dv);
  // the register-blocked kernel: 16-byte K rows (D % 8, strides % 8), 8-byte V pieces (DV % 4)
  bool strides_ok = true;
  for (int i = AT_K_SB; i <= AT_V_ST; ++i) strides_ok = strides_ok && op.ip[i] % 8 == 0;
  const int scn2 = (int)align_up((size_t)tk, AE_KT);
  st->exact2 = d % 8 == 0 && dv % 4 == 0 && strides_ok && attn2_smem(d, dv, scn2) <= 227 * 1024;
  if (st->exact2) {
    st->scn = scn2;
    st->smem = attn2_smem(d, dv, scn2);
    cudaError_t e =
        cudaFuncSetAttribute(attention_exact2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)st->smem);
    if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return 0;
  }
  st->scn = (int)align_up((size_t)tk, AT_KT);
  st->smem = attn_smem(d, dv, st->scn);
  if (st->smem > 227 * 1024) return fail(msg, n, 5, "Attention: %zu B shared memory for %d keys", st->smem, tk);
  cudaError_t e =
      cudaFuncSetAttribute(attention_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)st->smem);
  if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  return 0;
}

int launch_attention(const PlanOp& op, void* const* ptrs, const OpState* st_, const LaunchCtx& ctx, int* launches) {
  const AttnState* st = reinterpret_cast<const AttnState*>(st_);
  AttnParams p{};
  p.q = (const uint16_t*)ptrs[op.t[0]];
  p.k = (const uint16_t*)ptrs[op.t[1]];
  p.v = (const uint16_t*)ptrs[op.t[2]];
  p.o = (uint16_t*)ptrs[op.t[3]];
  uint32_t* stats = (uint32_t*)ptrs[op.t[4]];
  p.stats = stats;
  p.err = ctx.d_error;
  p.B = (int)eff_batch(ctx, op, op.ip[AT_B]);
  p.HQ = (int)op.ip[AT_HQ];
  p.group = (int)op.ip[AT_GROUP];
  p.TQ = (int)op.ip[AT_TQ];
  p.TK = (int)op.ip[AT_TK];
  p.past = (int)op.ip[AT_PAST];
  p.D = (int)op.ip[AT_D];
  p.DV = (int)op.ip[AT_DV];
  p.causal = (int)op.ip[AT_CAUSAL];
  p.scn = st->scn;
  p.scale = (float)op.fp[ATF_SCALE];
  const int64_t* s = &op.ip[AT_Q_SB];
  p.q_sb = s[0]; p.q_sh = s[1]; p.q_st = s[2];
  p.k_sb = s[3]; p.k_sh = s[4]; p.k_st = s[5];
  p.v_sb = s[6]; p.v_sh = s[7]; p.v_st = s[8];
  p.o_sb = s[9]; p.o_sh = s[10]; p.o_st = s[11];
  if (p.B <= 0 || p.TQ <= 0) return 0;
  const int64_t hkv = p.HQ / p.group;
  const int64_t nq = (int64_t)p.B * p.q_sb, nk = (int64_t)p.B * p.k_sb, nv = (int64_t)p.B * p.v_sb;
  (void)hkv;
  cudaError_t e = launch_pdl(attn_stats_reset_kernel, dim3(1), dim3(32), 0, ctx.stream, stats);
  ++*launches;
  if (e == cudaSuccess) {
    e = launch_pdl(attn_stats_kernel, dim3(ctx.num_sms * 4), dim3(256), 0, ctx.stream, p.q, nq, p.k, nk, p.v, nv,
                   stats);
    ++*launches;
  }
  if (e == cudaSuccess) {
    if (st->exact2) {
      dim3 grid((unsigned)((p.TQ + AE_QB - 1) / AE_QB), (unsigned)p.HQ, (unsigned)p.B);
      e = launch_pdl(attention_exact2_kernel, grid, dim3(AE_THREADS), st->smem, ctx.stream, p);
    } else {
      dim3 grid((unsigned)((p.TQ + AT_QB - 1) / AT_QB), (unsigned)p.HQ, (unsigned)p.B);
      e = launch_pdl(attention_exact_kernel, grid, dim3(AT_THREADS), st->smem, ctx.stream, p);
    }
    ++*launches;
  }
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
