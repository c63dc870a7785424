// ONNX LSTM, fp32, forward direction, layout 0, default activations
// (Sigmoid, Tanh, Tanh), in the reference's accumulation order.
//
// Reference (src/emx_onnx_cgen/templates/lstm_op.c.j2:49-123; gcc -O2 on
// x86-64, so no FMA contraction), per (batch b, step t, unit h) and gate
// g in (i, o, f, c):
//   gate = 0.0f;  for i < I: gate += x[t][b][i] * W[g*H+h][i];
//                 for j < H: gate += h_prev[b][j] * R[g*H+h][j];
//   gate += (Wb[g*H+h] + Rb[g*H+h]);
//   i = sigmoid(gate_i); f = sigmoid(gate_f); c = tanh(gate_c);
//   c_new = f * c_prev + i * c;  o = sigmoid(gate_o);  h_new = o * tanh(c_new)
// with sigmoid(a) = 1.0f / (1.0f + expf(-a)).  Every gate is one sequential
// chain of separately rounded multiplies and adds; the chain's first I terms
// do not depend on h, so:
//   1. one launch computes, for all T*B rows at once, the partial sums after
//      the x terms (Gx, an exact-order GEMM of X [T*B][I] with W^T);
//   2. one launch per step continues each chain from Gx with the H terms of
//      the previous step's h, adds the bias and applies the cell update in
//      the epilogue (the four gates of a unit sit in four adjacent columns:
//      the weight rows are interleaved as row 4h+g at plan time).
// Both use packed f32x2 multiplies and adds (two chains per instruction,
// each result rounded separately, never fused).  expf and tanhf are CUDA's
// (documented <= 2 ulp); the reference links glibc's, so results can differ
// in the last bits where the two libraries do, and the parity tests state
// that bound.
#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// acc[r][c] (c pairs packed) += A[m0 + ty*RM + r][k] * B[n0 + tx*RN + c][k] for
// k = 0 .. K-1 in ascending order; A [M][K] with row pitch lda, B [N][K] with
// row pitch ldb (both row-major, K contiguous).  Rows past M / columns past N
// read as 0 and are not stored by the callers.
template <int BM, int BN, int RM, int RN, int BK>
__device__ __forceinline__ void exact_chain_tile(const float* __restrict__ A, int lda, const float* __restrict__ B,
                                                 int ldb, int M, int N, int K, int m0, int n0,
                                                 uint64_t (&acc)[RM][RN / 2], float (*As)[BK][BM + 4],
                                                 float (*Bs)[BK][BN + 4]) {
  constexpr int TX = BN / RN, NT = (BM / RM) * TX;
  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;
  auto load = [&](int buf, int k0) {
    // BK consecutive k of a row as float4s (K % 4 == 0 and rows 16-byte aligned: host-checked)
    for (int e = tid; e < BM * (BK / 4); e += NT) {
      const int r = e / (BK / 4), kq = (e % (BK / 4)) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m0 + r < M && k0 + kq < K) v = *reinterpret_cast<const float4*>(A + (size_t)(m0 + r) * lda + k0 + kq);
      As[buf][kq + 0][r] = v.x;
      As[buf][kq + 1][r] = v.y;
      As[buf][kq + 2][r] = v.z;
      As[buf][kq + 3][r] = v.w;
    }
    for (int e = tid; e < BN * (BK / 4); e += NT) {
      const int r = e / (BK / 4), kq = (e % (BK / 4)) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (n0 + r < N && k0 + kq < K) v = *reinterpret_cast<const float4*>(B + (size_t)(n0 + r) * ldb + k0 + kq);
      Bs[buf][kq + 0][r] = v.x;
      Bs[buf][kq + 1][r] = v.y;
      Bs[buf][kq + 2][r] = v.z;
      Bs[buf][kq + 3][r] = v.w;
    }
  };
  const int ktiles = (K + BK - 1) / BK;
  if (ktiles > 0) load(0, 0);
  __syncthreads();
  for (int t = 0; t < ktiles; ++t) {
    const int cur = t & 1;
    if (t + 1 < ktiles) load(cur ^ 1, (t + 1) * BK);
    const int klen = min(BK, K - t * BK);  // never add past K
#pragma unroll 4
    for (int kk = 0; kk < klen; ++kk) {
      float a[RM];
      uint64_t b2[RN / 2];
#pragma unroll
      for (int r = 0; r < RM; r += 4) {
        const float4 v = *reinterpret_cast<const float4*>(&As[cur][kk][ty * RM + r]);
        a[r] = v.x;
        a[r + 1] = v.y;
        a[r + 2] = v.z;
        a[r + 3] = v.w;
      }
#pragma unroll
      for (int c = 0; c < RN / 2; c += 2) {
        const float4 v = *reinterpret_cast<const float4*>(&Bs[cur][kk][tx * RN + 2 * c]);
        b2[c] = f2_pack(v.x, v.y);
        b2[c + 1] = f2_pack(v.z, v.w);
      }
#pragma unroll
      for (int r = 0; r < RM; ++r) {
        const uint64_t a2 = f2_pack(a[r], a[r]);
#pragma unroll
        for (int c = 0; c < RN / 2; ++c) acc[r][c] = f2_add(acc[r][c], f2_mul(a2, b2[c]));
      }
    }
    __syncthreads();
  }
}

// ---- 1. x-part partial sums: Gx[m][n] = sum_i X[m][i] * Wp[n][i] (m = t*B + b)
constexpr int GX_BM = 64, GX_BN = 128, GX_RM = 8, GX_RN = 8, GX_BK = 16;
constexpr int GX_THREADS = (GX_BM / GX_RM) * (GX_BN / GX_RN);

__global__ void __launch_bounds__(GX_THREADS) lstm_gx_kernel(const float* __restrict__ x, const float* __restrict__ wp,
                                                             float* __restrict__ gx, int M, int N, int K) {
  __shared__ __align__(16) float As[2][GX_BK][GX_BM + 4];
  __shared__ __align__(16) float Bs[2][GX_BK][GX_BN + 4];
  pdl_wait();
  pdl_launch_dependents();
  const int m0 = blockIdx.y * GX_BM, n0 = blockIdx.x * GX_BN;
  uint64_t acc[GX_RM][GX_RN / 2];
#pragma unroll
  for (int r = 0; r < GX_RM; ++r)
#pragma unroll
    for (int c = 0; c < GX_RN / 2; ++c) acc[r][c] = 0;  // +0.0f pairs
  exact_chain_tile<GX_BM, GX_BN, GX_RM, GX_RN, GX_BK>(x, K, wp, K, M, N, K, m0, n0, acc, As, Bs);
  constexpr int TX = GX_BN / GX_RN;
  const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
#pragma unroll
  for (int r = 0; r < GX_RM; ++r) {
    const int m = m0 + ty * GX_RM + r;
    if (m >= M) continue;
#pragma unroll
    for (int c = 0; c < GX_RN / 2; ++c) {
      const int n = n0 + tx * GX_RN + 2 * c;
      if (n + 1 < N) {
        *reinterpret_cast<float2*>(gx + (size_t)m * N + n) = make_float2(f2_lo(acc[r][c]), f2_hi(acc[r][c]));
      } else if (n < N) {
        gx[(size_t)m * N + n] = f2_lo(acc[r][c]);
      }
    }
  }
}

// ---- 2. one recurrent step
constexpr int ST_BM = 64, ST_BN = 64, ST_RM = 8, ST_RN = 4, ST_BK = 16;
constexpr int ST_THREADS = (ST_BM / ST_RM) * (ST_BN / ST_RN);

struct LstmStepParams {
  const float* gx;     // [T*B][4H] (this step's rows start at t*B)
  const float* rp;     // [4H][H], row 4h+g
  const float* bsum;   // [4H]
  const float* h_prev; // [B][H]
  float* h_next;       // [B][H]
  float* c;            // [B][H], updated in place
  float* y;            // [T][1][B][H] or null
  float* y_h;          // [1][B][H] or null (written on the last step)
  float* y_c;
  int t, B, H, last;
};

__device__ __forceinline__ float sigmoid_ref(float a) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a))); }

__global__ void __launch_bounds__(ST_THREADS) lstm_step_kernel(const LstmStepParams p) {
  __shared__ __align__(16) float As[2][ST_BK][ST_BM + 4];
  __shared__ __align__(16) float Bs[2][ST_BK][ST_BN + 4];
  const int N = 4 * p.H;
  const int m0 = blockIdx.y * ST_BM, n0 = blockIdx.x * ST_BN;
  constexpr int TX = ST_BN / ST_RN;
  const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
  pdl_wait();  // h_prev and c come from the previous step
  pdl_launch_dependents();
  uint64_t acc[ST_RM][ST_RN / 2];
  const float* g0 = p.gx + (size_t)p.t * p.B * N;
#pragma unroll
  for (int r = 0; r < ST_RM; ++r) {
    const int m = m0 + ty * ST_RM + r;
    const int n = n0 + tx * ST_RN;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m < p.B && n < N) v = *reinterpret_cast<const float4*>(g0 + (size_t)m * N + n);
    acc[r][0] = f2_pack(v.x, v.y);
    acc[r][1] = f2_pack(v.z, v.w);
  }
  exact_chain_tile<ST_BM, ST_BN, ST_RM, ST_RN, ST_BK>(p.h_prev, p.H, p.rp, p.H, p.B, N, p.H, m0, n0, acc, As, Bs);
  const int n = n0 + tx * ST_RN;  // four gates (i, o, f, c) of unit n / 4
  if (n >= N) return;
  const int h = n >> 2;
  const float4 bs = *reinterpret_cast<const float4*>(p.bsum + n);
#pragma unroll
  for (int r = 0; r < ST_RM; ++r) {
    const int b = m0 + ty * ST_RM + r;
    if (b >= p.B) continue;
    const float gi = __fadd_rn(f2_lo(acc[r][0]), bs.x);
    const float go = __fadd_rn(f2_hi(acc[r][0]), bs.y);
    const float gf = __fadd_rn(f2_lo(acc[r][1]), bs.z);
    const float gc = __fadd_rn(f2_hi(acc[r][1]), bs.w);
    const float ig = sigmoid_ref(gi);
    const float fg = sigmoid_ref(gf);
    const float cg = tanhf(gc);
    const size_t bh = (size_t)b * p.H + h;
    const float c_new = __fadd_rn(__fmul_rn(fg, p.c[bh]), __fmul_rn(ig, cg));
    const float og = sigmoid_ref(go);
    const float h_new = __fmul_rn(og, tanhf(c_new));
    p.c[bh] = c_new;
    p.h_next[bh] = h_new;
    if (p.y) p.y[(size_t)p.t * p.B * p.H + bh] = h_new;
    if (p.last) {
      if (p.y_h) p.y_h[bh] = h_new;
      if (p.y_c) p.y_c[bh] = c_new;
    }
  }
}

__global__ void lstm_init_kernel(float* __restrict__ h0, float* __restrict__ c0, int64_t count) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    h0[i] = 0.0f;
    c0[i] = 0.0f;
  }
}

int launch_lstm_f32(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int T = (int)op.ip[LS_T], B = (int)op.ip[LS_B], I = (int)op.ip[LS_I], H = (int)op.ip[LS_H];
  if (T <= 0 || B <= 0) return 0;
  if (I % 4 || H % 4) return 5;  // float4 rows
  const float* x = (const float*)ptrs[op.t[0]];
  const float* wp = (const float*)ptrs[op.t[1]];
  const float* rp = (const float*)ptrs[op.t[2]];
  const float* bsum = (const float*)ptrs[op.t[3]];
  float* gx = (float*)ptrs[op.t[4]];
  float* hbuf = (float*)ptrs[op.t[5]];
  float* c = (float*)ptrs[op.t[6]];
  float* y = op.t[7] >= 0 ? (float*)ptrs[op.t[7]] : nullptr;
  float* y_h = op.t[8] >= 0 ? (float*)ptrs[op.t[8]] : nullptr;
  float* y_c = op.t[9] >= 0 ? (float*)ptrs[op.t[9]] : nullptr;
  if (((uintptr_t)x | (uintptr_t)wp | (uintptr_t)rp | (uintptr_t)bsum | (uintptr_t)gx | (uintptr_t)hbuf) & 15u)
    return 5;  // 16-byte aligned rows (the plan places every tensor on 256 bytes; a caller's X must be too)
  const int N = 4 * H;
  const int64_t bh = (int64_t)B * H;
  cudaError_t e = launch_pdl(lstm_init_kernel, dim3((unsigned)((bh + 255) / 256 < 1184 ? (bh + 255) / 256 : 1184)),
                             dim3(256), 0, ctx.stream, hbuf, c, bh);
  ++*launches;
  if (e != cudaSuccess) return 4;
  const int64_t M = (int64_t)T * B;
  dim3 ggrid((unsigned)((N + GX_BN - 1) / GX_BN), (unsigned)((M + GX_BM - 1) / GX_BM));
  e = launch_pdl(lstm_gx_kernel, ggrid, dim3(GX_THREADS), 0, ctx.stream, x, wp, gx, (int)M, N, I);
  ++*launches;
  if (e != cudaSuccess) return 4;
  dim3 sgrid((unsigned)((N + ST_BN - 1) / ST_BN), (unsigned)((B + ST_BM - 1) / ST_BM));
  for (int t = 0; t < T; ++t) {
    LstmStepParams sp{gx, rp, bsum, hbuf + (size_t)(t & 1) * bh, hbuf + (size_t)((t + 1) & 1) * bh, c, y, y_h, y_c,
                      t, B, H, t == T - 1};
    e = launch_pdl(lstm_step_kernel, sgrid, dim3(ST_THREADS), 0, ctx.stream, sp);
    ++*launches;
    if (e != cudaSuccess) return 4;
  }
  return 0;
}

}  // namespace emx
