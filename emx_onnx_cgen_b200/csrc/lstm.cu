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
//      the epilogue (a unit's four gates are the four columns one thread
//      owns: the weight rows are permuted at plan time, see kernels.h).
// Both run the cp.async-pipelined exact chains of exact_chain.cuh (every
// multiply and add rounded separately, never fused).  expf and tanhf are CUDA's
// (documented <= 2 ulp); the reference links glibc's, so results can differ
// in the last bits where the two libraries do, and the parity tests state
// that bound.
#include "exact_chain.cuh"
#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

__device__ __forceinline__ void st_evict_first(float* p, float v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(p), "f"(v), "l"(pol) : "memory");
}
__device__ __forceinline__ float ld_evict_first(const float* p, uint64_t pol) {
  float v;
  asm volatile("ld.global.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(pol) : "memory");
  return v;
}

// ---- 1. x-part partial sums: Gx[m][n] = sum_i X[m][i] * Wp[n][i] (m = t*B + b, n gate column)
using GxChain = ExactChain<64, 64, 4, 4, 32, 4>;
constexpr int GX_BM = 64, GX_BN = 64;

__global__ void __launch_bounds__(GxChain::NT) lstm_gx_kernel(const float* __restrict__ x, const float* __restrict__ wp,
                                                              float* __restrict__ gx, int M, int N, int K) {
  extern __shared__ __align__(16) float xc_smem[];
  pdl_wait();
  pdl_launch_dependents();
  const int m0 = blockIdx.y * GX_BM, n0 = blockIdx.x * GX_BN;
  uint64_t acc[4][2];
#pragma unroll
  for (int r = 0; r < 4; ++r) acc[r][0] = acc[r][1] = 0;  // +0.0f pairs
  GxChain::run(x, K, wp, K, M, N, K, m0, n0, acc, xc_smem);
  const int tx = threadIdx.x % GxChain::TX, ty = threadIdx.x / GxChain::TX;
  // the partials (T*B x 4Hp floats, read once by their step) must not push the
  // recurrent matrix that every step re-reads out of L2
  const uint64_t pol = l2_policy_evict_first();
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int m = m0 + ty * 4 + r;
    if (m >= M) continue;
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = n0 + GxChain::col(tx, c, h);
        if (n < N) st_evict_first(gx + (size_t)m * N + n, h ? xc_hi(acc[r][c]) : xc_lo(acc[r][c]), pol);
      }
  }
}

// ---- 2. one recurrent step.  A 64-column tile holds LS_TILE_UNITS = 16 units:
// thread tx's four columns tx + g*16 are gates g = i, o, f, c of unit
// tile*16 + tx, so the cell update runs in the thread that owns the chains.
constexpr int ST_RM = 4;  // batch rows per thread (8 warps' rows = the CTA's ST_BM)
using StChain = ExactChain<8 * ST_RM, 64, ST_RM, 4, 32, 4, true>;  // R kept in L2 across steps
constexpr int ST_BM = 8 * ST_RM, ST_BN = 64;
static_assert(StChain::TX == LS_TILE_UNITS && ST_BN == 4 * LS_TILE_UNITS, "gate tile layout");

struct LstmStepParams {
  const float* gx;     // [T*B][4Hp] (this step's rows start at t*B)
  const float* rp;     // [4Hp][H]
  const float* bsum;   // [4Hp]
  const float* h_prev; // [B][H]
  float* h_next;       // [B][H]
  float* c;            // [B][H], updated in place
  float* y;            // [T][1][B][H] or null
  float* y_h;          // [1][B][H] or null (written on the last step)
  float* y_c;
  int t, B, H, N, last;  // N = 4 * Hp gate columns
};

__device__ __forceinline__ float sigmoid_ref(float a) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a))); }

__global__ void __launch_bounds__(StChain::NT) lstm_step_kernel(const LstmStepParams p) {
  extern __shared__ __align__(16) float xc_smem[];
  const int m0 = blockIdx.y * ST_BM, n0 = blockIdx.x * ST_BN;
  const int tx = threadIdx.x % StChain::TX, ty = threadIdx.x / StChain::TX;
  pdl_wait();  // h_prev and c come from the previous step
  pdl_launch_dependents();
  uint64_t acc[ST_RM][2];
  const float* g0 = p.gx + (size_t)p.t * p.B * p.N;
  const uint64_t pol = l2_policy_evict_first();
#pragma unroll
  for (int r = 0; r < ST_RM; ++r) {  // continue the chains after their x terms
    const int m = m0 + ty * ST_RM + r;
    float g[4] = {0.f, 0.f, 0.f, 0.f};
    if (m < p.B)
#pragma unroll
      for (int q = 0; q < 4; ++q) g[q] = ld_evict_first(g0 + (size_t)m * p.N + n0 + tx + q * StChain::TX, pol);
    acc[r][0] = xc_pack(g[0], g[1]);
    acc[r][1] = xc_pack(g[2], g[3]);
  }
  StChain::run(p.h_prev, p.H, p.rp, p.H, p.B, p.N, p.H, m0, n0, acc, xc_smem);
  const int h = (n0 / ST_BN) * LS_TILE_UNITS + tx;
  if (h >= p.H) return;
  float bs[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) bs[q] = p.bsum[n0 + tx + q * StChain::TX];
#pragma unroll
  for (int r = 0; r < ST_RM; ++r) {
    const int b = m0 + ty * ST_RM + r;
    if (b >= p.B) continue;
    const float gi = __fadd_rn(xc_lo(acc[r][0]), bs[0]);
    const float go = __fadd_rn(xc_hi(acc[r][0]), bs[1]);
    const float gf = __fadd_rn(xc_lo(acc[r][1]), bs[2]);
    const float gc = __fadd_rn(xc_hi(acc[r][1]), bs[3]);
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

int prepare_lstm_f32(const PlanOp&, void* const*, OpState*, int, char* msg, size_t n) {
  cudaError_t e = cudaFuncSetAttribute(lstm_gx_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)GxChain::SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(lstm_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)StChain::SMEM_BYTES);
  if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  return 0;
}

int launch_lstm_f32(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int T = (int)op.ip[LS_T], B = (int)op.ip[LS_B], I = (int)op.ip[LS_I], H = (int)op.ip[LS_H];
  if (T <= 0 || B <= 0) return 0;
  if (I % 4 || H % 4) return 5;  // 16-byte rows
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
  const int hp = (H + LS_TILE_UNITS - 1) / LS_TILE_UNITS * LS_TILE_UNITS;
  const int N = 4 * hp;
  const int64_t bh = (int64_t)B * H;
  cudaError_t e = launch_pdl(lstm_init_kernel, dim3((unsigned)((bh + 255) / 256 < 1184 ? (bh + 255) / 256 : 1184)),
                             dim3(256), 0, ctx.stream, hbuf, c, bh);
  ++*launches;
  if (e != cudaSuccess) return 4;
  const int64_t M = (int64_t)T * B;
  dim3 ggrid((unsigned)((N + GX_BN - 1) / GX_BN), (unsigned)((M + GX_BM - 1) / GX_BM));
  e = launch_pdl(lstm_gx_kernel, ggrid, dim3(GxChain::NT), GxChain::SMEM_BYTES, ctx.stream, x, wp, gx, (int)M, N, I);
  ++*launches;
  if (e != cudaSuccess) return 4;
  dim3 sgrid((unsigned)(N / ST_BN), (unsigned)((B + ST_BM - 1) / ST_BM));
  for (int t = 0; t < T; ++t) {
    LstmStepParams sp{gx, rp, bsum, hbuf + (size_t)(t & 1) * bh, hbuf + (size_t)((t + 1) & 1) * bh, c, y, y_h, y_c,
                      t, B, H, N, t == T - 1};
    e = launch_pdl(lstm_step_kernel, sgrid, dim3(StChain::NT), StChain::SMEM_BYTES, ctx.stream, sp);
    ++*launches;
    if (e != cudaSuccess) return 4;
  }
  return 0;
}

}  // namespace emx
