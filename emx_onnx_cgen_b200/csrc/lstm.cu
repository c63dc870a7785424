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
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
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
    for (int c = 0; c < 4; ++c) {
      const int n = n0 + GxChain::col(tx, c);
      if (n < N) st_evict_first(gx + (size_t)m * N + n, acc[r][c], pol);
    }
  }
}

// ---- 2. one recurrent step.  A 64-column tile holds LS_TILE_UNITS = 16 units:
// thread tx's four columns tx + g*16 are gates g = i, o, f, c of unit
// tile*16 + tx, so the cell update runs in the thread that owns the chains.
constexpr int ST_RM = 4;  // batch rows per thread (16 row groups of threads = the CTA's ST_BM rows)
using StChain = ExactChain<16 * ST_RM, 64, ST_RM, 4, 32, 4>;
constexpr int ST_BM = 16 * ST_RM, ST_BN = 64;
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

__global__ void __launch_bounds__(StChain::NT) lstm_step_kernel(const __grid_constant__ LstmStepParams p) {
  extern __shared__ __align__(16) float xc_smem[];
  const int m0 = blockIdx.y * ST_BM, n0 = blockIdx.x * ST_BN;
  const int tx = threadIdx.x % StChain::TX, ty = threadIdx.x / StChain::TX;
  pdl_wait();  // h_prev and c come from the previous step
  pdl_launch_dependents();
  float acc[ST_RM][4];
  const float* g0 = p.gx + (size_t)p.t * p.B * p.N;
  const uint64_t pol = l2_policy_evict_first();
#pragma unroll
  for (int r = 0; r < ST_RM; ++r) {  // continue the chains after their x terms
    const int m = m0 + ty * ST_RM + r;
    float g[4] = {0.f, 0.f, 0.f, 0.f};
    if (m < p.B)
#pragma unroll
      for (int q = 0; q < 4; ++q) g[q] = ld_evict_first(g0 + (size_t)m * p.N + n0 + tx + q * StChain::TX, pol);
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[r][q] = g[q];
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
    const float gi = __fadd_rn(acc[r][0], bs[0]);
    const float go = __fadd_rn(acc[r][1], bs[1]);
    const float gf = __fadd_rn(acc[r][2], bs[2]);
    const float gc = __fadd_rn(acc[r][3], bs[3]);
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

// ---- persistent path: one launch for all T steps.
//
// CTA k owns hidden units [k*U, (k+1)*U): the W and R rows of their four gates
// (U * 4 * (I + H) floats) stay in shared memory for the whole sequence.
// Compute warp w serves unit w / WU and batch rows ((w % WU) * 32 * RB) + lane
// + 32 r (r < RB), so each thread holds RB x 4 exact-order chains (its rows'
// i, o, f, c gates of one unit) and the cell states of those (row, unit) pairs
// in registers.  One producer warp streams the activations through a ring of
// LP_STAGES chunks (LP_KC columns of every batch row) with 2-D TMA loads
// (32-byte swizzle), in the order the compute warps consume them: x_0; then
// per step t, x_{t+1} (its x terms are computed first, kept aside) and, once
// the grid counter says every CTA has written h_{t-1}, h_{t-1}.  The compute warps never synchronise CTA-wide
// inside a step: a chunk's full barrier carries its bytes, and each warp
// releases the chunk on its empty barrier once its lanes have read it.  Per
// step a compute warp adds the h terms, applies the bias and the cell update,
// stores h_t, and the compute warps' named barrier lets one thread arrive on
// the grid counter; the x terms of step t+1 follow at once, so that work
// overlaps the other CTAs finishing step t.  A step-0 h term adds h = 0 times
// R, i.e. +-0, which leaves every partial sum unchanged (a partial sum started
// at +0.0f is never -0), so step 0 has no h terms.  Every wait is bounded.
struct LstmPParams {
  CUtensorMap map_x;   // x as [T*B][I] f32, box (LP_KC, BPAD), 32-byte swizzle
  CUtensorMap map_h;   // h buffer as [2*B][H] f32, same box
  const float* wp;     // [4Hp][I], gate rows interleaved (kernels.h)
  const float* rp;     // [4Hp][H]
  const float* bsum;   // [4Hp]
  float* hbuf;         // [2][B][H]
  unsigned int* bar;   // grid counter: one arrival per CTA per step
  float* y;            // [T][1][B][H] or null
  float* y_h;          // [1][B][H] or null
  float* y_c;
  int T, B, I, H, U, WU, BPAD;
  int* err;
};

struct LpConfig {
  int rb, wu, u, grid, threads, bpad;
  size_t smem;
  bool ok;
};

// Shape of the persistent launch for batch B, input I, hidden H on `sms` SMs
// (threads: the compute warps plus the producer warp).
static LpConfig lp_config(int B, int I, int H, int sms) {
  LpConfig c{};
  c.rb = B > 64 ? 4 : (B > 32 ? 2 : 1);
  c.wu = (B + 32 * c.rb - 1) / (32 * c.rb);
  c.bpad = c.wu * 32 * c.rb;
  c.u = sms > 0 ? (H + sms - 1) / sms : H;
  c.grid = (H + c.u - 1) / c.u;
  c.threads = c.u * c.wu * 32 + 32;
  c.smem = 1024 + (size_t)c.u * 4 * (I + H) * sizeof(float) + (size_t)LP_STAGES * c.bpad * LP_KC * sizeof(float) +
           (size_t)(2 * LP_STAGES + 1) * 8;
  c.ok = I % LP_KC == 0 && H % LP_KC == 0 && c.bpad <= 256 && c.threads <= LP_MAX_THREADS &&
         c.smem <= (size_t)LP_SMEM_LIMIT && c.grid <= sms;
  return c;
}

// gate row of (unit u, gate g) in the interleaved weight layout
__device__ __forceinline__ int lp_row(int u, int g) {
  return (u / LS_TILE_UNITS) * (4 * LS_TILE_UNITS) + g * LS_TILE_UNITS + (u % LS_TILE_UNITS);
}

template <int RB>
__global__ void __launch_bounds__(LP_MAX_THREADS, 1) lstm_persistent_kernel(const __grid_constant__ LstmPParams p) {
  extern __shared__ __align__(1024) uint8_t lp_raw[];
  constexpr int KC = LP_KC, S = LP_STAGES;
  static_assert(KC == 8, "the ring's 32-byte swizzle assumes 8-float rows");
  const int KW = p.I + p.H;  // weight row: x part then h part
  uint8_t* base = lp_raw + ((1024u - (smem_u32(lp_raw) & 1023u)) & 1023u);
  float* ring = reinterpret_cast<float*>(base);                              // [S][BPAD][KC], 1024-aligned
  float* ws = ring + (size_t)S * p.BPAD * KC;                                // [U][4][KW]
  uint64_t* full = reinterpret_cast<uint64_t*>(ws + (size_t)p.U * 4 * KW);   // [S]
  uint64_t* empty = full + S;                                                // [S]
  uint64_t* step_done = empty + S;  // every compute warp has stored its h_t (one phase per step)
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int n_compute = p.U * p.WU;  // compute warps; the producer is warp n_compute
  const int B = p.B, I = p.I, H = p.H;
  int* const err = p.err;
  const uint32_t stage_bytes = (uint32_t)(p.BPAD * KC * sizeof(float));
  const int nx = I / KC, nh = H / KC;  // chunks of an x part / an h part

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], (uint32_t)n_compute);
    }
    mbar_init(step_done, (uint32_t)n_compute);
    fence_barrier_init();
  }
  pdl_wait();  // x and the zeroed counter come from preceding kernels
  pdl_launch_dependents();
  // this CTA's weight rows (plan constants) into shared memory
  {
    const int q_per_row = KW / 4;
    const int total = p.U * 4 * q_per_row;
    for (int e = tid; e < total; e += blockDim.x) {
      const int row = e / q_per_row, q = e - row * q_per_row;
      const int uu = blockIdx.x * p.U + row / 4, g = row % 4;
      const bool ok = uu < H;
      const int k = 4 * q;
      const float* src = !ok ? p.wp : (k < I ? p.wp + (size_t)lp_row(uu, g) * I + k
                                               : p.rp + (size_t)lp_row(uu, g) * H + (k - I));
      xc_cp16(ws + (size_t)row * KW + k, src, ok);
    }
    xc_commit();
    xc_wait<0>();
  }
  __syncthreads();

  if (warp == n_compute) {
    // ---------------- producer: chunks in consumption order
    if (lane == 0) {
      int cc = 0;  // chunks issued
      bool ok = true;
      auto issue = [&](const CUtensorMap* map, int x0, int y0) -> bool {
        const int s = cc % S;
        if (cc >= S && !mbar_wait(&empty[s], (uint32_t)((cc / S) - 1) & 1u, err, DEV_TIMEOUT_PRODUCER)) return false;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        tma_load_2d(ring + (size_t)s * p.BPAD * KC, map, &full[s], x0, y0);
        ++cc;
        return true;
      };
      // stream order = consumption order: x_0, then per step t: x_{t+1}, h_{t-1}
      for (int c = 0; c < nx && ok; ++c) ok = issue(&p.map_x, c * KC, 0);
      const unsigned int grid = gridDim.x;
      for (int t = 0; t < p.T && ok; ++t) {
        if (t + 1 < p.T)
          for (int c = 0; c < nx && ok; ++c) ok = issue(&p.map_x, c * KC, (t + 1) * B);
        if (!ok || t == 0) continue;
        // h_{t-1} needs every CTA's step t-1
        const unsigned int target = (unsigned int)t * grid;
        const uint64_t t0 = globaltimer_ns();
        const uint64_t budget = wait_budget_ns(err);
        uint32_t spins = 0;
        while (true) {
          unsigned int v;
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.bar) : "memory");
          if (v >= target) break;
          if ((++spins & 15u) == 0) {
            if (error_raised(err)) { ok = false; break; }
            if (globaltimer_ns() - t0 > budget) {
              record_error(err, DEV_TIMEOUT_GRID);
              ok = false;
              break;
            }
          }
          __nanosleep(64);
        }
        if (!ok) break;
        fence_proxy_async_global();  // the TMA reads h written by generic stores of other CTAs
        for (int c = 0; c < nh && ok; ++c) ok = issue(&p.map_h, c * KC, ((t - 1) & 1) * B);
      }
      // let every copy issued land before the CTA can exit
      for (int k = cc - S < 0 ? 0 : cc - S; k < cc; ++k) (void)mbar_wait(&full[k % S], (uint32_t)(k / S) & 1u, nullptr, 0);
    }
    return;
  }

  // ---------------- compute warps
  const int ul = warp / p.WU, wb = warp % p.WU;
  const int u = blockIdx.x * p.U + ul;
  const bool unit_ok = u < H;
  float bs[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) bs[g] = unit_ok ? p.bsum[lp_row(u, g)] : 0.0f;
  const float* wrow = ws + (size_t)ul * 4 * KW;
  const int row0 = wb * 32 * RB + lane;
  float acc[RB][4];
  float cst[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) cst[r] = 0.0f;
  int cc = 0;  // chunks consumed
  bool ok = true;
  // acc[r][g] += a[row][k] * W[g][wofs + k] over n chunks, k in order
  auto run_part = [&](int n, int wofs) {
    for (int ch = 0; ch < n; ++ch, ++cc) {
      const int s = cc % S;
      ok = mbar_wait(&full[s], (uint32_t)(cc / S) & 1u, err, DEV_TIMEOUT_MMA);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        return;
      }
      const float* a = ring + (size_t)s * p.BPAD * KC;
      const float* w = wrow + wofs + ch * KC;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float4 w4[4], a4[RB];
#pragma unroll
        for (int g = 0; g < 4; ++g) w4[g] = *reinterpret_cast<const float4*>(w + g * KW + 4 * half);
#pragma unroll
        for (int r = 0; r < RB; ++r) {  // 32-byte swizzle: 16-byte half h of row q sits at h ^ ((q >> 2) & 1)
          const int q = row0 + 32 * r;
          a4[r] = *reinterpret_cast<const float4*>(a + q * KC + 4 * (half ^ ((q >> 2) & 1)));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            const float av = j == 0 ? a4[r].x : j == 1 ? a4[r].y : j == 2 ? a4[r].z : a4[r].w;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const float wv = j == 0 ? w4[g].x : j == 1 ? w4[g].y : j == 2 ? w4[g].z : w4[g].w;
              acc[r][g] = __fadd_rn(acc[r][g], __fmul_rn(av, wv));
            }
          }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  };

  const size_t bh = (size_t)B * H;
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int g = 0; g < 4; ++g) acc[r][g] = 0.0f;
  run_part(nx, 0);  // x terms of step 0
  for (int t = 0; t < p.T && ok; ++t) {
    // x terms of step t are in acc; the h terms of h_{t-1} follow (none at step 0)
    float acc_x[RB][4];
    if (t + 1 < p.T) {
      // the chunk stream has x_{t+1} before h_{t-1}: the next step's x terms first, kept aside
#pragma unroll
      for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          acc_x[r][g] = acc[r][g];
          acc[r][g] = 0.0f;
        }
      run_part(nx, 0);
      if (!ok) break;
#pragma unroll
      for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const float nxt = acc[r][g];
          acc[r][g] = acc_x[r][g];
          acc_x[r][g] = nxt;
        }
    }
    if (t > 0) {
      run_part(nh, I);
      if (!ok) break;
    }
    // bias and cell update; h_t to global memory
    float* hn = p.hbuf + (size_t)(t & 1) * bh;
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const int b = row0 + 32 * r;
      if (!unit_ok || b >= B) continue;
      const float gi = __fadd_rn(acc[r][0], bs[0]);
      const float go = __fadd_rn(acc[r][1], bs[1]);
      const float gf = __fadd_rn(acc[r][2], bs[2]);
      const float gc = __fadd_rn(acc[r][3], bs[3]);
      const float ig = sigmoid_ref(gi);
      const float fg = sigmoid_ref(gf);
      const float cg = tanhf(gc);
      const float c_new = __fadd_rn(__fmul_rn(fg, cst[r]), __fmul_rn(ig, cg));
      const float og = sigmoid_ref(go);
      const float h_new = __fmul_rn(og, tanhf(c_new));
      cst[r] = c_new;
      const size_t o = (size_t)b * H + u;
      hn[o] = h_new;
      if (p.y) p.y[(size_t)t * bh + o] = h_new;
      if (t == p.T - 1) {
        if (p.y_h) p.y_h[o] = h_new;
        if (p.y_c) p.y_c[o] = c_new;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(step_done);  // this warp's h_t stores are issued
    if (tid == 0) {  // once every compute warp's are: one arrival on the grid counter
      if (!mbar_wait(step_done, (uint32_t)t & 1u, err, DEV_TIMEOUT_EPILOGUE)) break;
      __threadfence();
      atomicAdd(p.bar, 1u);
    }
    if (t + 1 < p.T) {
#pragma unroll
      for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int g = 0; g < 4; ++g) acc[r][g] = acc_x[r][g];
    }
  }
}

__global__ void lstm_counter_reset_kernel(unsigned int* bar) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) *bar = 0u;
}

int prepare_lstm_f32(const PlanOp&, void* const*, OpState*, int, char* msg, size_t n) {
  cudaError_t e = cudaFuncSetAttribute(lstm_gx_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)GxChain::SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(lstm_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)StChain::SMEM_BYTES);
  for (auto k : {lstm_persistent_kernel<1>, lstm_persistent_kernel<2>, lstm_persistent_kernel<4>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, LP_SMEM_LIMIT);
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
  // persistent path: one CTA per SM resident at once (checked by occupancy), weights in shared memory
  const LpConfig lc = lp_config(B, I, H, ctx.num_sms);
  if (lc.ok) {
    auto kern = lc.rb == 1 ? lstm_persistent_kernel<1> : (lc.rb == 2 ? lstm_persistent_kernel<2> : lstm_persistent_kernel<4>);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, lc.threads, lc.smem) != cudaSuccess || per_sm < 1)
      return 5;
    unsigned int* bar = reinterpret_cast<unsigned int*>(c);  // the c scratch: the persistent path keeps c in registers
    LstmPParams pp{};
    char msg[128];
    if (make_tmap_2d(&pp.map_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, (uint64_t)I, (uint64_t)T * B, (uint64_t)I * 4,
                     LP_KC, (uint32_t)lc.bpad, CU_TENSOR_MAP_SWIZZLE_32B, msg, sizeof(msg)) ||
        make_tmap_2d(&pp.map_h, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, hbuf, (uint64_t)H, (uint64_t)2 * B, (uint64_t)H * 4,
                     LP_KC, (uint32_t)lc.bpad, CU_TENSOR_MAP_SWIZZLE_32B, msg, sizeof(msg)))
      return 5;
    cudaError_t e = launch_pdl(lstm_counter_reset_kernel, dim3(1), dim3(32), 0, ctx.stream, bar);
    ++*launches;
    if (e != cudaSuccess) return 4;
    pp.wp = wp;
    pp.rp = rp;
    pp.bsum = bsum;
    pp.hbuf = hbuf;
    pp.bar = bar;
    pp.y = y;
    pp.y_h = y_h;
    pp.y_c = y_c;
    pp.T = T;
    pp.B = B;
    pp.I = I;
    pp.H = H;
    pp.U = lc.u;
    pp.WU = lc.wu;
    pp.BPAD = lc.bpad;
    pp.err = ctx.d_error;
    e = launch_pdl(kern, dim3(lc.grid), dim3(lc.threads), lc.smem, ctx.stream, pp);
    ++*launches;
    return e == cudaSuccess ? 0 : 4;
  }
  if (op.ip[LS_GX_PLACEHOLDER]) return 5;  // planned for the persistent path, which this device cannot run
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
