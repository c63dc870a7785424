// Gemm fp32 in the reference's accumulation order, + bias, + optional Relu.
//
// Reference (src/emx_onnx_cgen/templates/gemm_op.c.j2:1-40, "simple" fp32
// accumulation strategy, gcc -O2 on x86-64 = no FMA contraction):
//     acc = 0.0f;  for k ascending: acc += a[i][k] * b[k][j];   (two roundings per k)
//     y[i][j] = acc * alpha + bias * beta;
// Every output is one sequential chain over k, so the kernel keeps exactly
// that chain per output in a register (__fmul_rn then __fadd_rn, never an
// FMA, never split-K) and gets its parallelism from the M x N outputs only:
// the host picks the CTA tile that puts at least ~2 CTAs on each of the 148
// SMs.  Bound: FP32 issue rate at 2 instructions per multiply-add (FMUL +
// FADD), i.e. half the FFMA peak; HBM traffic (weights once) is far below it.
#include "exact_chain.cuh"
#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

struct GemmF32Params {
  const float* a;
  const float* b;
  const float* bias;
  float* y;
  int m, n, k;
  int trans_a, trans_b;
  int bias_mode;  // 0 none, 1 scalar, 2 per column [N], 3 per row [M], 4 full [M,N]
  float alpha, beta;
  int relu;
};

template <int BM, int BN, int RM, int RN>
__global__ void __launch_bounds__((BM / RM) * (BN / RN)) gemm_f32_kernel(const __grid_constant__ GemmF32Params p) {
  constexpr int BK = 16;
  constexpr int TX = BN / RN, TY = BM / RM, NT = TX * TY;
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  const int tid = threadIdx.x;
  const int tx = tid % TX, ty = tid / TX;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  pdl_wait();
  pdl_launch_dependents();

  float acc[RM][RN];
#pragma unroll
  for (int r = 0; r < RM; ++r)
#pragma unroll
    for (int c = 0; c < RN; ++c) acc[r][c] = 0.0f;

  // load one BK-slice of A (BM x BK) and B (BN x BK) into buffer `buf`
  auto load_tile = [&](int buf, int k0) {
    for (int e = tid; e < BM * BK; e += NT) {
      int mm, kk;
      if (p.trans_a) { mm = e % BM; kk = e / BM; } else { kk = e % BK; mm = e / BK; }
      const int gm = m0 + mm, gk = k0 + kk;
      float v = 0.0f;
      if (gm < p.m && gk < p.k) v = p.trans_a ? p.a[(size_t)gk * p.m + gm] : p.a[(size_t)gm * p.k + gk];
      As[buf][kk][mm] = v;
    }
    for (int e = tid; e < BN * BK; e += NT) {
      int nn, kk;
      if (p.trans_b) { kk = e % BK; nn = e / BK; } else { nn = e % BN; kk = e / BN; }
      const int gn = n0 + nn, gk = k0 + kk;
      float v = 0.0f;
      if (gn < p.n && gk < p.k) v = p.trans_b ? p.b[(size_t)gn * p.k + gk] : p.b[(size_t)gk * p.n + gn];
      Bs[buf][kk][nn] = v;
    }
  };

  const int ktiles = (p.k + BK - 1) / BK;
  if (ktiles > 0) load_tile(0, 0);
  __syncthreads();
  for (int t = 0; t < ktiles; ++t) {
    const int cur = t & 1;
    if (t + 1 < ktiles) load_tile(cur ^ 1, (t + 1) * BK);
    const int klen = min(BK, p.k - t * BK);  // never add past K: the reference performs no extra adds
    if (klen == BK) {
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        float av[RM], bv[RN];
#pragma unroll
        for (int r = 0; r < RM; ++r) av[r] = As[cur][kk][ty * RM + r];
#pragma unroll
        for (int c = 0; c < RN; ++c) bv[c] = Bs[cur][kk][tx * RN + c];
#pragma unroll
        for (int r = 0; r < RM; ++r)
#pragma unroll
          for (int c = 0; c < RN; ++c) acc[r][c] = __fadd_rn(acc[r][c], __fmul_rn(av[r], bv[c]));
      }
    } else {
      for (int kk = 0; kk < klen; ++kk) {
#pragma unroll
        for (int r = 0; r < RM; ++r)
#pragma unroll
          for (int c = 0; c < RN; ++c)
            acc[r][c] = __fadd_rn(acc[r][c], __fmul_rn(As[cur][kk][ty * RM + r], Bs[cur][kk][tx * RN + c]));
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int r = 0; r < RM; ++r) {
    const int i = m0 + ty * RM + r;
    if (i >= p.m) continue;
#pragma unroll
    for (int c = 0; c < RN; ++c) {
      const int j = n0 + tx * RN + c;
      if (j >= p.n) continue;
      float y;
      if (p.bias_mode) {
        float bias;
        switch (p.bias_mode) {
          case 1: bias = p.bias[0]; break;
          case 2: bias = p.bias[j]; break;
          case 3: bias = p.bias[i]; break;
          default: bias = p.bias[(size_t)i * p.n + j]; break;
        }
        y = __fadd_rn(__fmul_rn(acc[r][c], p.alpha), __fmul_rn(bias, p.beta));
      } else {
        y = __fmul_rn(acc[r][c], p.alpha);
      }
      if (p.relu) y = y > 0.0f ? y : 0.0f;  // ref_scalar_f32_relu
      p.y[(size_t)i * p.n + j] = y;
    }
  }
}

// Y = op(A) * B^T with A [M][K] and B [N][K] row-major (no transA, transB = 1:
// K contiguous in both): the cp.async-pipelined exact chains of exact_chain.cuh.
template <int BM, int BN, int RM, int RN, int BK = 32, int S = 4>
__global__ void __launch_bounds__((BM / RM) * (BN / RN)) gemm_f32_chain_kernel(const __grid_constant__ GemmF32Params p) {
  using XC = ExactChain<BM, BN, RM, RN, BK, S>;
  extern __shared__ __align__(16) float xc_smem[];
  pdl_wait();
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[RM][RN];
#pragma unroll
  for (int r = 0; r < RM; ++r)
#pragma unroll
    for (int c = 0; c < RN; ++c) acc[r][c] = 0.0f;
  XC::run(p.a, p.k, p.b, p.k, p.m, p.n, p.k, m0, n0, acc, xc_smem);
  // The next kernel's CTAs may be scheduled only now: launched at the start,
  // they would sit in their own pdl_wait holding shared memory and thread
  // slots that this grid's later CTAs need.
  pdl_launch_dependents();
  const int tx = threadIdx.x % XC::TX, ty = threadIdx.x / XC::TX;
#pragma unroll
  for (int r = 0; r < RM; ++r) {
    const int i = m0 + ty * RM + r;
    if (i >= p.m) continue;
#pragma unroll
    for (int c = 0; c < RN; ++c) {
        const int j = n0 + XC::col(tx, c);
        if (j >= p.n) continue;
        const float a = acc[r][c];
        float y;
        if (p.bias_mode) {
          float bias;
          switch (p.bias_mode) {
            case 1: bias = p.bias[0]; break;
            case 2: bias = p.bias[j]; break;
            case 3: bias = p.bias[i]; break;
            default: bias = p.bias[(size_t)i * p.n + j]; break;
          }
          y = __fadd_rn(__fmul_rn(a, p.alpha), __fmul_rn(bias, p.beta));
        } else {
          y = __fmul_rn(a, p.alpha);
        }
        if (p.relu) y = y > 0.0f ? y : 0.0f;  // ref_scalar_f32_relu
        p.y[(size_t)i * p.n + j] = y;
      }
  }
}

typedef void (*GemmKernel)(const GemmF32Params);
struct ChainVariant {
  int bm, bn, threads;
  size_t smem;
  GemmKernel fn;
};
#define EMX_CHAIN_VARIANT(BM, BN, RM, RN, BK, S)                                                 \
  {BM, BN, (BM / RM) * (BN / RN), ExactChain<BM, BN, RM, RN, BK, S>::SMEM_BYTES,                 \
   gemm_f32_chain_kernel<BM, BN, RM, RN, BK, S>}
// Several CTAs per SM (many outputs).  64-wide K stages where the tile is
// small enough to keep three to four CTAs on an SM (64 x 4096, K 1024: 39 ->
// 37.5 us alone on B200).
static const ChainVariant kChainVariants[] = {
    EMX_CHAIN_VARIANT(64, 64, 4, 4, 32, 4), EMX_CHAIN_VARIANT(32, 64, 4, 4, 32, 4),
    EMX_CHAIN_VARIANT(32, 32, 2, 2, 64, 4), EMX_CHAIN_VARIANT(16, 32, 2, 2, 64, 4),
    EMX_CHAIN_VARIANT(16, 16, 2, 2, 32, 4), EMX_CHAIN_VARIANT(8, 16, 1, 2, 32, 4),
};
// Long chains over few outputs (K >= 1024, 256 to 1024 outputs per SM):
// 256-thread CTAs of 2 chains per thread (two rows of one column) with 64-wide
// K stages, so each SM holds enough warps to hide the chains' latency.  A
// sweep of 29 tile shapes on 64 x 1024, K 4096 (the MLP's second Gemm) on
// B200 put this one first (57.5 us alone; 1-chain tiles 72 us, 4-chain tiles
// 68-70 us, 148 CTAs of 14 columns 68 us, deeper rings of 6 or 8 stages no
// faster: shared-memory operand reads, not the copy latency, bound it).
static const ChainVariant kLongKVariants[] = {
    EMX_CHAIN_VARIANT(32, 16, 2, 1, 64, 4),
};
#undef EMX_CHAIN_VARIANT

int prepare_gemm_f32(const PlanOp&, void* const*, OpState*, int, char* msg, size_t n) {
  for (const auto* table : {kChainVariants, kLongKVariants}) {
    const size_t count = table == kChainVariants ? sizeof(kChainVariants) / sizeof(kChainVariants[0])
                                                 : sizeof(kLongKVariants) / sizeof(kLongKVariants[0]);
    for (size_t i = 0; i < count; ++i) {
      cudaError_t e = cudaFuncSetAttribute(table[i].fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)table[i].smem);
      if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
  }
  return 0;
}

struct GemmVariant {
  int bm, bn, threads;
  GemmKernel fn;
};
static const GemmVariant kGemmVariants[] = {
    {64, 64, 256, gemm_f32_kernel<64, 64, 4, 4>},
    {32, 64, 128, gemm_f32_kernel<32, 64, 4, 4>},
    {32, 32, 256, gemm_f32_kernel<32, 32, 2, 2>},
    {16, 32, 128, gemm_f32_kernel<16, 32, 2, 2>},
    {16, 16, 64, gemm_f32_kernel<16, 16, 2, 2>},
};

int launch_gemm_f32(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  GemmF32Params p{};
  p.a = (const float*)ptrs[op.t[0]];
  p.b = (const float*)ptrs[op.t[1]];
  p.bias = op.t[2] >= 0 ? (const float*)ptrs[op.t[2]] : nullptr;
  p.y = (float*)ptrs[op.t[3]];
  p.m = (int)eff_batch(ctx, op, op.ip[GM_M]);
  p.n = (int)op.ip[GM_N];
  p.k = (int)op.ip[GM_K];
  p.trans_a = (int)op.ip[GM_TRANS_A];
  p.trans_b = (int)op.ip[GM_TRANS_B];
  p.bias_mode = p.bias ? (int)op.ip[GM_BIAS_MODE] : 0;
  p.relu = (int)op.ip[GM_RELU];
  p.alpha = (float)op.fp[GMF_ALPHA];
  p.beta = (float)op.fp[GMF_BETA];
  if (p.trans_a && p.m != op.ip[GM_M]) return 5;  // a transposed A cannot be sliced by rows
  if (p.m <= 0 || p.n <= 0) return 0;
  if (!p.trans_a && p.trans_b && p.k % 4 == 0 && !(((uintptr_t)p.a | (uintptr_t)p.b) & 15u)) {
    // long chains over few outputs; else the largest tile that still gives
    // >= 3 CTAs per SM; else the smallest tile
    const ChainVariant* v = nullptr;
    const long outputs = (long)p.m * p.n;
    if (p.k >= 1024 && outputs >= 256L * ctx.num_sms && outputs < 1024L * ctx.num_sms) v = &kLongKVariants[0];
    if (!v) {
      v = &kChainVariants[sizeof(kChainVariants) / sizeof(kChainVariants[0]) - 1];
      for (const auto& c : kChainVariants) {
        const long ctas = (long)((p.m + c.bm - 1) / c.bm) * ((p.n + c.bn - 1) / c.bn);
        if (ctas >= 3L * ctx.num_sms) {
          v = &c;
          break;
        }
      }
    }
    dim3 grid((unsigned)((p.n + v->bn - 1) / v->bn), (unsigned)((p.m + v->bm - 1) / v->bm));
    cudaError_t e = launch_pdl(v->fn, grid, dim3(v->threads), v->smem, ctx.stream, p);
    ++*launches;
    return e == cudaSuccess ? 0 : 4;
  }
  // the largest tile that still gives >= 2 CTAs per SM; else the smallest tile
  const GemmVariant* v = &kGemmVariants[sizeof(kGemmVariants) / sizeof(kGemmVariants[0]) - 1];
  for (const auto& c : kGemmVariants) {
    const long ctas = (long)((p.m + c.bm - 1) / c.bm) * ((p.n + c.bn - 1) / c.bn);
    if (ctas >= 2L * ctx.num_sms) {
      v = &c;
      break;
    }
  }
  dim3 grid((unsigned)((p.n + v->bn - 1) / v->bn), (unsigned)((p.m + v->bm - 1) / v->bm));
  cudaError_t e = launch_pdl(v->fn, grid, dim3(v->threads), 0, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ Relu (standalone)
__global__ void relu_f32_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float a = x[i];
    y[i] = a > 0.0f ? a : 0.0f;
  }
}

int launch_relu_f32(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t rows = op.ip[EW_ROWS] > 0 ? eff_batch(ctx, op, op.ip[EW_ROWS]) : 1;
  const int64_t n = op.ip[EW_COUNT] / (op.ip[EW_ROWS] > 0 ? op.ip[EW_ROWS] : 1) * rows;
  if (n == 0) return 0;
  const int blocks = (int)((n + 255) / 256 < 148 * 32 ? (n + 255) / 256 : 148 * 32);
  cudaError_t e = launch_pdl(relu_f32_kernel, dim3(blocks), dim3(256), 0, ctx.stream, (const float*)ptrs[op.t[0]],
                             (float*)ptrs[op.t[1]], n);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
