// The remaining lowered ops of the hot-path list, each repeating its
// reference template's arithmetic (CUDA cores, one output per thread unless
// noted):
//   QLinearMatMul  templates/qlinear_matmul_op.c.j2:1-81 (ir/ops/nn.py:710-769):
//                  int32 sum of (a - za)(b - zb); either the integer requant
//                  (acc * multiplier, round-half-even shift) when the host found
//                  the double multiplier exact in 31 fractional bits, or
//                  llrint((double)acc * (double)scale + zy), scale the float
//                  expression sa * sb / sy; clamp.
//   MatMulInteger  templates/matmul_integer_op.c.j2: int32 sum of (a - za)(b - zb).
//   Conv (fp32)    templates/conv_op.c.j2: acc = bias; in-bounds taps in
//                  (ic, kh, kw) order, acc += x * w (separately rounded, no FMA);
//                  tiled through shared memory, 16 outputs per thread.
//   Softmax (fp32) templates/softmax_op.c.j2: fmaxf chain, expf, sequential float
//                  sum, division (one warp per row; the sum stays sequential;
//                  contiguous rows are staged in shared memory).
//   QuantizeLinear / DequantizeLinear  templates/quantize_linear_op.c.j2,
//                  dequantize_linear_op.c.j2: per tensor or per axis index.
// Integer work is exact in any order; the float steps use explicitly rounded
// operations in the reference's order.  Softmax calls CUDA's expf (<= 2 ulp)
// where the reference calls glibc's.
#include "host_util.h"
#include "kernels.h"
#include "qmatmul.cuh"
#include "tc100.cuh"

namespace emx {

__device__ __forceinline__ int32_t load8(const uint8_t* p, int64_t i, int is_signed) {
  return is_signed ? (int32_t)(int8_t)p[i] : (int32_t)p[i];
}

// ------------------------------------------------------------------ QLinearMatMul / MatMulInteger
__global__ void qmatmul_kernel(const __grid_constant__ QMatMulParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x * 32 + (threadIdx.x & 31);
  const int64_t m = (int64_t)blockIdx.y * 8 + (threadIdx.x >> 5);
  if (n >= p.n || m >= p.m) return;
  const uint8_t* arow = p.a + m * p.k;
  int32_t acc = 0;
  for (int k = 0; k < p.k; ++k)
    acc += (load8(arow, k, p.a_signed) - p.za) * (load8(p.b, (int64_t)k * p.n + n, p.b_signed) - p.zb);
  const int64_t o = m * p.n + n;
  if (!p.quantized)
    reinterpret_cast<int32_t*>(p.y)[o] = acc;
  else
    reinterpret_cast<uint8_t*>(p.y)[o] = qm_requant(acc, p);
}

int prepare_qmatmul(const PlanOp& op, void* const*, OpState*, int, char* msg, size_t n) {
  if (op.n_tensors > 5 && op.t[3] >= 0 && prepare_qgemm_tc())
    return fail(msg, n, 4, "cudaFuncSetAttribute (QLinearMatMul tensor-core kernel) failed");
  return 0;
}

int launch_qmatmul(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  QMatMulParams p{};
  p.a = (const uint8_t*)ptrs[op.t[0]];
  p.b = (const uint8_t*)ptrs[op.t[1]];
  p.y = ptrs[op.t[2]];
  const int64_t rpb = op.ip[QM_ROWS_PER_BATCH];
  p.m = op.ip[IP_BATCHED] && ctx.batch > 0 && rpb > 0 ? ctx.batch * rpb : op.ip[QM_M];
  p.k = (int)op.ip[QM_K];
  p.n = (int)op.ip[QM_N];
  p.a_signed = (int)op.ip[QM_A_SIGNED];
  p.b_signed = (int)op.ip[QM_B_SIGNED];
  p.za = (int)op.ip[QM_A_ZERO];
  p.zb = (int)op.ip[QM_B_ZERO];
  p.quantized = (int)op.ip[QM_QUANTIZED];
  p.use_int = (int)op.ip[QM_USE_INT];
  p.frac_bits = (int)op.ip[QM_FRAC_BITS];
  p.mult = op.ip[QM_MULT];
  p.zy = (int)op.ip[QM_Y_ZERO];
  p.y_signed = (int)op.ip[QM_Y_SIGNED];
  p.scale = (float)op.fp[QMF_SCALE];
  if (p.m <= 0 || p.n <= 0) return 0;
  if (op.n_tensors > 5 && op.t[3] >= 0 && op.t[4] >= 0 && op.t[5] >= 0) {  // planned for the tensor cores
    const int r = launch_qgemm_tc(op, ptrs, ctx, p, launches);
    if (r >= 0) return r;
  }
  dim3 grid((unsigned)((p.n + 31) / 32), (unsigned)((p.m + 7) / 8));
  if (grid.y > 65535u) return 5;
  cudaError_t e = launch_pdl(qmatmul_kernel, grid, dim3(256), 0, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ Conv fp32 (2-D)
struct ConvF32Params {
  const float* x;
  const float* w;
  const float* bias;
  float* y;
  int n, c, h, wd, oc, kh, kw, oh, ow, sh, sw, pt, pl, dh, dw, group;
  int zero_taps_ok;  // out-of-image taps may be added as zeros (planner-checked weights and bias)
};

__global__ void conv2d_f32_kernel(const __grid_constant__ ConvF32Params p) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = (int64_t)p.n * p.oc * p.oh * p.ow;
  const int gic = p.c / p.group, goc = p.oc / p.group;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int ox = (int)(idx % p.ow);
    const int oy = (int)((idx / p.ow) % p.oh);
    const int og = (int)((idx / ((int64_t)p.ow * p.oh)) % p.oc);
    const int b = (int)(idx / ((int64_t)p.ow * p.oh * p.oc));
    const int g = og / goc;
    float acc = p.bias ? p.bias[og] : 0.0f;
    for (int ic = 0; ic < gic; ++ic) {
      const int icg = g * gic + ic;
      const float* xp = p.x + ((int64_t)b * p.c + icg) * p.h * p.wd;
      const float* wp = p.w + ((int64_t)og * gic + ic) * p.kh * p.kw;
      for (int a = 0; a < p.kh; ++a) {
        const int iy = oy * p.sh + a * p.dh - p.pt;
        if (iy < 0 || iy >= p.h) continue;
        for (int bb = 0; bb < p.kw; ++bb) {
          const int ix = ox * p.sw + bb * p.dw - p.pl;
          if (ix < 0 || ix >= p.wd) continue;
          acc = __fadd_rn(acc, __fmul_rn(xp[(int64_t)iy * p.wd + ix], wp[a * p.kw + bb]));
        }
      }
    }
    p.y[idx] = acc;
  }
}

// Tiled form, for kernels of at most CT_MAX_TAPS taps: a block computes CT_OC
// output channels of one group x CT_P output pixels of one image; thread
// (tx = t % 16, ty = t / 16) owns channels ty*CT_RI .. +CT_RI-1 and pixels tx + 16j
// (j < 4).  Per input channel, ascending, the block stages in shared memory
// the input value of every (tap, pixel) and the weight of every (tap,
// channel); each thread then adds its 16 outputs' terms tap by tap (kh, kw
// ascending), multiply and add rounded separately, so every output sees the
// reference's statements in the reference's order.  A tap outside the image
// is skipped, as in the reference (not added as zero: acc + (+0) turns -0 into
// +0, and 0 * inf is NaN), through a per-pixel bit mask computed once per
// block (warps whose pixels are all interior skip the test, and so does every
// warp when the planner found that adding x = 0 for those taps cannot change
// a result: finite weights and no -0 bias; the taps are then staged as zeros).  The next
// channel's entries arrive by cp.async while the current one is summed (two
// shared-memory buffers).  3 x 3 kernels get the tap loop unrolled.
constexpr int CT_RI = 4;  // output channels per thread
constexpr int CT_OC = 8 * CT_RI, CT_P = 64, CT_THREADS = 128, CT_MAX_TAPS = 32;

// One input channel's terms for a thread's CT_RI channels x 4 pixels, taps in
// order; CHECK: test each (pixel, tap) against the in-image mask (border
// pixels), otherwise every tap is in the image.
template <int TAPS, bool CHECK>
__device__ __forceinline__ void conv_tile_channel(float (&acc)[CT_RI][4], const float* xsb, const float* wsb, int taps_rt,
                                                  const uint32_t (&msk)[4], int tx, int ty) {
  const int taps = TAPS > 0 ? TAPS : taps_rt;
#pragma unroll
  for (int tap = 0; tap < taps; ++tap) {
    float wv[CT_RI];
#pragma unroll
    for (int i = 0; i < CT_RI; i += 4) {
      const float4 w4 = *reinterpret_cast<const float4*>(wsb + tap * CT_OC + ty * CT_RI + i);
      wv[i] = w4.x;
      wv[i + 1] = w4.y;
      wv[i + 2] = w4.z;
      wv[i + 3] = w4.w;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (!CHECK || ((msk[j] >> tap) & 1u)) {
        const float xv = xsb[tap * CT_P + tx + 16 * j];
#pragma unroll
        for (int i = 0; i < CT_RI; ++i) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(xv, wv[i]));
      }
    }
  }
}

template <int TAPS>
__global__ void __launch_bounds__(CT_THREADS) conv2d_f32_tiled_kernel(const __grid_constant__ ConvF32Params p, int p_tiles,
                                                                      int oc_tiles) {
  __shared__ __align__(16) float xs[2][CT_MAX_TAPS * CT_P];   // [tap][pixel]
  __shared__ __align__(16) float ws[2][CT_MAX_TAPS * CT_OC];  // [tap][channel]
  __shared__ int s_base[CT_P];                                // iy0 * W + ix0 of each pixel
  __shared__ uint32_t s_mask[CT_P];                           // bit tap: the tap reads inside the image
  __shared__ int s_tapoff[CT_MAX_TAPS];                       // kh * dh * W + kw * dw
  pdl_wait();
  pdl_launch_dependents();
  const int taps = p.kh * p.kw;
  const int gic = p.c / p.group, goc = p.oc / p.group;
  const int npix = p.oh * p.ow;
  int bid = blockIdx.x;
  const int ptile = bid % p_tiles;
  bid /= p_tiles;
  const int otile = bid % oc_tiles;
  bid /= oc_tiles;
  const int g = bid % p.group, b = bid / p.group;
  const int p0 = ptile * CT_P, oc0 = otile * CT_OC;
  const int t = threadIdx.x;
  if (t < CT_P) {
    const int pix = p0 + t;
    uint32_t m = 0;
    int base = 0;
    if (pix < npix) {
      const int oy = pix / p.ow, ox = pix - oy * p.ow;
      const int iy0 = oy * p.sh - p.pt, ix0 = ox * p.sw - p.pl;
      base = iy0 * p.wd + ix0;
      for (int a = 0; a < p.kh; ++a)
        for (int c = 0; c < p.kw; ++c) {
          const int iy = iy0 + a * p.dh, ix = ix0 + c * p.dw;
          if (iy >= 0 && iy < p.h && ix >= 0 && ix < p.wd) m |= 1u << (a * p.kw + c);
        }
    }
    s_base[t] = base;
    s_mask[t] = m;
  } else if (t - CT_P < taps) {
    const int tap = t - CT_P, a = tap / p.kw, c = tap - a * p.kw;
    s_tapoff[tap] = a * p.dh * p.wd + c * p.dw;
  }
  __syncthreads();

  const int64_t plane = (int64_t)p.h * p.wd;
  const float* xb = p.x + ((int64_t)b * p.c + (int64_t)g * gic) * plane;
  const float* wb = p.w + (int64_t)(g * goc + oc0) * gic * taps;  // OIHW
  // asynchronous 4-byte copies of one input channel's entries into buffer
  // `buf`; entries of taps outside the image are never read, so not copied
  auto issue = [&](int ic, int buf) {
    const float* xc = xb + (int64_t)ic * plane;
    for (int e = t; e < taps * CT_P; e += CT_THREADS) {
      const int tap = e / CT_P, px = e % CT_P;
      if ((s_mask[px] >> tap) & 1u)
        cp_async4(&xs[buf][e], xc + s_base[px] + s_tapoff[tap]);
      else if (p.zero_taps_ok)
        xs[buf][e] = 0.0f;
    }
    for (int e = t; e < taps * CT_OC; e += CT_THREADS) {
      const int tap = e / CT_OC, o = e % CT_OC;
      if (oc0 + o < goc)
        cp_async4(&ws[buf][e], wb + ((int64_t)o * gic + ic) * taps + tap);
      else
        ws[buf][e] = 0.0f;
    }
    cp_async_commit();
  };

  const int tx = t & 15, ty = t >> 4;
  float acc[CT_RI][4];
  uint32_t msk[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) msk[j] = s_mask[tx + 16 * j];
  const uint32_t all_taps = taps == 32 ? 0xFFFFFFFFu : (1u << taps) - 1u;
  // warp-uniform, so a warp never runs both forms
  const bool interior =
      p.zero_taps_ok || __all_sync(0xffffffffu, (msk[0] & msk[1] & msk[2] & msk[3]) == all_taps);
#pragma unroll
  for (int i = 0; i < CT_RI; ++i) {
    const int o = oc0 + ty * CT_RI + i;
    const float bias = p.bias && o < goc ? p.bias[g * goc + o] : 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = bias;
  }
  issue(0, 0);
  for (int ic = 0; ic < gic; ++ic) {
    const int buf = ic & 1;
    if (ic + 1 < gic) {
      issue(ic + 1, buf ^ 1);
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    __syncthreads();  // every thread's copies of channel ic have landed
    if (interior)
      conv_tile_channel<TAPS, false>(acc, xs[buf], ws[buf], taps, msk, tx, ty);
    else
      conv_tile_channel<TAPS, true>(acc, xs[buf], ws[buf], taps, msk, tx, ty);
    __syncthreads();  // channel ic read by all before the next issue refills this buffer
  }
#pragma unroll
  for (int i = 0; i < CT_RI; ++i) {
    const int o = oc0 + ty * CT_RI + i;
    if (o >= goc) continue;
    float* yo = p.y + ((int64_t)b * p.oc + g * goc + o) * npix;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int pix = p0 + tx + 16 * j;
      if (pix < npix) yo[pix] = acc[i][j];
    }
  }
}

int launch_conv_f32(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  ConvF32Params p{};
  p.x = (const float*)ptrs[op.t[0]];
  p.w = (const float*)ptrs[op.t[1]];
  p.bias = op.t[2] >= 0 ? (const float*)ptrs[op.t[2]] : nullptr;
  p.y = (float*)ptrs[op.t[3]];
  p.n = (int)eff_batch(ctx, op, op.ip[CF_N]);
  p.c = (int)op.ip[CF_C];
  p.h = (int)op.ip[CF_H];
  p.wd = (int)op.ip[CF_W];
  p.oc = (int)op.ip[CF_OC];
  p.kh = (int)op.ip[CF_KH];
  p.kw = (int)op.ip[CF_KW];
  p.oh = (int)op.ip[CF_OH];
  p.ow = (int)op.ip[CF_OW];
  p.sh = (int)op.ip[CF_SH];
  p.sw = (int)op.ip[CF_SW];
  p.pt = (int)op.ip[CF_PT];
  p.pl = (int)op.ip[CF_PL];
  p.dh = (int)op.ip[CF_DH];
  p.dw = (int)op.ip[CF_DW];
  p.group = (int)op.ip[CF_GROUP];
  p.zero_taps_ok = (int)op.ip[CF_ZERO_TAPS_OK];
  const int64_t total = (int64_t)p.n * p.oc * p.oh * p.ow;
  if (total == 0) return 0;
  if (p.kh * p.kw <= CT_MAX_TAPS && p.c / p.group > 0) {
    const int64_t p_tiles = ((int64_t)p.oh * p.ow + CT_P - 1) / CT_P;
    const int64_t oc_tiles = (p.oc / p.group + CT_OC - 1) / CT_OC;
    const int64_t blocks = (int64_t)p.n * p.group * oc_tiles * p_tiles;
    if (blocks < (int64_t(1) << 31)) {
      void (*fn)(ConvF32Params, int, int) =
          p.kh * p.kw == 9 ? conv2d_f32_tiled_kernel<9> : conv2d_f32_tiled_kernel<0>;
      cudaError_t e =
          launch_pdl(fn, dim3((unsigned)blocks), dim3(CT_THREADS), 0, ctx.stream, p, (int)p_tiles, (int)oc_tiles);
      ++*launches;
      return e == cudaSuccess ? 0 : 4;
    }
  }
  const int64_t blocks64 = (total + 255) / 256;
  const int blocks = (int)(blocks64 < 148 * 64 ? blocks64 : 148 * 64);
  cudaError_t e = launch_pdl(conv2d_f32_kernel, dim3(blocks), dim3(256), 0, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ Softmax fp32
__global__ void softmax_f32_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t axis,
                                   int64_t inner) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t o = row / inner, i = row - o * inner;
    const int64_t base = o * axis * inner + i;
    float mx = x[base];  // fmaxf is order-free (NaN ignored) up to the sign of zero, which cannot change x - max
    for (int64_t a = 1 + lane; a < axis; a += 32) mx = fmaxf(mx, x[base + a * inner]);
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    for (int64_t a = lane; a < axis; a += 32) y[base + a * inner] = expf(__fsub_rn(x[base + a * inner], mx));
    __syncwarp();
    // the reference's sequential sum (k ascending, one rounding per add); the
    // next 16 terms are loaded ahead so the chain waits on adds, not on loads
    float sum = 0.0f;
    if (lane == 0) {
      int64_t a = 0;
      for (; a + 16 <= axis; a += 16) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = y[base + (a + j) * inner];
#pragma unroll
        for (int j = 0; j < 16; ++j) sum = __fadd_rn(sum, v[j]);
      }
      for (; a < axis; ++a) sum = __fadd_rn(sum, y[base + a * inner]);
    }
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int64_t a = lane; a < axis; a += 32) y[base + a * inner] = __fdiv_rn(y[base + a * inner], sum);
    __syncwarp();
  }
}

// Contiguous rows (inner == 1) that fit in shared memory: a block stages one
// row per warp, so x is read once and y written once (the strided kernel above
// re-reads y twice).  The arithmetic is the same statement for statement: the
// fmaxf reduction, expf(x - max) stored, the sequential sum, the division.
// The sums of the block's rows run side by side in the lanes of warp 0 (lane r
// adds row r's terms in order, four per shared-memory load, the next loads
// issued before the current adds), so a row's add chain costs a quarter of a
// warp instruction per term rather than a whole one.  Row r starts at
// r * stride floats with stride = 4 (mod 32), which puts the lanes' loads in
// different banks.
constexpr int SMX_ROWS = 4;
constexpr int64_t SMX_MAX_BYTES = 200 * 1024;
constexpr int SMX_MIN_ROWS_PER_SM = 12;

__device__ __forceinline__ void cp_async16_cg(float* smem_dst, const float* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}

template <bool VEC>
__global__ void softmax_rows_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t axis,
                                    int64_t stride) {
  extern __shared__ __align__(16) float smx[];
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nr = blockDim.x >> 5;
  float* s = smx + warp * stride;
  float* s_sum = smx + nr * stride;
  const int n = (int)axis;
  for (int64_t g = blockIdx.x; g * nr < rows; g += gridDim.x) {
    const int64_t row = g * nr + warp;
    const bool live = row < rows;
    float mx = 0.0f;
    if (live) {
      const float* xr = x + row * axis;
      // the whole row in flight at once: asynchronous copies into the row's
      // shared-memory slot, no registers held while they land
      if (VEC) {
        for (int a = lane; a < (n >> 2); a += 32) cp_async16_cg(s + 4 * a, xr + 4 * a);
      } else {
        for (int a = lane; a < n; a += 32) cp_async4(s + a, xr + a);
      }
      cp_async_commit();
      cp_async_wait_group<0>();
      __syncwarp();
      mx = s[0];  // fmaxf is order-free (NaN ignored) up to the sign of zero, which cannot change x - max
      if (VEC) {
        for (int a = lane; a < (n >> 2); a += 32) {
          const float4 v = reinterpret_cast<const float4*>(s)[a];
          mx = fmaxf(fmaxf(fmaxf(fmaxf(mx, v.x), v.y), v.z), v.w);
        }
      } else {
        for (int a = lane; a < n; a += 32) mx = fmaxf(mx, s[a]);
      }
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      if (VEC) {
        for (int a = lane; a < (n >> 2); a += 32) {
          float4 v = reinterpret_cast<float4*>(s)[a];
          v.x = expf(__fsub_rn(v.x, mx));
          v.y = expf(__fsub_rn(v.y, mx));
          v.z = expf(__fsub_rn(v.z, mx));
          v.w = expf(__fsub_rn(v.w, mx));
          reinterpret_cast<float4*>(s)[a] = v;
        }
      } else {
        for (int a = lane; a < n; a += 32) s[a] = expf(__fsub_rn(s[a], mx));
      }
    }
    __syncthreads();
    if (warp == 0 && lane < nr && g * nr + lane < rows) {
      const float* sr = smx + lane * stride;
      const float4* s4 = reinterpret_cast<const float4*>(sr);
      const int n16 = n >> 4;
      float sum = 0.0f;
      float4 v[4];
      if (n16 > 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = s4[j];
      }
      for (int q = 0; q < n16; ++q) {
        float4 w[4];
        const int nq = q + 1 < n16 ? q + 1 : q;
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = s4[4 * nq + j];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, v[j].x), v[j].y), v[j].z), v[j].w);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = w[j];
      }
      for (int a = 16 * n16; a < n; ++a) sum = __fadd_rn(sum, sr[a]);
      s_sum[lane] = sum;
    }
    __syncthreads();
    if (live) {
      const float sum = s_sum[warp];
      float* yr = y + row * axis;
      if (VEC) {
        for (int a = lane; a < (n >> 2); a += 32) {
          float4 v = reinterpret_cast<const float4*>(s)[a];
          v.x = __fdiv_rn(v.x, sum);
          v.y = __fdiv_rn(v.y, sum);
          v.z = __fdiv_rn(v.z, sum);
          v.w = __fdiv_rn(v.w, sum);
          __stcs(reinterpret_cast<float4*>(yr) + a, v);
        }
      } else {
        for (int a = lane; a < n; a += 32) __stcs(yr + a, __fdiv_rn(s[a], sum));
      }
    }
    // the next group's stores into row `warp` follow this warp's own reads;
    // the next sums are written only after the next group's first barrier
  }
}

// Contiguous rows of a multiple of four floats: the exponentials are staged in
// y itself (L2-resident between the passes) instead of shared memory, so a
// block holds no row in shared memory and six blocks per SM keep 24 rows in
// flight.  Per group of SMX_ROWS rows: each warp reads its row's max (pass 1,
// HBM), writes expf(x - max) into y (pass 2, x again from L2); lanes 0..3 of
// warp 0 add their rows' terms in order, streamed through a per-lane cp.async
// ring (SML_ST chunks of SML_CH floats, SML_ST - 1 in flight); each warp then
// divides its row in place (pass 3).  Same statements as the kernels above.
constexpr int SML_CH = 64;
constexpr int SML_ST = 6;
constexpr int SML_LANE = SML_ST * SML_CH + 4;  // = 4 (mod 32): the lanes' rings sit in different banks
constexpr int SML_BLOCKS_PER_SM = 6;
constexpr int SML_LOADS = 4;   // passes 2 and 3 (L2)
constexpr int SML_LOADS_HBM = 6;  // pass 1

__global__ void __launch_bounds__(32 * SMX_ROWS, SML_BLOCKS_PER_SM) softmax_stream_kernel(const float* __restrict__ x,
                                                                       float* __restrict__ y, int64_t rows,
                                                                       int64_t axis) {
  __shared__ __align__(16) float ring[SMX_ROWS * SML_LANE];
  __shared__ float s_sum[SMX_ROWS];
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = (int)axis, n4 = n >> 2;
  for (int64_t g = blockIdx.x; g * SMX_ROWS < rows; g += gridDim.x) {
    const int64_t row = g * SMX_ROWS + warp;
    const bool live = row < rows;
    if (live) {
      const float4* xr = reinterpret_cast<const float4*>(x + row * axis);
      float4* yr = reinterpret_cast<float4*>(y + row * axis);
      float mx = x[row * axis];  // fmaxf is order-free (NaN ignored) up to the sign of zero
      for (int a0 = lane; a0 < n4; a0 += 32 * SML_LOADS_HBM) {
        float4 v[SML_LOADS_HBM];
#pragma unroll
        for (int j = 0; j < SML_LOADS_HBM; ++j)
          if (a0 + 32 * j < n4) v[j] = xr[a0 + 32 * j];
#pragma unroll
        for (int j = 0; j < SML_LOADS_HBM; ++j)
          if (a0 + 32 * j < n4) mx = fmaxf(fmaxf(fmaxf(fmaxf(mx, v[j].x), v[j].y), v[j].z), v[j].w);
      }
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      for (int a0 = lane; a0 < n4; a0 += 32 * SML_LOADS) {
        float4 v[SML_LOADS];
#pragma unroll
        for (int j = 0; j < SML_LOADS; ++j)
          if (a0 + 32 * j < n4) v[j] = __ldcs(xr + a0 + 32 * j);
#pragma unroll
        for (int j = 0; j < SML_LOADS; ++j)
          if (a0 + 32 * j < n4) {
            v[j].x = expf(__fsub_rn(v[j].x, mx));
            v[j].y = expf(__fsub_rn(v[j].y, mx));
            v[j].z = expf(__fsub_rn(v[j].z, mx));
            v[j].w = expf(__fsub_rn(v[j].w, mx));
            yr[a0 + 32 * j] = v[j];
          }
      }
    }
    __syncthreads();
    if (warp == 0 && lane < SMX_ROWS && g * SMX_ROWS + lane < rows) {
      const float* er = y + (g * SMX_ROWS + lane) * axis;
      float* rg = ring + lane * SML_LANE;
      const int nch = (n + SML_CH - 1) / SML_CH;
      // chunk c goes to ring slot c % SML_ST; issued after the adds of chunk
      // c - SML_ST + 1, so the slot it overwrites was read one chunk earlier
      auto issue = [&](int c) {
        if (c < nch) {
          const int b0 = c * SML_CH, cnt = min(SML_CH, n - b0) >> 2;
          float* dst = rg + (c % SML_ST) * SML_CH;
          for (int j = 0; j < cnt; ++j) cp_async16_cg(dst + 4 * j, er + b0 + 4 * j);
        }
        cp_async_commit();
      };
#pragma unroll
      for (int c = 0; c < SML_ST - 1; ++c) issue(c);
      float sum = 0.0f;
      for (int c = 0; c < nch; ++c) {
        cp_async_wait_group<SML_ST - 2>();
        const float* src = rg + (c % SML_ST) * SML_CH;
        const int cnt = min(SML_CH, n - c * SML_CH);
        if (cnt == SML_CH) {
#pragma unroll
          for (int j = 0; j < SML_CH / 4; ++j) {
            const float4 v = reinterpret_cast<const float4*>(src)[j];
            sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, v.x), v.y), v.z), v.w);
          }
        } else {
          for (int k = 0; k < cnt; ++k) sum = __fadd_rn(sum, src[k]);
        }
        issue(c + SML_ST - 1);
      }
      cp_async_wait_group<0>();
      s_sum[lane] = sum;
    }
    __syncthreads();
    if (live) {
      const float sum = s_sum[warp];
      float4* yr = reinterpret_cast<float4*>(y + row * axis);
      for (int a0 = lane; a0 < n4; a0 += 32 * SML_LOADS) {
        float4 v[SML_LOADS];
#pragma unroll
        for (int j = 0; j < SML_LOADS; ++j)
          if (a0 + 32 * j < n4) v[j] = __ldcg(yr + a0 + 32 * j);
#pragma unroll
        for (int j = 0; j < SML_LOADS; ++j)
          if (a0 + 32 * j < n4) {
            v[j].x = __fdiv_rn(v[j].x, sum);
            v[j].y = __fdiv_rn(v[j].y, sum);
            v[j].z = __fdiv_rn(v[j].z, sum);
            v[j].w = __fdiv_rn(v[j].w, sum);
            __stcs(yr + a0 + 32 * j, v[j]);
          }
      }
    }
  }
}

int launch_softmax_f32(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t outer_full = op.ip[SM_OUTER];
  const int64_t outer = op.ip[IP_BATCHED] && ctx.batch > 0 && op.ip[SM_OUTER_PER_BATCH] > 0
                            ? ctx.batch * op.ip[SM_OUTER_PER_BATCH]
                            : outer_full;
  const int64_t rows = outer * op.ip[SM_INNER];
  if (rows == 0 || op.ip[SM_AXIS] == 0) return 0;
  const int64_t axis = op.ip[SM_AXIS];
  const float* x = (const float*)ptrs[op.t[0]];
  float* y = (float*)ptrs[op.t[1]];
  const bool vec = (axis & 3) == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0;
  // rows staged in shared memory while at least SMX_MIN_ROWS_PER_SM fit per
  // SM; longer rows of a multiple of four floats stream through L2
  // (shared-memory row stride 4 (mod 32) floats: 16-byte rows, and the summing
  // lanes read different banks)
  const int64_t stride = ((axis + 31) & ~int64_t(31)) + 4;
  const bool fits = op.ip[SM_INNER] == 1 && (stride + 1) * 4 <= SMX_MAX_BYTES;
  int nr = 1, per_sm = 0;
  size_t smem = 0;
  void (*fn)(const float*, float*, int64_t, int64_t, int64_t) =
      vec ? softmax_rows_kernel<true> : softmax_rows_kernel<false>;
  if (fits) {
    nr = (stride + 1) * 4 * SMX_ROWS <= SMX_MAX_BYTES ? SMX_ROWS : 1;
    smem = (size_t)(stride * nr + nr) * 4;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 32 * nr, smem);
    if (e != cudaSuccess) return 4;
  }
  if (op.ip[SM_INNER] == 1 && vec && axis < (int64_t(1) << 30) && (int64_t)per_sm * nr < SMX_MIN_ROWS_PER_SM) {
    const int64_t blocks64 = (rows + SMX_ROWS - 1) / SMX_ROWS;
    const int64_t cap = 148 * SML_BLOCKS_PER_SM;
    const int blocks = (int)(blocks64 < cap ? blocks64 : cap);
    cudaError_t e =
        launch_pdl(softmax_stream_kernel, dim3(blocks), dim3(32 * SMX_ROWS), 0, ctx.stream, x, y, rows, axis);
    ++*launches;
    return e == cudaSuccess ? 0 : 4;
  }
  if (fits) {
    const int64_t blocks64 = (rows + nr - 1) / nr;
    const int64_t cap = 148 * (int64_t)(per_sm > 0 ? per_sm : 1);
    const int blocks = (int)(blocks64 < cap ? blocks64 : cap);
    cudaError_t e = launch_pdl(fn, dim3(blocks), dim3(32 * nr), smem, ctx.stream, x, y, rows, axis, stride);
    ++*launches;
    return e == cudaSuccess ? 0 : 4;
  }
  const int64_t blocks64 = (rows + 7) / 8;
  const int blocks = (int)(blocks64 < 148 * 32 ? blocks64 : 148 * 32);
  cudaError_t e =
      launch_pdl(softmax_f32_kernel, dim3(blocks), dim3(256), 0, ctx.stream, x, y, rows, axis, op.ip[SM_INNER]);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ Quantize / Dequantize
__global__ void quantize_linear_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                       const uint8_t* __restrict__ zp, uint8_t* __restrict__ y, int64_t count,
                                       int64_t axis_len, int64_t inner, int y_signed) {
  pdl_wait();
  pdl_launch_dependents();
  const float lo = y_signed ? -128.0f : 0.0f, hi = y_signed ? 127.0f : 255.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t a = axis_len > 1 ? (i / inner) % axis_len : 0;
    const float z = zp ? (float)load8(zp, a, y_signed) : 0.0f;
    float r = __fadd_rn(rintf(__fdiv_rn(x[i], scale[a])), z);
    r = fminf(fmaxf(r, lo), hi);
    y[i] = y_signed ? (uint8_t)(int8_t)r : (uint8_t)r;
  }
}

__global__ void dequantize_linear_kernel(const uint8_t* __restrict__ x, const float* __restrict__ scale,
                                         const uint8_t* __restrict__ zp, float* __restrict__ y, int64_t count,
                                         int64_t axis_len, int64_t inner, int x_signed) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t a = axis_len > 1 ? (i / inner) % axis_len : 0;
    const float z = zp ? (float)load8(zp, a, x_signed) : 0.0f;
    y[i] = __fmul_rn(__fsub_rn((float)load8(x, i, x_signed), z), scale[a]);
  }
}

// Per-tensor scale and zero point, four elements per thread (16-byte float
// side, 4-byte byte side), the same statements per element.
__global__ void quantize_linear_x4_kernel(const float4* __restrict__ x, const float* __restrict__ scale,
                                          const uint8_t* __restrict__ zp, uint32_t* __restrict__ y, int64_t n4,
                                          int y_signed) {
  pdl_wait();
  pdl_launch_dependents();
  const float lo = y_signed ? -128.0f : 0.0f, hi = y_signed ? 127.0f : 255.0f;
  const float s = scale[0], z = zp ? (float)load8(zp, 0, y_signed) : 0.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = __ldcs(x + i);
    const float f[4] = {v.x, v.y, v.z, v.w};
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float r = __fadd_rn(rintf(__fdiv_rn(f[j], s)), z);
      r = fminf(fmaxf(r, lo), hi);
      const uint8_t b = y_signed ? (uint8_t)(int8_t)r : (uint8_t)r;
      w |= (uint32_t)b << (8 * j);
    }
    __stcs(reinterpret_cast<unsigned int*>(y + i), w);
  }
}

__global__ void dequantize_linear_x4_kernel(const uint32_t* __restrict__ x, const float* __restrict__ scale,
                                            const uint8_t* __restrict__ zp, float4* __restrict__ y, int64_t n4,
                                            int x_signed) {
  pdl_wait();
  pdl_launch_dependents();
  const float s = scale[0], z = zp ? (float)load8(zp, 0, x_signed) : 0.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t w = __ldcs(reinterpret_cast<const unsigned int*>(x + i));
    float f[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t b = (w >> (8 * j)) & 0xFFu;
      const float q = x_signed ? (float)(int32_t)(int8_t)b : (float)b;
      f[j] = __fmul_rn(__fsub_rn(q, z), s);
    }
    __stcs(y + i, make_float4(f[0], f[1], f[2], f[3]));
  }
}

int launch_quant(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t rows = op.ip[QL_ROWS];
  const int64_t count = rows > 0 && op.ip[IP_BATCHED] && ctx.batch > 0 ? op.ip[QL_COUNT] / rows * ctx.batch
                                                                        : op.ip[QL_COUNT];
  if (count == 0) return 0;
  const int64_t blocks64 = (count + 255) / 256;
  const int blocks = (int)(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
  const uint8_t* zp = op.t[2] >= 0 ? (const uint8_t*)ptrs[op.t[2]] : nullptr;
  const void* xp = ptrs[op.t[0]];
  void* yp = ptrs[op.t[3]];
  cudaError_t e;
  if (op.ip[QL_AXIS_LEN] <= 1 && count % 4 == 0 && ((uintptr_t)xp & 15) == 0 && ((uintptr_t)yp & 15) == 0) {
    const int64_t n4 = count / 4, b64 = (n4 + 255) / 256;
    const int b4 = (int)(b64 < 148 * 16 ? b64 : 148 * 16);
    if (op.kernel == K_QUANTIZE_LINEAR)
      e = launch_pdl(quantize_linear_x4_kernel, dim3(b4), dim3(256), 0, ctx.stream, (const float4*)xp,
                     (const float*)ptrs[op.t[1]], zp, (uint32_t*)yp, n4, (int)op.ip[QL_SIGNED]);
    else
      e = launch_pdl(dequantize_linear_x4_kernel, dim3(b4), dim3(256), 0, ctx.stream, (const uint32_t*)xp,
                     (const float*)ptrs[op.t[1]], zp, (float4*)yp, n4, (int)op.ip[QL_SIGNED]);
    ++*launches;
    return e == cudaSuccess ? 0 : 4;
  }
  if (op.kernel == K_QUANTIZE_LINEAR)
    e = launch_pdl(quantize_linear_kernel, dim3(blocks), dim3(256), 0, ctx.stream, (const float*)ptrs[op.t[0]],
                   (const float*)ptrs[op.t[1]], zp, (uint8_t*)ptrs[op.t[3]], count, op.ip[QL_AXIS_LEN],
                   op.ip[QL_INNER], (int)op.ip[QL_SIGNED]);
  else
    e = launch_pdl(dequantize_linear_kernel, dim3(blocks), dim3(256), 0, ctx.stream, (const uint8_t*)ptrs[op.t[0]],
                   (const float*)ptrs[op.t[1]], zp, (float*)ptrs[op.t[3]], count, op.ip[QL_AXIS_LEN],
                   op.ip[QL_INNER], (int)op.ip[QL_SIGNED]);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
