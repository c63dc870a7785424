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
//                  (ic, kh, kw) order, acc += x * w (separately rounded, no FMA).
//   Softmax (fp32) templates/softmax_op.c.j2: fmaxf chain, expf, sequential float
//                  sum, division (one warp per row; the sum stays sequential).
//   QuantizeLinear / DequantizeLinear  templates/quantize_linear_op.c.j2,
//                  dequantize_linear_op.c.j2: per tensor or per axis index.
// Integer work is exact in any order; the float steps use explicitly rounded
// operations in the reference's order.  Softmax calls CUDA's expf (<= 2 ulp)
// where the reference calls glibc's.
#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

__device__ __forceinline__ int32_t load8(const uint8_t* p, int64_t i, int is_signed) {
  return is_signed ? (int32_t)(int8_t)p[i] : (int32_t)p[i];
}

// ------------------------------------------------------------------ QLinearMatMul / MatMulInteger
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

__global__ void qmatmul_kernel(const QMatMulParams p) {
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
  if (!p.quantized) {
    reinterpret_cast<int32_t*>(p.y)[o] = acc;
    return;
  }
  int64_t q;
  if (p.use_int) {
    int64_t r = (int64_t)acc * p.mult;
    if (p.frac_bits > 0) {
      const uint64_t mag = r < 0 ? (uint64_t)(-r) : (uint64_t)r;
      uint64_t quo = mag >> p.frac_bits;
      const uint64_t rem = mag & ((1ull << p.frac_bits) - 1ull), half = 1ull << (p.frac_bits - 1);
      if (rem > half || (rem == half && (quo & 1ull))) ++quo;
      r = r < 0 ? -(int64_t)quo : (int64_t)quo;
    }
    q = r + (int64_t)p.zy;
  } else {
    q = __double2ll_rn(__dadd_rn(__dmul_rn((double)acc, (double)p.scale), (double)p.zy));
  }
  const int64_t lo = p.y_signed ? -128 : 0, hi = p.y_signed ? 127 : 255;
  q = q < lo ? lo : (q > hi ? hi : q);
  reinterpret_cast<uint8_t*>(p.y)[o] = (uint8_t)q;
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
};

__global__ void conv2d_f32_kernel(const ConvF32Params p) {
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
  const int64_t total = (int64_t)p.n * p.oc * p.oh * p.ow;
  if (total == 0) return 0;
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
    float sum = 0.0f;
    if (lane == 0)
      for (int64_t a = 0; a < axis; ++a) sum = __fadd_rn(sum, y[base + a * inner]);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int64_t a = lane; a < axis; a += 32) y[base + a * inner] = __fdiv_rn(y[base + a * inner], sum);
    __syncwarp();
  }
}

int launch_softmax_f32(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t outer_full = op.ip[SM_OUTER];
  const int64_t outer = op.ip[IP_BATCHED] && ctx.batch > 0 && op.ip[SM_OUTER_PER_BATCH] > 0
                            ? ctx.batch * op.ip[SM_OUTER_PER_BATCH]
                            : outer_full;
  const int64_t rows = outer * op.ip[SM_INNER];
  if (rows == 0 || op.ip[SM_AXIS] == 0) return 0;
  const int64_t blocks64 = (rows + 7) / 8;
  const int blocks = (int)(blocks64 < 148 * 32 ? blocks64 : 148 * 32);
  cudaError_t e = launch_pdl(softmax_f32_kernel, dim3(blocks), dim3(256), 0, ctx.stream, (const float*)ptrs[op.t[0]],
                             (float*)ptrs[op.t[1]], rows, op.ip[SM_AXIS], op.ip[SM_INNER]);
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

int launch_quant(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t rows = op.ip[QL_ROWS];
  const int64_t count = rows > 0 && op.ip[IP_BATCHED] && ctx.batch > 0 ? op.ip[QL_COUNT] / rows * ctx.batch
                                                                        : op.ip[QL_COUNT];
  if (count == 0) return 0;
  const int64_t blocks64 = (count + 255) / 256;
  const int blocks = (int)(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
  const uint8_t* zp = op.t[2] >= 0 ? (const uint8_t*)ptrs[op.t[2]] : nullptr;
  cudaError_t e;
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
