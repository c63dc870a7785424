// Layout and pooling ops of the QOperator models (the reference's in-tree
// micro_kws_m_static_qoperator.onnx uses each of them once or twice), in the
// reference's arithmetic:
//
//   Reshape            (templates/reshape_op.c.j2): the same bytes; the plan
//                      aliases the tensor, K_COPY only when the result is a
//                      graph output;
//   Transpose          (transpose_op.c.j2): y[o] = x[sum o_i * stride(perm[i])];
//   MaxPool, 8-bit     (maxpool_op.c.j2): start from the type's minimum, max
//                      over the in-bounds taps (out-of-image taps skipped);
//   QLinearAveragePool (qlinear_average_pool_op.c.j2, float compute):
//                      acc = sum (x - zx) over in-bounds taps (int32), denom =
//                      count_include_pad ? KH*KW : in-bounds count, mean =
//                      (float)acc / (float)denom, y = clamp((int)roundf(mean *
//                      scale) + zy) with scale = (float)xs / (float)ys;
//   QLinearSoftmax     (qlinear_softmax_op.c.j2): v = (float)(x - zx) * xs,
//                      max over the row, sum = sum expf(v - max) in row order,
//                      y = clamp(nearbyintf((expf(v - max) * inv) / sum) + zy)
//                      with inv = floorf(1 / (float)ys) (the reference follows
//                      ONNX Runtime's floored reciprocal here); expf values
//                      come from a planner-built table (see qsoftmax8_kernel).
// Every float operation is rounded on its own (no contraction).
#include <stdint.h>

#include <algorithm>

#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

__device__ __forceinline__ int ld8(const uint8_t* p, int64_t i, bool s) {
  return s ? (int)(int8_t)p[i] : (int)p[i];
}

__device__ __forceinline__ uint8_t clamp8(int v, bool s) {
  const int lo = s ? -128 : 0, hi = s ? 127 : 255;
  return (uint8_t)(v < lo ? lo : (v > hi ? hi : v));
}

// ------------------------------------------------------------------ copy
__global__ void copy_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n16 = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) ? 0 : n / 16;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += stride)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  for (int64_t i = n16 * 16 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) dst[i] = src[i];
}

int launch_copy(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t full = op.ip[CP_BATCH] > 0 ? op.ip[CP_BATCH] : 1;
  const int64_t n = op.ip[CP_BYTES] / full * (op.ip[CP_BATCH] > 0 ? eff_batch(ctx, op, full) : 1);
  if (n <= 0) return 0;
  const int blocks = (int)std::min<int64_t>((n / 16 + 255) / 256 + 1, (int64_t)ctx.num_sms * 8);
  cudaError_t e = launch_pdl(copy_kernel, dim3(blocks), dim3(256), 0, ctx.stream, (const uint8_t*)ptrs[op.t[0]],
                             (uint8_t*)ptrs[op.t[1]], n);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ transpose
struct TransposeParams {
  int64_t d[6], s[6];  // output dims, x stride of each output dim
  int64_t count;
};

template <typename T>
__global__ void transpose_kernel(const T* __restrict__ x, T* __restrict__ y, const __grid_constant__ TransposeParams p) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < p.count; o += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = o, src = 0;
#pragma unroll
    for (int i = 5; i >= 0; --i) {
      const int64_t c = rem % p.d[i];
      rem /= p.d[i];
      src += c * p.s[i];
    }
    y[o] = x[src];
  }
}

int launch_transpose(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  TransposeParams p{};
  p.count = 1;
  for (int i = 0; i < 6; ++i) {
    p.d[i] = op.ip[TR_D0 + i];
    p.s[i] = op.ip[TR_S0 + i];
    if (p.d[i] < 0) return 5;
  }
  const int64_t ba = op.ip[TR_BATCH_AXIS];
  if (ba >= 0 && ba < 6) p.d[ba] = eff_batch(ctx, op, p.d[ba]);
  for (int i = 0; i < 6; ++i) p.count *= p.d[i];
  if (p.count == 0) return 0;
  const int blocks = (int)std::min<int64_t>((p.count + 255) / 256, (int64_t)ctx.num_sms * 8);
  cudaError_t e;
  switch (op.ip[TR_ELEM]) {
    case 1: e = launch_pdl(transpose_kernel<uint8_t>, dim3(blocks), dim3(256), 0, ctx.stream,
                           (const uint8_t*)ptrs[op.t[0]], (uint8_t*)ptrs[op.t[1]], p); break;
    case 2: e = launch_pdl(transpose_kernel<uint16_t>, dim3(blocks), dim3(256), 0, ctx.stream,
                           (const uint16_t*)ptrs[op.t[0]], (uint16_t*)ptrs[op.t[1]], p); break;
    case 4: e = launch_pdl(transpose_kernel<uint32_t>, dim3(blocks), dim3(256), 0, ctx.stream,
                           (const uint32_t*)ptrs[op.t[0]], (uint32_t*)ptrs[op.t[1]], p); break;
    default: return 5;
  }
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ pooling
struct PoolParams {
  const uint8_t* x;
  uint8_t* y;
  int n, c, h, w, oh, ow, kh, kw, sh, sw, dh, dw, pt, pl;
  int x_signed, y_signed, count_pad, x_zero, y_zero;
  float scale;
};

// one thread per output element
__global__ void maxpool8_kernel(const __grid_constant__ PoolParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = (int64_t)p.n * p.c * p.oh * p.ow;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
    const int ox = (int)(o % p.ow);
    const int oy = (int)((o / p.ow) % p.oh);
    const int64_t nc = o / ((int64_t)p.ow * p.oh);
    const uint8_t* plane = p.x + nc * p.h * p.w;
    int m = p.x_signed ? -128 : 0;
    for (int ky = 0; ky < p.kh; ++ky) {
      const int iy = oy * p.sh + ky * p.dh - p.pt;
      if (iy < 0 || iy >= p.h) continue;
      for (int kx = 0; kx < p.kw; ++kx) {
        const int ix = ox * p.sw + kx * p.dw - p.pl;
        if (ix < 0 || ix >= p.w) continue;
        const int v = ld8(plane, (int64_t)iy * p.w + ix, p.x_signed);
        m = v > m ? v : m;
      }
    }
    p.y[o] = (uint8_t)m;
  }
}

__global__ void qavgpool8_kernel(const __grid_constant__ PoolParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = (int64_t)p.n * p.c * p.oh * p.ow;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
    const int ox = (int)(o % p.ow);
    const int oy = (int)((o / p.ow) % p.oh);
    const int64_t nc = o / ((int64_t)p.ow * p.oh);
    const uint8_t* plane = p.x + nc * p.h * p.w;
    int acc = 0, count = 0;
    for (int ky = 0; ky < p.kh; ++ky) {
      const int iy = oy * p.sh + ky * p.dh - p.pt;
      for (int kx = 0; kx < p.kw; ++kx) {
        const int ix = ox * p.sw + kx * p.dw - p.pl;
        if (iy >= 0 && iy < p.h && ix >= 0 && ix < p.w) {
          acc += ld8(plane, (int64_t)iy * p.w + ix, p.x_signed) - p.x_zero;
          ++count;
        } else if (p.count_pad) {
          ++count;
        }
      }
    }
    const int denom = p.count_pad ? p.kh * p.kw : count;
    const float mean = denom > 0 ? __fdiv_rn(__int2float_rn(acc), __int2float_rn(denom)) : 0.0f;
    const int r = (int)roundf(__fmul_rn(mean, p.scale)) + p.y_zero;
    p.y[o] = clamp8(r, p.y_signed);
  }
}

static int pool_params(const PlanOp& op, void* const* ptrs, const LaunchCtx& ctx, PoolParams& p) {
  p.x = (const uint8_t*)ptrs[op.t[0]];
  p.y = (uint8_t*)ptrs[op.t[1]];
  p.n = (int)eff_batch(ctx, op, op.ip[PL_N]);
  p.c = (int)op.ip[PL_C];
  p.h = (int)op.ip[PL_H];
  p.w = (int)op.ip[PL_W];
  p.oh = (int)op.ip[PL_OH];
  p.ow = (int)op.ip[PL_OW];
  p.kh = (int)op.ip[PL_KH];
  p.kw = (int)op.ip[PL_KW];
  p.sh = (int)op.ip[PL_SH];
  p.sw = (int)op.ip[PL_SW];
  p.dh = (int)op.ip[PL_DH];
  p.dw = (int)op.ip[PL_DW];
  p.pt = (int)op.ip[PL_PT];
  p.pl = (int)op.ip[PL_PL];
  p.x_signed = (int)op.ip[PL_X_SIGNED];
  p.y_signed = (int)op.ip[PL_Y_SIGNED];
  p.count_pad = (int)op.ip[PL_COUNT_PAD];
  p.x_zero = (int)op.ip[PL_X_ZERO];
  p.y_zero = (int)op.ip[PL_Y_ZERO];
  p.scale = (float)op.fp[PLF_SCALE];
  return (int64_t)p.n * p.c * p.oh * p.ow > 0 ? 1 : 0;
}

static int launch_pool(void (*kern)(const PoolParams), const PoolParams& p, const LaunchCtx& ctx, int* launches) {
  const int64_t total = (int64_t)p.n * p.c * p.oh * p.ow;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)ctx.num_sms * 8);
  cudaError_t e = launch_pdl(kern, dim3(blocks), dim3(256), 0, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

int launch_maxpool(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  PoolParams p{};
  if (!pool_params(op, ptrs, ctx, p)) return 0;
  return launch_pool(maxpool8_kernel, p, ctx, launches);
}

int launch_qlinear_avgpool(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  PoolParams p{};
  if (!pool_params(op, ptrs, ctx, p)) return 0;
  return launch_pool(qavgpool8_kernel, p, ctx, launches);
}

// ------------------------------------------------------------------ QLinearSoftmax
struct QSoftmaxParams {
  const uint8_t* x;
  uint8_t* y;
  const float* exp_table;  // [256][256]: expf(v(b) - v(bm)) for raw bytes b, bm
  int64_t outer, axis, inner;
  int x_signed, y_signed, x_zero, y_zero;
  float x_scale, y_inv;
};

// One thread per (outer, inner) row; the row sum is one sequential chain in
// row order.  v(q) = (float)(q - zx) * xs is a function of the byte, so every
// exp argument v(q) - max is one of 256 x 256 values: the planner evaluates
// them once with the C library's expf (the function the reference calls) and
// the kernel reads them, indexed by the element's byte and the byte that gave
// the row maximum (equal v values give equal table rows).
__global__ void qsoftmax8_kernel(const __grid_constant__ QSoftmaxParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t rows = p.outer * p.inner;
  const float y_zero = (float)p.y_zero;
  const float lo = p.y_signed ? -128.0f : 0.0f, hi = p.y_signed ? 127.0f : 255.0f;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x) {
    const int64_t base = (r / p.inner) * p.axis * p.inner + r % p.inner;
    int bm = p.x[base];
    float mx = __fmul_rn(__int2float_rn(ld8(p.x, base, p.x_signed) - p.x_zero), p.x_scale);
    for (int64_t a = 1; a < p.axis; ++a) {
      const int b = p.x[base + a * p.inner];
      const float v = __fmul_rn(__int2float_rn(ld8(p.x, base + a * p.inner, p.x_signed) - p.x_zero), p.x_scale);
      if (v > mx) {
        mx = v;
        bm = b;
      }
    }
    const float* ex = p.exp_table + bm;
    float sum = 0.0f;
    for (int64_t a = 0; a < p.axis; ++a) sum = __fadd_rn(sum, ex[(int)p.x[base + a * p.inner] * 256]);
    for (int64_t a = 0; a < p.axis; ++a) {
      const float e = ex[(int)p.x[base + a * p.inner] * 256];
      const float scaled = __fdiv_rn(__fmul_rn(e, p.y_inv), sum);
      float rr = __fadd_rn(rintf(scaled), y_zero);
      rr = fminf(fmaxf(rr, lo), hi);
      p.y[base + a * p.inner] = (uint8_t)(int)rr;
    }
  }
}

int launch_qlinear_softmax(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  QSoftmaxParams p{};
  p.x = (const uint8_t*)ptrs[op.t[0]];
  p.y = (uint8_t*)ptrs[op.t[1]];
  p.exp_table = (const float*)ptrs[op.t[2]];
  p.outer = eff_batch(ctx, op, op.ip[QS_OUTER]);
  p.axis = op.ip[QS_AXIS];
  p.inner = op.ip[QS_INNER];
  p.x_signed = (int)op.ip[QS_X_SIGNED];
  p.y_signed = (int)op.ip[QS_Y_SIGNED];
  p.x_zero = (int)op.ip[QS_X_ZERO];
  p.y_zero = (int)op.ip[QS_Y_ZERO];
  p.x_scale = (float)op.fp[QSF_X_SCALE];
  p.y_inv = (float)op.fp[QSF_Y_INV];
  const int64_t rows = p.outer * p.inner;
  if (rows <= 0 || p.axis <= 0) return 0;
  const int blocks = (int)std::min<int64_t>((rows + 127) / 128, (int64_t)ctx.num_sms * 8);
  cudaError_t e = launch_pdl(qsoftmax8_kernel, dim3(blocks), dim3(128), 0, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
