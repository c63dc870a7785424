// QLinearConv (any stride / pad / dilation / group, CUDA cores) and standalone
// QLinearAdd: the reference loop nests one output element per thread
// (src/emx_onnx_cgen/templates/qlinear_conv_op.c.j2:1-45,
// qlinear_add_op.c.j2:1-21).  They run every QLinearConv the tensor-core path
// does not take and every QLinearAdd that is not fused into a convolution.
#include "host_util.h"
#include "kernels.h"
#include "qmath.cuh"
#include "tc100.cuh"

namespace emx {

// ------------------------------------------------------------------ generic QLinearConv
// One thread per output element, the reference loop nest verbatim (in-bounds
// taps only, per-channel weight zero points, groups, strides, dilations).
struct QConvGenericParams {
  const uint8_t* x;
  const uint8_t* w;
  const float* ws;
  const int32_t* wz;
  const int32_t* bias;
  uint8_t* y;
  int n, c, h, wd, oc, kh, kw, oh, ow, sh, sw, pt, pl, dh, dw, group;
  int x_signed, w_signed, y_signed, x_zero, y_zero, ws_pc, wz_pc;
  float xs, ys;
};

__global__ void qconv_generic_kernel(const __grid_constant__ QConvGenericParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = (int64_t)p.n * p.oc * p.oh * p.ow;
  const int gic = p.c / p.group, goc = p.oc / p.group;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int ow = (int)(idx % p.ow);
    const int oh = (int)((idx / p.ow) % p.oh);
    const int ocg = (int)((idx / ((int64_t)p.ow * p.oh)) % p.oc);
    const int n = (int)(idx / ((int64_t)p.ow * p.oh * p.oc));
    const int g = ocg / goc;
    const float scale = __fdiv_rn(__fmul_rn(p.xs, p.ws[p.ws_pc ? ocg : 0]), p.ys);
    const int32_t wzero = p.wz ? p.wz[p.wz_pc ? ocg : 0] : 0;
    int32_t acc = p.bias ? p.bias[ocg] : 0;
    for (int ic = 0; ic < gic; ++ic) {
      const int icg = g * gic + ic;
      for (int a = 0; a < p.kh; ++a) {
        const int ih = oh * p.sh + a * p.dh - p.pt;
        if (ih < 0 || ih >= p.h) continue;
        for (int b = 0; b < p.kw; ++b) {
          const int iw = ow * p.sw + b * p.dw - p.pl;
          if (iw < 0 || iw >= p.wd) continue;
          const uint8_t xb = p.x[(((size_t)n * p.c + icg) * p.h + ih) * p.wd + iw];
          const uint8_t wb = p.w[(((size_t)ocg * gic + ic) * p.kh + a) * p.kw + b];
          const int32_t xv = load_8bit(xb, p.x_signed) - p.x_zero;
          const int32_t wv = load_8bit(wb, p.w_signed) - wzero;
          acc += xv * wv;
        }
      }
    }
    p.y[idx] = (uint8_t)requant_exact(acc, scale, (float)p.y_zero, p.y_signed);
  }
}

int launch_qconv_generic(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  QConvGenericParams p{};
  p.x = (const uint8_t*)ptrs[op.t[0]];
  p.w = (const uint8_t*)ptrs[op.t[1]];
  p.ws = (const float*)ptrs[op.t[2]];
  p.wz = op.t[3] >= 0 ? (const int32_t*)ptrs[op.t[3]] : nullptr;
  p.bias = op.t[4] >= 0 ? (const int32_t*)ptrs[op.t[4]] : nullptr;
  p.y = (uint8_t*)ptrs[op.t[5]];
  p.n = (int)eff_batch(ctx, op, op.ip[QG_N]);
  p.c = (int)op.ip[QG_C];
  p.h = (int)op.ip[QG_H];
  p.wd = (int)op.ip[QG_W];
  p.oc = (int)op.ip[QG_OC];
  p.kh = (int)op.ip[QG_KH];
  p.kw = (int)op.ip[QG_KW];
  p.oh = (int)op.ip[QG_OH];
  p.ow = (int)op.ip[QG_OW];
  p.sh = (int)op.ip[QG_SH];
  p.sw = (int)op.ip[QG_SW];
  p.pt = (int)op.ip[QG_PT];
  p.pl = (int)op.ip[QG_PL];
  p.dh = (int)op.ip[QG_DH];
  p.dw = (int)op.ip[QG_DW];
  p.group = (int)op.ip[QG_GROUP];
  p.x_signed = (int)op.ip[QG_X_SIGNED];
  p.w_signed = (int)op.ip[QG_W_SIGNED];
  p.y_signed = (int)op.ip[QG_Y_SIGNED];
  p.x_zero = (int)op.ip[QG_X_ZERO];
  p.y_zero = (int)op.ip[QG_Y_ZERO];
  p.ws_pc = (int)op.ip[QG_WS_PER_CH];
  p.wz_pc = (int)op.ip[QG_WZ_PER_CH];
  p.xs = (float)op.fp[QGF_X_SCALE];
  p.ys = (float)op.fp[QGF_Y_SCALE];
  const int64_t total = (int64_t)p.n * p.oc * p.oh * p.ow;
  if (total == 0) return 0;
  const int64_t blocks64 = (total + 255) / 256;
  const int blocks = (int)(blocks64 < 65535 * 16 ? blocks64 : 65535 * 16);
  cudaError_t e = launch_pdl(qconv_generic_kernel, dim3(blocks), dim3(256), 0, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ QLinearAdd (same shape)
__global__ void qlinear_add_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b,
                                   uint8_t* __restrict__ y, int64_t count, int as, int bs, int ys_signed, int az,
                                   int bz, float sa, float sb, float sy, float yz) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = (uint8_t)qadd_exact(load_8bit(a[i], as), az, sa, load_8bit(b[i], bs), bz, sb, sy, yz, ys_signed);
  }
}

int launch_qlinear_add(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t full_batch = op.ip[QA_BATCH] > 0 ? op.ip[QA_BATCH] : 1;
  const int64_t count = op.ip[QA_COUNT] / full_batch * (op.ip[QA_BATCH] > 0 ? eff_batch(ctx, op, full_batch) : 1);
  if (count == 0) return 0;
  const int64_t blocks64 = (count + 255) / 256;
  const int blocks = (int)(blocks64 < 148 * 64 ? blocks64 : 148 * 64);
  cudaError_t e = launch_pdl(
      qlinear_add_kernel, dim3(blocks), dim3(256), 0, ctx.stream, (const uint8_t*)ptrs[op.t[0]],
      (const uint8_t*)ptrs[op.t[1]], (uint8_t*)ptrs[op.t[2]], count, (int)op.ip[QA_A_SIGNED], (int)op.ip[QA_B_SIGNED],
      (int)op.ip[QA_Y_SIGNED], (int)op.ip[QA_A_ZERO], (int)op.ip[QA_B_ZERO], (float)op.fp[QAF_A_SCALE],
      (float)op.fp[QAF_B_SCALE], (float)op.fp[QAF_Y_SCALE], (float)op.ip[QA_Y_ZERO]);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
