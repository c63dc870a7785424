// emx_b200_qlinear_conv3x3_noalloc: one QLinearConv (3x3, stride 1, pad 1)
// through the tensor-core convolution path, without any device allocation.
//
// Who needs it: callers that must not allocate device memory once they are
// running -- integrations whose device-memory footprint has to be fixed when
// the library is loaded (embedded / real-time deployments of the kind the
// reference's generated C serves with static buffers only), and processes
// that share a GPU under a fixed memory budget where a cudaMalloc in the
// middle of serving may fail or stall.  The plan API (emx_b200_plan_load)
// allocates its arena and weight buffers at load time; this entry point
// instead works in a file-scope static device array of fixed size.
//
// Scratch: kNoAllocScratchBytes (8 MiB) of static __device__ memory holding,
// per call, the zero-bordered swizzled NHWC copy of the input, the
// tensor-core weight image and the requantisation table.  Calls whose
// geometry needs more are rejected with EMX_ERR_INVALID_ARGUMENT (e.g. a
// batch of 32 x 64 x 56 x 56 needs 6.98 MB and fits).  The activation region
// must start at zero wherever the layout has a border or tail row; every call
// clears the region it uses (cudaMemsetAsync on the caller's stream) before
// writing the interior, so the result never depends on an earlier call.
//
// Set-up: the first call on a device (with that device current) looks up the
// scratch address with cudaGetSymbolAddress and caches it; make that first
// call before any stream capture begins.
//
// Concurrency: all calls on one device share the one scratch array.  Calls
// that may overlap in time (different streams, host threads) race on it and
// give wrong results; serialise them (one stream, or events).
//
// The kernels are the plan path's own (layout kernel + qconv_tc); only the
// buffers differ, so results are bit-identical to emx_b200_run on a plan of
// the same QLinearConv.  The call only enqueues work: it returns argument and
// launch errors only.  Every device-side error -- a bounded wait that gives
// up, or a kernel finding an inconsistent configuration -- is recorded in a
// word inside the scratch, which the next call clears; none of them is
// reported by this entry point, and the output of such a call is undefined.
//
// Cost to every user: the static array (8 MiB + 256 B) is reserved on each
// device whose context loads this library's module, whether or not this
// entry point is ever called (plan-only users included).
#include <mutex>

#include "emx_b200.h"
#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

int emx_report_error(int code, const char* msg);

namespace emx {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kNoAllocMaxDevices = 64;

// Zero-initialised at module load; the last 256 bytes hold the device error word.
__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes + 256];

// OIHW int8 weights -> [tap][oc][cin] image with each oc row's 16-byte chunks
// at their swizzled positions (the qconv_tc B operand), plus the epilogue
// table: scale[oc] = ((float)xs * (float)ws[oc]) / (float)ys, bias[oc].
__global__ void noalloc_conv_prep_kernel(const int8_t* __restrict__ w, const float* __restrict__ ws,
                                         const int32_t* __restrict__ bias, uint8_t* __restrict__ img,
                                         float* __restrict__ epi, int oc, int cin, float xs, float ys) {
  const int total = 9 * oc * cin;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int ci = i % cin, o = (i / cin) % oc, tap = i / (cin * oc);
    const int8_t v = w[((size_t)o * cin + ci) * 9 + tap];
    img[((size_t)tap * oc + o) * cin + 16 * swz_chunk(o, ci / 16, cin) + (ci % 16)] = (uint8_t)v;
  }
  for (int o = blockIdx.x * blockDim.x + threadIdx.x; o < oc; o += gridDim.x * blockDim.x) {
    epi[o] = __fdiv_rn(__fmul_rn(xs, ws[o]), ys);
    reinterpret_cast<int32_t*>(epi + oc)[o] = bias ? bias[o] : 0;
  }
}

namespace {
std::mutex g_noalloc_mu;
uint8_t* g_noalloc_ptr[kNoAllocMaxDevices] = {};

int report(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return emx_report_error(code, buf);
}
}  // namespace

}  // namespace emx

extern "C" int emx_b200_qlinear_conv3x3_noalloc(const uint8_t* x, const int8_t* w, const float* w_scale,
                                                const int32_t* bias, float x_scale, int x_zero_point,
                                                float y_scale, int y_zero_point, int n, int c, int h, int wd,
                                                int oc, uint8_t* y, void* stream_) {
  using namespace emx;
  if (!x || !w || !w_scale || !y) return report(EMX_ERR_INVALID_ARGUMENT, "noalloc conv: null pointer");
  if (n <= 0 || h <= 0 || wd <= 0) return report(EMX_ERR_INVALID_ARGUMENT, "noalloc conv: empty shape");
  const bool variant = (c == 32 || c == 64 || c == 128) && (oc == 32 || oc == 64 || oc == 128) &&
                       !(c == 32 && oc == 128) && !(c == 128 && oc == 32);
  if (!variant) return report(EMX_ERR_UNSUPPORTED, "noalloc conv: no tensor-core variant for C=%d OC=%d", c, oc);
  if (x_zero_point != 0 && x_zero_point != 128)
    return report(EMX_ERR_UNSUPPORTED, "noalloc conv: x_zero_point must be 0 or 128 (got %d)", x_zero_point);
  if (y_zero_point < 0 || y_zero_point > 255)
    return report(EMX_ERR_INVALID_ARGUMENT, "noalloc conv: y_zero_point %d outside uint8", y_zero_point);
  if ((size_t)2 * c * ((wd + 4) & ~3) > 48 * 1024)  // the layout kernel stages two input rows in shared memory
    return report(EMX_ERR_UNSUPPORTED, "noalloc conv: width %d too large for the layout kernel", wd);

  // scratch layout: [planar activations][weight image][epilogue table]
  const int hp = h + 2, wp = wd + 2;
  const int64_t rows = (int64_t)n * hp * wp + 9 * wp + 264;  // same tail as the plan emitter
  const size_t act_bytes = align_up((size_t)rows * c, 1024);
  const size_t img_bytes = align_up((size_t)9 * oc * c, 1024);
  const size_t epi_bytes = (size_t)oc * 8;
  const size_t need = act_bytes + img_bytes + epi_bytes;
  if (need > kNoAllocScratchBytes)
    return report(EMX_ERR_INVALID_ARGUMENT,
                  "noalloc conv: N=%d C=%d H=%d W=%d OC=%d needs %zu bytes of scratch; the static scratch holds %zu",
                  n, c, h, wd, oc, need, kNoAllocScratchBytes);

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return report(EMX_ERR_CUDA, "noalloc conv: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return report(EMX_ERR_INVALID_ARGUMENT, "noalloc conv: device %d", dev);
  uint8_t* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return report(EMX_ERR_CUDA, "noalloc conv: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
    }
    scratch = g_noalloc_ptr[dev];
  }
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return report(EMX_ERR_CUDA, "noalloc conv: SM count: %s", cudaGetErrorString(e));
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  uint8_t* act = scratch;
  uint8_t* img = scratch + act_bytes;
  float* epi = reinterpret_cast<float*>(scratch + act_bytes + img_bytes);
  int* d_err = reinterpret_cast<int*>(scratch + kNoAllocScratchBytes);

  // The weight image and epilogue table first: the conv kernel reads them
  // before its programmatic-dependency wait (they are load-time constants on
  // the plan path), so they must be complete before the layout kernel starts.
  // The memsets below are not kernels and end any programmatic overlap, so the
  // stream fully orders this kernel before the layout and conv kernels.
  noalloc_conv_prep_kernel<<<64, 256, 0, stream>>>(w, w_scale, bias, img, epi, oc, c, x_scale, y_scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) return report(EMX_ERR_CUDA, "noalloc conv: weight image: %s", cudaGetErrorString(e));
  // the border and tail rows of the planar copy must read as zero; the
  // device error word starts clear on every call
  e = cudaMemsetAsync(act, 0, (size_t)rows * c, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(d_err, 0, sizeof(int), stream);
  if (e != cudaSuccess) return report(EMX_ERR_CUDA, "noalloc conv: clearing scratch: %s", cudaGetErrorString(e));

  // the plan path's two ops, pointed at the scratch
  void* ptrs[5] = {const_cast<uint8_t*>(x), act, img, epi, y};
  PlanOp pad{};
  pad.kernel = K_PAD_NHWC;
  pad.n_tensors = 2;
  pad.t[0] = 0;
  pad.t[1] = 1;
  pad.ip[PAD_N] = n;
  pad.ip[PAD_C] = c;
  pad.ip[PAD_H] = h;
  pad.ip[PAD_W] = wd;
  pad.ip[PAD_TOP] = 1;
  pad.ip[PAD_LEFT] = 1;
  pad.ip[PAD_HP] = hp;
  pad.ip[PAD_WP] = wp;
  pad.ip[PAD_XOR] = x_zero_point == 128 ? 0x80 : 0;
  pad.ip[PAD_ROWS] = rows;
  PlanOp conv{};
  conv.kernel = K_QCONV_TC;
  conv.n_tensors = 6;
  conv.t[5] = -1;  // no fused add
  conv.t[0] = 1;
  conv.t[1] = 2;
  conv.t[2] = 3;
  conv.t[3] = -1;
  conv.t[4] = 4;
  conv.ip[QC_N] = n;
  conv.ip[QC_CIN] = c;
  conv.ip[QC_OC] = oc;
  conv.ip[QC_KH] = 3;
  conv.ip[QC_KW] = 3;
  conv.ip[QC_HP] = hp;
  conv.ip[QC_WP] = wp;
  conv.ip[QC_OH] = h;
  conv.ip[QC_OW] = wd;
  conv.ip[QC_A_SIGNED] = x_zero_point == 128 ? 1 : 0;  // zp 128: bytes XOR 0x80 are x - 128 as int8
  conv.ip[QC_Y_ZERO] = y_zero_point;
  conv.ip[QC_Y_LAYOUT] = 1;  // NCHW output
  conv.ip[QC_X_ROWS] = rows;
  OpState st{};
  char msg[256] = {0};
  int rc = prepare_qconv_tc(conv, ptrs, &st, dev, msg, sizeof(msg));
  if (rc) return report(rc, "noalloc conv: %s", msg);
  LaunchCtx ctx{stream, d_err, 0, sms};
  int launches = 0;
  rc = launch_pad_nhwc(pad, ptrs, nullptr, ctx, &launches);
  if (!rc) rc = launch_qconv_tc(conv, ptrs, &st, ctx, &launches);
  if (rc) {
    e = cudaGetLastError();
    return report(rc == EMX_ERR_CUDA ? EMX_ERR_CUDA : rc, "noalloc conv: launch failed: %s", cudaGetErrorString(e));
  }
  return EMX_OK;
}
