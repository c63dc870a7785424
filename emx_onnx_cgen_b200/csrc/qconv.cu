// QLinearConv / QLinearAdd kernels (int8 ResNet-style stacks).
//
// Reference arithmetic (src/emx_onnx_cgen/templates/qlinear_conv_op.c.j2:1-45,
// qlinear_add_op.c.j2:1-21, ir/ops/nn.py:4875-4951):
//   acc   = bias[oc] + sum over in-bounds taps (x - zx) * (w - zw)      (int32)
//   scale = ((float)xs * (float)ws[oc]) / (float)ys
//   y     = clamp((float)(nearbyint((double)((float)acc * scale)) + zy))
//   add   = clamp(nearbyintf(((float)(a-za)*sa + (float)(b-zb)*sb) / ys + zy))
// Integer accumulation is exact in any order, so the tensor-core kernel is
// bit-exact as long as the epilogue repeats the float steps one rounding at a
// time (__fmul_rn/__fadd_rn/__fdiv_rn: no FMA contraction, IEEE division).
//
// Tensor-core path (K_QCONV_TC), stride 1 / dilation 1 / group 1 convolutions:
//   * activations live in a zero-bordered NHWC layout [N][Hp][Wp][C] (Hp, Wp
//     include the conv's pads).  Output pixel (oh, ow) of image n is the
//     "pitched" row q = n*Hp*Wp + oh*Wp + ow; tap (kh, kw) then reads padded
//     row q + kh*Wp + kw.  A tile of 128 consecutive pitched rows therefore
//     needs, per kh, one contiguous window of 128+KW-1 input rows, and the KW
//     taps of that kh are the same window shifted by kw rows.  Rows that fall
//     on the pad columns / pad rows produce discarded outputs.
//   * the window is fetched by TMA as C/16 planes of [rows][16 bytes] (one 2-D
//     tile load per 16-byte channel chunk), which is exactly the SWIZZLE_NONE
//     K-major canonical layout with SBO = 128 (8 rows x 16 B) and LBO = plane
//     pitch; the kw shift is a 16*kw byte offset of the descriptor start.
//   * zero padding must mean "real zero": when the activation zero point is
//     128 on uint8 storage the producer stores x ^ 0x80 (= x - 128 as int8)
//     and the MMA runs s8 x s8; when it is 0 the MMA runs u8 x s8 on the raw
//     bytes.  Other zero points use the generic kernel.
//   * weights (all taps, [tap][C/16][OC][16 B]) stay in shared memory for the
//     CTA's lifetime; the int32 accumulator (128 x OC) is double-buffered in
//     TMEM so the epilogue of tile i overlaps the MMAs of tile i+1.
//   * warp roles: warp 0 TMA producer, warp 1 MMA issuer, warp 2 TMEM owner,
//     warps 4-7 epilogue (TMEM lane quarter = warp % 4).
#include <cuda_fp16.h>

#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

// ------------------------------------------------------------------ epilogue math
__device__ __forceinline__ int requant(int32_t acc, float scale, float zero, bool is_signed) {
  float v = __fmul_rn(__int2float_rn(acc), scale);
  float r = __fadd_rn(rintf(v), zero);
  r = fmaxf(r, is_signed ? -128.0f : 0.0f);
  r = fminf(r, is_signed ? 127.0f : 255.0f);
  return (int)r;
}

__device__ __forceinline__ int qadd(int a, int za, float sa, int b, int zb, float sb, float ys, float yz,
                                    bool is_signed) {
  float ar = __fmul_rn(__int2float_rn(a - za), sa);
  float br = __fmul_rn(__int2float_rn(b - zb), sb);
  float s = __fadd_rn(__fdiv_rn(__fadd_rn(ar, br), ys), yz);
  float r = rintf(s);
  r = fmaxf(r, is_signed ? -128.0f : 0.0f);
  r = fminf(r, is_signed ? 127.0f : 255.0f);
  return (int)r;
}

__device__ __forceinline__ int load_8bit(uint32_t byte, bool is_signed) {
  return is_signed ? (int)(int8_t)(uint8_t)byte : (int)(uint8_t)byte;
}

// ------------------------------------------------------------------ tcgen05 conv
struct QConvTcParams {
  const uint8_t* w_img;
  const float* scale;
  const int32_t* bias;
  const uint8_t* resid;
  uint8_t* y;
  int* err;
  int batch, kh, kw, hp, wp, oh, ow;
  int rows_box, stages, n_tiles;
  uint32_t idesc, b_bytes, stage_bytes, plane_bytes;
  float y_zero;
  int y_layout, y_xor, y_hp, y_wp, y_pt, y_pl, y_signed;
  int has_add;
  float c_scale, r_scale, add_scale, add_zero;
  int c_zero, r_zero, r_xor, r_signed, r_hp, r_wp, r_pt, r_pl, add_signed;
};

constexpr int QC_THREADS = 256;
constexpr int QC_TILE_M = 128;

template <int CIN, int OC>
__global__ void __launch_bounds__(QC_THREADS, 1)
    qconv_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const QConvTcParams p) {
  constexpr int CHUNKS = CIN / 16;  // 16-byte channel chunks per pixel
  constexpr int KSTEPS = CIN / 32;  // kind::i8 MMAs (K = 32) per tap
  constexpr uint32_t TMEM_COLS = (2 * OC < 32) ? 32 : 2 * OC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_b = smem;
  uint8_t* s_a = smem + align_up_dev(p.b_bytes, 1024);
  float* s_scale = reinterpret_cast<float*>(s_a + (size_t)p.stages * p.stage_bytes);
  int32_t* s_bias = reinterpret_cast<int32_t*>(s_scale + OC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_bias + OC);
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  uint64_t* accf = bars + 2 * p.stages;
  uint64_t* acce = accf + 2;
  uint64_t* bbar = acce + 2;
  uint64_t* drain = bbar + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 128);
    }
    mbar_init(bbar, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp >= 4) {
    for (int i = threadIdx.x - 128; i < OC; i += 128) {
      s_scale[i] = p.scale[i];
      s_bias[i] = p.bias[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: weights once, then one window per (tile, kh)
      mbar_arrive_expect_tx(bbar, p.b_bytes);
      for (uint32_t off = 0; off < p.b_bytes; off += 16384u) {
        const uint32_t n = min(16384u, p.b_bytes - off);
        bulk_load(s_b + off, p.w_img + off, n, bbar);
      }
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued = 0;  // bit s: stage s has a window in flight or landed, parity in `parity_of`
      uint32_t parity_of = 0;
      for (int tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
        const int q0 = tile * QC_TILE_M;
        for (int kh = 0; kh < p.kh; ++kh) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* dst = s_a + (size_t)stage * p.stage_bytes;
          mbar_arrive_expect_tx(&full[stage], p.stage_bytes);
#pragma unroll
          for (int c = 0; c < CHUNKS; ++c)
            tma_load_2d(dst + (size_t)c * p.plane_bytes, &tmap_x, &full[stage], c * 16, q0 + kh * p.wp);
          issued |= 1u << stage;
          parity_of = (parity_of & ~(1u << stage)) | (phase << stage);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // error path: let every window this thread issued land before the CTA exits
      if (!ok) {
        for (int s2 = 0; s2 < p.stages; ++s2)
          if (issued & (1u << s2)) (void)mbar_wait(&full[s2], (parity_of >> s2) & 1u, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      bool ok = mbar_wait(bbar, 0, p.err, DEV_TIMEOUT_MMA);
      tc_fence_after();
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      const uint32_t b_plane = OC * 16u;
      const uint32_t a_base = smem_u32(s_a);
      const uint32_t b_base = smem_u32(s_b);
      for (int tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x, ++it) {
        const int acc = it & 1;
        if (!mbar_wait(&acce[acc], ((it >> 1) & 1) ^ 1u, p.err, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * OC);
        for (int kh = 0; kh < p.kh; ++kh) {
          if (!mbar_wait(&full[stage], phase, p.err, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_stage = a_base + (uint32_t)stage * p.stage_bytes;
          for (int kw = 0; kw < p.kw; ++kw) {
            const int tap = kh * p.kw + kw;
#pragma unroll
            for (int s = 0; s < KSTEPS; ++s) {
              const uint64_t adesc =
                  smem_desc_k_noswizzle(a_stage + (uint32_t)kw * 16u + (uint32_t)(2 * s) * p.plane_bytes,
                                        p.plane_bytes, 128u);
              const uint64_t bdesc = smem_desc_k_noswizzle(
                  b_base + ((uint32_t)(tap * CHUNKS + 2 * s)) * b_plane, b_plane, 128u);
              mma_i8(d_tmem, adesc, bdesc, p.idesc, (kh | kw | s) != 0 ? 1u : 0u);
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&accf[acc]);
      }
      if (!ok) {  // error path: wait for this thread's MMAs before TMEM is released
        tc_commit(drain);
        (void)mbar_wait(drain, 0, nullptr, 0);
      }
    }
  } else if (warp >= 4) {
    // ---------------- epilogue: TMEM -> registers -> requant (+ QLinearAdd) -> global
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int hpwp = p.hp * p.wp;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++it) {
      __syncwarp();
      const int acc = it & 1;
      bool ok = mbar_wait(&accf[acc], (it >> 1) & 1, p.err, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      uint32_t v[OC];
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * OC);
#pragma unroll
      for (int c = 0; c < OC / 16; ++c) tmem_ld16(taddr + c * 16, *reinterpret_cast<uint32_t(*)[16]>(&v[c * 16]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&acce[acc]);

      const int q = tile * QC_TILE_M + row;
      const int n = q / hpwp;
      const int rem = q - n * hpwp;
      const int oh = rem / p.wp;
      const int ow = rem - oh * p.wp;
      if (n >= p.batch || oh >= p.oh || ow >= p.ow) continue;

      uint32_t rbytes[OC / 4];
      if (p.has_add) {
        const size_t rpix = ((size_t)n * p.r_hp + oh + p.r_pt) * p.r_wp + ow + p.r_pl;
        const uint4* rp = reinterpret_cast<const uint4*>(p.resid + rpix * OC);
#pragma unroll
        for (int c = 0; c < OC / 16; ++c) {
          uint4 t = rp[c];
          rbytes[4 * c + 0] = t.x;
          rbytes[4 * c + 1] = t.y;
          rbytes[4 * c + 2] = t.z;
          rbytes[4 * c + 3] = t.w;
        }
      }
      uint32_t out[OC / 4];
#pragma unroll
      for (int j = 0; j < OC / 4; ++j) out[j] = 0;
#pragma unroll
      for (int oc = 0; oc < OC; ++oc) {
        const int32_t a = (int32_t)v[oc] + s_bias[oc];
        int yv = requant(a, s_scale[oc], p.y_zero, p.y_signed);
        if (p.has_add) {
          const uint32_t rb = ((rbytes[oc >> 2] >> (8 * (oc & 3))) & 0xFFu) ^ (uint32_t)p.r_xor;
          yv = qadd(yv, p.c_zero, p.c_scale, load_8bit(rb, p.r_signed), p.r_zero, p.r_scale, p.add_scale,
                    p.add_zero, p.add_signed);
        }
        out[oc >> 2] |= (((uint32_t)yv & 0xFFu) ^ (uint32_t)p.y_xor) << (8 * (oc & 3));
      }
      if (p.y_layout == 0) {
        const size_t ypix = ((size_t)n * p.y_hp + oh + p.y_pt) * p.y_wp + ow + p.y_pl;
        uint4* yp = reinterpret_cast<uint4*>(p.y + ypix * OC);
#pragma unroll
        for (int c = 0; c < OC / 16; ++c)
          yp[c] = make_uint4(out[4 * c + 0], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]);
      } else {
        const size_t plane = (size_t)p.oh * p.ow;
        uint8_t* yb = p.y + (size_t)n * OC * plane + (size_t)oh * p.ow + ow;
#pragma unroll
        for (int oc = 0; oc < OC; ++oc) yb[(size_t)oc * plane] = (uint8_t)(out[oc >> 2] >> (8 * (oc & 3)));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
struct QConvTcState {
  CUtensorMap tmap;  // 128 bytes, 64-aligned
  int variant;       // index into the instantiation table
  int stages;
  int rows_box;
  uint32_t stage_bytes, plane_bytes, b_bytes;
  size_t smem_bytes;
};
static_assert(sizeof(QConvTcState) <= sizeof(OpState), "state fits");

typedef void (*QcKernel)(const CUtensorMap, const QConvTcParams);
struct QcVariant {
  int cin, oc;
  QcKernel fn;
};
static const QcVariant kQcVariants[] = {
    {32, 32, qconv_tc_kernel<32, 32>},   {32, 64, qconv_tc_kernel<32, 64>},
    {64, 32, qconv_tc_kernel<64, 32>},   {64, 64, qconv_tc_kernel<64, 64>},
    {64, 128, qconv_tc_kernel<64, 128>}, {128, 64, qconv_tc_kernel<128, 64>},
    {128, 128, qconv_tc_kernel<128, 128>},
};

static size_t qconv_smem_bytes(uint32_t b_bytes, int stages, uint32_t stage_bytes, int oc) {
  size_t s = 1024;  // alignment slack
  s += align_up(b_bytes, 1024);
  s += (size_t)stages * stage_bytes;
  s += (size_t)oc * 8;
  s += (size_t)(2 * stages + 6) * 8 + 16;
  return s;
}

int prepare_qconv_tc(const PlanOp& op, void* const* ptrs, OpState* st_, int device, char* msg, size_t n) {
  QConvTcState* st = reinterpret_cast<QConvTcState*>(st_);
  const int cin = (int)op.ip[QC_CIN], oc = (int)op.ip[QC_OC];
  st->variant = -1;
  for (int i = 0; i < (int)(sizeof(kQcVariants) / sizeof(kQcVariants[0])); ++i)
    if (kQcVariants[i].cin == cin && kQcVariants[i].oc == oc) st->variant = i;
  if (st->variant < 0) return fail(msg, n, 5, "QLinearConv tensor-core path: no variant for C=%d OC=%d", cin, oc);
  const int kw = (int)op.ip[QC_KW], kh = (int)op.ip[QC_KH];
  st->rows_box = (int)align_up((size_t)(QC_TILE_M + kw - 1), 8);
  if (st->rows_box > 256) return fail(msg, n, 5, "kernel width %d too large for one TMA box", kw);
  st->plane_bytes = (uint32_t)st->rows_box * 16u;
  st->stage_bytes = st->plane_bytes * (uint32_t)(cin / 16);
  st->b_bytes = (uint32_t)(kh * kw * cin * oc);
  const size_t budget = 200 * 1024;
  int stages = 9;
  while (stages > 2 && qconv_smem_bytes(st->b_bytes, stages, st->stage_bytes, oc) > budget) --stages;
  st->stages = stages;
  st->smem_bytes = qconv_smem_bytes(st->b_bytes, stages, st->stage_bytes, oc);
  if (st->smem_bytes > 227 * 1024) return fail(msg, n, 5, "QLinearConv tensor-core path needs %zu B smem", st->smem_bytes);
  const int64_t rows = op.ip[QC_N] * op.ip[QC_HP] * op.ip[QC_WP];
  int rc = make_tmap_2d(&st->tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ptrs[op.t[0]], (uint64_t)cin, (uint64_t)rows,
                        (uint64_t)cin, 16, (uint32_t)st->rows_box, CU_TENSOR_MAP_SWIZZLE_NONE, msg, n);
  if (rc) return rc;
  cudaError_t e = cudaFuncSetAttribute(kQcVariants[st->variant].fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)st->smem_bytes);
  if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  (void)device;
  return 0;
}

int launch_qconv_tc(const PlanOp& op, void* const* ptrs, const OpState* st_, const LaunchCtx& ctx, int* launches) {
  const QConvTcState* st = reinterpret_cast<const QConvTcState*>(st_);
  const int oc = (int)op.ip[QC_OC];
  QConvTcParams p{};
  p.w_img = (const uint8_t*)ptrs[op.t[1]];
  p.scale = (const float*)ptrs[op.t[2]];
  p.bias = (const int32_t*)((const float*)ptrs[op.t[2]] + oc);
  p.resid = op.t[3] >= 0 ? (const uint8_t*)ptrs[op.t[3]] : nullptr;
  p.y = (uint8_t*)ptrs[op.t[4]];
  p.err = ctx.d_error;
  p.batch = (int)eff_batch(ctx, op.ip[QC_N]);
  p.kh = (int)op.ip[QC_KH];
  p.kw = (int)op.ip[QC_KW];
  p.hp = (int)op.ip[QC_HP];
  p.wp = (int)op.ip[QC_WP];
  p.oh = (int)op.ip[QC_OH];
  p.ow = (int)op.ip[QC_OW];
  p.rows_box = st->rows_box;
  p.stages = st->stages;
  const int64_t q_last = ((int64_t)p.batch - 1) * p.hp * p.wp + (int64_t)(p.oh - 1) * p.wp + p.ow;  // one past last valid
  p.n_tiles = (int)((q_last + QC_TILE_M - 1) / QC_TILE_M);
  p.idesc = make_idesc(2u, op.ip[QC_A_SIGNED] ? 1u : 0u, 1u, 128u, (uint32_t)oc);
  p.b_bytes = st->b_bytes;
  p.stage_bytes = st->stage_bytes;
  p.plane_bytes = st->plane_bytes;
  p.y_zero = (float)op.ip[QC_Y_ZERO];
  p.y_layout = (int)op.ip[QC_Y_LAYOUT];
  p.y_xor = (int)op.ip[QC_Y_XOR];
  p.y_hp = (int)op.ip[QC_Y_HP];
  p.y_wp = (int)op.ip[QC_Y_WP];
  p.y_pt = (int)op.ip[QC_Y_PT];
  p.y_pl = (int)op.ip[QC_Y_PL];
  p.y_signed = (int)op.ip[QC_Y_SIGNED];
  p.has_add = (int)op.ip[QC_HAS_ADD];
  p.c_scale = (float)op.fp[QCF_C_SCALE];
  p.r_scale = (float)op.fp[QCF_R_SCALE];
  p.add_scale = (float)op.fp[QCF_ADD_SCALE];
  p.add_zero = (float)op.ip[QC_ADD_ZERO];
  p.c_zero = (int)op.ip[QC_C_ZERO];
  p.r_zero = (int)op.ip[QC_R_ZERO];
  p.r_xor = (int)op.ip[QC_R_XOR];
  p.r_signed = (int)op.ip[QC_R_SIGNED];
  p.r_hp = (int)op.ip[QC_R_HP];
  p.r_wp = (int)op.ip[QC_R_WP];
  p.r_pt = (int)op.ip[QC_R_PT];
  p.r_pl = (int)op.ip[QC_R_PL];
  p.add_signed = (int)op.ip[QC_ADD_SIGNED];
  if (p.n_tiles <= 0) return 0;
  const int grid = p.n_tiles < ctx.num_sms ? p.n_tiles : ctx.num_sms;
  kQcVariants[st->variant].fn<<<grid, QC_THREADS, st->smem_bytes, ctx.stream>>>(st->tmap, p);
  ++*launches;
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ NCHW -> padded NHWC
// One block per (image, input row).  Coalesced row reads, coalesced pixel writes.
__global__ void pad_nhwc_kernel(const uint8_t* __restrict__ x, uint8_t* __restrict__ y, int c, int h, int w, int pt,
                                int pl, int hp, int wp, uint32_t xr) {
  extern __shared__ uint8_t s[];
  const int row = blockIdx.x, n = blockIdx.y;
  const uint8_t* src = x + ((size_t)n * c * h + row) * w;
  for (int i = threadIdx.x; i < c * w; i += blockDim.x) {
    const int ch = i / w, col = i - ch * w;
    s[col * c + ch] = src[(size_t)ch * h * w + col] ^ (uint8_t)xr;
  }
  __syncthreads();
  uint8_t* dst = y + (((size_t)n * hp + row + pt) * wp + pl) * c;
  if ((c & 15) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(s);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int i = threadIdx.x; i < c * w / 16; i += blockDim.x) d4[i] = s4[i];
  } else {
    for (int i = threadIdx.x; i < c * w; i += blockDim.x) dst[i] = s[i];
  }
}

int launch_pad_nhwc(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int c = (int)op.ip[PAD_C], h = (int)op.ip[PAD_H], w = (int)op.ip[PAD_W];
  const size_t smem = (size_t)c * w;
  if (smem > 48 * 1024) return 5;
  dim3 grid((unsigned)h, (unsigned)eff_batch(ctx, op.ip[PAD_N]));
  pad_nhwc_kernel<<<grid, 256, smem, ctx.stream>>>((const uint8_t*)ptrs[op.t[0]], (uint8_t*)ptrs[op.t[1]], c, h, w,
                                                   (int)op.ip[PAD_TOP], (int)op.ip[PAD_LEFT], (int)op.ip[PAD_HP],
                                                   (int)op.ip[PAD_WP], (uint32_t)op.ip[PAD_XOR]);
  ++*launches;
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

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

__global__ void qconv_generic_kernel(const QConvGenericParams p) {
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
    p.y[idx] = (uint8_t)requant(acc, scale, (float)p.y_zero, p.y_signed);
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
  p.n = (int)eff_batch(ctx, op.ip[QG_N]);
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
  qconv_generic_kernel<<<blocks, 256, 0, ctx.stream>>>(p);
  ++*launches;
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ QLinearAdd (same shape)
__global__ void qlinear_add_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b,
                                   uint8_t* __restrict__ y, int64_t count, int as, int bs, int ys_signed, int az,
                                   int bz, float sa, float sb, float sy, float yz) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = (uint8_t)qadd(load_8bit(a[i], as), az, sa, load_8bit(b[i], bs), bz, sb, sy, yz, ys_signed);
  }
}

int launch_qlinear_add(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t full_batch = op.ip[QA_BATCH] > 0 ? op.ip[QA_BATCH] : 1;
  const int64_t count = op.ip[QA_COUNT] / full_batch * (op.ip[QA_BATCH] > 0 ? eff_batch(ctx, full_batch) : 1);
  if (count == 0) return 0;
  const int64_t blocks64 = (count + 255) / 256;
  const int blocks = (int)(blocks64 < 148 * 64 ? blocks64 : 148 * 64);
  qlinear_add_kernel<<<blocks, 256, 0, ctx.stream>>>(
      (const uint8_t*)ptrs[op.t[0]], (const uint8_t*)ptrs[op.t[1]], (uint8_t*)ptrs[op.t[2]], count,
      (int)op.ip[QA_A_SIGNED], (int)op.ip[QA_B_SIGNED], (int)op.ip[QA_Y_SIGNED], (int)op.ip[QA_A_ZERO],
      (int)op.ip[QA_B_ZERO], (float)op.fp[QAF_A_SCALE], (float)op.fp[QAF_B_SCALE], (float)op.fp[QAF_Y_SCALE],
      (float)op.ip[QA_Y_ZERO]);
  ++*launches;
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

}  // namespace emx
