// QLinearConv (+ fused QLinearAdd) on tcgen05 kind::i8, for the int8
// ResNet-style stacks: stride 1, dilation 1, group 1, C in {32,64,128}.
//
// Reference arithmetic (src/emx_onnx_cgen/templates/qlinear_conv_op.c.j2:1-45,
// qlinear_add_op.c.j2:1-21, ir/ops/nn.py:4875-4951):
//   acc   = bias[oc] + sum over in-bounds taps (x - zx) * (w - zw)      (int32)
//   scale = ((float)xs * (float)ws[oc]) / (float)ys
//   y     = clamp((float)(nearbyint((double)((float)acc * scale)) + zy))
//   add   = clamp(nearbyintf(((float)(a-za)*sa + (float)(b-zb)*sb) / ys + zy))
// Integer accumulation is exact in any order, so the tensor cores reproduce
// acc exactly; the epilogue repeats the float steps one rounding at a time
// (qmath.cuh).
//
// Activation layout between these kernels: "swizzled NHWC, zero-bordered":
// [rows][C bytes], row = n*Hp*Wp + hp*Wp + wp over the image padded by the
// conv's pads (Hp = H+pads, Wp = W+pads), plus a tail of spare rows.  Inside a
// row the 16-byte channel chunks are permuted by the tensor-core swizzle of a
// C-byte row (swz_chunk in tc100.cuh).  Border rows are zero, never written.
//   * Output pixel (oh, ow) of image n is the "pitched" row q = n*Hp*Wp +
//     oh*Wp + ow; tap (kh, kw) reads input row q + kh*Wp + kw.  A tile of 128
//     consecutive pitched rows therefore reads, for all taps together, the
//     window of 128 + (KH-1)*Wp + KW-1 consecutive rows starting at q0; tap
//     (kh, kw) is the 128-row slice starting kh*Wp + kw rows into it.
//     Pitched rows on pad columns / pad rows give outputs that are discarded.
//   * That window is contiguous: one bulk copy per tile (cp.async.bulk, no
//     tensor map, no multicast) lands it in shared memory already in the
//     swizzled K-major canonical layout (tile starts are multiples of 8 rows
//     and stages are 1024-byte aligned, so the swizzle phase carries over); a
//     tap is a (kh*Wp+kw)*C byte offset of the descriptor start, with the
//     descriptor's base offset carrying the shifted phase.  Bulk copies here
//     have a round trip of ~2 us, so throughput comes from keeping ~120 KB of
//     windows in flight per SM (8 stages of one tile each).  The swizzle keeps
//     the tensor cores' operand reads conflict-free (without it each MMA
//     waited ~5x its math time on shared memory).
//   * each CTA takes a contiguous range of tiles (neighbouring windows share
//     most rows, which stay hot in L2).
//   * zero padding must mean "real zero": for zero point 128 on uint8 storage
//     the producer stores x ^ 0x80 (= x - 128 as int8) and the MMA runs
//     s8 x s8; for zero point 0 the MMA runs on the raw bytes (u8 or s8).
//   * weights (all taps, [tap][C/16][OC][16 B]) stay in shared memory for the
//     CTA's lifetime; the int32 accumulator tile (128 x OC) is double-buffered
//     in TMEM so the epilogue of tile i overlaps the MMAs of tile i+1.
//   * warps: 0 producer, 1 MMA issuer, 2 TMEM owner, 3 idle, 4-19 epilogue
//     (four warps per TMEM lane quarter, each taking a quarter of the OC
//     columns).
#include "host_util.h"
#include "kernels.h"
#include "qmath.cuh"
#include "tc100.cuh"

namespace emx {

struct QConvTcParams {
  const uint8_t* x;
  const uint8_t* w_img;
  const float* scale;
  const int32_t* bias;
  const uint8_t* resid;
  uint8_t* y;
  int* err;
  int64_t x_rows;  // rows allocated in the input
  uint64_t hpwp_mul, wp_mul;  // ceil(2^40 / (Hp*Wp)), ceil(2^40 / Wp)
  int batch, kh, kw, hp, wp, oh, ow;
  int win_rows, stages, n_tiles;
  uint32_t idesc, b_bytes, stage_bytes, win_bytes;
  float y_lo, y_hi, y_m_minus_zero;
  int y_layout, y_xor, y_hp, y_wp, y_pt, y_pl;
  int has_add, fast_div;
  float c_scale, r_scale, add_scale, add_inv_scale, add_zero, c_zero, r_zero, add_lo, add_hi;
  int r_xor, r_signed, r_hp, r_wp, r_pt, r_pl;
  // residual rows of a tile are contiguous when the residual has the input's
  // padded geometry: row q + r_off for pitched row q; they are then staged in
  // shared memory by one bulk copy per tile (r_bulk)
  int r_bulk;
  int64_t r_off;
  // fused add by table: out byte = lut[(conv byte << 8) | residual byte], staged in shared memory
  const uint8_t* lut;
};

constexpr int QC_RSTAGES = 3;  // residual ring depth (tiles)

// Warp roles: warp 0 producer, warps 1..P MMA issuers (one partial
// accumulator each: one issuing thread completes a tcgen05.mma every ~150
// cycles whatever its N, so with N = OC = 64 several issuers keep more of the
// tensor core busy), warp P+1 residual producer, then 16 epilogue warps from
// the next multiple of 4.  P = 4 while 2 tiles x P partials x OC columns fit
// the 512 TMEM columns (OC <= 64), else 2.
constexpr int QC_MMA_WARPS = 4;  // most issuers of any variant
constexpr int QC_EPI_WARPS = 16;
__host__ __device__ constexpr int qc_partials(int oc) { return 2 * QC_MMA_WARPS * oc <= 512 ? QC_MMA_WARPS : 256 / oc; }
__host__ __device__ constexpr int qc_epi_warp0(int oc) { return (qc_partials(oc) + 2 + 3) & ~3; }
__host__ __device__ constexpr int qc_threads(int oc) { return 32 * (qc_epi_warp0(oc) + QC_EPI_WARPS); }
constexpr int QC_TILE_M = 128;

// bytes of a clamped integer-valued float (see float_to_byte): gather the low
// byte of four bit patterns into one word.
__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d) {
  const uint32_t ba = (uint32_t)__float_as_int(__fadd_rn(a, kMagic));
  const uint32_t bb = (uint32_t)__float_as_int(__fadd_rn(b, kMagic));
  const uint32_t bc = (uint32_t)__float_as_int(__fadd_rn(c, kMagic));
  const uint32_t bd = (uint32_t)__float_as_int(__fadd_rn(d, kMagic));
  return __byte_perm(__byte_perm(ba, bb, 0x0040), __byte_perm(bc, bd, 0x0040), 0x5410);
}

// Store G output bytes (G/4 words) of one pixel.
template <int OC, int G>
__device__ __forceinline__ void qc_store(const QConvTcParams& p, const uint32_t (&out)[G / 4], int col0, int n, int oh,
                                         int ow) {
  if (p.y_layout == 0) {
    const int64_t ypix = ((int64_t)n * p.y_hp + oh + p.y_pt) * p.y_wp + ow + p.y_pl;
    uint8_t* row = p.y + (uint64_t)ypix * OC;
    if constexpr (G == 8) {
      *reinterpret_cast<uint2*>(row + 16 * swz_chunk(ypix, col0 / 16, OC) + (col0 % 16)) = make_uint2(out[0], out[1]);
    } else {
#pragma unroll
      for (int c = 0; c < G / 16; ++c)
        *reinterpret_cast<uint4*>(row + 16 * swz_chunk(ypix, col0 / 16 + c, OC)) =
            make_uint4(out[4 * c + 0], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]);
    }
  } else {
    const int64_t plane = (int64_t)p.oh * p.ow;
    uint8_t* yb = p.y + ((int64_t)n * OC + col0) * plane + (int64_t)oh * p.ow + ow;
#pragma unroll
    for (int c = 0; c < G; ++c) yb[(int64_t)c * plane] = (uint8_t)(out[c >> 2] >> (8 * (c & 3)));
  }
}

template <int OC, int G>
__device__ __forceinline__ void qc_load_resid(const QConvTcParams& p, uint32_t (&rb)[G / 4], int col0, int n, int oh,
                                              int ow) {
  const int64_t rpix = ((int64_t)n * p.r_hp + oh + p.r_pt) * p.r_wp + ow + p.r_pl;
  const uint8_t* row = p.resid + (uint64_t)rpix * OC;
  if constexpr (G == 8) {
    const uint2 t = *reinterpret_cast<const uint2*>(row + 16 * swz_chunk(rpix, col0 / 16, OC) + (col0 % 16));
    rb[0] = t.x;
    rb[1] = t.y;
  } else {
#pragma unroll
    for (int c = 0; c < G / 16; ++c) {
      const uint4 t = *reinterpret_cast<const uint4*>(row + 16 * swz_chunk(rpix, col0 / 16 + c, OC));
      rb[4 * c + 0] = t.x;
      rb[4 * c + 1] = t.y;
      rb[4 * c + 2] = t.z;
      rb[4 * c + 3] = t.w;
    }
  }
}

// G consecutive accumulator columns of this warp's 32 TMEM lanes (asynchronous; tmem_wait_ld before use)
template <int G>
__device__ __forceinline__ void qc_tmem_ld(uint32_t taddr, uint32_t (&r)[G]) {
  if constexpr (G == 8) {
    tmem_ld8(taddr, r);
  } else {
#pragma unroll
    for (int c = 0; c < G / 16; ++c) tmem_ld16(taddr + c * 16, *reinterpret_cast<uint32_t(*)[16]>(&r[c * 16]));
  }
}

template <int CIN, int OC>
__global__ void __launch_bounds__(qc_threads(OC), 1) qconv_tc_kernel(const QConvTcParams p) {
  constexpr int KSTEPS = CIN / 32;  // kind::i8 MMAs (K = 32) per tap
  constexpr int G = OC / 4;         // columns per epilogue warp
  // partial accumulators (= issuing warps) per tile: 2 tiles x P x OC <= 512 TMEM columns
  constexpr int P = qc_partials(OC);
  constexpr int QC_RESID_WARP = P + 1;
  constexpr int QC_EPI_WARP0 = qc_epi_warp0(OC);
  constexpr uint32_t TMEM_COLS = 512;
  static_assert(G % 8 == 0, "OC must be a multiple of 32");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_b = smem;
  uint8_t* s_lut = smem + align_up_dev(p.b_bytes, 1024);  // 64 KB when p.lut
  uint8_t* s_a = s_lut + (p.lut ? 65536 : 0);
  float* s_scale = reinterpret_cast<float*>(s_a + (size_t)p.stages * p.stage_bytes);
  int32_t* s_bias = reinterpret_cast<int32_t*>(s_scale + OC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_bias + OC);
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  uint64_t* accf = bars + 2 * p.stages;
  uint64_t* acce = accf + 2;
  uint64_t* bbar = acce + 2;
  uint64_t* drain = bbar + 1;  // one per MMA warp
  uint64_t* rfull = drain + QC_MMA_WARPS;
  uint64_t* rempty = rfull + QC_RSTAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(rempty + QC_RSTAGES);
  // residual ring after the barrier block (16-byte aligned)
  uint8_t* s_r = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tmem_holder + 4) + 127) & ~uintptr_t(127));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_mma = p.kh * p.kw * KSTEPS;   // MMAs per tile
  const int PE = n_mma < P ? n_mma : P;     // partials (and issuing warps) in use
  // contiguous tile range of this CTA
  const int t_begin = (int)((int64_t)blockIdx.x * p.n_tiles / gridDim.x);
  const int t_end = (int)((int64_t)(blockIdx.x + 1) * p.n_tiles / gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], PE);  // one commit per MMA warp
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], PE);
      mbar_init(&acce[a], QC_EPI_WARPS);  // one arrive per epilogue warp
    }
    mbar_init(bbar, 1);
    for (int w = 0; w < QC_MMA_WARPS; ++w) mbar_init(&drain[w], 1);
    for (int r = 0; r < QC_RSTAGES; ++r) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], QC_EPI_WARPS);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp >= QC_EPI_WARP0) {
    for (int i = threadIdx.x - 32 * QC_EPI_WARP0; i < OC; i += 32 * QC_EPI_WARPS) {
      s_scale[i] = p.scale[i];
      s_bias[i] = p.bias[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: weights once, then one window per tile
      mbar_arrive_expect_tx(bbar, p.b_bytes + (p.lut ? 65536u : 0u));
      for (uint32_t off = 0; off < p.b_bytes; off += 16384u) {
        const uint32_t n = min(16384u, p.b_bytes - off);
        bulk_load(s_b + off, p.w_img + off, n, bbar);
      }
      if (p.lut)
        for (uint32_t off = 0; off < 65536u; off += 16384u) bulk_load(s_lut + off, p.lut + off, 16384u, bbar);
      pdl_wait();  // activations come from the preceding kernel
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued = 0, parity_of = 0;  // per stage: window issued, and in which phase
      for (int tile = t_begin; tile < t_end; ++tile) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.err, DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        const int64_t row0 = (int64_t)tile * QC_TILE_M;
        uint8_t* dst = s_a + (size_t)stage * p.stage_bytes;
        if (row0 + p.win_rows > p.x_rows) {  // the plan guarantees this never happens; never read past a plane
          record_error(p.err, DEV_BAD_CONFIG);
          mbar_arrive(&full[stage]);
        } else {
          mbar_arrive_expect_tx(&full[stage], p.win_bytes);
          bulk_load(dst, p.x + (uint64_t)row0 * CIN, p.win_bytes, &full[stage]);
        }
        issued |= 1u << stage;
        parity_of = (parity_of & ~(1u << stage)) | (phase << stage);
        if (++stage == p.stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {  // error path: let every window this thread issued land before the CTA exits
        for (int s2 = 0; s2 < p.stages; ++s2)
          if (issued & (1u << s2)) (void)mbar_wait(&full[s2], (parity_of >> s2) & 1u, nullptr, 0);
      }
    }
  } else if (warp >= 1 && warp <= PE) {
    if (lane == 0) {
      // ---------------- MMA issuers: warp 1+j issues MMAs k = j, j+P, j+2P, ...
      // of every tile into partial accumulator j
      const int my = warp - 1;
      bool ok = mbar_wait(bbar, 0, p.err, DEV_TIMEOUT_MMA);
      tc_fence_after();
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      const uint32_t a_base = smem_u32(s_a);
      const uint32_t b_base = smem_u32(s_b);
      for (int tile = t_begin; tile < t_end && ok; ++tile, ++it) {
        const int acc = it & 1;
        if (!mbar_wait(&acce[acc], ((it >> 1) & 1) ^ 1u, p.err, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&full[stage], phase, p.err, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // MMA number k of the tile accumulates into partial k % P (integer
        // partial sums are exact in any order; the epilogue adds the P
        // partials), issued by warp 1 + k % P.
        const uint32_t d_tmem = tmem_base + (uint32_t)((acc * P + my) * OC);
        const uint32_t a_stage = a_base + (uint32_t)stage * p.stage_bytes;
        for (int k = my; k < n_mma; k += PE) {
          const int tap = k / KSTEPS, s = k - tap * KSTEPS;
          const int kh = tap / p.kw, kw = tap - kh * p.kw;
          const uint32_t a_tap = a_stage + (uint32_t)(kh * p.wp + kw) * CIN;
          const uint32_t b_tap = b_base + (uint32_t)tap * (OC * CIN);
          const uint64_t adesc = smem_desc_k_swizzled(a_tap + 32u * s, CIN);
          const uint64_t bdesc = smem_desc_k_swizzled(b_tap + 32u * s, CIN);
          mma_i8(d_tmem, adesc, bdesc, p.idesc, k >= PE ? 1u : 0u);
        }
        tc_commit(&empty[stage]);
        tc_commit(&accf[acc]);
        if (++stage == p.stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {  // error path: wait for this thread's MMAs before TMEM is released
        tc_commit(&drain[my]);
        (void)mbar_wait(&drain[my], 0, nullptr, 0);
      }
    }
  } else if (warp == QC_RESID_WARP) {
    if (lane == 0 && p.has_add && p.r_bulk) {
      // ---------------- residual producer: the tile's residual rows, one bulk copy each
      pdl_wait();  // the residual may come from the preceding kernel
      int rs = 0;
      uint32_t rph = 0, issued = 0, parity_of = 0;
      bool ok = true;
      const uint32_t rbytes = (uint32_t)QC_TILE_M * OC;
      for (int tile = t_begin; tile < t_end; ++tile) {
        if (!mbar_wait(&rempty[rs], rph ^ 1u, p.err, DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&rfull[rs], rbytes);
        bulk_load(s_r + (size_t)rs * rbytes, p.resid + (uint64_t)((int64_t)tile * QC_TILE_M + p.r_off) * OC, rbytes,
                  &rfull[rs]);
        issued |= 1u << rs;
        parity_of = (parity_of & ~(1u << rs)) | (rph << rs);
        if (++rs == QC_RSTAGES) {
          rs = 0;
          rph ^= 1u;
        }
      }
      if (!ok)
        for (int s2 = 0; s2 < QC_RSTAGES; ++s2)
          if (issued & (1u << s2)) (void)mbar_wait(&rfull[s2], (parity_of >> s2) & 1u, nullptr, 0);
    }
  } else if (warp >= QC_EPI_WARP0) {
    // ---------------- epilogue: TMEM -> registers -> requant (+ QLinearAdd) -> global
    const int quarter = warp & 3;
    const int col0 = ((warp - QC_EPI_WARP0) >> 2) * G;
    const int row = quarter * 32 + lane;
    const int64_t hpwp = (int64_t)p.hp * p.wp;
    const uint32_t yx4 = (uint32_t)p.y_xor * 0x01010101u;
    pdl_wait();  // residual reads and output writes follow the preceding kernel
    if (p.lut && !__all_sync(0xffffffffu, mbar_wait(bbar, 0, p.err, DEV_TIMEOUT_EPILOGUE))) {
      // the add table never arrived (an error is recorded); nothing to do
    } else {
    int it = 0;
    for (int tile = t_begin; tile < t_end; ++tile, ++it) {
      __syncwarp();
      const int acc = it & 1;
      bool ok = mbar_wait(&accf[acc], (it >> 1) & 1, p.err, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      // the PE partial accumulators in use (PE >= 1), summed as they arrive
      uint32_t v[G];
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * P * OC + col0);
      {
        uint32_t t[G];
        qc_tmem_ld<G>(taddr, v);
        if (PE > 1) qc_tmem_ld<G>(taddr + OC, t);
        tmem_wait_ld();
        if (PE > 1) {
#pragma unroll
          for (int c = 0; c < G; ++c) v[c] += t[c];
        }
      }
#pragma unroll
      for (int pp = 2; pp < P; pp += 2) {
        if (pp < PE) {
          uint32_t t0[G], t1[G];
          qc_tmem_ld<G>(taddr + pp * OC, t0);
          if (pp + 1 < PE) qc_tmem_ld<G>(taddr + (pp + 1) * OC, t1);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < G; ++c) v[c] += pp + 1 < PE ? t0[c] + t1[c] : t0[c];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[acc]);
      const bool rb_on = p.has_add && p.r_bulk;
      const int rs = it % QC_RSTAGES;
      if (rb_on) {
        ok = mbar_wait(&rfull[rs], (uint32_t)(it / QC_RSTAGES) & 1u, p.err, DEV_TIMEOUT_EPILOGUE);
        if (!__all_sync(0xffffffffu, ok)) break;
      }

      // pixel of pitched row q: divisions by Hp*Wp and Wp as multiply-shift
      // with host-computed ceil(2^40 / d) (exact for q * d < 2^40, checked on the host)
      const uint32_t q = (uint32_t)tile * QC_TILE_M + (uint32_t)row;
      const int n = (int)(((uint64_t)q * p.hpwp_mul) >> 40);
      const int rem = (int)(q - (uint32_t)n * (uint32_t)hpwp);
      const int oh = (int)(((uint64_t)(uint32_t)rem * p.wp_mul) >> 40);
      const int ow = rem - oh * p.wp;
      if (n < p.batch && oh < p.oh && ow < p.ow) {
      float r[G];
#pragma unroll
      for (int c4 = 0; c4 < G / 4; ++c4) {
        const float4 sc = *reinterpret_cast<const float4*>(&s_scale[col0 + 4 * c4]);
        const int4 bi = *reinterpret_cast<const int4*>(&s_bias[col0 + 4 * c4]);
        r[4 * c4 + 0] = requant_fast((int32_t)v[4 * c4 + 0] + bi.x, sc.x, p.y_m_minus_zero, p.y_lo, p.y_hi);
        r[4 * c4 + 1] = requant_fast((int32_t)v[4 * c4 + 1] + bi.y, sc.y, p.y_m_minus_zero, p.y_lo, p.y_hi);
        r[4 * c4 + 2] = requant_fast((int32_t)v[4 * c4 + 2] + bi.z, sc.z, p.y_m_minus_zero, p.y_lo, p.y_hi);
        r[4 * c4 + 3] = requant_fast((int32_t)v[4 * c4 + 3] + bi.w, sc.w, p.y_m_minus_zero, p.y_lo, p.y_hi);
      }
      if (p.has_add) {
        uint32_t rb[G / 4];
        if (p.r_bulk) {
          const uint8_t* rrow = s_r + ((size_t)rs * QC_TILE_M + row) * OC;
          const int64_t rpix = (int64_t)q + p.r_off;
          if constexpr (G == 8) {
            const uint2 t = *reinterpret_cast<const uint2*>(rrow + 16 * swz_chunk(rpix, col0 / 16, OC) + (col0 % 16));
            rb[0] = t.x;
            rb[1] = t.y;
          } else {
#pragma unroll
            for (int c = 0; c < G / 16; ++c) {
              const uint4 t = *reinterpret_cast<const uint4*>(rrow + 16 * swz_chunk(rpix, col0 / 16 + c, OC));
              rb[4 * c + 0] = t.x;
              rb[4 * c + 1] = t.y;
              rb[4 * c + 2] = t.z;
              rb[4 * c + 3] = t.w;
            }
          }
        } else {
          qc_load_resid<OC, G>(p, rb, col0, n, oh, ow);
        }
        if (p.lut) {
          // out byte = table[(conv byte << 8) | residual byte]
          uint32_t out[G / 4];
#pragma unroll
          for (int c4 = 0; c4 < G / 4; ++c4) {
            uint32_t word = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int c = 4 * c4 + j;
              const uint32_t ab = float_to_byte(r[c]);
              const uint32_t bb = ((rb[c >> 2] >> (8 * (c & 3))) ^ (uint32_t)p.r_xor) & 0xFFu;
              word |= (uint32_t)s_lut[(ab << 8) | bb] << (8 * j);
            }
            out[c4] = word ^ yx4;
          }
          qc_store<OC, G>(p, out, col0, n, oh, ow);
          goto tile_done;
        }
        if (p.fast_div) {
#pragma unroll
          for (int c = 0; c < G; ++c) {
            const int rv = load_8bit(((rb[c >> 2] >> (8 * (c & 3))) ^ (uint32_t)p.r_xor) & 0xFFu, p.r_signed);
            r[c] = qadd_fast<true>(r[c], p.c_zero, p.c_scale, rv, p.r_zero, p.r_scale, p.add_scale, p.add_inv_scale,
                                   p.add_zero, p.add_lo, p.add_hi);
          }
        } else {
#pragma unroll
          for (int c = 0; c < G; ++c) {
            const int rv = load_8bit(((rb[c >> 2] >> (8 * (c & 3))) ^ (uint32_t)p.r_xor) & 0xFFu, p.r_signed);
            r[c] = qadd_fast<false>(r[c], p.c_zero, p.c_scale, rv, p.r_zero, p.r_scale, p.add_scale,
                                    p.add_inv_scale, p.add_zero, p.add_lo, p.add_hi);
          }
        }
      }
      uint32_t out[G / 4];
#pragma unroll
      for (int c4 = 0; c4 < G / 4; ++c4)
        out[c4] = pack4(r[4 * c4 + 0], r[4 * c4 + 1], r[4 * c4 + 2], r[4 * c4 + 3]) ^ yx4;
      qc_store<OC, G>(p, out, col0, n, oh, ow);
      }
    tile_done:
      if (rb_on) {  // this warp is done with the tile's residual rows
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[rs]);
      }
    }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Exhaustive check, for one fused QLinearAdd, that the refined-reciprocal
// division gives the same output byte as __fdiv_rn for every (conv value,
// residual byte) pair.  mismatch[0] counts differing pairs.
__global__ void qadd_fastdiv_check_kernel(QConvTcParams p, int* mismatch) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 65536) return;
  const int a8 = i >> 8, r8 = i & 255;
  const float cv = p.y_lo < 0.0f ? (float)(int8_t)a8 : (float)a8;  // conv output value (already clamped)
  const int r = load_8bit((uint32_t)r8, p.r_signed);
  const float f = qadd_fast<true>(cv, p.c_zero, p.c_scale, r, p.r_zero, p.r_scale, p.add_scale, p.add_inv_scale,
                                  p.add_zero, p.add_lo, p.add_hi);
  const int e = qadd_exact((int)cv, (int)p.c_zero, p.c_scale, r, (int)p.r_zero, p.r_scale, p.add_scale, p.add_zero,
                           p.add_lo < 0.0f);
  if ((int)f != e) atomicAdd(mismatch, 1);
}

// ------------------------------------------------------------------ host side
struct QConvTcState {
  int variant;
  int resid_ring;  // stage the fused add's residual rows in shared memory
  int use_lut;     // stage the fused add's table in shared memory
  int stages;
  int win_rows;
  int fast_div;
  uint32_t stage_bytes, win_bytes, b_bytes;
  size_t smem_bytes;
};
static_assert(sizeof(QConvTcState) <= sizeof(OpState), "state fits");

typedef void (*QcKernel)(const QConvTcParams);
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

static size_t qconv_smem_bytes(uint32_t b_bytes, int stages, uint32_t stage_bytes, int oc, bool resid_ring,
                               bool lut) {
  size_t s = 1024;  // alignment slack
  s += align_up(b_bytes, 1024) + (lut ? 65536 : 0);
  s += (size_t)stages * stage_bytes;
  s += (size_t)oc * 8;
  s += (size_t)(2 * stages + 5 + QC_MMA_WARPS + 2 * QC_RSTAGES) * 8 + 16;
  if (resid_ring) s += 128 + (size_t)QC_RSTAGES * QC_TILE_M * oc;
  return s;
}

static void fill_params(QConvTcParams& p, const PlanOp& op, void* const* ptrs, const QConvTcState* st,
                        int64_t batch) {
  const int oc = (int)op.ip[QC_OC];
  p.x = (const uint8_t*)ptrs[op.t[0]];
  p.w_img = (const uint8_t*)ptrs[op.t[1]];
  p.scale = (const float*)ptrs[op.t[2]];
  p.bias = (const int32_t*)((const float*)ptrs[op.t[2]] + oc);
  p.resid = op.t[3] >= 0 ? (const uint8_t*)ptrs[op.t[3]] : nullptr;
  p.y = (uint8_t*)ptrs[op.t[4]];
  p.x_rows = op.ip[QC_X_ROWS];
  p.batch = (int)batch;
  p.kh = (int)op.ip[QC_KH];
  p.kw = (int)op.ip[QC_KW];
  p.hp = (int)op.ip[QC_HP];
  p.wp = (int)op.ip[QC_WP];
  p.oh = (int)op.ip[QC_OH];
  p.ow = (int)op.ip[QC_OW];
  p.win_rows = st->win_rows;
  p.stages = st->stages;
  const uint64_t hpwp = (uint64_t)p.hp * (uint64_t)p.wp;
  p.hpwp_mul = ((1ull << 40) + hpwp - 1) / hpwp;
  p.wp_mul = ((1ull << 40) + (uint64_t)p.wp - 1) / (uint64_t)p.wp;
  const int64_t q_end = (batch - 1) * p.hp * p.wp + (int64_t)(p.oh - 1) * p.wp + p.ow;  // one past last valid
  p.n_tiles = batch > 0 ? (int)((q_end + QC_TILE_M - 1) / QC_TILE_M) : 0;
  p.idesc = make_idesc(2u, op.ip[QC_A_SIGNED] ? 1u : 0u, 1u, 128u, (uint32_t)oc);
  p.b_bytes = st->b_bytes;
  p.stage_bytes = st->stage_bytes;
  p.win_bytes = st->win_bytes;
  const bool ys = op.ip[QC_Y_SIGNED] != 0;
  p.y_lo = ys ? -128.0f : 0.0f;
  p.y_hi = ys ? 127.0f : 255.0f;
  p.y_m_minus_zero = kMagic - (float)op.ip[QC_Y_ZERO];
  p.y_layout = (int)op.ip[QC_Y_LAYOUT];
  p.y_xor = (int)op.ip[QC_Y_XOR];
  p.y_hp = (int)op.ip[QC_Y_HP];
  p.y_wp = (int)op.ip[QC_Y_WP];
  p.y_pt = (int)op.ip[QC_Y_PT];
  p.y_pl = (int)op.ip[QC_Y_PL];
  p.has_add = (int)op.ip[QC_HAS_ADD];
  p.fast_div = st->fast_div;
  p.c_scale = (float)op.fp[QCF_C_SCALE];
  p.r_scale = (float)op.fp[QCF_R_SCALE];
  p.add_scale = (float)op.fp[QCF_ADD_SCALE];
  p.add_inv_scale = p.has_add ? 1.0f / p.add_scale : 0.0f;
  p.add_zero = (float)op.ip[QC_ADD_ZERO];
  p.c_zero = (float)op.ip[QC_C_ZERO];
  p.r_zero = (float)op.ip[QC_R_ZERO];
  const bool as = op.ip[QC_ADD_SIGNED] != 0;
  p.add_lo = as ? -128.0f : 0.0f;
  p.add_hi = as ? 127.0f : 255.0f;
  p.r_xor = (int)op.ip[QC_R_XOR];
  p.r_signed = (int)op.ip[QC_R_SIGNED];
  p.r_hp = (int)op.ip[QC_R_HP];
  p.r_wp = (int)op.ip[QC_R_WP];
  p.r_pt = (int)op.ip[QC_R_PT];
  p.r_pl = (int)op.ip[QC_R_PL];
  // residual rows of a tile are contiguous when the residual's padded geometry equals the input's
  p.lut = st->use_lut && op.t[5] >= 0 ? (const uint8_t*)ptrs[op.t[5]] : nullptr;
  p.r_bulk = 0;
  p.r_off = 0;
  if (p.has_add && st->resid_ring && p.r_hp == p.hp && p.r_wp == p.wp) {
    p.r_off = (int64_t)p.r_pt * p.wp + p.r_pl;
    const int64_t last_row = (int64_t)((op.ip[QC_N] * (int64_t)p.hp * p.wp + QC_TILE_M - 1) / QC_TILE_M) *
                                 QC_TILE_M + p.r_off;
    p.r_bulk = last_row <= op.ip[QC_R_ROWS] ? 1 : 0;
  }
}

int prepare_qconv_tc(const PlanOp& op, void* const* ptrs, OpState* st_, int device, char* msg, size_t n) {
  QConvTcState* st = reinterpret_cast<QConvTcState*>(st_);
  const int cin = (int)op.ip[QC_CIN], oc = (int)op.ip[QC_OC];
  st->variant = -1;
  for (int i = 0; i < (int)(sizeof(kQcVariants) / sizeof(kQcVariants[0])); ++i)
    if (kQcVariants[i].cin == cin && kQcVariants[i].oc == oc) st->variant = i;
  if (st->variant < 0) return fail(msg, n, 5, "QLinearConv tensor-core path: no variant for C=%d OC=%d", cin, oc);
  const int kw = (int)op.ip[QC_KW], kh = (int)op.ip[QC_KH];
  const int64_t wp = op.ip[QC_WP];
  st->win_rows = (int)align_up((size_t)(QC_TILE_M + (kh - 1) * wp + kw - 1), 8);
  st->win_bytes = (uint32_t)st->win_rows * (uint32_t)cin;
  st->stage_bytes = (uint32_t)align_up(st->win_bytes, 1024);  // stages keep the 1024-byte swizzle alignment
  st->b_bytes = (uint32_t)(kh * kw * cin * oc);
  // pitched-row arithmetic: 32-bit rows and exact multiply-shift division (q * Hp*Wp < 2^40)
  const int64_t hpwp = op.ip[QC_HP] * wp;
  const int64_t q_max = op.ip[QC_N] * hpwp + QC_TILE_M;
  if (q_max >= (1ll << 31) || (double)q_max * (double)hpwp >= (double)(1ull << 40))
    return fail(msg, n, 5, "QLinearConv tensor-core path: %lld pitched rows too many for one launch",
                (long long)q_max);
  // every window the kernel can request must stay inside the input planes
  const int64_t rows_needed = op.ip[QC_N] * op.ip[QC_HP] * wp + st->win_rows;
  if (op.ip[QC_X_ROWS] < rows_needed)
    return fail(msg, n, 2, "input planes have %lld rows, windows need %lld", (long long)op.ip[QC_X_ROWS],
                (long long)rows_needed);
  const size_t budget = 210 * 1024;
  int stages = 8;
  // fused-add helpers in shared memory only where at least 4 window stages remain
  bool lut = op.ip[QC_HAS_ADD] != 0 && op.t[5] >= 0;
  if (lut && qconv_smem_bytes(st->b_bytes, 4, st->stage_bytes, oc, false, true) > budget) lut = false;
  bool ring = op.ip[QC_HAS_ADD] != 0;
  if (ring && qconv_smem_bytes(st->b_bytes, 4, st->stage_bytes, oc, true, lut) > budget) ring = false;
  st->use_lut = lut ? 1 : 0;
  st->resid_ring = ring ? 1 : 0;
  while (stages > 2 && qconv_smem_bytes(st->b_bytes, stages, st->stage_bytes, oc, ring, lut) > budget) --stages;
  st->stages = stages;
  st->smem_bytes = qconv_smem_bytes(st->b_bytes, stages, st->stage_bytes, oc, ring, lut);
  if (st->smem_bytes > 227 * 1024)
    return fail(msg, n, 5, "QLinearConv tensor-core path needs %zu B smem", st->smem_bytes);
  cudaError_t e = cudaFuncSetAttribute(kQcVariants[st->variant].fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)st->smem_bytes);
  if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  st->fast_div = 0;
  if (op.ip[QC_HAS_ADD]) {
    QConvTcParams p{};
    fill_params(p, op, ptrs, st, op.ip[QC_N]);
    int* d_mis = nullptr;
    int mis = -1;
    if (cudaMalloc(&d_mis, sizeof(int)) != cudaSuccess) return fail(msg, n, 7, "check buffer");
    cudaMemset(d_mis, 0, sizeof(int));
    qadd_fastdiv_check_kernel<<<256, 256>>>(p, d_mis);
    e = cudaMemcpy(&mis, d_mis, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(d_mis);
    if (e != cudaSuccess) return fail(msg, n, 4, "fast-division check: %s", cudaGetErrorString(e));
    st->fast_div = mis == 0 ? 1 : 0;
  }
  (void)device;
  return 0;
}

int launch_qconv_tc(const PlanOp& op, void* const* ptrs, const OpState* st_, const LaunchCtx& ctx, int* launches) {
  const QConvTcState* st = reinterpret_cast<const QConvTcState*>(st_);
  QConvTcParams p{};
  fill_params(p, op, ptrs, st, eff_batch(ctx, op, op.ip[QC_N]));
  p.err = ctx.d_error;
  if (p.n_tiles <= 0) return 0;
  const int grid = p.n_tiles < ctx.num_sms ? p.n_tiles : ctx.num_sms;
  cudaError_t e = launch_pdl(kQcVariants[st->variant].fn, dim3(grid), dim3(qc_threads(kQcVariants[st->variant].oc)),
                             st->smem_bytes, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ NCHW -> swizzled NHWC, zero-bordered
// One block per (image, PAD_ROWS_PER_BLOCK input rows).  Phase 1: each warp
// copies whole channel rows (4-byte words when W % 4 == 0) into shared memory
// [rows][C][W+4]; phase 2: thread per (pixel, 4-channel word) packs the word
// and stores it at its swizzled position in the pixel's C-byte row (a warp
// writes whole pixels: contiguous 128-byte runs).  No runtime divisions.
constexpr int PAD_ROWS_PER_BLOCK = 2;

template <int C>
__global__ void __launch_bounds__(256) pad_planar_kernel(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                                                         int h, int w, int pt, int pl, int hp, int wp, uint32_t xr) {
  extern __shared__ __align__(16) uint8_t s[];  // [PAD_ROWS_PER_BLOCK][C][ws]
  constexpr int WPP = C / 4;                    // 4-byte words per pixel
  const int row_base = blockIdx.x * PAD_ROWS_PER_BLOCK, n = blockIdx.y;
  const int ws = (w + 4) & ~3;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  const int rows = min(PAD_ROWS_PER_BLOCK, h - row_base);
  // asynchronous global -> shared copies (no register round trip), all in flight at once
  for (int t = warp; t < rows * C; t += 8) {  // one channel row per warp iteration
    const int r = t / C, ch = t - r * C;      // C is a compile-time power of two
    const uint8_t* src = x + (((size_t)n * C + ch) * h + row_base + r) * w;
    uint8_t* dst = s + (r * C + ch) * ws;
    if ((w & 3) == 0) {
      for (int k = lane; k < (w >> 2); k += 32)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst + 4 * k)), "l"(src + 4 * k)
                     : "memory");
    } else {
      for (int k = lane; k < w; k += 32) dst[k] = src[k];
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const uint32_t x4 = xr * 0x01010101u;
  for (int i = threadIdx.x; i < rows * w * WPP; i += 256) {
    const int g4 = i % WPP, pix = i / WPP;  // compile-time power-of-two divisor
    const int r = pix / w, col = pix - r * w;
    const uint8_t* sc = s + (r * C + 4 * g4) * ws + col;
    const uint32_t word =
        __byte_perm(__byte_perm(sc[0], sc[ws], 0x0040), __byte_perm(sc[2 * ws], sc[3 * ws], 0x0040), 0x5410) ^ x4;
    const int64_t g = ((int64_t)n * hp + row_base + r + pt) * wp + pl + col;
    *reinterpret_cast<uint32_t*>(y + (uint64_t)g * C + 16 * swz_chunk(g, g4 >> 2, C) + 4 * (g4 & 3)) = word;
  }
}

// Widths that are multiples of 4 (the common case): no shared memory.  One
// thread per (image, row, 4-pixel quad, 16-channel chunk) loads the 16
// channel words (4 pixels each) straight from NCHW -- a warp covers 8 quads x
// 4 chunks, so every channel row is read as 32 contiguous bytes -- turns them
// into 4 pixels x 16 channels with 4x4 byte transposes (8 PRMT each) and
// stores each pixel's 16-byte chunk at its swizzled position.
template <int C>
__global__ void __launch_bounds__(256) pad_planar_q4_kernel(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                                                            int n_img, int h, int w, int pt, int pl, int hp, int wp,
                                                            uint32_t xr) {
  constexpr int CG = C / 16;
  pdl_wait();
  pdl_launch_dependents();
  const int wq = w >> 2;
  const int64_t items = (int64_t)n_img * h * wq * CG;
  const uint32_t x4 = xr * 0x01010101u;
  for (int64_t it = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it < items; it += (int64_t)gridDim.x * blockDim.x) {
    const int cg = (int)(it % CG);
    const int64_t r = it / CG;
    const int pq = (int)(r % wq);
    const int64_t nh = r / wq;  // n * h + row
    const int row = (int)(nh % h), n = (int)(nh / h);
    const uint8_t* src = x + (((int64_t)n * C + 16 * cg) * h + row) * w + 4 * pq;
    const int64_t plane = (int64_t)h * w;
    uint32_t v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = *reinterpret_cast<const uint32_t*>(src + k * plane);
    uint32_t o[4][4];  // [pixel][word of 4 channels]
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // channels 4q .. 4q+3
      const uint32_t t0 = __byte_perm(v[4 * q], v[4 * q + 1], 0x5140), t1 = __byte_perm(v[4 * q], v[4 * q + 1], 0x7362);
      const uint32_t t2 = __byte_perm(v[4 * q + 2], v[4 * q + 3], 0x5140),
                     t3 = __byte_perm(v[4 * q + 2], v[4 * q + 3], 0x7362);
      o[0][q] = __byte_perm(t0, t2, 0x5410) ^ x4;
      o[1][q] = __byte_perm(t0, t2, 0x7632) ^ x4;
      o[2][q] = __byte_perm(t1, t3, 0x5410) ^ x4;
      o[3][q] = __byte_perm(t1, t3, 0x7632) ^ x4;
    }
    const int64_t g0 = ((int64_t)n * hp + row + pt) * wp + pl + 4 * pq;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int64_t g = g0 + p;
      *reinterpret_cast<uint4*>(y + (uint64_t)g * C + 16 * swz_chunk(g, cg, C)) =
          make_uint4(o[p][0], o[p][1], o[p][2], o[p][3]);
    }
  }
}

int launch_pad_nhwc(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int c = (int)op.ip[PAD_C], h = (int)op.ip[PAD_H], w = (int)op.ip[PAD_W];
  if ((w & 3) == 0 && ((uintptr_t)ptrs[op.t[0]] & 3) == 0 && (c == 32 || c == 64 || c == 128)) {
    const int n_img = (int)eff_batch(ctx, op, op.ip[PAD_N]);
    const int64_t items = (int64_t)n_img * h * (w / 4) * (c / 16);
    if (items == 0) return 0;
    const int64_t blocks64 = (items + 255) / 256;
    const int blocks = (int)(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
    auto kq = c == 32 ? pad_planar_q4_kernel<32> : (c == 64 ? pad_planar_q4_kernel<64> : pad_planar_q4_kernel<128>);
    cudaError_t e = launch_pdl(kq, dim3(blocks), dim3(256), 0, ctx.stream, (const uint8_t*)ptrs[op.t[0]],
                               (uint8_t*)ptrs[op.t[1]], n_img, h, w, (int)op.ip[PAD_TOP], (int)op.ip[PAD_LEFT],
                               (int)op.ip[PAD_HP], (int)op.ip[PAD_WP], (uint32_t)op.ip[PAD_XOR]);
    ++*launches;
    return e == cudaSuccess ? 0 : 4;
  }
  const size_t smem = (size_t)PAD_ROWS_PER_BLOCK * c * ((w + 4) & ~3);
  if (smem > 48 * 1024 || (c != 32 && c != 64 && c != 128)) return 5;
  dim3 grid((unsigned)((h + PAD_ROWS_PER_BLOCK - 1) / PAD_ROWS_PER_BLOCK), (unsigned)eff_batch(ctx, op, op.ip[PAD_N]));
  auto kern = c == 32 ? pad_planar_kernel<32> : (c == 64 ? pad_planar_kernel<64> : pad_planar_kernel<128>);
  cudaError_t e = launch_pdl(kern, grid, dim3(256), smem, ctx.stream, (const uint8_t*)ptrs[op.t[0]],
                             (uint8_t*)ptrs[op.t[1]], h, w, (int)op.ip[PAD_TOP], (int)op.ip[PAD_LEFT],
                             (int)op.ip[PAD_HP], (int)op.ip[PAD_WP], (uint32_t)op.ip[PAD_XOR]);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
