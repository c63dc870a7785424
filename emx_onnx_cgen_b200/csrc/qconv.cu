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
//   * each CTA takes every gridDim.x-th tile: in each round the CTAs load
//     consecutive windows, which share most rows (hot in L2).
//   * zero padding must mean "real zero": for zero point 128 on uint8 storage
//     the producer stores x ^ 0x80 (= x - 128 as int8) and the MMA runs
//     s8 x s8; for zero point 0 the MMA runs on the raw bytes (u8 or s8).
//   * weights (all taps, [tap][C/16][OC][16 B]) stay in shared memory for the
//     CTA's lifetime; the int32 accumulator tile (128 x OC) is double-buffered
//     in TMEM so the epilogue of tile i overlaps the MMAs of tile i+1.
//   * warps: 0 producer, 1 MMA issuer, 2 TMEM owner, 3 idle, 4-19 epilogue
//     (four warps per TMEM lane quarter, each taking a quarter of the OC
//     columns).
#include <algorithm>

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
  // chain layer whose output the residual is (its progress is waited for), or
  // -1: a tensor written before the launch
  int r_src;
  // fused add by table: out byte = lut[(conv byte << 8) | residual byte], staged in shared memory
  const uint8_t* lut;
  int rq_int;  // integer requantisation (QC_RQ_INT)
  int rq_sub;  // bits(1.5 * 2^23) - output zero point
};

constexpr int QC_RSTAGES = 3;  // residual ring depth (tiles)

// Warp roles: warp 0 producer, warps 1..P MMA issuers (one partial
// accumulator each: one issuing thread completes a tcgen05.mma every ~150
// cycles whatever its N, so with N = OC = 64 several issuers keep more of the
// tensor core busy), warp P+1 residual producer, then 16 epilogue warps from
// the next multiple of 4, then the chain's progress publisher.  Each waiting
// role has a warp of its own: two lanes of one warp spinning in different
// loops delay each other by microseconds.
constexpr int QC_MMA_WARPS = 4;  // most issuers of any variant
constexpr int QC_EPI_WARPS = 16;
__host__ __device__ constexpr int qc_partials(int oc) { return oc <= 64 ? 2 : 256 / oc; }
__host__ __device__ constexpr int qc_epi_warp0(int oc) { return (qc_partials(oc) + 2 + 3) & ~3; }
__host__ __device__ constexpr int qc_pub_warp(int oc) { return qc_epi_warp0(oc) + QC_EPI_WARPS; }
__host__ __device__ constexpr int qc_threads(int oc) { return 32 * (qc_pub_warp(oc) + 1); }
constexpr int QC_TILE_M = 128;

// A chain of up to QC_MAX_CHAIN convolutions run by one launch (see
// qconv_chain_kernel); layer[0] also carries the geometry every layer shares.
constexpr int QC_MAX_CHAIN = 8;
struct QConvChainParams {
  QConvTcParams layer[QC_MAX_CHAIN];
  int n_layers;
  int use_lut;   // a table buffer is in shared memory
  int use_ring;  // a residual ring is in shared memory
  int dlo, dhi;  // layer l+1's tile t reads rows layer l's tiles t-dlo .. t+dhi write
  int rlo, rhi;  // tile t's residual rows were written by tiles t-rlo .. t+rhi
  unsigned long long* state;  // [0] run epoch, [1] CTAs finished, [2 + t] progress of tile t; null for L = 1
  int* err;
  // failure-detection test hook (emx_b200_set_fault): the publisher never
  // advances the progress words, so the next layer's bounded waits run out
  int drop_progress;
};

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

// Chain progress publisher (one thread): tiles every epilogue warp has
// stored are made visible GPU-wide and their progress words advanced.  One
// fence (which waits for the stores to drain) covers every tile completed
// since the last one, so the fences adapt to the backlog, not the tile count.
__device__ __forceinline__ void qc_publish(const QConvChainParams& cp, const uint32_t* s_stored,
                                           unsigned long long* progress, int n_tiles, int t_first, int t_step) {
  int* const err = cp.err;
  const int L = cp.n_layers;
  pdl_wait();
  const unsigned long long epoch = ld_acquire_u64(cp.state);
  const int per_layer = (n_tiles - t_first + t_step - 1) / t_step;  // tiles of this CTA
  const uint32_t total = (uint32_t)(per_layer * (L - 1));
  uint32_t published = 0;
  uint64_t t_last = globaltimer_ns();
  const uint64_t budget = wait_budget_ns(err);
  uint32_t spins = 0;
  while (published < total) {
    uint32_t done = total;
    for (int w = 0; w < QC_EPI_WARPS; ++w) done = min(done, ld_acquire_cta_u32(&s_stored[w]));
    if (done > published) {
      __threadfence();
      for (uint32_t k = published; k < done; ++k) {
        const int l = (int)(k / (uint32_t)per_layer);
        const int tile = t_first + (int)(k % (uint32_t)per_layer) * t_step;
        if (!cp.drop_progress) st_relaxed_u64(progress + tile, epoch * 64ull + (unsigned)(l + 1));
      }
      published = done;
      t_last = globaltimer_ns();
      continue;
    }
    if ((++spins & 15u) == 0) {
      if (error_raised(err)) break;
      if (globaltimer_ns() - t_last > budget) {
        record_error(err, DEV_TIMEOUT_EPILOGUE);
        break;
      }
    }
    __nanosleep(32);
  }
}

// One launch runs a chain of L convolutions with the same geometry (L = 1:
// a single convolution).  Every CTA owns the same strided set of tiles in
// every layer and walks the items (layer, tile) in order.  Layer l+1's tile t
// reads rows that layer l's tiles t-dlo .. t+dhi write (and residual rows of
// tiles t-rlo .. t+rhi of an earlier layer), so before loading them the
// producer waits until those tiles' progress words say "layer l done";
// the epilogue publishes a tile's progress once all its rows are stored.
// Progress words carry the run's epoch (layers done + 64 * epoch), so no
// reset is needed between runs: the last CTA to finish advances the epoch.
// No layer waits on a later one, and every CTA owns at least one tile (grid
// <= tiles), so the waits form no cycle; all waits are bounded.
template <int CIN, int OC>
__global__ void __launch_bounds__(qc_threads(OC), 1) qconv_chain_kernel(const __grid_constant__ QConvChainParams cp) {
  constexpr int KSTEPS = CIN / 32;  // kind::i8 MMAs (K = 32) per tap
  constexpr int G = OC / 4;         // columns per epilogue warp
  // partial accumulators (= issuing warps) per tile: 2 tiles x P x OC <= 512 TMEM columns
  constexpr int P = qc_partials(OC);
  constexpr int RESID_WARP = P + 1;
  constexpr int EPI_WARP0 = qc_epi_warp0(OC);
  constexpr int PUB_WARP = qc_pub_warp(OC);
  constexpr uint32_t TMEM_COLS = 512;
  static_assert(G % 8 == 0, "OC must be a multiple of 32");
  const QConvTcParams& g = cp.layer[0];  // geometry shared by every layer
  const int L = cp.n_layers;
  const bool chained = cp.state != nullptr;
  int* const err = cp.err;
  // Shared-memory regions are carved out by adding byte offsets to the
  // extern __shared__ array (never through integer casts), so the compiler
  // keeps them in the shared state space: LDS/STS with 32-bit addresses
  // instead of generic loads and stores.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  // weights: one buffer, or two for a chain (layer l uses buffer l & 1, so
  // layer l+1's weights load while layer l's MMAs run)
  const int wbufs = L > 1 ? 2 : 1;
  const uint32_t wbuf_bytes = (uint32_t)align_up_dev(g.b_bytes, 1024);
  uint8_t* s_b = smem;
  uint8_t* s_lut = smem + (size_t)wbufs * wbuf_bytes;  // 64 KB when cp.use_lut
  uint8_t* s_a = s_lut + (cp.use_lut ? 65536 : 0);
  // per epilogue warp, per layer parity: its G scales and biases
  float* s_scale = reinterpret_cast<float*>(s_a + (size_t)g.stages * g.stage_bytes);
  int32_t* s_bias = reinterpret_cast<int32_t*>(s_scale + 2 * QC_EPI_WARPS * G);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_bias + 2 * QC_EPI_WARPS * G);
  uint64_t* full = bars;
  uint64_t* empty = bars + g.stages;
  uint64_t* accf = bars + 2 * g.stages;
  uint64_t* acce = accf + 2;
  uint64_t* bbar = acce + 2;    // [2] weights of a layer landed in buffer b (one phase per layer using b)
  uint64_t* lbar = bbar + 2;    // table of a layer landed (one phase per layer with a table)
  uint64_t* wfree = lbar + 1;   // [2] MMAs of a layer using buffer b done: its weights may be replaced
  // Epilogue warps drift up to two tiles (and two layers) apart, so the
  // barrier they all arrive on per layer is a ring of 4: a fast warp's next
  // arrival never lands in a phase a slow warp still owes.
  uint64_t* lfree = wfree + 2;  // [4] epilogue done with layer l (l % 4): table may be replaced
  uint64_t* drain = lfree + 4;  // one per MMA warp
  uint64_t* rfull = drain + QC_MMA_WARPS;
  uint64_t* rempty = rfull + QC_RSTAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(rempty + QC_RSTAGES);
  // per epilogue warp: how many published tiles it has stored (monotonic; the publisher reads them)
  uint32_t* s_stored = tmem_holder + 4;
  // per MMA k of a tile: offsets of its A (window) and B (weights) operands in
  // 16-byte units, the unit of a descriptor's start-address field
  uint32_t* s_koff = s_stored + QC_EPI_WARPS;  // [2 * MMAs per tile], 8-byte aligned
  // residual ring after that (128-byte aligned)
  uint8_t* s_r = smem + ((uint32_t)(reinterpret_cast<uint8_t*>(s_koff + 2 * g.kh * g.kw * KSTEPS) - smem) + 127u & ~127u);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_mma = g.kh * g.kw * KSTEPS;  // MMAs per tile
  const int PE = n_mma < P ? n_mma : P;    // partials (and issuing warps) in use
  const int n_tiles = g.n_tiles;
  // tiles of this CTA in every layer: blockIdx.x, + gridDim.x, ... (strided, so
  // that a tile's neighbours of the previous layer were done a round earlier
  // by the neighbouring CTAs, and each round's windows are consecutive rows)
  const int t_first = blockIdx.x, t_step = gridDim.x;
  unsigned long long* progress = chained ? cp.state + 2 : nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], PE);  // one commit per MMA warp
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], PE);
      mbar_init(&acce[a], QC_EPI_WARPS);  // one arrive per epilogue warp
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bbar[b], 1);
      mbar_init(&wfree[b], PE);
    }
    mbar_init(lbar, 1);
    for (int r = 0; r < 4; ++r) mbar_init(&lfree[r], QC_EPI_WARPS);
    for (int w = 0; w < QC_EPI_WARPS; ++w) s_stored[w] = 0;
    for (int k = 0; k < g.kh * g.kw * KSTEPS; ++k) {
      const int tap = k / KSTEPS, s = k - tap * KSTEPS;
      const int kh = tap / g.kw, kw = tap - kh * g.kw;
      s_koff[2 * k] = ((uint32_t)(kh * g.wp + kw) * CIN + 32u * s) >> 4;
      s_koff[2 * k + 1] = ((uint32_t)tap * (OC * CIN) + 32u * s) >> 4;
    }
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: weights, tables and one window per tile.
      // Weights of layers 0 and 1 load at once; those of layer l+1 after layer
      // l's windows are issued (into the buffer layer l-1 used).  The table of
      // the next layer with a fused add loads as soon as the epilogue is done
      // with the previous table, at the end of the next layer's windows at the
      // latest (so no barrier runs two phases ahead of its waiter).
      auto issue_weights = [&](int l) {
        const int b = l & 1;
        mbar_arrive_expect_tx(&bbar[b], g.b_bytes);
        for (uint32_t off = 0; off < g.b_bytes; off += 16384u)
          bulk_load(s_b + (size_t)b * wbuf_bytes + off, cp.layer[l].w_img + off, min(16384u, g.b_bytes - off),
                    &bbar[b]);
      };
      auto next_lut_layer = [&](int from) {
        for (int m = from; m < L; ++m)
          if (cp.layer[m].lut) return m;
        return L;
      };
      auto issue_lut = [&](int m) {
        mbar_arrive_expect_tx(lbar, 65536u);
        for (uint32_t off = 0; off < 65536u; off += 16384u) bulk_load(s_lut + off, cp.layer[m].lut + off, 16384u, lbar);
      };
      int w_issued = 0, luts = 0;  // weight loads and tables issued so far
      issue_weights(0);
      ++w_issued;
      if (L > 1) {
        issue_weights(1);
        ++w_issued;
      }
      int lut_prev = next_lut_layer(0);  // layer whose table is (being) loaded
      if (lut_prev < L) {
        issue_lut(lut_prev);
        ++luts;
      }
      int lut_next = lut_prev < L ? next_lut_layer(lut_prev + 1) : L;
      pdl_wait();  // activations come from the preceding kernel
      const unsigned long long epoch = chained ? ld_acquire_u64(cp.state) : 0ull;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued = 0, parity_of = 0;  // per stage: window issued, and in which phase
      for (int l = 0; l < L && ok; ++l) {
        const QConvTcParams& lp = cp.layer[l];
        for (int tile = t_first; tile < n_tiles; tile += t_step) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (chained && l > 0) {  // the rows of this window are layer l-1 outputs of neighbouring tiles
            if (!wait_flags_at_least(progress, tile - cp.dlo, tile + cp.dhi, n_tiles, epoch * 64ull + (unsigned)l,
                                     err, DEV_TIMEOUT_GRID)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
          }
          const int64_t row0 = (int64_t)tile * QC_TILE_M;
          uint8_t* dst = s_a + (size_t)stage * g.stage_bytes;
          if (row0 + g.win_rows > lp.x_rows) {  // the plan guarantees this never happens; never read past a plane
            record_error(err, DEV_BAD_CONFIG);
            mbar_arrive(&full[stage]);
          } else {
            mbar_arrive_expect_tx(&full[stage], g.win_bytes);
            bulk_load(dst, lp.x + (uint64_t)row0 * CIN, g.win_bytes, &full[stage]);
          }
          issued |= 1u << stage;
          parity_of = (parity_of & ~(1u << stage)) | (phase << stage);
          if (++stage == g.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (l + 1 < L && l + 1 >= 2) {  // buffer (l+1) & 1 is free once layer l-1's MMAs are done
          if (!mbar_wait(&wfree[(l + 1) & 1], (uint32_t)((l - 1) >> 1) & 1u, err, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          issue_weights(l + 1);
          ++w_issued;
        }
        if (lut_next < L && (l >= lut_prev + 1 || lut_next == l + 1)) {
          if (!mbar_wait(&lfree[lut_prev & 3], (uint32_t)(lut_prev >> 2) & 1u, err, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          issue_lut(lut_next);
          ++luts;
          lut_prev = lut_next;
          lut_next = next_lut_layer(lut_prev + 1);
        }
      }
      if (!ok) {  // error path: let every copy this thread issued land before the CTA exits
        for (int s2 = 0; s2 < g.stages; ++s2)
          if (issued & (1u << s2)) (void)mbar_wait(&full[s2], (parity_of >> s2) & 1u, nullptr, 0);
        for (int k = w_issued - 2 < 0 ? 0 : w_issued - 2; k < w_issued; ++k)
          (void)mbar_wait(&bbar[k & 1], (uint32_t)(k >> 1) & 1u, nullptr, 0);
        if (luts > 0) (void)mbar_wait(lbar, (uint32_t)(luts - 1) & 1u, nullptr, 0);
      }
    }
  } else if (warp >= 1 && warp <= PE) {
    if (lane == 0) {
      // ---------------- MMA issuers: warp 1+j issues MMAs k = j, j+P, j+2P, ...
      // of every tile into partial accumulator j
      const int my = warp - 1;
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      const uint32_t a_base = smem_u32(s_a);
      for (int l = 0; l < L && ok; ++l) {
        const uint32_t idesc = cp.layer[l].idesc;
        const int wb = wbufs == 2 ? (l & 1) : 0;
        const uint64_t b_desc0 = smem_desc_k_swizzled(smem_u32(s_b + (size_t)wb * wbuf_bytes), CIN);
        if (!mbar_wait(&bbar[wb], (uint32_t)(wbufs == 2 ? (l >> 1) : l) & 1u, err, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int tile = t_first; tile < n_tiles; tile += t_step, ++it) {
          const int acc = it & 1;
          if (!mbar_wait(&acce[acc], ((it >> 1) & 1) ^ 1u, err, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&full[stage], phase, err, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // MMA number k of the tile accumulates into partial k % P (integer
          // partial sums are exact in any order; the epilogue adds the P
          // partials), issued by warp 1 + k % P.
          // An operand's descriptor is its base's plus the operand offset: the
          // start-address field holds address >> 4 in 14 bits and every shared
          // address stays below 256 KB, so the sum never carries out of the field.
          const uint32_t d_tmem = tmem_base + (uint32_t)((acc * P + my) * OC);
          const uint64_t a_desc0 = smem_desc_k_swizzled(a_base + (uint32_t)stage * g.stage_bytes, CIN);
          for (int k = my; k < n_mma; k += PE) {
            const uint2 o = *reinterpret_cast<const uint2*>(&s_koff[2 * k]);
            mma_i8(d_tmem, a_desc0 + o.x, b_desc0 + o.y, idesc, k >= PE ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          tc_commit(&accf[acc]);
          if (++stage == g.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) tc_commit(&wfree[wb]);  // arrives once this warp's MMAs of layer l have read the weights
      }
      if (!ok) {  // error path: wait for this thread's MMAs before TMEM is released
        tc_commit(&drain[my]);
        (void)mbar_wait(&drain[my], 0, nullptr, 0);
      }
    }
  } else if (warp == PUB_WARP) {
    if (lane == 0 && chained && L > 1) qc_publish(cp, s_stored, progress, n_tiles, t_first, t_step);
  } else if (warp == RESID_WARP) {
    if (lane == 0 && cp.use_ring) {
      // ---------------- residual producer: the tile's residual rows, one bulk copy each
      pdl_wait();  // the residual may come from the preceding kernel
      const unsigned long long epoch = chained ? ld_acquire_u64(cp.state) : 0ull;
      int rs = 0;
      uint32_t rph = 0, issued = 0, parity_of = 0;
      bool ok = true;
      const uint32_t rbytes = (uint32_t)QC_TILE_M * OC;
      for (int l = 0; l < L && ok; ++l) {
        const QConvTcParams& lp = cp.layer[l];
        if (!(lp.has_add && lp.r_bulk)) continue;
        for (int tile = t_first; tile < n_tiles; tile += t_step) {
          if (!mbar_wait(&rempty[rs], rph ^ 1u, err, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (chained && lp.r_src >= 0) {  // the residual is layer r_src's output: wait for those rows
            if (!wait_flags_at_least(progress, tile - cp.rlo, tile + cp.rhi, n_tiles,
                                     epoch * 64ull + (unsigned)(lp.r_src + 1), err, DEV_TIMEOUT_GRID)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
          }
          mbar_arrive_expect_tx(&rfull[rs], rbytes);
          bulk_load(s_r + (size_t)rs * rbytes, lp.resid + (uint64_t)((int64_t)tile * QC_TILE_M + lp.r_off) * OC,
                    rbytes, &rfull[rs]);
          issued |= 1u << rs;
          parity_of = (parity_of & ~(1u << rs)) | (rph << rs);
          if (++rs == QC_RSTAGES) {
            rs = 0;
            rph ^= 1u;
          }
        }
      }
      if (!ok)
        for (int s2 = 0; s2 < QC_RSTAGES; ++s2)
          if (issued & (1u << s2)) (void)mbar_wait(&rfull[s2], (parity_of >> s2) & 1u, nullptr, 0);
    }
  } else if (warp >= EPI_WARP0 && warp < PUB_WARP) {
    // ---------------- epilogue: TMEM -> registers -> requant (+ QLinearAdd) -> global
    const int ew = warp - EPI_WARP0;
    const int quarter = warp & 3;
    const int col0 = (ew >> 2) * G;
    const int row = quarter * 32 + lane;
    // geometry shared by every layer, in registers
    const uint32_t hpwp = (uint32_t)g.hp * (uint32_t)g.wp;
    const uint64_t hpwp_mul = g.hpwp_mul, wp_mul = g.wp_mul;
    const int gwp = g.wp, gbatch = g.batch, goh = g.oh, gow = g.ow;
    auto fetch_consts = [&](int l) {  // this warp's slice of layer l's scales and biases, parity l & 1
      if (lane < G) {
        cp_async4(s_scale + ((l & 1) * QC_EPI_WARPS + ew) * G + lane, cp.layer[l].scale + col0 + lane);
        cp_async4(s_bias + ((l & 1) * QC_EPI_WARPS + ew) * G + lane, cp.layer[l].bias + col0 + lane);
      }
      cp_async_commit();
    };
    fetch_consts(0);  // plan constants: not written by the preceding kernel
    if (L > 1) fetch_consts(1);
    pdl_wait();  // residual reads and output writes follow the preceding kernel
    int it = 0, rit = 0, luts = 0;
    uint32_t pub = 0;
    bool ok = true;
    bool pend = false;  // a stored tile not yet published
    for (int l = 0; l < L && ok; ++l) {
      // Layer constants, read once per layer: the layer table is indexed at run
      // time, so each field read is a memory load that must stay out of the tile loop.
      const QConvTcParams& lp = cp.layer[l];
      uint8_t* const ybase = lp.y;
      const int y_layout = lp.y_layout;
      const uint32_t yx4 = (uint32_t)lp.y_xor * 0x01010101u;
      const int y_hp = lp.y_hp, y_wp = lp.y_wp, y_pt = lp.y_pt, y_pl = lp.y_pl;
      const int64_t yplane = (int64_t)lp.oh * lp.ow;
      const float ymz = lp.y_m_minus_zero, ylo = lp.y_lo, yhi = lp.y_hi;
      const bool y_signed = lp.y_lo < 0.0f;
      const int has_add = lp.has_add;
      const bool use_lut = lp.lut != nullptr;
      // integer requantisation (rint + zero point + clamp as one saturating pack)
      // where the planner proved it exact; the float fused add needs float values.
      // Signed outputs saturate y + 128 to [0, 255] and flip the top bit back.
      const bool int_rq = lp.rq_int && (!has_add || use_lut);
      const int rq_sub = lp.rq_sub - (y_signed ? 128 : 0);
      const uint32_t sx4 = y_signed ? 0x80808080u : 0u;
      const int64_t r_off = lp.r_off;
      const uint32_t rx4 = (uint32_t)lp.r_xor * 0x01010101u;
      const bool rb_on = has_add && lp.r_bulk;
      // this warp's scales and biases of layer l (its own slice: no cross-warp
      // barrier), fetched asynchronously one layer ahead
      float* sc = s_scale + ((l & 1) * QC_EPI_WARPS + ew) * G;
      int32_t* bi = s_bias + ((l & 1) * QC_EPI_WARPS + ew) * G;
      __syncwarp();  // every lane is done with layer l-1's slice, which layer l+1 reuses
      if (l >= 1 && l + 1 < L) fetch_consts(l + 1);
      if (l + 1 < L)
        cp_async_wait_group<1>();
      else
        cp_async_wait_group<0>();
      __syncwarp();
      if (use_lut) {
        ok = __all_sync(0xffffffffu, mbar_wait(lbar, (uint32_t)luts & 1u, err, DEV_TIMEOUT_EPILOGUE));
        ++luts;
        if (!ok) break;
      }
      const bool publish = chained && l + 1 < L;
      for (int tile = t_first; tile < n_tiles; tile += t_step, ++it) {
        __syncwarp();
        const int acc = it & 1;
        ok = mbar_wait(&accf[acc], (it >> 1) & 1, err, DEV_TIMEOUT_EPILOGUE);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
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
        const int rs = rit % QC_RSTAGES;
        if (rb_on) {
          ok = mbar_wait(&rfull[rs], (uint32_t)(rit / QC_RSTAGES) & 1u, err, DEV_TIMEOUT_EPILOGUE);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
        }

        // pixel of pitched row q: divisions by Hp*Wp and Wp as multiply-shift
        // with host-computed ceil(2^40 / d) (exact for q * d < 2^40, checked on the host)
        const uint32_t q = (uint32_t)tile * QC_TILE_M + (uint32_t)row;
        const int n = (int)(((uint64_t)q * hpwp_mul) >> 40);
        const uint32_t rem = q - (uint32_t)n * hpwp;
        const int oh = (int)(((uint64_t)rem * wp_mul) >> 40);
        const int ow = (int)rem - oh * gwp;
        const bool valid = n < gbatch && oh < goh && ow < gow;
        // the tile's residual bytes of this warp's G channels (a fused add)
        auto load_rb = [&](uint32_t(&rb)[G / 4]) {
          if (rb_on) {
            const uint8_t* rrow = s_r + ((size_t)rs * QC_TILE_M + row) * OC;
            const int64_t rpix = (int64_t)q + r_off;
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
            qc_load_resid<OC, G>(lp, rb, col0, n, oh, ow);
          }
        };
        uint32_t out[G / 4];
        if (valid) {
          if (int_rq) {
#pragma unroll
            for (int c4 = 0; c4 < G / 4; ++c4) {
              const float4 s4 = *reinterpret_cast<const float4*>(&sc[4 * c4]);
              const int4 b4 = *reinterpret_cast<const int4*>(&bi[4 * c4]);
              const int y0 = requant_int((int32_t)v[4 * c4 + 0] + b4.x, s4.x, rq_sub);
              const int y1 = requant_int((int32_t)v[4 * c4 + 1] + b4.y, s4.y, rq_sub);
              const int y2 = requant_int((int32_t)v[4 * c4 + 2] + b4.z, s4.z, rq_sub);
              const int y3 = requant_int((int32_t)v[4 * c4 + 3] + b4.w, s4.w, rq_sub);
              out[c4] = pack_sat_u8x4(y0, y1, y2, y3) ^ sx4;
            }
          } else {
            float r[G];
#pragma unroll
            for (int c4 = 0; c4 < G / 4; ++c4) {
              const float4 s4 = *reinterpret_cast<const float4*>(&sc[4 * c4]);
              const int4 b4 = *reinterpret_cast<const int4*>(&bi[4 * c4]);
              r[4 * c4 + 0] = requant_fast((int32_t)v[4 * c4 + 0] + b4.x, s4.x, ymz, ylo, yhi);
              r[4 * c4 + 1] = requant_fast((int32_t)v[4 * c4 + 1] + b4.y, s4.y, ymz, ylo, yhi);
              r[4 * c4 + 2] = requant_fast((int32_t)v[4 * c4 + 2] + b4.z, s4.z, ymz, ylo, yhi);
              r[4 * c4 + 3] = requant_fast((int32_t)v[4 * c4 + 3] + b4.w, s4.w, ymz, ylo, yhi);
            }
            if (has_add && !use_lut) {  // the fused add in float, one channel at a time
              uint32_t rb[G / 4];
              load_rb(rb);
              if (lp.fast_div) {
#pragma unroll
                for (int c = 0; c < G; ++c) {
                  const int rv = load_8bit(((rb[c >> 2] >> (8 * (c & 3))) ^ (uint32_t)lp.r_xor) & 0xFFu, lp.r_signed);
                  r[c] = qadd_fast<true>(r[c], lp.c_zero, lp.c_scale, rv, lp.r_zero, lp.r_scale, lp.add_scale,
                                         lp.add_inv_scale, lp.add_zero, lp.add_lo, lp.add_hi);
                }
              } else {
#pragma unroll
                for (int c = 0; c < G; ++c) {
                  const int rv = load_8bit(((rb[c >> 2] >> (8 * (c & 3))) ^ (uint32_t)lp.r_xor) & 0xFFu, lp.r_signed);
                  r[c] = qadd_fast<false>(r[c], lp.c_zero, lp.c_scale, rv, lp.r_zero, lp.r_scale, lp.add_scale,
                                          lp.add_inv_scale, lp.add_zero, lp.add_lo, lp.add_hi);
                }
              }
            }
#pragma unroll
            for (int c4 = 0; c4 < G / 4; ++c4)
              out[c4] = pack4(r[4 * c4 + 0], r[4 * c4 + 1], r[4 * c4 + 2], r[4 * c4 + 3]);
          }
          if (has_add && use_lut) {
            // out byte = table[(conv byte << 8) | residual byte]: the conv
            // bytes packed four to a word, the 16-bit indices of two
            // channels built by one byte permute from the two words
            uint32_t rb[G / 4];
            load_rb(rb);
#pragma unroll
            for (int c4 = 0; c4 < G / 4; ++c4) {
              const uint32_t cw = out[c4];
              const uint32_t rw = rb[c4] ^ rx4;
              const uint32_t t01 = __byte_perm(rw, cw, 0x5140);  // [r0, c0, r1, c1]
              const uint32_t t23 = __byte_perm(rw, cw, 0x7362);  // [r2, c2, r3, c3]
              const uint32_t b0 = s_lut[t01 & 0xFFFFu], b1 = s_lut[t01 >> 16];
              const uint32_t b2 = s_lut[t23 & 0xFFFFu], b3 = s_lut[t23 >> 16];
              out[c4] = __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
            }
          }
#pragma unroll
          for (int c4 = 0; c4 < G / 4; ++c4) out[c4] ^= yx4;
        }
        // Publish the previous tile now: its stores were issued a tile ago, so
        // the proxy fence (which waits for this thread's earlier global writes)
        // finds them drained instead of stalling right behind them.
        if (pend) {
          fence_proxy_async_global();
          __syncwarp();
          ++pub;
          if (lane == 0) st_release_cta_u32(&s_stored[ew], (uint32_t)pub);
          pend = false;
        }
        if (valid) {
          if (y_layout == 0) {  // swizzled NHWC: G bytes of the pixel's OC-byte row
            const int64_t ypix = ((int64_t)n * y_hp + oh + y_pt) * y_wp + ow + y_pl;
            uint8_t* yrow = ybase + (uint64_t)ypix * OC;
            if constexpr (G == 8) {
              st_global_v2(yrow + 16 * swz_chunk(ypix, col0 / 16, OC) + (col0 % 16), out[0], out[1]);
            } else {
#pragma unroll
              for (int c = 0; c < G / 16; ++c)
                st_global_v4(yrow + 16 * swz_chunk(ypix, col0 / 16 + c, OC), out[4 * c + 0], out[4 * c + 1],
                             out[4 * c + 2], out[4 * c + 3]);
            }
          } else {  // NCHW: one byte per channel plane
            uint8_t* yb = ybase + ((int64_t)n * OC + col0) * yplane + (int64_t)oh * gow + ow;
#pragma unroll
            for (int c = 0; c < G; ++c) st_global_u8(yb + (int64_t)c * yplane, out[c >> 2] >> (8 * (c & 3)));
          }
        }
        if (rb_on) {  // this warp is done with the tile's residual rows
          __syncwarp();
          if (lane == 0) mbar_arrive(&rempty[rs]);
          ++rit;
        }
        pend = publish;  // this warp's rows of the tile are stored: published with the next tile
      }
      if (pend) {  // the layer's last tile
        fence_proxy_async_global();
        __syncwarp();
        ++pub;
        if (lane == 0) st_release_cta_u32(&s_stored[ew], (uint32_t)pub);
        pend = false;
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&lfree[l & 3]);  // this warp is done with layer l's table
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (chained && threadIdx.x == 0) {
    // the last CTA to finish advances the run epoch (read by the next run after its pdl_wait)
    __threadfence();
    const unsigned long long done = atomicAdd(cp.state + 1, 1ull);
    if (done == gridDim.x - 1) {
      cp.state[1] = 0ull;
      __threadfence();
      atomicAdd(cp.state, 1ull);
    }
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

typedef void (*QcKernel)(const QConvChainParams);
struct QcVariant {
  int cin, oc;
  QcKernel fn;
};
static const QcVariant kQcVariants[] = {
    {32, 32, qconv_chain_kernel<32, 32>},   {32, 64, qconv_chain_kernel<32, 64>},
    {64, 32, qconv_chain_kernel<64, 32>},   {64, 64, qconv_chain_kernel<64, 64>},
    {64, 128, qconv_chain_kernel<64, 128>}, {128, 64, qconv_chain_kernel<128, 64>},
    {128, 128, qconv_chain_kernel<128, 128>},
};
constexpr size_t QC_SMEM_BUDGET = 210 * 1024;
constexpr size_t QC_SMEM_MAX = 227 * 1024;

// Shared memory of qconv_chain_kernel (the layout at its top).
static size_t qconv_smem_bytes(uint32_t b_bytes, int stages, uint32_t stage_bytes, int oc, bool resid_ring,
                               bool lut, int wbufs = 1) {
  size_t s = 1024;  // alignment slack
  s += (size_t)wbufs * align_up(b_bytes, 1024) + (lut ? 65536 : 0);
  s += (size_t)stages * stage_bytes;
  s += (size_t)2 * QC_EPI_WARPS * (oc / 4) * 8;  // per-warp scales + biases, two layer parities
  s += (size_t)(2 * stages + 4 + 5 + 4 + QC_MMA_WARPS + 2 * QC_RSTAGES) * 8 + 16 + 4 * QC_EPI_WARPS;
  s += (size_t)8 * (b_bytes / (32u * (uint32_t)oc));  // MMA operand offsets: 2 words per MMA of a tile
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
  p.rq_int = (int)op.ip[QC_RQ_INT];
  p.rq_sub = kMagicBits - (int)op.ip[QC_Y_ZERO];
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
  p.r_src = -1;
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
  const size_t budget = QC_SMEM_BUDGET;
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
  if (st->smem_bytes > QC_SMEM_MAX)
    return fail(msg, n, 5, "QLinearConv tensor-core path needs %zu B smem", st->smem_bytes);
  // a chain launch may combine a table and a residual ring of different members: allow the maximum
  cudaError_t e = cudaFuncSetAttribute(kQcVariants[st->variant].fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)QC_SMEM_MAX);
  if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  // A chain's CTAs wait on each other's progress words, so its grid (at most
  // one CTA per SM) must be resident all at once: refuse at load time, rather
  // than time out at run time, where this device cannot hold one CTA per SM.
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kQcVariants[st->variant].fn,
                                                    qc_threads(kQcVariants[st->variant].oc), QC_SMEM_MAX);
  if (e != cudaSuccess) return fail(msg, n, 4, "occupancy query: %s", cudaGetErrorString(e));
  if (per_sm < 1)
    return fail(msg, n, 5, "QLinearConv tensor-core path: no CTA of %d threads and %zu B shared memory fits an SM",
                qc_threads(kQcVariants[st->variant].oc), QC_SMEM_MAX);
  st->fast_div = 0;
  if (op.ip[QC_HAS_ADD]) {
    QConvTcParams p{};
    fill_params(p, op, ptrs, st, op.ip[QC_N]);
    int* d_mis = nullptr;
    int mis = -1;
    if (cudaMalloc(&d_mis, sizeof(int)) != cudaSuccess) return fail(msg, n, 7, "check buffer");
    // the fast division is kept only when the check itself ran to the end
    e = cudaMemset(d_mis, 0, sizeof(int));
    if (e == cudaSuccess) {
      qadd_fastdiv_check_kernel<<<256, 256>>>(p, d_mis);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(&mis, d_mis, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(d_mis);
    if (e != cudaSuccess) return fail(msg, n, 4, "fast-division check: %s", cudaGetErrorString(e));
    st->fast_div = mis == 0 ? 1 : 0;
  }
  (void)device;
  return 0;
}

static int floor_div(int64_t a, int64_t b) { return (int)(a >= 0 ? a / b : -((-a + b - 1) / b)); }

// One member launched alone (a chain of one).
static int launch_single(const PlanOp& op, void* const* ptrs, const QConvTcState* st, const LaunchCtx& ctx,
                         int* launches) {
  QConvChainParams cp{};
  QConvTcParams& p = cp.layer[0];
  fill_params(p, op, ptrs, st, eff_batch(ctx, op, op.ip[QC_N]));
  if (p.n_tiles <= 0) return 0;
  cp.n_layers = 1;
  cp.use_lut = p.lut != nullptr;
  cp.use_ring = p.has_add && p.r_bulk;
  cp.err = ctx.d_error;
  const int grid = p.n_tiles < ctx.num_sms ? p.n_tiles : ctx.num_sms;
  cudaError_t e = launch_pdl(kQcVariants[st->variant].fn, dim3(grid), dim3(qc_threads(kQcVariants[st->variant].oc)),
                             st->smem_bytes, ctx.stream, cp);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// The chain headed by `op` (ctx.index) as one launch; false when the members
// do not qualify (the caller then launches them one by one).
static bool build_chain(const PlanOp& op, void* const* ptrs, const LaunchCtx& ctx, int L, QConvChainParams& cp,
                        size_t* smem, const QConvTcState** head_st) {
  const QConvTcState* st0 = reinterpret_cast<const QConvTcState*>(&ctx.states[ctx.index]);
  *head_st = st0;
  if (L > QC_MAX_CHAIN || op.t[6] < 0) return false;
  const int64_t batch = eff_batch(ctx, op, op.ip[QC_N]);
  bool any_lut = false, any_add = false;
  for (int k = 0; k < L; ++k) {
    const PlanOp& m = ctx.ops[ctx.index + k];
    const QConvTcState* st = reinterpret_cast<const QConvTcState*>(&ctx.states[ctx.index + k]);
    if (m.kernel != op.kernel || st->variant != st0->variant) return false;
    for (int f : {QC_N, QC_CIN, QC_OC, QC_KH, QC_KW, QC_HP, QC_WP, QC_OH, QC_OW})
      if (m.ip[f] != op.ip[f]) return false;
    if (k > 0 && m.t[0] != ctx.ops[ctx.index + k - 1].t[4]) return false;  // layer k reads layer k-1's output
    if (k + 1 < L && m.ip[QC_Y_LAYOUT] != 0) return false;
    QConvTcParams& p = cp.layer[k];
    fill_params(p, m, ptrs, st, batch);
    if (p.has_add) {  // chained adds read their residual rows by bulk copy (the ring)
      any_add = true;
      if (m.ip[QC_R_HP] != m.ip[QC_HP] || m.ip[QC_R_WP] != m.ip[QC_WP]) return false;
      p.r_off = (int64_t)p.r_pt * p.wp + p.r_pl;
      const int64_t last_row = (int64_t)((m.ip[QC_N] * (int64_t)p.hp * p.wp + QC_TILE_M - 1) / QC_TILE_M) *
                                   QC_TILE_M + p.r_off;
      if (last_row > m.ip[QC_R_ROWS]) return false;
      p.r_bulk = 1;
      for (int j = 0; j < k; ++j)  // written inside the chain, by layer j?
        if (m.t[3] == ctx.ops[ctx.index + j].t[4]) p.r_src = j;
      p.lut = m.t[5] >= 0 ? (const uint8_t*)ptrs[m.t[5]] : nullptr;
      any_lut = any_lut || p.lut != nullptr;
    }
  }
  // shared memory: weights + (table) + ring + as many window stages as fit, at least 2
  const QConvTcParams& g = cp.layer[0];
  const int oc = (int)op.ip[QC_OC];
  // (two weight buffers; a window takes well under a tile's MMA time to land, so 3 stages keep the MMAs fed)
  bool lut = any_lut;
  if (lut && qconv_smem_bytes(st0->b_bytes, 3, st0->stage_bytes, oc, any_add, true, 2) > QC_SMEM_MAX) lut = false;
  int stages = 8;
  while (stages > 2 && qconv_smem_bytes(st0->b_bytes, stages, st0->stage_bytes, oc, any_add, lut, 2) > QC_SMEM_MAX)
    --stages;
  *smem = qconv_smem_bytes(st0->b_bytes, stages, st0->stage_bytes, oc, any_add, lut, 2);
  if (*smem > QC_SMEM_MAX) return false;
  for (int k = 0; k < L; ++k) {
    cp.layer[k].stages = stages;
    if (!lut) cp.layer[k].lut = nullptr;
  }
  cp.n_layers = L;
  cp.use_lut = lut;
  cp.use_ring = any_add;
  // rows of layer l's window, written by layer l-1 at output row q + off for pitched row q
  const int kh = g.kh, kw = g.kw;
  const int64_t win_true = QC_TILE_M + (int64_t)(kh - 1) * g.wp + kw - 1;
  int dlo = 0, dhi = 0;
  for (int k = 0; k + 1 < L; ++k) {
    const QConvTcParams& p = cp.layer[k];
    const int64_t off = (int64_t)p.y_pt * p.y_wp + p.y_pl;
    if (p.y_hp != g.hp || p.y_wp != g.wp) return false;  // the next layer reads it in the shared geometry
    dlo = std::max(dlo, -floor_div(-off, QC_TILE_M));
    dhi = std::max(dhi, floor_div(win_true - 1 - off, QC_TILE_M));
  }
  cp.dlo = dlo;
  cp.dhi = dhi;
  cp.rlo = 0;  // a chained residual has the shared geometry: tile t's rows are tile t's outputs
  cp.rhi = 0;
  cp.state = (unsigned long long*)ptrs[op.t[6]];
  cp.err = ctx.d_error;
  cp.drop_progress = (ctx.fault & FAULT_DROP_CHAIN_PROGRESS) ? 1 : 0;
  return true;
}

int launch_qconv_tc(const PlanOp& op, void* const* ptrs, const OpState* st_, const LaunchCtx& ctx, int* launches) {
  const QConvTcState* st = reinterpret_cast<const QConvTcState*>(st_);
  const int64_t chain = op.ip[QC_CHAIN];
  if (chain < 0) return 0;  // a chain member: launched by the chain's first op
  if (chain <= 1) return launch_single(op, ptrs, st, ctx, launches);
  if (!ctx.ops || ctx.index + (size_t)chain > ctx.n_ops) return 5;
  QConvChainParams cp{};
  size_t smem = 0;
  const QConvTcState* st0 = nullptr;
  if (!build_chain(op, ptrs, ctx, (int)chain, cp, &smem, &st0)) {
    for (int k = 0; k < chain; ++k) {
      int rc = launch_single(ctx.ops[ctx.index + k], ptrs,
                             reinterpret_cast<const QConvTcState*>(&ctx.states[ctx.index + k]), ctx, launches);
      if (rc) return rc;
    }
    return 0;
  }
  const int n_tiles = cp.layer[0].n_tiles;
  if (n_tiles <= 0) return 0;
  const int grid = n_tiles < ctx.num_sms ? n_tiles : ctx.num_sms;
  cudaError_t e = launch_pdl(kQcVariants[st0->variant].fn, dim3(grid), dim3(qc_threads(kQcVariants[st0->variant].oc)),
                             smem, ctx.stream, cp);
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
