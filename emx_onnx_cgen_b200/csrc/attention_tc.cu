// ONNX Attention (opset 23), fp16 in and out, on the tensor cores: the fast
// mode of the Attention op (the exact mode, attention.cu, repeats the
// reference's statement-by-statement fp16 rounding on CUDA cores).
//
// What it computes is the same function as the reference
// (src/emx_onnx_cgen/templates/attention_op.c.j2:47-188): per (b, h, query
// row) softmax over the visible keys of scale * q.k, times V, with the causal
// mask key > query + past -> excluded.  The arithmetic differs: scores and
// P.V accumulate in fp32 on tcgen05 kind::f16 MMAs, the softmax runs online in
// fp32 (exp2 with the scale folded into log2 units), P is rounded to fp16 for
// the P.V MMA and the row sum adds those same rounded values, and the output
// is normalised once at the end.  The reference rounds every statement to
// fp16, so this mode is closer to the exact value than the reference is; the
// tests hold it to that (max ULP against a float64 evaluation no larger than
// the reference's own).
//
// Work split: one CTA per (128 query rows, head, batch); heads in groups of 8
// run all their query tiles together (K/V stay in L2), heaviest causal query
// tiles first within a group.  Two CTAs share an SM (112 KB of shared memory
// and 256 TMEM columns each), so each scheduler holds two softmax warps: one
// CTA's exponentials overlap the other's MMAs and TMEM loads.  Warp 0: TMA
// producer (the Q tile once, then K and V tiles of 64 keys, double-buffered).  Warp 1: issues S_j = Q K_j^T into one
// of two TMEM score buffers.  Warp 2: issues O += P_j V_j into the TMEM output
// accumulator.  Warps 4-7: one thread per query row -- scores from TMEM,
// running max, exponentials, P_j (fp16) into shared memory, row sums, and the
// final O / l epilogue.  The output accumulator is rescaled only when a row's
// running max grows by more than 8 (log2 units): until then exponentials are
// taken against the stale max and stay below 2^8, which fp16 P and the fp32
// accumulators hold exactly as well.
//
// Operands in shared memory, all 128-byte swizzled (the TMA writes them so):
//   Q tile [128 rows][128 d] and K tiles [64 keys][128 d] fp16 as two 64-wide
//   slabs [rows][128 B]: the K-major A / B operands of S = Q K^T;
//   P [128 queries][64 keys] fp16, one such slab, written by the softmax
//   threads: the K-major A operand of O += P V;
//   V tile [64 keys][128 d] as two 64-wide d slabs: the B operand of P V in
//   MN-major form (N = d contiguous), slabs 8 KB apart (LBO), 8-key groups
//   1 KB apart (SBO).
// The shared-memory window must start on a 1 KB boundary (the swizzle atom);
// the kernel checks it and reports DEV_BAD_CONFIG otherwise.
// Every wait is bounded (tc100.cuh) and reports through the plan's error word.
#include <type_traits>
#include <cuda_fp16.h>

#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

constexpr int ATC_M = 128;        // query rows per CTA
constexpr int ATC_N = 64;         // keys per K / V tile
constexpr int ATC_D = 128;        // head size (Q/K and V)
constexpr int ATC_THREADS = 256;  // 8 warps
constexpr uint32_t ATC_QSLAB = (uint32_t)ATC_M * 128u;  // one 64-wide d slab of the Q tile: 16 KB
constexpr uint32_t ATC_QTILE = 2u * ATC_QSLAB;          // Q tile: 32 KB
constexpr uint32_t ATC_KSLAB = (uint32_t)ATC_N * 128u;  // one 64-wide d slab of a K or V tile: 8 KB
constexpr uint32_t ATC_KTILE = 2u * ATC_KSLAB;          // K or V tile: 16 KB
constexpr uint32_t ATC_PTILE = (uint32_t)ATC_M * ATC_N * 2u;  // P: 16 KB (one 128-byte-row slab)
constexpr uint32_t ATC_TMEM_COLS = 256;  // score buffers at columns 0 and ATC_N, output at ATC_O_COL
constexpr uint32_t ATC_O_COL = 2u * ATC_N;
constexpr float ATC_RESCALE = 8.0f;            // lazy-rescale threshold, log2 units
constexpr int ATC_GROUP = 8;                   // heads whose query tiles run together

struct AttnTcParams {
  CUtensorMap map_q, map_k, map_v;  // 4-D (d, t, h, b), box (64, 128, 1, 1), 128-byte swizzle
  uint16_t* o;
  int64_t o_sb, o_sh, o_st;
  int B, HQ, group, TQ, TK, past, causal, n_qtiles;
  float scale_log2;  // scale * log2(e)
  int* err;
};

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// 32 TMEM lanes x 32 bits, 32 consecutive columns <-> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// c + (the fp16 value h), rounded to fp32: one mixed-precision add
__device__ __forceinline__ float add_f16(uint16_t h, float c) {
  float d;
  asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(h), "f"(c));
  return d;
}

// K-major SW128 operand descriptor: 128-byte rows, 8-row atoms 1 KB apart.
__device__ __forceinline__ uint64_t atc_desc_k(uint32_t saddr) { return smem_desc_k_sw128(saddr, 1024); }

// MN-major SW128 operand descriptor: 64-element (128-byte) rows along MN,
// 64-wide MN slabs `lbo` bytes apart, 8-row K groups `sbo` bytes apart.
__device__ __forceinline__ uint64_t atc_desc_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

__global__ void __launch_bounds__(ATC_THREADS, 2) attention_tc_kernel(const __grid_constant__ AttnTcParams p) {
  extern __shared__ __align__(1024) uint8_t atc_raw[];
  if (smem_u32(atc_raw) & 1023u) {  // the swizzled operands need a 1 KB aligned window
    if (threadIdx.x == 0) record_error(p.err, DEV_BAD_CONFIG);
    return;
  }
  uint8_t* sm = atc_raw;
  uint8_t* s_q = sm;
  uint8_t* s_k = sm + ATC_QTILE;          // [2] K stages
  uint8_t* s_v = s_k + 2 * ATC_KTILE;     // [2] V stages
  uint8_t* s_p = s_v + 2 * ATC_KTILE;     // P
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_p + ATC_PTILE);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2] score buffer b holds S_j (j % 2 == b)
  uint64_t* s_empty = bars + 11; // [2] softmax warps are done reading score buffer b
  uint64_t* p_full = bars + 13;  // P_j written (and O rescaled) by the softmax warps
  uint64_t* o_done = bars + 14;  // P_j V_j accumulated into O (P may be rewritten)
  uint64_t* drain = bars + 15;   // [2] every MMA of the S / P.V issuer has completed
  uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 17);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* const err = p.err;
  // CTA order: heads in groups of ATC_GROUP, every query tile of a group before
  // the next group (a head's K and V, 1 MB at 2048 x 128, stay in L2 while its
  // query tiles run), heaviest causal tiles first within a group
  const int bh_count = p.HQ * p.B;
  const int grp = (int)(blockIdx.x / (unsigned)(ATC_GROUP * p.n_qtiles));
  const int gsize = min(ATC_GROUP, bh_count - grp * ATC_GROUP);
  const int within = (int)blockIdx.x - grp * ATC_GROUP * p.n_qtiles;
  const int qt = p.n_qtiles - 1 - within / gsize;
  const int bh = grp * ATC_GROUP + within % gsize;
  const int h = bh % p.HQ, b = bh / p.HQ;
  const int kvh = h / p.group;
  const int q0 = qt * ATC_M;
  int kend = p.TK;  // keys the tile's last row sees
  if (p.causal) kend = min(kend, q0 + ATC_M - 1 + p.past + 1);
  const int J = kend > 0 ? (kend + ATC_N - 1) / ATC_N : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(holder, ATC_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;  // score buffers at columns 0 and ATC_N, output accumulator at ATC_O_COL
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0 && J > 0) {
      // ---------------- producer
      pdl_wait();  // Q, K, V may come from the preceding kernel
      bool ok = true;
      int k_last[2] = {-1, -1}, v_last[2] = {-1, -1};  // per stage: last tile whose loads were issued
      mbar_arrive_expect_tx(q_full, ATC_QTILE);
      tma_load_4d(s_q, &p.map_q, q_full, 0, q0, h, b);
      tma_load_4d(s_q + ATC_QSLAB, &p.map_q, q_full, 64, q0, h, b);
      for (int j = 0; j < J && ok; ++j) {
        const int s = j & 1;
        const int key0 = j * ATC_N;
        if (j >= 2 && !mbar_wait(&k_empty[s], (uint32_t)((j >> 1) - 1) & 1u, err, DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[s], ATC_KTILE);
        tma_load_4d(s_k + s * ATC_KTILE, &p.map_k, &k_full[s], 0, key0, kvh, b);
        tma_load_4d(s_k + s * ATC_KTILE + ATC_KSLAB, &p.map_k, &k_full[s], 64, key0, kvh, b);
        k_last[s] = j;
        if (j >= 2 && !mbar_wait(&v_empty[s], (uint32_t)((j >> 1) - 1) & 1u, err, DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&v_full[s], ATC_KTILE);
        tma_load_4d(s_v + s * ATC_KTILE, &p.map_v, &v_full[s], 0, key0, kvh, b);
        tma_load_4d(s_v + s * ATC_KTILE + ATC_KSLAB, &p.map_v, &v_full[s], 64, key0, kvh, b);
        v_last[s] = j;
      }
      if (!ok) {  // error path: let the copies in flight land before the CTA exits
        (void)mbar_wait(q_full, 0, nullptr, 0);
        for (int st = 0; st < 2; ++st) {
          if (k_last[st] >= 0) (void)mbar_wait(&k_full[st], (uint32_t)(k_last[st] >> 1) & 1u, nullptr, 0);
          if (v_last[st] >= 0) (void)mbar_wait(&v_full[st], (uint32_t)(v_last[st] >> 1) & 1u, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && J > 0) {
      // ---------------- S issuer: S_j = Q K_j^T into score buffer j % 2
      const uint32_t idesc = make_idesc(1u, 0u, 0u, ATC_M, ATC_N);
      bool ok = mbar_wait(q_full, 0, err, DEV_TIMEOUT_MMA);
      for (int j = 0; j < J && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (uint32_t)(j >> 1) & 1u, err, DEV_TIMEOUT_MMA)) break;
        if (j >= 2 && !mbar_wait(&s_empty[s], (uint32_t)((j >> 1) - 1) & 1u, err, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t qa = smem_u32(s_q), kb = smem_u32(s_k + s * ATC_KTILE);
#pragma unroll
        for (int ks = 0; ks < ATC_D / 16; ++ks) {
          const uint32_t qoff = (uint32_t)(ks >> 2) * ATC_QSLAB + (uint32_t)(ks & 3) * 32u;
          const uint32_t koff = (uint32_t)(ks >> 2) * ATC_KSLAB + (uint32_t)(ks & 3) * 32u;
          mma_f16(tmem + (uint32_t)(s * ATC_N), atc_desc_k(qa + qoff), atc_desc_k(kb + koff), idesc,
                  ks > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[s]);
        tc_commit(&k_empty[s]);
      }
      // every MMA this thread issued completes before TMEM is released
      tc_commit(&drain[0]);
      (void)mbar_wait(&drain[0], 0, nullptr, 0);
    }
  } else if (warp == 2) {
    if (lane == 0 && J > 0) {
      // ---------------- P.V issuer: O += P_j V_j (V as the MN-major B operand)
      const uint32_t idesc = make_idesc(1u, 0u, 0u, ATC_M, ATC_D) | (1u << 16);
      for (int j = 0; j < J; ++j) {
        const int s = j & 1;
        if (!mbar_wait(p_full, (uint32_t)j & 1u, err, DEV_TIMEOUT_MMA)) break;
        if (!mbar_wait(&v_full[s], (uint32_t)(j >> 1) & 1u, err, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t pa = smem_u32(s_p), vb = smem_u32(s_v + s * ATC_KTILE);
#pragma unroll
        for (int kk = 0; kk < ATC_N / 16; ++kk) {
          const uint32_t aoff = (uint32_t)kk * 32u;  // P is one 128-byte-row slab: 16 keys = 32 bytes
          const uint64_t bdesc = atc_desc_mn(vb + (uint32_t)kk * 16u * 128u, ATC_KSLAB, 1024u);
          mma_f16(tmem + ATC_O_COL, atc_desc_k(pa + aoff), bdesc, idesc, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(o_done);
        tc_commit(&v_empty[s]);
      }
      tc_commit(&drain[1]);
      (void)mbar_wait(&drain[1], 0, nullptr, 0);
    }
  } else if (warp >= 4) {
    // ---------------- softmax and epilogue: thread = query row
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    // last key index this row sees
    const int row_last = p.causal ? min(p.TK - 1, qi + p.past) : p.TK - 1;
    float m_used = -INFINITY;  // running max in log2 units, as used by the exponentials
    float l = 0.0f;            // row sum of the fp16-rounded exponentials
    bool ok = true;
    for (int j = 0; j < J && ok; ++j) {
      const int s = j & 1;
      ok = mbar_wait(&s_full[s], (uint32_t)(j >> 1) & 1u, err, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      constexpr int NC = ATC_N / 32;  // 32-column chunks of a score row
      uint32_t sv[NC][32];
#pragma unroll
      for (int c = 0; c < NC; ++c) tmem_ld32(tmem + lane_base + (uint32_t)(s * ATC_N + 32 * c), sv[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[s]);  // the score buffer may be overwritten
      const int nvalid = min(ATC_N, max(0, row_last - j * ATC_N + 1));  // keys [0, nvalid) of the tile are visible
      // Row maximum in 4 independent partials (max is exact in any order).  With a
      // positive scale the maximum of the scaled scores is the scaled maximum
      // (rounding is monotone), so the scores stay raw and each exponential takes
      // one fma: 2^(s * scale_log2 - m).
      const float sc = p.scale_log2;
      const bool pos = sc > 0.0f;
      float mxp[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      // tiles whose keys are all visible (every tile but a causal row block's
      // last) run the element loops without the per-key visibility test
      const bool full_tile = nvalid == ATC_N;
      auto row_max = [&](auto full_c) {
        constexpr bool FULL = decltype(full_c)::value;
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float x = __uint_as_float(sv[c][i]);
            if (!pos) {
              x *= sc;
              sv[c][i] = __float_as_uint(x);
            }
            if (FULL || 32 * c + i < nvalid) mxp[i & 3] = fmaxf(mxp[i & 3], x);
          }
      };
      if (full_tile)
        row_max(std::true_type{});
      else
        row_max(std::false_type{});
      float mx = fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3]));
      if (pos) mx *= sc;
      const float mul = pos ? sc : 1.0f;
      float m_new = m_used;
      bool rescale = false;
      if (mx > m_used + ATC_RESCALE || m_used == -INFINITY) {
        m_new = mx;
        rescale = j > 0 && m_used != -INFINITY;
      }
      const float alpha = rescale ? ex2_approx(m_used - m_new) : 1.0f;
      // exponentials against m_new, rounded to fp16 (the P.V operand); the row sum adds the same
      // values, in 4 independent partials
      uint32_t pw[NC][16];
      float lp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const float neg_m = -m_new;
      auto exps = [&](auto full_c) {
        constexpr bool FULL = decltype(full_c)::value;
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int k0 = 32 * c + 2 * i;
            const float e0 =
                FULL || k0 < nvalid ? ex2_approx(fmaf(__uint_as_float(sv[c][2 * i]), mul, neg_m)) : 0.0f;
            const float e1 =
                FULL || k0 + 1 < nvalid ? ex2_approx(fmaf(__uint_as_float(sv[c][2 * i + 1]), mul, neg_m)) : 0.0f;
            pw[c][i] = pack_f16x2(e0, e1);
            lp[i & 3] = add_f16((uint16_t)(pw[c][i] >> 16), add_f16((uint16_t)pw[c][i], lp[i & 3]));
          }
      };
      if (full_tile)
        exps(std::true_type{});
      else
        exps(std::false_type{});
      l = l * alpha + ((lp[0] + lp[1]) + (lp[2] + lp[3]));
      m_used = m_new;
      // P_{j-1} V_{j-1} must be done before P is overwritten and O rescaled
      if (j > 0) {
        ok = mbar_wait(o_done, (uint32_t)(j - 1) & 1u, err, DEV_TIMEOUT_EPILOGUE);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_base + ATC_O_COL + 32u * c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tmem + lane_base + ATC_O_COL + 32u * c, o);
          }
          tmem_wait_st();
        }
      }
      // P row r: keys 8g .. 8g+7 are 16-byte chunk g of the row, swizzled by the row
#pragma unroll
      for (int g = 0; g < ATC_N / 8; ++g) {
        const int c = g >> 2, i = (g & 3) * 4;
        uint8_t* dst = s_p + r * 128 + ((g ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pw[c][i], pw[c][i + 1], pw[c][i + 2], pw[c][i + 3]);
      }
      fence_async_shared();  // the generic writes of P become visible to the tensor cores
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // ---------------- epilogue: O / l -> fp16
    if (ok && J > 0) {
      ok = mbar_wait(o_done, (uint32_t)(J - 1) & 1u, err, DEV_TIMEOUT_EPILOGUE);
      ok = __all_sync(0xffffffffu, ok);
    }
    pdl_wait();  // the output may still be read by the preceding kernel
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      uint16_t* orow = p.o + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)qi * p.o_st;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        if (J > 0) {
          tmem_ld32(tmem + lane_base + ATC_O_COL + 32u * c, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (qi < p.TQ) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack_f16x2(__uint_as_float(o[i + 0]) * inv, __uint_as_float(o[i + 1]) * inv);
            w.y = pack_f16x2(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
            w.z = pack_f16x2(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
            w.w = pack_f16x2(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + 32 * c + i) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ATC_TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
// no alignment slack: two CTAs of this size fit one SM only without it (the
// kernel checks that the window starts on a 1 KB boundary)
constexpr size_t ATC_SMEM = (size_t)ATC_QTILE + 4 * (size_t)ATC_KTILE + ATC_PTILE + 256;

// The fast mode needs 128-wide fp16 heads and 16-byte aligned token strides.
int prepare_attention_tc(const PlanOp& op, void* const*, OpState*, int, char* msg, size_t n) {
  if (op.ip[AT_D] != ATC_D || op.ip[AT_DV] != ATC_D)
    return fail(msg, n, 5, "Attention tensor-core mode: head sizes %lld/%lld, needs 128", (long long)op.ip[AT_D],
                (long long)op.ip[AT_DV]);
  for (int s = AT_Q_SB; s <= AT_O_ST; ++s)
    if ((op.ip[s] * 2) % 16 != 0) return fail(msg, n, 5, "Attention tensor-core mode: strides must be 16-byte multiples");
  cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATC_SMEM);
  if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  return 0;
}

// 4-D map (d, t, h, b) over an fp16 tensor with element strides (1, st, sh, sb),
// boxes of 64 d x `rows` tokens.
static int make_tmap_attn(CUtensorMap* map, const void* base, int64_t t, int64_t heads, int64_t batch, int64_t st,
                          int64_t sh, int64_t sb, uint32_t rows) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc || ((uintptr_t)base & 15u)) return 5;
  cuuint64_t dims[4] = {(cuuint64_t)ATC_D, (cuuint64_t)t, (cuuint64_t)heads, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)st * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 4;
}

int launch_attention_tc(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  AttnTcParams p{};
  const int64_t* s = &op.ip[AT_Q_SB];
  p.B = (int)eff_batch(ctx, op, op.ip[AT_B]);
  p.HQ = (int)op.ip[AT_HQ];
  p.group = (int)op.ip[AT_GROUP];
  p.TQ = (int)op.ip[AT_TQ];
  p.TK = (int)op.ip[AT_TK];
  p.past = (int)op.ip[AT_PAST];
  p.causal = (int)op.ip[AT_CAUSAL];
  p.n_qtiles = (p.TQ + ATC_M - 1) / ATC_M;
  p.scale_log2 = (float)op.fp[ATF_SCALE] * 1.4426950408889634f;
  p.o = (uint16_t*)ptrs[op.t[3]];
  p.o_sb = s[9];
  p.o_sh = s[10];
  p.o_st = s[11];
  p.err = ctx.d_error;
  if (p.B <= 0 || p.TQ <= 0) return 0;
  const int hkv = p.HQ / p.group;
  int rc = make_tmap_attn(&p.map_q, ptrs[op.t[0]], p.TQ, p.HQ, p.B, s[2], s[1], s[0], ATC_M);
  if (!rc) rc = make_tmap_attn(&p.map_k, ptrs[op.t[1]], p.TK, hkv, p.B, s[5], s[4], s[3], ATC_N);
  if (!rc) rc = make_tmap_attn(&p.map_v, ptrs[op.t[2]], p.TK, hkv, p.B, s[8], s[7], s[6], ATC_N);
  if (rc) return rc;
  const unsigned grid = (unsigned)(p.n_qtiles * p.HQ * p.B);
  cudaError_t e = launch_pdl(attention_tc_kernel, dim3(grid), dim3(ATC_THREADS), ATC_SMEM, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
