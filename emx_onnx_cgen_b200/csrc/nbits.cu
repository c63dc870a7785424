// com.microsoft MatMulNBits (bits 4, fp16 activations, accuracy_level 0) on
// tcgen05 kind::f16, with the int4 weights dequantised inside the kernel, and
// the fused form for a Llama-style MLP: gate and up projections of the same
// activations in one kernel whose epilogue applies Swish(gate) * up.
//
// Reference arithmetic (src/emx_onnx_cgen/templates/matmul_nbits_op.c.j2:1-58,
// ir/ops/nn.py:1035-1283; float accumulator for fp16 inputs):
//   q   = (B[n][k / bs][(k % bs) / 2] >> (4 * (k % 2))) & 15
//   deq = ((float)q - (float)zp) * (float)scale[n][k / bs]       (zp = 8 by default)
//   acc = sum_k (float)A[m][k] * deq;  acc += (float)bias[n];  Y = (_Float16)acc
// Swish (shared/scalar_functions.py:880-896) and Mul on fp16 are
//   S = (_Float16)(g / (1.0 + exp((double)(-(float)alpha * (float)g))))
//   P = (_Float16)((float)S * (float)U)
// deq has at most 15 significant bits ((q - zp) has 4, the fp16 scale 11), so
// it is split exactly into two fp16 operands hi = fp16(deq) and
// lo = fma(q - zp, scale, -hi) (the rounding remainder, exactly representable)
// and every K slice is multiplied twice, A x hi + A x lo, into the same fp32
// accumulator: products are exact, only the summation order differs from the
// reference's sequential float sum, and Y agrees within the fp16 ULP bound
// the parity tests state.  (A plan may drop the lo half -- one MMA per slice,
// deq rounded to fp16 -- trading that accuracy for MMA throughput.)  Swish and
// Mul are evaluated exactly as above (double exp and division, one rounding
// to fp16; fp16 product rounded once).
//
// Tiling (the operands are swapped so that the dequantised side is the
// smaller one): MMA M = 128 weight rows (output columns n), MMA N = 256
// activation rows m, K steps of 64 fp16 (one 128-byte swizzled row).
//   * activations A[m][k] arrive by TMA (tensor map, SWIZZLE_128B, box
//     64 x 256; rows/columns past the tensor read as zero);
//   * the weights of a 128-row tile and one K step form one contiguous image
//     block, loaded by one bulk copy: [2][128 rows][16 B] packed nibbles
//     (eight 4-byte words per row, nibbles of each word permuted so that
//     (w >> 4i) & 0x000F000F holds the pair k = 2i, 2i+1 of the word's eight)
//     followed by [128 rows][G groups] words (fp16 scale, fp16 -(1024 + zp));
//   * four dequant warps turn a block into the 128 x 64 fp16 operands hi and
//     lo: a nibble OR 0x6400 is the fp16 value 1024 + q, adding -(1024 + zp)
//     gives c = q - zp exactly, hi = c * scale rounded once, lo = fma(c,
//     scale, -hi) exact;
//   * the 128 x 256 fp32 accumulator is double-buffered in TMEM (2 x 256
//     columns) so the epilogue of a tile overlaps the main loop of the next;
//   * epilogue: TMEM -> registers -> fp16 -> a per-warp 32 x 32 staging tile
//     -> TMA store (rows/columns past the output are clipped).  Fused mode:
//     tile rows 0-63 are gate columns n0..n0+63, rows 64-127 up columns
//     n0..n0+63; the two warps holding the same n exchange through shared
//     memory and split the Swish/Mul work.
//   * warps: 0 activation producer, 1 MMA issuer + TMEM owner, 2 weight
//     producer, 3 idle, 4-7 dequant, 8-11 epilogue (TMEM lane quarter =
//     warp % 4).  Persistent CTAs walk tiles n-major so that the CTAs in
//     flight share weight tiles and the activations stay in L2.
#include <cuda_fp16.h>

#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

constexpr int NB_TILE_N = 128;  // weight rows per tile (MMA M)
constexpr int NB_TILE_M = 256;  // activation rows per tile (MMA N)
constexpr int NB_KSTEP = 64;    // fp16 elements per K step
constexpr int NB_THREADS = 384;
constexpr int NB_SX = 3;  // activation stages (32 KB each)
constexpr int NB_SA = 2;  // dequantised weight stages (hi + lo, 2 x 16 KB each)
constexpr int NB_SW = 4;  // packed weight stages
constexpr uint32_t NB_X_BYTES = NB_TILE_M * NB_KSTEP * 2;
constexpr uint32_t NB_A_BYTES = NB_TILE_N * NB_KSTEP * 2;
constexpr uint32_t NB_PACKED_BYTES = NB_TILE_N * NB_KSTEP / 2;
constexpr uint32_t NB_STG_BYTES = 32 * 32 * 2;  // one 32 x 32 fp16 staging tile

struct NbitsParams {
  CUtensorMap map_a;  // activations [rows][K] fp16, box 64 x 256, SWIZZLE_128B
  CUtensorMap map_y;  // output [rows][N] fp16, box 32 x 32
  const uint8_t* w_img;
  const float* bias;  // [n_tiles * 128] or null
  int* err;
  int rows, k_steps, n_tiles, m_tiles, groups, fused, exact;
  uint32_t w_stage_bytes, idesc;
  float alpha;
};

__device__ __forceinline__ uint32_t h2_add(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint16_t f32_to_f16_rn(float v) {
  uint16_t r;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ float f16_to_f32(uint16_t h) {
  float r;
  asm("cvt.f32.f16 %0, %1;" : "=f"(r) : "h"(h));
  return r;
}

__device__ __forceinline__ uint16_t f64_to_f16_rn(double v) {
  uint16_t r;
  asm("cvt.rn.f16.f64 %0, %1;" : "=h"(r) : "d"(v));
  return r;
}

// Swish of an fp16 value as the reference evaluates it: the exponent argument
// -(alpha * g) is an exact float product, exp and the division run in double,
// the quotient is rounded once to fp16.
__device__ __forceinline__ uint16_t swish_f16(uint16_t g, float alpha) {
  const float gf = f16_to_f32(g);
  const double e = exp((double)(-__fmul_rn(alpha, gf)));
  return f64_to_f16_rn((double)gf / (1.0 + e));
}

// Same value, cheaper: the quotient is first formed in float with expf (CUDA
// documents <= 2 ulp), one rounded add and an IEEE division, a relative error
// below 1.5 * 2^-22.  When the float quotient widened by a 2^-20 relative
// margin on both sides still rounds to a single fp16 value, that value is the
// correctly rounded fp16 of the exact quotient, and hence of the double
// evaluation (whose own error is ~2^-52); otherwise -- about one value in a
// thousand, close to an fp16 rounding boundary -- the double evaluation runs.
// Exhaustively checked against the reference helper over all 65536 inputs.
__device__ __forceinline__ uint16_t swish_f16_fast(uint16_t g, float alpha) {
  const float gf = f16_to_f32(g);
  const float r = __fdiv_rn(gf, __fadd_rn(1.0f, expf(-__fmul_rn(alpha, gf))));
  const uint16_t lo = f32_to_f16_rn(__fmul_rn(r, 1.0f - 0x1p-20f));
  const uint16_t hi = f32_to_f16_rn(__fmul_rn(r, 1.0f + 0x1p-20f));
  if (lo == hi && !isnan(r)) return lo;
  return swish_f16(g, alpha);
}

// fp16 product rounded once (the float product of two fp16 values is exact).
__device__ __forceinline__ uint16_t mul_f16(uint16_t a, uint16_t b) {
  return f32_to_f16_rn(__fmul_rn(f16_to_f32(a), f16_to_f32(b)));
}

__global__ void __launch_bounds__(NB_THREADS, 1) nbits_gemm_kernel(const __grid_constant__ NbitsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_x = smem;                                  // NB_SX x 32 KB
  uint8_t* s_a = s_x + NB_SX * NB_X_BYTES;              // NB_SA x (hi 16 KB, lo 16 KB)
  uint8_t* s_stg = s_a + NB_SA * 2 * NB_A_BYTES;        // 8 staging tiles
  uint8_t* s_w = s_stg + 8 * NB_STG_BYTES;              // NB_SW x w_stage_bytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_w + NB_SW * p.w_stage_bytes);
  uint64_t* x_full = bars;
  uint64_t* x_empty = x_full + NB_SX;
  uint64_t* w_full = x_empty + NB_SX;
  uint64_t* w_empty = w_full + NB_SW;
  uint64_t* a_full = w_empty + NB_SW;
  uint64_t* a_empty = a_full + NB_SA;
  uint64_t* acc_full = a_empty + NB_SA;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* pair_ok = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [4], fused epilogue

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_work = p.n_tiles * p.m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NB_SX; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < NB_SW; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 4);
    }
    for (int s = 0; s < NB_SA; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&a_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- activation producer
      pdl_wait();  // activations may come from the preceding kernel
      int s = 0;
      uint32_t ph = 0, issued = 0, parity_of = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_work && ok; t += gridDim.x) {
        const int m0 = (t % p.m_tiles) * NB_TILE_M;
        for (int ks = 0; ks < p.k_steps; ++ks) {
          if (!mbar_wait(&x_empty[s], ph ^ 1u, p.err, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&x_full[s], NB_X_BYTES);
          tma_load_2d(s_x + s * NB_X_BYTES, &p.map_a, &x_full[s], ks * NB_KSTEP, m0);
          issued |= 1u << s;
          parity_of = (parity_of & ~(1u << s)) | (ph << s);
          if (++s == NB_SX) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok)  // error path: let every load this thread issued land before the CTA exits
        for (int s2 = 0; s2 < NB_SX; ++s2)
          if (issued & (1u << s2)) (void)mbar_wait(&x_full[s2], (parity_of >> s2) & 1u, nullptr, 0);
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ---------------- weight producer (constants: no wait on the preceding kernel)
      int s = 0;
      uint32_t ph = 0, issued = 0, parity_of = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_work && ok; t += gridDim.x) {
        const int nt = t / p.m_tiles;
        const uint8_t* src = p.w_img + (size_t)nt * p.k_steps * p.w_stage_bytes;
        for (int ks = 0; ks < p.k_steps; ++ks) {
          if (!mbar_wait(&w_empty[s], ph ^ 1u, p.err, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&w_full[s], p.w_stage_bytes);
          bulk_load(s_w + s * p.w_stage_bytes, src + (size_t)ks * p.w_stage_bytes, p.w_stage_bytes, &w_full[s]);
          issued |= 1u << s;
          parity_of = (parity_of & ~(1u << s)) | (ph << s);
          if (++s == NB_SW) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok)
        for (int s2 = 0; s2 < NB_SW; ++s2)
          if (issued & (1u << s2)) (void)mbar_wait(&w_full[s2], (parity_of >> s2) & 1u, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      int sx = 0, sa = 0, it = 0;
      uint32_t phx = 0, pha = 0;
      bool ok = true;
      const uint32_t x_base = smem_u32(s_x), a_base = smem_u32(s_a);
      for (int t = blockIdx.x; t < n_work && ok; t += gridDim.x, ++it) {
        const int b = it & 1;
        if (!mbar_wait(&acc_empty[b], ((it >> 1) & 1) ^ 1u, p.err, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(b * NB_TILE_M);
        for (int ks = 0; ks < p.k_steps; ++ks) {
          if (!mbar_wait(&x_full[sx], phx, p.err, DEV_TIMEOUT_MMA) ||
              !mbar_wait(&a_full[sa], pha, p.err, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_base + (uint32_t)sa * 2 * NB_A_BYTES;
          const uint32_t x_addr = x_base + (uint32_t)sx * NB_X_BYTES;
#pragma unroll
          for (int kk = 0; kk < NB_KSTEP / 16; ++kk) {
            const uint64_t bdesc = smem_desc_k_swizzled(x_addr + 32u * kk, 128);
            mma_f16(d_tmem, smem_desc_k_swizzled(a_addr + 32u * kk, 128), bdesc, p.idesc, (ks | kk) != 0 ? 1u : 0u);
            if (p.exact) mma_f16(d_tmem, smem_desc_k_swizzled(a_addr + NB_A_BYTES + 32u * kk, 128), bdesc, p.idesc, 1u);
          }
          tc_commit(&x_empty[sx]);
          tc_commit(&a_empty[sa]);
          if (++sx == NB_SX) {
            sx = 0;
            phx ^= 1u;
          }
          if (++sa == NB_SA) {
            sa = 0;
            pha ^= 1u;
          }
        }
        if (ok) tc_commit(&acc_full[b]);
      }
      if (!ok) {  // error path: wait for this thread's MMAs before TMEM is released
        tc_commit(drain);
        (void)mbar_wait(drain, 0, nullptr, 0);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------- dequant: thread r converts weight row r of every K step
    const int r = threadIdx.x - 128;
    const uint32_t swz = (uint32_t)(r & 7);
    int sw = 0, sa = 0;
    uint32_t phw = 0, pha = 0;
    for (int t = blockIdx.x; t < n_work; t += gridDim.x) {
      bool ok = true;
      for (int ks = 0; ks < p.k_steps; ++ks) {
        ok = mbar_wait(&w_full[sw], phw, p.err, DEV_TIMEOUT_PRODUCER);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        const uint8_t* wst = s_w + sw * p.w_stage_bytes;
        const uint4 q0 = *reinterpret_cast<const uint4*>(wst + r * 16);
        const uint4 q1 = *reinterpret_cast<const uint4*>(wst + 2048 + r * 16);
        const uint32_t* sst = reinterpret_cast<const uint32_t*>(wst + NB_PACKED_BYTES) + r * p.groups;
        uint32_t sc[4] = {0u, 0u, 0u, 0u};
        sc[0] = sst[0];
        sc[1] = sst[1];
        if (p.groups == 4) {
          sc[2] = sst[2];
          sc[3] = sst[3];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&w_empty[sw]);
        if (++sw == NB_SW) {
          sw = 0;
          phw ^= 1u;
        }
        ok = mbar_wait(&a_empty[sa], pha ^ 1u, p.err, DEV_TIMEOUT_PRODUCER);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        uint8_t* arow = s_a + sa * 2 * NB_A_BYTES + r * 128;
        const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // scale group of chunk j: 2 groups (of 32) or 4 groups (of 16) per K step
          const uint32_t g = p.groups == 4 ? sc[j >> 1] : sc[j >> 2];
          const uint32_t s2 = __byte_perm(g, 0, 0x1010);   // (scale, scale)
          const uint32_t nb2 = __byte_perm(g, 0, 0x3232);  // (-(1024+zp), -(1024+zp))
          const uint32_t w = words[j];
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t c = h2_add(((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u, nb2);  // q - zp, exact
            hi[i] = h2_mul(c, s2);
            lo[i] = h2_fma(c, s2, hi[i] ^ 0x80008000u);  // c * scale - hi, exact
          }
          *reinterpret_cast<uint4*>(arow + ((j ^ swz) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          if (p.exact)
            *reinterpret_cast<uint4*>(arow + NB_A_BYTES + ((j ^ swz) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
        if (++sa == NB_SA) {
          sa = 0;
          pha ^= 1u;
        }
      }
      if (!ok) break;
    }
  } else if (warp >= 8) {
    // ---------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter: tile rows 32q .. 32q+31
    const int ew = warp - 8;
    uint8_t* stg = s_stg + ew * 2 * NB_STG_BYTES;
    pdl_wait();  // outputs may still be read by the preceding kernel
    int it = 0;
    uint32_t store_groups = 0;
    const bool issuer = p.fused ? (q >= 2 && lane == 0) : lane == 0;
    for (int t = blockIdx.x; t < n_work; t += gridDim.x, ++it) {
      const int nt = t / p.m_tiles, m0 = (t % p.m_tiles) * NB_TILE_M;
      const int b = it & 1;
      bool ok = mbar_wait(&acc_full[b], (it >> 1) & 1, p.err, DEV_TIMEOUT_EPILOGUE);
      ok = __all_sync(0xffffffffu, ok);
      if (p.fused) {
        // the two warps of a pair meet at named barriers below: they leave together or not at all
        if (lane == 0) pair_ok[q] = ok ? 1 : 0;
        named_barrier(1 + (q & 1), 64);
        ok = pair_ok[q & 1] && pair_ok[(q & 1) + 2];
        named_barrier(1 + (q & 1), 64);
      }
      if (!ok) break;
      tc_fence_after();
      const int row = q * 32 + lane;
      const float bias = p.bias ? p.bias[nt * NB_TILE_N + row] : 0.0f;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * NB_TILE_M);
      for (int c = 0; c < NB_TILE_M / 32; ++c) {
        uint32_t v[32];
        tmem_ld16(taddr + c * 32, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
        tmem_ld16(taddr + c * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
        tmem_wait_ld();
        if (c == NB_TILE_M / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (!p.fused) {
          uint8_t* buf = stg + (c & 1) * NB_STG_BYTES;
          if (lane == 0 && store_groups >= 2) bulk_wait_group_read<1>();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            *reinterpret_cast<uint16_t*>(buf + j * 64 + lane * 2) =
                f32_to_f16_rn(__fadd_rn(__uint_as_float(v[j]), bias));
          fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&p.map_y, buf, nt * NB_TILE_N + q * 32, m0 + c * 32);
            bulk_commit_group();
            ++store_groups;
          }
        } else {
          // warps q and q+2 hold gate and up of the same 32 output columns
          const int pair = q & 1;
          uint8_t* pbase = s_stg + pair * 4 * NB_STG_BYTES;  // [gate][up][out0][out1]
          uint8_t* xv = pbase + (q >> 1) * NB_STG_BYTES;
          uint8_t* out = pbase + (2 + (c & 1)) * NB_STG_BYTES;
          if (issuer && store_groups >= 2) bulk_wait_group_read<1>();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            *reinterpret_cast<uint16_t*>(xv + j * 64 + lane * 2) =
                f32_to_f16_rn(__fadd_rn(__uint_as_float(v[j]), bias));
          named_barrier(1 + pair, 64);
          const int tid64 = (q >> 1) * 32 + lane;
#pragma unroll 4
          for (int e = tid64; e < 1024; e += 64) {
            const uint16_t g = *reinterpret_cast<const uint16_t*>(pbase + 2 * e);
            const uint16_t u = *reinterpret_cast<const uint16_t*>(pbase + NB_STG_BYTES + 2 * e);
            *reinterpret_cast<uint16_t*>(out + 2 * e) = mul_f16(swish_f16_fast(g, p.alpha), u);
          }
          fence_async_shared();
          named_barrier(1 + pair, 64);
          if (issuer) {
            tma_store_2d(&p.map_y, out, nt * (NB_TILE_N / 2) + pair * 32, m0 + c * 32);
            bulk_commit_group();
            ++store_groups;
          }
        }
      }
    }
    if (store_groups) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ------------------------------------------------------------------ host side
struct NbitsState {
  uint32_t w_stage_bytes;
  size_t smem_bytes;
};
static_assert(sizeof(NbitsState) <= sizeof(OpState), "state fits");

static size_t nbits_smem_bytes(uint32_t w_stage_bytes) {
  size_t s = 1024;  // alignment slack
  s += (size_t)NB_SX * NB_X_BYTES + (size_t)NB_SA * 2 * NB_A_BYTES + 8 * NB_STG_BYTES;
  s += (size_t)NB_SW * w_stage_bytes;
  s += (size_t)(2 * NB_SX + 2 * NB_SW + 2 * NB_SA + 4 + 1) * 8 + 32;
  return s;
}

int prepare_nbits(const PlanOp& op, void* const*, OpState* st_, int, char* msg, size_t n) {
  NbitsState* st = reinterpret_cast<NbitsState*>(st_);
  const int groups = (int)op.ip[NB_GROUPS];
  if (groups != 2 && groups != 4) return fail(msg, n, 5, "MatMulNBits: %d scale groups per K step", groups);
  if (op.ip[NB_KSTEPS] <= 0 || op.ip[NB_NTILES] <= 0) return fail(msg, n, 5, "MatMulNBits: empty weight image");
  if ((op.ip[NB_A_PITCH] * 2) % 16 || (op.ip[NB_Y_PITCH] * 2) % 16)
    return fail(msg, n, 5, "MatMulNBits: row pitches must be multiples of 16 bytes");
  st->w_stage_bytes = NB_PACKED_BYTES + (uint32_t)(NB_TILE_N * groups * 4);
  st->smem_bytes = nbits_smem_bytes(st->w_stage_bytes);
  if (st->smem_bytes > 227 * 1024) return fail(msg, n, 5, "MatMulNBits needs %zu B smem", st->smem_bytes);
  cudaError_t e =
      cudaFuncSetAttribute(nbits_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)st->smem_bytes);
  if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  return 0;
}

int launch_nbits(const PlanOp& op, void* const* ptrs, const OpState* st_, const LaunchCtx& ctx, int* launches) {
  const NbitsState* st = reinterpret_cast<const NbitsState*>(st_);
  const int64_t rpb = op.ip[NB_ROWS_PER_BATCH] > 0 ? op.ip[NB_ROWS_PER_BATCH] : 1;
  const int64_t rows = op.ip[IP_BATCHED] && ctx.batch > 0 ? ctx.batch * rpb : op.ip[NB_ROWS];
  if (rows <= 0) return 0;
  NbitsParams p{};
  char msg[256];
  if (make_tmap_2d(&p.map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ptrs[op.t[0]], (uint64_t)op.ip[NB_K], (uint64_t)rows,
                   (uint64_t)op.ip[NB_A_PITCH] * 2, NB_KSTEP, NB_TILE_M, CU_TENSOR_MAP_SWIZZLE_128B, msg,
                   sizeof(msg)))
    return 4;
  if (make_tmap_2d(&p.map_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ptrs[op.t[3]], (uint64_t)op.ip[NB_N_OUT],
                   (uint64_t)rows, (uint64_t)op.ip[NB_Y_PITCH] * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE, msg,
                   sizeof(msg)))
    return 4;
  p.w_img = (const uint8_t*)ptrs[op.t[1]];
  p.bias = op.t[2] >= 0 ? (const float*)ptrs[op.t[2]] : nullptr;
  p.err = ctx.d_error;
  p.rows = (int)rows;
  p.k_steps = (int)op.ip[NB_KSTEPS];
  p.n_tiles = (int)op.ip[NB_NTILES];
  p.m_tiles = (int)((rows + NB_TILE_M - 1) / NB_TILE_M);
  p.groups = (int)op.ip[NB_GROUPS];
  p.fused = (int)op.ip[NB_FUSED];
  p.exact = op.ip[NB_ROUNDED_DEQUANT] ? 0 : 1;
  p.w_stage_bytes = st->w_stage_bytes;
  p.idesc = make_idesc(1u, 0u, 0u, NB_TILE_N, NB_TILE_M);
  p.alpha = (float)op.fp[NBF_ALPHA];
  const int64_t work = (int64_t)p.n_tiles * p.m_tiles;
  const int grid = (int)(work < ctx.num_sms ? work : ctx.num_sms);
  cudaError_t e = launch_pdl(nbits_gemm_kernel, dim3(grid), dim3(NB_THREADS), st->smem_bytes, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

// ------------------------------------------------------------------ Swish / Mul fp16 (unfused)
__global__ void swish_f16_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int64_t count,
                                 float alpha) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = swish_f16_fast(x[i], alpha);
}

__global__ void mul_f16_kernel(const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                               uint16_t* __restrict__ y, int64_t count) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = mul_f16(a[i], b[i]);
}

// Eight fp16 values per thread (16-byte loads and stores), same statements.
__global__ void mul_f16_x8_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b, uint4* __restrict__ y,
                                  int64_t n8) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 va = __ldcs(a + i), vb = __ldcs(b + i);
    const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
    uint32_t wy[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      wy[j] = (uint32_t)mul_f16((uint16_t)(wa[j] & 0xFFFFu), (uint16_t)(wb[j] & 0xFFFFu)) |
              ((uint32_t)mul_f16((uint16_t)(wa[j] >> 16), (uint16_t)(wb[j] >> 16)) << 16);
    __stcs(y + i, make_uint4(wy[0], wy[1], wy[2], wy[3]));
  }
}

// Standalone Swish through a table: an fp16 input has 65536 values, so the
// plan reserves a 128 KB table per Swish op that load time fills with
// swish_f16_fast of every input (the function the direct kernel evaluates,
// so the results are the same bits); a run is then a gather.  Persistent
// blocks copy the table into shared memory once and stream the tensor in
// 16-byte pieces (eight values per thread).
constexpr int SW_TABLE = 65536;
constexpr int SW_THREADS = 1024;

__global__ void swish_table_kernel(uint16_t* __restrict__ table, float alpha) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < SW_TABLE; i += gridDim.x * blockDim.x)
    table[i] = swish_f16_fast((uint16_t)i, alpha);
}

__global__ void __launch_bounds__(SW_THREADS) swish_f16_table_kernel(const uint4* __restrict__ x,
                                                                     uint4* __restrict__ y,
                                                                     const uint4* __restrict__ table, int64_t n8) {
  extern __shared__ uint4 s_table[];  // SW_TABLE fp16 values
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < SW_TABLE / 8; i += SW_THREADS) s_table[i] = table[i];  // filled at load time
  __syncthreads();
  pdl_wait();
  const uint16_t* t = reinterpret_cast<const uint16_t*>(s_table);
  for (int64_t i = blockIdx.x * (int64_t)SW_THREADS + threadIdx.x; i < n8; i += (int64_t)gridDim.x * SW_THREADS) {
    const uint4 v = __ldcs(x + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = (uint32_t)t[w[j] & 0xFFFFu] | ((uint32_t)t[w[j] >> 16] << 16);
    __stcs(y + i, make_uint4(o[0], o[1], o[2], o[3]));
  }
}

int prepare_swish_f16(const PlanOp& op, void* const* ptrs, OpState*, int, char* msg, size_t n) {
  if (op.n_tensors < 3 || op.t[2] < 0) return 0;
  cudaError_t e = cudaFuncSetAttribute(swish_f16_table_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SW_TABLE * 2);
  if (e == cudaSuccess) {
    swish_table_kernel<<<64, 1024>>>((uint16_t*)ptrs[op.t[2]], (float)op.fp[EWF_ALPHA]);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(msg, n, 4, "Swish table: %s", cudaGetErrorString(e));
  return 0;
}

static int64_t ew_count(const PlanOp& op, const LaunchCtx& ctx) {
  const int64_t rows = op.ip[EW_ROWS];
  if (rows > 0 && op.ip[IP_BATCHED] && ctx.batch > 0) return op.ip[EW_COUNT] / rows * ctx.batch;
  return op.ip[EW_COUNT];
}

int launch_swish_f16(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t count = ew_count(op, ctx);
  if (count == 0) return 0;
  const void* x = ptrs[op.t[0]];
  void* y = ptrs[op.t[1]];
  if (op.n_tensors > 2 && op.t[2] >= 0 && count % 8 == 0 && (((uintptr_t)x | (uintptr_t)y) & 15) == 0) {
    const int64_t n8 = count / 8, b64 = (n8 + SW_THREADS - 1) / SW_THREADS;
    cudaError_t e = launch_pdl(swish_f16_table_kernel, dim3((unsigned)(b64 < ctx.num_sms ? b64 : ctx.num_sms)),
                               dim3(SW_THREADS), (size_t)SW_TABLE * 2, ctx.stream, (const uint4*)x, (uint4*)y,
                               (const uint4*)ptrs[op.t[2]], n8);
    ++*launches;
    return e == cudaSuccess ? 0 : 4;
  }
  const int64_t blocks64 = (count + 255) / 256;
  const int blocks = (int)(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
  cudaError_t e = launch_pdl(swish_f16_kernel, dim3(blocks), dim3(256), 0, ctx.stream, (const uint16_t*)x,
                             (uint16_t*)y, count, (float)op.fp[EWF_ALPHA]);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

int launch_mul_f16(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t count = ew_count(op, ctx);
  if (count == 0) return 0;
  const int64_t blocks64 = (count + 255) / 256;
  const int blocks = (int)(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
  const void *a = ptrs[op.t[0]], *b = ptrs[op.t[1]];
  void* y = ptrs[op.t[2]];
  cudaError_t e;
  if (count % 8 == 0 && (((uintptr_t)a | (uintptr_t)b | (uintptr_t)y) & 15) == 0) {
    const int64_t n8 = count / 8, b64 = (n8 + 255) / 256;
    e = launch_pdl(mul_f16_x8_kernel, dim3((unsigned)(b64 < 148 * 16 ? b64 : 148 * 16)), dim3(256), 0, ctx.stream,
                   (const uint4*)a, (const uint4*)b, (uint4*)y, n8);
  } else {
    e = launch_pdl(mul_f16_kernel, dim3(blocks), dim3(256), 0, ctx.stream, (const uint16_t*)a, (const uint16_t*)b,
                   (uint16_t*)y, count);
  }
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
