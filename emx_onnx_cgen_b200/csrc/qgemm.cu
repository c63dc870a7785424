// QLinearMatMul / MatMulInteger on tcgen05 kind::i8 (reference
// templates/qlinear_matmul_op.c.j2:1-81, matmul_integer_op.c.j2; lowering
// ir/ops/nn.py:710-769).  The reference sums (a - za) * (b - zb) in int32; the
// tensor cores sum the raw 8-bit products a * b exactly in int32 (signed or
// unsigned per operand), and the epilogue restores the zero points with
//   sum (a - za)(b - zb) = sum a*b - zb * rowsum(A)[m] - za * colsum(B)[n] + K * za * zb,
// all modulo 2^32, so the result equals the reference's int32 sum whenever
// that sum is defined (no int32 overflow).  K <= 32768 keeps even the raw sum
// of u8 * u8 products below 2^31, so no accumulator ever wraps.  The output
// then goes through the CUDA-core kernel's requantisation (qm_requant_int or
// qm_requant_double, the form the plan selected, one per kernel instantiation).
//
// B^T (K-major rows [N][K], the layout the MMA reads) and B's column sums are
// packed by the planner when B is an initializer; otherwise a preparation
// launch writes them every run.  A's row sums (needed when zb != 0) come from
// that launch too.  Then the GEMM:
//   * tiles of 128 A rows x 256 output columns, K in steps of 128 bytes (one
//     128-byte swizzled row; four MMAs of K = 32); A and B^T arrive by TMA
//     (SWIZZLE_128B; rows and columns past the matrices read as zero) into a
//     ring of QG_STAGES stages;
//   * the 128 x 256 int32 accumulator is double-buffered in TMEM (2 x 256
//     columns), so the epilogue of a tile overlaps the main loop of the next;
//   * warps: 0 TMA producer, 1 MMA issuer + TMEM owner, 2-9 epilogue (TMEM
//     lane quarter = warp % 4, two warps per quarter on alternate 16-column
//     chunks; thread = one output row, 16 columns per tcgen05.ld).  Persistent CTAs walk the tiles m-fastest, so the CTAs in
//     flight share B^T tiles through L2.
#include "host_util.h"
#include "kernels.h"
#include "qmatmul.cuh"
#include "tc100.cuh"

namespace emx {

constexpr int QG_BM = 128;
constexpr int QG_BN = 256;
constexpr int QG_BK = 128;
constexpr int QG_STAGES = 4;
constexpr int QG_THREADS = 320;
constexpr int QG_EPI_WARPS = 8;
constexpr uint32_t QG_A_BYTES = QG_BM * QG_BK;
constexpr uint32_t QG_B_BYTES = QG_BN * QG_BK;
constexpr uint32_t QG_STAGE_BYTES = QG_A_BYTES + QG_B_BYTES;
constexpr size_t QG_SMEM = 1024 + (size_t)QG_STAGES * QG_STAGE_BYTES + (2 * QG_STAGES + 5) * 8 + 16;
constexpr int QG_PREP_COLS = 32;   // B columns per preparation block
constexpr int QG_PREP_K = 64;      // K rows per shared-memory transpose step
constexpr int QG_PREP_KSPLIT = 256;  // K rows per preparation block

struct QGemmParams {
  CUtensorMap map_a;  // A [M][K] bytes, box 128 x 128, SWIZZLE_128B
  CUtensorMap map_b;  // B^T [N][K] bytes, box 128 x 256, SWIZZLE_128B
  QMatMulParams q;
  const int32_t* rowsum;  // [M], or null when zb == 0
  const int32_t* colsum;  // [N], or null when za == 0
  int* err;
  int m_tiles, n_tiles, k_steps;
  int y_vec;  // Y rows start 16-byte aligned and hold whole 16-byte groups: vector stores
  uint32_t idesc;
};

struct QGemmPrepParams {
  const uint8_t* a;
  const uint8_t* b;
  uint8_t* bt;
  int32_t* rowsum;  // null: not needed
  int32_t* colsum;  // null: not needed (zeroed before the launch otherwise)
  int64_t m;
  int k, n, a_signed, b_signed, b_blocks, k_splits;
};

// Blocks [0, b_blocks): a 32-column x QG_PREP_KSPLIT-row slab of B, transposed
// through shared memory into B^T, its column sums added into colsum.  Blocks
// after that: eight A rows each (one warp per row), summed into rowsum.
__global__ void __launch_bounds__(256) qgemm_prep_kernel(const __grid_constant__ QGemmPrepParams p) {
  __shared__ uint8_t tile[QG_PREP_K][QG_PREP_COLS + 1];
  pdl_wait();
  pdl_launch_dependents();
  const int t = threadIdx.x;
  if ((int)blockIdx.x < p.b_blocks) {
    const int n0 = (blockIdx.x / p.k_splits) * QG_PREP_COLS;
    const int kbeg = (blockIdx.x % p.k_splits) * QG_PREP_KSPLIT;
    const int kend = min(p.k, kbeg + QG_PREP_KSPLIT);
    const int c = t >> 3, kk = (t & 7) * 8;  // writer: column c, 8 K bytes from kk
    const int n = n0 + c;
    int32_t part = 0;
    for (int k0 = kbeg; k0 < kend; k0 += QG_PREP_K) {
      {  // reader: row k0 + t/4, 8 columns from 8 * (t % 4)
        const int kr = k0 + (t >> 2), cb = 8 * (t & 3);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int nn = n0 + cb + j;
          tile[t >> 2][cb + j] = (kr < kend && nn < p.n) ? p.b[(int64_t)kr * p.n + nn] : (uint8_t)0;
        }
      }
      __syncthreads();
      const int kb = k0 + kk;
      if (n < p.n && kb < kend) {  // K % 16 == 0: eight bytes are all in range or all out
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint8_t v = tile[kk + j][c];
          w[j >> 2] |= (uint32_t)v << (8 * (j & 3));
          part += p.b_signed ? (int32_t)(int8_t)v : (int32_t)v;
        }
        *reinterpret_cast<uint2*>(p.bt + (int64_t)n * p.k + kb) = make_uint2(w[0], w[1]);
      }
      __syncthreads();
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    part += __shfl_xor_sync(0xffffffffu, part, 4);
    if (p.colsum && (t & 7) == 0 && n < p.n) atomicAdd(p.colsum + n, part);
  } else {
    const int lane = t & 31;
    const int64_t row = (int64_t)(blockIdx.x - p.b_blocks) * 8 + (t >> 5);
    if (row >= p.m || !p.rowsum) return;
    const uint4* ar = reinterpret_cast<const uint4*>(p.a + row * p.k);  // K % 16 == 0, A 16-byte aligned
    int32_t s = 0;
    for (int i = lane; i < p.k / 16; i += 32) {
      const uint4 v = ar[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t byte = (w[j] >> (8 * b)) & 0xFFu;
          s += p.a_signed ? (int32_t)(int8_t)byte : (int32_t)byte;
        }
    }
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) p.rowsum[row] = s;
  }
}

// MODE: QG_OUT_I32 (MatMulInteger), QG_OUT_REQ_INT / QG_OUT_REQ_DOUBLE (QLinearMatMul's two
// requantisations), so each instantiation's epilogue carries one form only.
enum { QG_OUT_I32, QG_OUT_REQ_INT, QG_OUT_REQ_DOUBLE };

template <int MODE>
__global__ void __launch_bounds__(QG_THREADS, 1) qgemm_tc_kernel(const __grid_constant__ QGemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + QG_STAGES * QG_STAGE_BYTES);
  uint64_t* empty = full + QG_STAGES;
  uint64_t* acc_full = empty + QG_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_work = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < QG_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], QG_EPI_WARPS);
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
      // ---------------- TMA producer
      pdl_wait();  // A from the preceding kernels, B^T from the preparation launch
      int s = 0;
      uint32_t ph = 0, issued = 0, parity_of = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_work && ok; t += gridDim.x) {
        const int m0 = (t % p.m_tiles) * QG_BM, n0 = (t / p.m_tiles) * QG_BN;
        for (int ks = 0; ks < p.k_steps; ++ks) {
          if (!mbar_wait(&empty[s], ph ^ 1u, p.err, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * QG_STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], QG_STAGE_BYTES);
          tma_load_2d(st, &p.map_a, &full[s], ks * QG_BK, m0);
          tma_load_2d(st + QG_A_BYTES, &p.map_b, &full[s], ks * QG_BK, n0);
          issued |= 1u << s;
          parity_of = (parity_of & ~(1u << s)) | (ph << s);
          if (++s == QG_STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok)  // error path: let every load this thread issued land before the CTA exits
        for (int s2 = 0; s2 < QG_STAGES; ++s2)
          if (issued & (1u << s2)) (void)mbar_wait(&full[s2], (parity_of >> s2) & 1u, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      int s = 0, it = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint32_t base = smem_u32(smem);
      for (int t = blockIdx.x; t < n_work && ok; t += gridDim.x, ++it) {
        const int b = it & 1;
        if (!mbar_wait(&acc_empty[b], ((it >> 1) & 1) ^ 1u, p.err, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(b * QG_BN);
        for (int ks = 0; ks < p.k_steps; ++ks) {
          if (!mbar_wait(&full[s], ph, p.err, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = base + (uint32_t)s * QG_STAGE_BYTES, b_addr = a_addr + QG_A_BYTES;
#pragma unroll
          for (int kk = 0; kk < QG_BK / 32; ++kk)
            mma_i8(d_tmem, smem_desc_k_swizzled(a_addr + 32u * kk, 128), smem_desc_k_swizzled(b_addr + 32u * kk, 128),
                   p.idesc, (ks | kk) != 0 ? 1u : 0u);
          tc_commit(&empty[s]);
          if (++s == QG_STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) tc_commit(&acc_full[b]);
      }
      if (!ok) {  // error path: wait for this thread's MMAs before TMEM is released
        tc_commit(drain);
        (void)mbar_wait(drain, 0, nullptr, 0);
      }
    }
  } else {
    // ---------------- epilogue: thread = output row q*32 + lane of the tile; the
    // two warps of a lane quarter take alternate 16-column chunks
    const int q = warp & 3, half = (warp - 2) >> 2;
    pdl_wait();  // row/column sums from the preparation launch; Y may still be read upstream
    const QMatMulParams& qp = p.q;
    const uint32_t kzz = (uint32_t)qp.k * (uint32_t)qp.za * (uint32_t)qp.zb;
    const bool vec = p.y_vec != 0;
    int it = 0;
    for (int t = blockIdx.x; t < n_work; t += gridDim.x, ++it) {
      const int m0 = (t % p.m_tiles) * QG_BM, n0 = (t / p.m_tiles) * QG_BN;
      const int b = it & 1;
      bool ok = mbar_wait(&acc_full[b], (it >> 1) & 1, p.err, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int64_t m = m0 + q * 32 + lane;
      const bool row_ok = m < qp.m;
      // sum a*b - zb * rowsum - za * colsum + K * za * zb, modulo 2^32
      const uint32_t row_corr = kzz - (uint32_t)qp.zb * (uint32_t)(p.rowsum && row_ok ? p.rowsum[m] : 0);
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * QG_BN);
      const int nc = min(QG_BN / 16, (qp.n - n0 + 15) / 16);
      for (int c = half; c < nc; c += 2) {
        uint32_t v[16];
        tmem_ld16(taddr + c * 16, v);
        tmem_wait_ld();
        const int nb = n0 + c * 16;
        int32_t acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = nb + j;
          const uint32_t cs = p.colsum && n < qp.n ? (uint32_t)p.colsum[n] : 0u;
          acc[j] = (int32_t)(v[j] + row_corr - (uint32_t)qp.za * cs);
        }
        if (!row_ok) continue;
        if (MODE != QG_OUT_I32) {
          uint8_t* yr = reinterpret_cast<uint8_t*>(qp.y) + m * qp.n;
          if (vec) {  // n % 16 == 0: the 16 columns are all in range
            uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
            for (int j = 0; j < 16; ++j)
              w[j >> 2] |= (uint32_t)(MODE == QG_OUT_REQ_INT ? qm_requant_int(acc[j], qp) : qm_requant_double(acc[j], qp))
                           << (8 * (j & 3));
            *reinterpret_cast<uint4*>(yr + nb) = make_uint4(w[0], w[1], w[2], w[3]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (nb + j < qp.n)
                yr[nb + j] = MODE == QG_OUT_REQ_INT ? qm_requant_int(acc[j], qp) : qm_requant_double(acc[j], qp);
          }
        } else {
          int32_t* yr = reinterpret_cast<int32_t*>(qp.y) + m * qp.n;
          if (vec && nb + 16 <= qp.n) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<int4*>(yr + nb + j) = make_int4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (nb + j < qp.n) yr[nb + j] = acc[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ------------------------------------------------------------------ host side
int prepare_qgemm_tc() {
  for (auto fn : {qgemm_tc_kernel<QG_OUT_I32>, qgemm_tc_kernel<QG_OUT_REQ_INT>, qgemm_tc_kernel<QG_OUT_REQ_DOUBLE>})
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QG_SMEM) != cudaSuccess) return 4;
  return 0;
}

// t[3] = B^T scratch [N][K], t[4] = column sums [N] int32, t[5] = row sums [M] int32.
// Returns -1 when the tensor-core path does not apply to these pointers (the
// caller then runs the CUDA-core kernel).
int launch_qgemm_tc(const PlanOp& op, void* const* ptrs, const LaunchCtx& ctx, const QMatMulParams& q,
                    int* launches) {
  if (q.k % 16 || q.k > 32768 || ((uintptr_t)q.a & 15u)) return -1;
  const bool packed = op.ip[QM_B_PACKED] != 0;
  uint8_t* bt = (uint8_t*)ptrs[op.t[3]];
  int32_t* colsum = q.za ? (int32_t*)ptrs[op.t[4]] : nullptr;
  int32_t* rowsum = q.zb ? (int32_t*)ptrs[op.t[5]] : nullptr;
  QGemmPrepParams pp{};
  pp.a = q.a;
  pp.b = q.b;
  pp.bt = bt;
  pp.rowsum = rowsum;
  pp.colsum = packed ? nullptr : colsum;
  pp.m = q.m;
  pp.k = q.k;
  pp.n = q.n;
  pp.a_signed = q.a_signed;
  pp.b_signed = q.b_signed;
  pp.k_splits = (q.k + QG_PREP_KSPLIT - 1) / QG_PREP_KSPLIT;
  pp.b_blocks = packed ? 0 : (q.n + QG_PREP_COLS - 1) / QG_PREP_COLS * pp.k_splits;
  const int64_t a_blocks = rowsum ? (q.m + 7) / 8 : 0;
  if (pp.colsum && cudaMemsetAsync(pp.colsum, 0, (size_t)q.n * 4, ctx.stream) != cudaSuccess) return 4;
  cudaError_t e = cudaSuccess;
  if (pp.b_blocks + a_blocks > 0) {
    e = launch_pdl(qgemm_prep_kernel, dim3((unsigned)(pp.b_blocks + a_blocks)), dim3(256), 0, ctx.stream, pp);
    ++*launches;
    if (e != cudaSuccess) return 4;
  }

  QGemmParams p{};
  char msg[256];
  if (make_tmap_2d(&p.map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q.a, (uint64_t)q.k, (uint64_t)q.m, (uint64_t)q.k, QG_BK,
                   QG_BM, CU_TENSOR_MAP_SWIZZLE_128B, msg, sizeof(msg)))
    return 4;
  if (make_tmap_2d(&p.map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, bt, (uint64_t)q.k, (uint64_t)q.n, (uint64_t)q.k, QG_BK,
                   QG_BN, CU_TENSOR_MAP_SWIZZLE_128B, msg, sizeof(msg)))
    return 4;
  p.q = q;
  p.rowsum = rowsum;
  p.colsum = colsum;
  p.err = ctx.d_error;
  p.m_tiles = (int)((q.m + QG_BM - 1) / QG_BM);
  p.n_tiles = (q.n + QG_BN - 1) / QG_BN;
  p.k_steps = (q.k + QG_BK - 1) / QG_BK;
  p.y_vec = ((uintptr_t)q.y & 15u) == 0 && (q.quantized ? q.n % 16 == 0 : q.n % 4 == 0);
  p.idesc = make_idesc(2u, (uint32_t)q.a_signed, (uint32_t)q.b_signed, QG_BM, QG_BN);
  const int64_t work = (int64_t)p.m_tiles * p.n_tiles;
  const int grid = (int)(work < ctx.num_sms ? work : ctx.num_sms);
  void (*fn)(QGemmParams) = !q.quantized ? qgemm_tc_kernel<QG_OUT_I32>
                            : q.use_int ? qgemm_tc_kernel<QG_OUT_REQ_INT>
                                        : qgemm_tc_kernel<QG_OUT_REQ_DOUBLE>;
  e = launch_pdl(fn, dim3(grid), dim3(QG_THREADS), QG_SMEM, ctx.stream, p);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
