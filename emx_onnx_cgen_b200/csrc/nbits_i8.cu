// com.microsoft MatMulNBits, accuracy_level 4, fp16 activations: the int8
// activation path (reference: templates/matmul_nbits_int8_op.c.j2:1-78,
// selected by ir/ops/nn.py:1183-1190).
//
// Reference arithmetic, per row of A and K block (float accumulator):
//   amax    = max |a|                 a_scale = amax / 127
//   a_inv   = amax > 0 ? 127 / amax : 0
//   qa      = (int8) clamp(nearbyintf(a * a_inv), -128, 127)
// and per output, blocks in order:
//   acc += (float)isum * (a_scale * b_scale),  isum = sum qa * (q - zp)  (exact int32)
//   acc += bias;  y = (fp16) acc
// Two launches: the quantiser writes qa [rows][KP] and a_scale [rows][NBLK]
// (scratch in the arena); the block GEMM sums each block with dp4a (exact
// int32, any order) and repeats the float statements one rounding at a time
// (__fmul_rn / __fadd_rn, never contracted into an FMA).  The planner packs the
// weights as int8 (q - zp) [N][KP] (|q - zp| <= 15), zero-padded past K, so a
// partial last block adds exact zeros, and the scales as float [N][NBLK].
#include "host_util.h"
#include "kernels.h"
#include "tc100.cuh"

#include <cuda_fp16.h>

namespace emx {

// One warp per (row, block): the block's |a| maximum (NaN never wins a
// comparison, as in the reference's `if (av > amax)`), its scale, and the
// quantised bytes.  Bytes in [K, KP) are written as zero.
__global__ void __launch_bounds__(256) nbits_i8_quant_kernel(const __half* __restrict__ a, int64_t rows, int k,
                                                             int kp, int block, int nblk, int8_t* __restrict__ qa,
                                                             float* __restrict__ a_scale) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t item = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); item < rows * nblk;
       item += warps) {
    const int64_t row = item / nblk;
    const int blk = (int)(item - row * nblk);
    const __half* ar = a + row * (int64_t)k;
    const int k0 = blk * block;
    float amax = 0.0f;
    for (int kk = lane; kk < block; kk += 32) {
      const int kx = k0 + kk;
      if (kx < k) {
        const float av = fabsf(__half2float(ar[kx]));
        if (av > amax) amax = av;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float other = __shfl_xor_sync(0xffffffffu, amax, o);
      if (other > amax) amax = other;
    }
    const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    if (lane == 0) a_scale[row * nblk + blk] = __fdiv_rn(amax, 127.0f);
    int8_t* qr = qa + row * (int64_t)kp;
    for (int kk = lane; kk < block; kk += 32) {
      const int kx = k0 + kk;
      if (kx >= kp) break;
      int8_t q = 0;
      if (kx < k) {
        float v = rintf(__fmul_rn(__half2float(ar[kx]), inv));
        if (v > 127.0f) v = 127.0f;
        if (v < -128.0f) v = -128.0f;
        q = (int8_t)__float2int_rz(v);  // NaN -> 0, as the x86 conversion's low byte
      }
      qr[kx] = q;
    }
  }
}

constexpr int NI_BM = 64, NI_BN = 64, NI_THREADS = 256;

// Block GEMM: CTA tile 64 rows x 64 columns, thread (tx, ty) owns rows
// 4*ty .. 4*ty+3 and columns tx + 16*c (c < 4).  Each K block of qa and of the
// packed weights is staged in shared memory (row pitch block + 16 bytes:
// conflict-free 16-byte loads); its int32 sums come from dp4a over 4-byte
// words, then every output takes the block's float step in block order.
__global__ void __launch_bounds__(NI_THREADS) nbits_i8_gemm_kernel(const int8_t* __restrict__ qa,
                                                                   const float* __restrict__ a_scale,
                                                                   const int8_t* __restrict__ w,
                                                                   const float* __restrict__ b_scale,
                                                                   const float* __restrict__ bias, __half* __restrict__ y,
                                                                   int64_t rows, int n, int kp, int block, int nblk) {
  extern __shared__ __align__(16) uint8_t ni_smem[];
  const int pitch = block + 16;
  uint8_t* sa = ni_smem;                       // [NI_BM][pitch]
  uint8_t* sw = ni_smem + NI_BM * pitch;       // [NI_BN][pitch]
  float* s_as = reinterpret_cast<float*>(sw + NI_BN * pitch);  // [NI_BM]
  float* s_bs = s_as + NI_BM;                                  // [NI_BN]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * NI_BM;
  const int n0 = blockIdx.x * NI_BN;
  pdl_wait();
  pdl_launch_dependents();
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
  const int chunks = block / 16;  // 16-byte chunks per row of a block
  for (int blk = 0; blk < nblk; ++blk) {
    const int64_t kb = (int64_t)blk * block;
    for (int e = tid; e < (NI_BM + NI_BN) * chunks; e += NI_THREADS) {
      const int rr = e / chunks, ch = e - rr * chunks;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (rr < NI_BM) {
        if (m0 + rr < rows) v = *reinterpret_cast<const uint4*>(qa + (m0 + rr) * kp + kb + 16 * ch);
        *reinterpret_cast<uint4*>(sa + rr * pitch + 16 * ch) = v;
      } else {
        const int cc = rr - NI_BM;
        if (n0 + cc < n) v = *reinterpret_cast<const uint4*>(w + (int64_t)(n0 + cc) * kp + kb + 16 * ch);
        *reinterpret_cast<uint4*>(sw + cc * pitch + 16 * ch) = v;
      }
    }
    if (tid < NI_BM) s_as[tid] = m0 + tid < rows ? a_scale[(m0 + tid) * nblk + blk] : 0.0f;
    else if (tid < NI_BM + NI_BN) {
      const int cc = tid - NI_BM;
      s_bs[cc] = n0 + cc < n ? b_scale[(int64_t)(n0 + cc) * nblk + blk] : 0.0f;
    }
    __syncthreads();
    int isum[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) isum[r][c] = 0;
    for (int ch = 0; ch < chunks; ++ch) {
      uint4 av[4], wv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) av[r] = *reinterpret_cast<const uint4*>(sa + (4 * ty + r) * pitch + 16 * ch);
#pragma unroll
      for (int c = 0; c < 4; ++c) wv[c] = *reinterpret_cast<const uint4*>(sw + (tx + 16 * c) * pitch + 16 * ch);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          int s = isum[r][c];
          s = __dp4a((int)av[r].x, (int)wv[c].x, s);
          s = __dp4a((int)av[r].y, (int)wv[c].y, s);
          s = __dp4a((int)av[r].z, (int)wv[c].z, s);
          s = __dp4a((int)av[r].w, (int)wv[c].w, s);
          isum[r][c] = s;
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float as = s_as[4 * ty + r];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float sc = __fmul_rn(as, s_bs[tx + 16 * c]);
        acc[r][c] = __fadd_rn(acc[r][c], __fmul_rn(__int2float_rn(isum[r][c]), sc));
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t i = m0 + 4 * ty + r;
    if (i >= rows) continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = n0 + tx + 16 * c;
      if (j >= n) continue;
      float v = acc[r][c];
      if (bias) v = __fadd_rn(v, bias[j]);
      y[i * n + j] = __float2half_rn(v);
    }
  }
}

int prepare_nbits_i8(const PlanOp& op, void* const*, OpState*, int, char* msg, size_t n) {
  const int64_t block = op.ip[NI_BLOCK], kp = op.ip[NI_KP];
  if (block < 16 || block % 16 || block > 4096 || kp % block || op.ip[NI_NBLK] * block != kp)
    return fail(msg, n, 5, "MatMulNBits int8 path: block %lld, padded K %lld", (long long)block, (long long)kp);
  const size_t smem = (size_t)(NI_BM + NI_BN) * (size_t)(block + 16) + (NI_BM + NI_BN) * sizeof(float);
  if (smem > 227 * 1024) return fail(msg, n, 5, "MatMulNBits int8 path needs %zu B smem", smem);
  cudaError_t e = cudaFuncSetAttribute(nbits_i8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(msg, n, 4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  return 0;
}

int launch_nbits_i8(const PlanOp& op, void* const* ptrs, const OpState*, const LaunchCtx& ctx, int* launches) {
  const int64_t rpb = op.ip[NI_ROWS_PER_BATCH] > 0 ? op.ip[NI_ROWS_PER_BATCH] : 1;
  const int64_t rows = op.ip[IP_BATCHED] && ctx.batch > 0 ? ctx.batch * rpb : op.ip[NI_ROWS];
  if (rows <= 0) return 0;
  const int k = (int)op.ip[NI_K], kp = (int)op.ip[NI_KP], n = (int)op.ip[NI_N];
  const int block = (int)op.ip[NI_BLOCK], nblk = (int)op.ip[NI_NBLK];
  int8_t* qa = (int8_t*)ptrs[op.t[4]];
  float* as = (float*)ptrs[op.t[5]];
  const int64_t items = rows * nblk;
  const int64_t qblocks = (items + 7) / 8;
  cudaError_t e = launch_pdl(nbits_i8_quant_kernel, dim3((unsigned)(qblocks < 148 * 64 ? qblocks : 148 * 64)),
                             dim3(256), 0, ctx.stream, (const __half*)ptrs[op.t[0]], rows, k, kp, block, nblk, qa, as);
  ++*launches;
  if (e != cudaSuccess) return 4;
  const size_t smem = (size_t)(NI_BM + NI_BN) * (size_t)(block + 16) + (NI_BM + NI_BN) * sizeof(float);
  dim3 grid((unsigned)((n + NI_BN - 1) / NI_BN), (unsigned)((rows + NI_BM - 1) / NI_BM));
  e = launch_pdl(nbits_i8_gemm_kernel, grid, dim3(NI_THREADS), smem, ctx.stream, (const int8_t*)qa, (const float*)as,
                 (const int8_t*)ptrs[op.t[1]], (const float*)ptrs[op.t[2]],
                 op.t[3] >= 0 ? (const float*)ptrs[op.t[3]] : nullptr, (__half*)ptrs[op.t[6]], rows, n, kp, block,
                 nblk);
  ++*launches;
  return e == cudaSuccess ? 0 : 4;
}

}  // namespace emx
