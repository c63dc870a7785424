// Exact-order fp32 dot-product chains for the reference's `acc += a * b`
// loops (gcc -O2 on x86-64: every multiply and every add rounded separately,
// k ascending, no FMA):  acc[m][n] += A[m][k] * B[n][k] for k = 0 .. K-1.
//
// Each output is one sequential chain, so parallelism comes only from the
// M x N outputs; the chains are fed from shared memory that a cp.async ring
// of S stages (BK columns of K each) keeps filled several stages ahead, so
// the chains never wait on global-memory latency.  Every step is a
// __fmul_rn followed by a __fadd_rn, which CUDA never merges into an FMA.
// (Packed f32x2 multiply/add pairs were measured to be contracted into
// fused multiply-adds by the code generator here, which changes the
// rounding, so they are not used.)  Accumulators are plain floats: packing
// them as pairs in 64-bit integers cost integer instructions per step.
//
// Thread (tx, ty) of the CTA owns rows m0 + ty*RM + r (r < RM) and columns
// n0 + tx + c*TX (c < RN, TX = BN / RN), accumulator acc[r][c]: columns are strided so that the
// threads of a quarter warp read consecutive shared-memory rows
// (conflict-free 16-byte loads).  A is [M][K] with row pitch lda, B is [N][K]
// with row pitch ldb (K contiguous in both), K % 4 == 0, both bases and pitches
// 16-byte aligned; rows past M / columns past N read as zero.
#pragma once
#include <stdint.h>

namespace emx {

__device__ __forceinline__ void xc_cp16(float* dst, const float* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
// cp.async with an L2 cache policy (createpolicy), e.g. evict-last for a
// matrix that every step re-reads while a larger stream passes through L2
__device__ __forceinline__ void xc_cp16_policy(float* dst, const float* src, bool valid, uint64_t policy) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(d), "l"(src),
               "r"(valid ? 16 : 0), "l"(policy)
               : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void xc_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void xc_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// B_KEEP: B's rows are loaded with an L2 evict-last policy (B re-read by later launches).
template <int BM, int BN, int RM, int RN, int BK, int S, bool B_KEEP = false>
struct ExactChain {
  static_assert(RN >= 1 && BK % 4 == 0 && RM >= 1, "tile shape");
  static constexpr int TX = BN / RN, TY = BM / RM, NT = TX * TY;
  static constexpr int PITCH = BK + 4;  // floats per shared-memory row (keeps 16-byte rows, shifts banks)
  static constexpr size_t SMEM_BYTES = (size_t)S * (BM + BN) * PITCH * sizeof(float);

  static __device__ __forceinline__ void load_stage(float* As, float* Bs, const float* A, int lda, const float* B,
                                                    int ldb, int M, int N, int K, int m0, int n0, int k0) {
    constexpr int CQ = BK / 4;  // 16-byte chunks per row
    for (int e = threadIdx.x; e < (BM + BN) * CQ; e += NT) {
      const int row = e / CQ, cq = e - row * CQ;
      const int k = k0 + 4 * cq;
      if (row < BM) {
        const bool ok = m0 + row < M && k < K;
        xc_cp16(As + row * PITCH + 4 * cq, ok ? A + (size_t)(m0 + row) * lda + k : A, ok);
      } else {
        const int r = row - BM;
        const bool ok = n0 + r < N && k < K;
        if constexpr (B_KEEP)
          xc_cp16_policy(Bs + r * PITCH + 4 * cq, ok ? B + (size_t)(n0 + r) * ldb + k : B, ok, l2_policy_evict_last());
        else
          xc_cp16(Bs + r * PITCH + 4 * cq, ok ? B + (size_t)(n0 + r) * ldb + k : B, ok);
      }
    }
  }

  static __device__ __forceinline__ void run(const float* __restrict__ A, int lda, const float* __restrict__ B,
                                             int ldb, int M, int N, int K, int m0, int n0, float (&acc)[RM][RN],
                                             float* smem) {
    const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
    float* As = smem;                          // [S][BM][PITCH]
    float* Bs = smem + (size_t)S * BM * PITCH;  // [S][BN][PITCH]
    const int KT = (K + BK - 1) / BK;
#pragma unroll
    for (int s = 0; s < S - 1; ++s) {
      if (s < KT) load_stage(As + s * BM * PITCH, Bs + s * BN * PITCH, A, lda, B, ldb, M, N, K, m0, n0, s * BK);
      xc_commit();
    }
    for (int t = 0; t < KT; ++t) {
      xc_wait<S - 2>();
      __syncthreads();  // stage t is complete for every thread; stage t-1 is no longer read
      const int tn = t + S - 1;
      if (tn < KT) {
        const int sn = tn % S;
        load_stage(As + sn * BM * PITCH, Bs + sn * BN * PITCH, A, lda, B, ldb, M, N, K, m0, n0, tn * BK);
      }
      xc_commit();
      const float* as = As + (t % S) * BM * PITCH + ty * RM * PITCH;
      const float* bs = Bs + (t % S) * BN * PITCH + tx * PITCH;
      const int klen = min(BK, K - t * BK);  // a multiple of 4: never add past K
      for (int kk = 0; kk < klen; kk += 4) {
        float4 a4[RM], b4[RN];
#pragma unroll
        for (int r = 0; r < RM; ++r) a4[r] = *reinterpret_cast<const float4*>(as + r * PITCH + kk);
#pragma unroll
        for (int c = 0; c < RN; ++c) b4[c] = *reinterpret_cast<const float4*>(bs + c * TX * PITCH + kk);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float bj[RN];
#pragma unroll
          for (int c = 0; c < RN; ++c) bj[c] = j == 0 ? b4[c].x : j == 1 ? b4[c].y : j == 2 ? b4[c].z : b4[c].w;
#pragma unroll
          for (int r = 0; r < RM; ++r) {
            const float a = j == 0 ? a4[r].x : j == 1 ? a4[r].y : j == 2 ? a4[r].z : a4[r].w;
#pragma unroll
            for (int c = 0; c < RN; ++c) acc[r][c] = __fadd_rn(acc[r][c], __fmul_rn(a, bj[c]));
          }
        }
      }
    }
    xc_wait<0>();
    __syncthreads();
  }

  // column of accumulator c (0..RN-1) for thread tx
  static __device__ __forceinline__ int col(int tx, int c) { return tx + c * TX; }
};

}  // namespace emx
