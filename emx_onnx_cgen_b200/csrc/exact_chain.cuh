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

// Shared memory holds S stages, each one contiguous block of BM rows of A then
// BN rows of B ([BM + BN][PITCH] floats).  A thread's 16-byte copies are the
// same (row, chunk) pairs in every stage, only shifted along K, so their
// global row addresses and shared offsets are computed once; a stage then
// costs one address add and one cp.async per copy.  Full-width stages
// (BK columns inside K, all but possibly the last) run a fully unrolled
// inner loop, which lets the compiler hoist the next shared-memory loads
// above the current multiply-adds.
template <int BM, int BN, int RM, int RN, int BK, int S>
struct ExactChain {
  static_assert(RN >= 1 && BK % 4 == 0 && RM >= 1, "tile shape");
  static constexpr int TX = BN / RN, TY = BM / RM, NT = TX * TY;
  static constexpr int PITCH = BK + 4;  // floats per shared-memory row (keeps 16-byte rows, shifts banks)
  static constexpr int STAGE = (BM + BN) * PITCH;  // floats per stage
  static constexpr size_t SMEM_BYTES = (size_t)S * STAGE * sizeof(float);
  static constexpr int CQ = BK / 4;                            // 16-byte chunks per row and stage
  static constexpr int NCOPY = ((BM + BN) * CQ + NT - 1) / NT;  // copies per thread and stage
  static constexpr bool EVEN = NCOPY * NT == (BM + BN) * CQ;

  struct Copies {
    const float* src[NCOPY];  // global address of the chunk at k = 0, or nullptr for a row past M / N
    uint32_t dst[NCOPY];      // byte offset of the chunk within a stage
    int kq[NCOPY];            // the chunk's first column within a stage
  };

  static __device__ __forceinline__ void plan_copies(Copies& cp, const float* A, int lda, const float* B, int ldb,
                                                     int M, int N, int m0, int n0) {
#pragma unroll
    for (int i = 0; i < NCOPY; ++i) {
      const int e = threadIdx.x + i * NT;
      const int row = e / CQ, cq = e - row * CQ;
      cp.kq[i] = 4 * cq;
      cp.dst[i] = (uint32_t)((row * PITCH + 4 * cq) * sizeof(float));
      const float* src = nullptr;
      if (row < BM) {
        if (m0 + row < M) src = A + (size_t)(m0 + row) * lda + 4 * cq;
      } else if (row < BM + BN) {
        if (n0 + row - BM < N) src = B + (size_t)(n0 + row - BM) * ldb + 4 * cq;
      }
      cp.src[i] = src;
    }
  }

  // one stage's copies: columns k0 .. k0+BK-1; chunks past K or rows past M / N are zero-filled
  static __device__ __forceinline__ void load_stage(const Copies& cp, uint32_t stage_addr, const float* fallback,
                                                    int K, int k0) {
    const bool full = k0 + BK <= K;
#pragma unroll
    for (int i = 0; i < NCOPY; ++i) {
      if (!EVEN && threadIdx.x + i * NT >= (BM + BN) * CQ) continue;
      const bool ok = cp.src[i] != nullptr && (full || k0 + cp.kq[i] < K);
      const float* src = ok ? cp.src[i] + k0 : fallback;
      const uint32_t d = stage_addr + cp.dst[i];
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(ok ? 16 : 0) : "memory");
    }
  }

  // four k-steps of every chain of this thread from shared memory (the
  // compiler's own schedule of the unrolled stage was measured faster than
  // explicitly double-buffered fragments)
  static __device__ __forceinline__ void step4(const float* as, const float* bs, int kk, float (&acc)[RM][RN]) {
    float4 a4[RM], b4[RN];
#pragma unroll
    for (int r = 0; r < RM; ++r) a4[r] = *reinterpret_cast<const float4*>(as + r * PITCH + kk);
#pragma unroll
    for (int c = 0; c < RN; ++c) b4[c] = *reinterpret_cast<const float4*>(bs + c * TX * PITCH + kk);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int r = 0; r < RM; ++r) {
        const float a = j == 0 ? a4[r].x : j == 1 ? a4[r].y : j == 2 ? a4[r].z : a4[r].w;
#pragma unroll
        for (int c = 0; c < RN; ++c) {
          const float b = j == 0 ? b4[c].x : j == 1 ? b4[c].y : j == 2 ? b4[c].z : b4[c].w;
          acc[r][c] = __fadd_rn(acc[r][c], __fmul_rn(a, b));
        }
      }
    }
  }

  static __device__ __forceinline__ void run(const float* __restrict__ A, int lda, const float* __restrict__ B,
                                             int ldb, int M, int N, int K, int m0, int n0, float (&acc)[RM][RN],
                                             float* smem) {
    const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
    const uint32_t smem_addr = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    Copies cp;
    plan_copies(cp, A, lda, B, ldb, M, N, m0, n0);
    const int KT = (K + BK - 1) / BK;
#pragma unroll
    for (int s = 0; s < S - 1; ++s) {
      if (s < KT) load_stage(cp, smem_addr + (uint32_t)(s * STAGE * sizeof(float)), A, K, s * BK);
      xc_commit();
    }
    for (int t = 0; t < KT; ++t) {
      xc_wait<S - 2>();
      __syncthreads();  // stage t is complete for every thread; stage t-1 is no longer read
      const int tn = t + S - 1;
      if (tn < KT) load_stage(cp, smem_addr + (uint32_t)((tn % S) * STAGE * sizeof(float)), A, K, tn * BK);
      xc_commit();
      const float* stage = smem + (t % S) * STAGE;
      const float* as = stage + ty * RM * PITCH;
      const float* bs = stage + (BM + tx) * PITCH;
      if (t * BK + BK <= K) {
#pragma unroll
        for (int kk = 0; kk < BK; kk += 4) step4(as, bs, kk, acc);
      } else {
        const int klen = K - t * BK;  // a multiple of 4: never add past K
        for (int kk = 0; kk < klen; kk += 4) step4(as, bs, kk, acc);
      }
    }
    xc_wait<0>();
    __syncthreads();
  }

  // column of accumulator c (0..RN-1) for thread tx
  static __device__ __forceinline__ int col(int tx, int c) { return tx + c * TX; }
};

}  // namespace emx
