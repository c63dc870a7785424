// Thin inline-PTX layer for sm_100a: mbarriers with bounded waits, TMA tile
// loads (no multicast anywhere), bulk copies, TMEM allocation, tcgen05.mma and
// tcgen05.ld.  Every wait gives up after a wall-clock budget and records an
// error code in a device word the host reads back (emx_b200_sync), so a broken
// pipeline returns EMX_ERR_DEVICE_TIMEOUT instead of hanging the GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace emx {

// Error codes written to the device error word (first writer wins).
enum DeviceError : int {
  DEV_OK = 0,
  DEV_TIMEOUT_PRODUCER = 1,
  DEV_TIMEOUT_MMA = 2,
  DEV_TIMEOUT_EPILOGUE = 3,
  DEV_TIMEOUT_GRID = 4,
  DEV_BAD_CONFIG = 5,
};

// Bounded waits: give up after this many nanoseconds of %globaltimer.  The
// default; a plan can set its own (emx_b200_set_wait_budget), stored in the
// 64-bit word 8 bytes after its device error word.
#ifndef EMX_WAIT_BUDGET_NS
#define EMX_WAIT_BUDGET_NS 2000000000ull
#endif

__host__ __device__ __forceinline__ constexpr size_t align_up_dev(size_t v, size_t a) { return (v + a - 1) / a * a; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ bool error_raised(const int* err) {
  return err && *reinterpret_cast<const volatile int*>(err) != 0;
}

// Wait budget of the plan owning `err` (read when a wait starts spinning, not
// on the fast path): the word 8 bytes after the error word, 0 = the default.
__device__ __forceinline__ uint64_t wait_budget_ns(const int* err) {
  if (!err) return EMX_WAIT_BUDGET_NS;
  const uint64_t v = *reinterpret_cast<const volatile unsigned long long*>(err + 2);
  return v ? v : EMX_WAIT_BUDGET_NS;
}

// ----------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed.  Returns false
// (and records `code`) when the budget runs out or another role already
// failed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t budget = wait_budget_ns(err);
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (error_raised(err)) return false;
      if (globaltimer_ns() - t0 > budget) {
        record_error(err, code);
        return false;
      }
    }
  }
}

// ----------------------------------------------------------------- cross-CTA flags
// Generic-proxy writes of this thread are ordered before later async-proxy
// (bulk copy) accesses to global memory, and vice versa.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void st_release_cta_u32(uint32_t* smem_p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(smem_p)), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_cta_u32(const uint32_t* smem_p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(smem_p)) : "memory");
  return v;
}

// Wait until flags[i] >= target for every i in [lo, hi] (clipped to [0, n)).
// The flags are read 8 at a time with independent loads (one memory round
// trip for a typical range), then any that are not there yet are polled.
// Returns false (recording `code`) when the budget runs out or another role
// already failed.
__device__ __forceinline__ bool wait_flags_at_least(const unsigned long long* flags, int lo, int hi, int n,
                                                    unsigned long long target, int* err, int code) {
  if (lo < 0) lo = 0;
  if (hi > n - 1) hi = n - 1;
  for (int base = lo; base <= hi; base += 8) {
    unsigned long long v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = base + j <= hi ? ld_acquire_u64(flags + base + j) : target;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (v[j] >= target) continue;
      const uint64_t t0 = globaltimer_ns();
      const uint64_t budget = wait_budget_ns(err);
      uint32_t spins = 0;
      while (ld_acquire_u64(flags + base + j) < target) {
        if ((++spins & 15u) == 0) {
          if (error_raised(err)) return false;
          if (globaltimer_ns() - t0 > budget) {
            record_error(err, code);
            return false;
          }
        }
        __nanosleep(64);
      }
    }
  }
  return true;
}

// ----------------------------------------------------------------- TMA / bulk
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 4-byte asynchronous copy global -> shared (cp.async), grouped by commit.
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Plain (untiled) bulk copy global -> shared; dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// TMA tile store shared -> global (bulk-group completion).  Coordinates must be
// non-negative; the inner coordinate times the element size a multiple of 16.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N committed bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every committed bulk group of this thread has completed.
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Named barrier over `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ----------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive (once) on `bar` when every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor, SWIZZLE_NONE, K-major canonical layout
// ((8,m),(T,2k)):((16B,SBO),(1,LBO)): rows of one 8-row core matrix 16 bytes
// apart, 8-row groups SBO bytes apart, 16-byte K chunks LBO bytes apart.
__device__ __forceinline__ uint64_t smem_desc_k_noswizzle(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version for tcgen05
  return d;                 // base offset 0, layout type 0 (no swizzle)
}

// Shared-memory matrix descriptor, 128-byte swizzle, K-major: rows of 128 bytes,
// 8-row swizzle atoms SBO (=1024) bytes apart.  Advancing along K inside the
// 128-byte row is done by adding the byte offset to the start address.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(1u) << 16;  // LBO unused for swizzled K-major
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;  // SWIZZLE_128B
  return d;
}

// Shared-memory matrix descriptor for a K-major operand stored with the
// swizzle whose atom row equals the operand's row pitch: 32, 64 or 128 bytes
// per row (SWIZZLE_32B / 64B / 128B), 8-row atoms SBO = 8 * row_bytes apart,
// LBO = 16 bytes (the two 16-byte halves of one K = 32-byte step).  16-byte
// chunk j of row r sits at chunk position j ^ (((r * row_bytes) >> 7) &
// (row_bytes / 16 - 1)) counted from a 1024-byte aligned base.  The start may
// sit anywhere on a 16-byte boundary (a row offset for a conv tap, +32 bytes
// for the next K step): the tensor cores apply the swizzle to the absolute
// shared-memory address bits, so the base-offset field stays 0 (checked on
// B200: a start shifted by a non-multiple of 8 rows reads the right chunks with
// base offset 0 and the wrong ones with base offset (start >> 7) & 7).
__device__ __forceinline__ uint64_t smem_desc_k_swizzled(uint32_t saddr, uint32_t row_bytes) {
  const uint64_t layout = row_bytes == 128 ? 2u : (row_bytes == 64 ? 4u : 6u);
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;                                    // LBO: 16 bytes
  d |= (uint64_t)(((8u * row_bytes) >> 4) & 0x3FFFu) << 32;  // SBO: one 8-row atom
  d |= (uint64_t)1u << 46;                                    // descriptor version for tcgen05
  d |= layout << 61;
  return d;
}

// Chunk position of 16-byte chunk j in row `row` of a swizzled K-major array
// with `row_bytes` per row (the data layout smem_desc_k_swizzled reads).
__host__ __device__ __forceinline__ int swz_chunk(int64_t row, int j, int row_bytes) {
  return j ^ (int)(((row * row_bytes) >> 7) & (row_bytes / 16 - 1));
}

// Instruction descriptor (kind::f16 / kind::tf32 / kind::i8), dense, K-major A and B.
//   c_fmt: 0 F16, 1 F32, 2 S32;  a_fmt/b_fmt: f16 kinds 0 F16 1 BF16 2 TF32, i8 kinds 0 U8 1 S8
__host__ __device__ __forceinline__ constexpr uint32_t make_idesc(uint32_t c_fmt, uint32_t a_fmt, uint32_t b_fmt,
                                                                  uint32_t m, uint32_t n) {
  return (c_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 TMEM lanes x 32 bits, 16 consecutive columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 TMEM lanes x 32 bits, 8 consecutive columns -> 8 registers per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

// Programmatic dependent launch.  Every kernel of this library is launched
// with programmatic stream serialisation allowed, so the next kernel may start
// its independent prologue while this one drains.  pdl_wait() blocks until the
// preceding grid has completed and its memory is visible: it must come before
// the first read of a predecessor's output and the first write of anything a
// predecessor may still read.  pdl_launch_dependents() lets the next grid be
// scheduled (its CTAs then wait in their own pdl_wait()).  Both are no-ops
// when the kernel was launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

}  // namespace emx
