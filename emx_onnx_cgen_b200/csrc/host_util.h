// Host-side helpers shared by the kernel families: error formatting and the
// driver's tensor-map encoder (fetched through the runtime so the library
// does not link libcuda directly).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include "plan_format.h"

namespace emx {

inline int fail(char* msg, size_t n, int code, const char* fmt, ...) {
  if (msg && n) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, n, fmt, ap);
    va_end(ap);
  }
  return code;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D tile map over a row-major [rows][inner] byte-addressed matrix with row
// pitch `pitch_bytes`; box = box_inner x box_rows elements.  Out-of-range
// rows/columns read as zero.
inline int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, size_t elem_bytes, const void* base,
                        uint64_t inner, uint64_t rows, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_rows,
                        CUtensorMapSwizzle swz, char* msg, size_t n) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(msg, n, 4, "cuTensorMapEncodeTiled unavailable");
  if (((uintptr_t)base & 15u) || (pitch_bytes & 15u) || ((box_inner * elem_bytes) & 15u))
    return fail(msg, n, 5, "tensor map alignment (base %p pitch %llu box %u)", base,
                (unsigned long long)pitch_bytes, box_inner);
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(msg, n, 4, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return 0;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace emx
