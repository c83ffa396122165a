// Host-side TMA tensor-map encoding (driver entry point fetched through the runtime, so the
// extension needs no direct libcuda symbol at load time).
#include <cuda.h>
#include <cuda_runtime.h>

#include "launchers.h"

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
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
}  // namespace

// 2-D map over a row-major matrix of packed FP4 (two per byte, K contiguous) that unpacks into the
// shared-memory layout of the tcgen05 8/6/4-bit kinds (16 values in the first 8 bytes of every 16-byte
// chunk) with the 128-byte swizzle: a box of 128 values x box_rows rows fills box_rows x 128 bytes.
int make_tmap_fp4_unpacked(void* out, const void* base, uint64_t k_elems, uint64_t rows, uint64_t row_bytes,
                           uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  const cuuint64_t dims[2] = {k_elems, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return (int)fn(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2,
                 const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// General tiled map of packed FP4 (K innermost, `rank` <= 5 dims, strides in bytes for dims 1..rank-1)
// with the same unpacking / swizzle; box[0] must be 128.
int make_tmap_fp4_unpacked_nd(void* out, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                              const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i) st[i - 1] = strides[i - 1];
  }
  return (int)fn(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, (cuuint32_t)rank,
                 const_cast<void*>(base), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// 2-D map over a row-major bf16 matrix (K contiguous) with the 128-byte swizzle: a box of 64 values x
// box_rows rows fills box_rows x 128 bytes in the K-major SW128 layout of tcgen05 operands.
int make_tmap_bf16_sw128(void* out, const void* base, uint64_t k_elems, uint64_t rows, uint64_t row_bytes,
                         uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  const cuuint64_t dims[2] = {k_elems, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return (int)fn(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
                 dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// 2-D map over a row-major matrix of bytes (E4M3 codes, K contiguous) with the 128-byte swizzle: a box of
// 128 values x box_rows rows fills box_rows x 128 bytes in the K-major SW128 layout of the 8-bit tcgen05
// kinds.  Rows past `rows` read as zero.
int make_tmap_u8_sw128(void* out, const void* base, uint64_t k_elems, uint64_t rows, uint64_t row_bytes,
                       uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  const cuuint64_t dims[2] = {k_elems, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return (int)fn(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base),
                 dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}
