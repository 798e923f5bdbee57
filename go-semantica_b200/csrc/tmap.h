// Host-side TMA tensor-map encoding shared by the tcgen05 kernels.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace sem {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major [rows][cols] 2-D map with a box of box_cols x box_rows; the base
// must be 16-byte aligned and a row a multiple of 16 bytes.
inline cudaError_t tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int esize, const void* base, int64_t rows,
                           int64_t cols, int box_cols, int box_rows, CUtensorMapSwizzle swz) {
  auto enc = tmap_encoder();
  if (!enc) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * esize) % 16) return cudaErrorMisalignedAddress;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * esize)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// General map of rank 2..5: dims[0] innermost (elements), strides[i] the byte
// stride of dimension i + 1 (multiples of 16), box[] in elements.
inline cudaError_t tmap_nd(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank,
                           const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                           CUtensorMapSwizzle swz) {
  auto enc = tmap_encoder();
  if (!enc) return cudaErrorNotSupported;
  if (rank < 2 || rank > 5 || (reinterpret_cast<uintptr_t>(base) & 15)) return cudaErrorInvalidValue;
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) {
      if (strides[i] % 16) return cudaErrorMisalignedAddress;
      st[i] = strides[i];
    }
  }
  CUresult r = enc(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace sem
