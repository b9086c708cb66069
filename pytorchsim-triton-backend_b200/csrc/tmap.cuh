// Tensor maps for TMA (cuTensorMapEncodeTiled through the runtime's driver entry point).
#pragma once
#include <cudaTypedefs.h>
#include "common.cuh"

namespace ptsim {

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row stride `ld` elements, box
// {box_cols (inner), box_rows}, zero fill outside the matrix; 128-byte swizzle (the MMA operand layout) or
// none (rows of up to 256 elements copied as they are).
static int make_tmap_2d(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                        uint32_t box_rows, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto enc = get_encode_tiled();
  if (enc == nullptr) return fail(PTSIM_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(PTSIM_E_ARGS, "TMA base address not 16-byte aligned");
  if ((ld * 2) % 16 != 0) return fail(PTSIM_E_ARGS, "TMA row stride %llu elements is not a multiple of 16 bytes", (unsigned long long)ld);
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PTSIM_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return PTSIM_OK;
}

}  // namespace ptsim
