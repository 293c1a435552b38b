// Tensor-map encoding through the driver entry point (no libcuda link).
#include <cudaTypedefs.h>

#include "amc_internal.h"
#include "amc_tc.cuh"

namespace amc {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess && fn) encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  }
  return encode;
}
}  // namespace

int make_tmap_2d_f32_swz(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                         uint32_t box_cols, uint32_t box_rows, TmapSwizzle swizzle) {
  auto encode = encoder();
  if (!encode) return fail(AMC_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (((uintptr_t)base & 15) || ((pitch_elems * 4) & 15)) return fail(AMC_ERR_INVALID, "tensor map: base or pitch not 16-byte aligned");
  const uint32_t span = swizzle == TmapSwizzle::k32 ? 32 : swizzle == TmapSwizzle::kNone ? 0 : 128;
  // a swizzled box row spans exactly the swizzle width
  if ((box_cols * 4) % 16 || (span && box_cols * 4 != span)) return fail(AMC_ERR_INVALID, "tensor map: bad box width");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle == TmapSwizzle::k128         ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle == TmapSwizzle::k128Atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                : swizzle == TmapSwizzle::k32        ? CU_TENSOR_MAP_SWIZZLE_32B
                                                                     : CU_TENSOR_MAP_SWIZZLE_NONE;
  // out-of-range elements of a load read as zero (OOB_FILL_NONE)
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AMC_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return AMC_OK;
}

int make_tmap_2d_f32_box(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                         uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  return make_tmap_2d_f32_swz(map, base, rows, cols, pitch_elems, box_cols, box_rows,
                              swizzle128 ? TmapSwizzle::k128 : TmapSwizzle::kNone);
}

int make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                     uint32_t box_rows) {
  return make_tmap_2d_f32_box(map, base, rows, cols, pitch_elems, 32, box_rows, true);
}

}  // namespace amc
