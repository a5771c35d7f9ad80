// tma.cpp - CUtensorMap encoding through the driver entry point (the library links the CUDA
// runtime statically and does not link libcuda, so it loads on machines without a driver).
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

#include "kernels.h"

namespace dv3 {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn(std::string *err) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn && err) *err = "cuTensorMapEncodeTiled is unavailable";
  return fn;
}

bool encode_map_f16(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                    uint32_t box_cols, uint32_t box_rows, std::string *err) {
  return encode_map_f16_swizzled(map, base, cols, rows, box_cols, box_rows, 128, err);
}

bool encode_map_f16_swizzled(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                             uint32_t box_cols, uint32_t box_rows, uint32_t swizzle_bytes,
                             std::string *err) {
  auto fn = encode_fn(err);
  if (!fn) return false;
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default:
      if (err) *err = "tensor map: unsupported swizzle";
      return false;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0 || rows == 0 ||
      box_cols * 2 != swizzle_bytes || box_rows == 0 || box_rows > 256) {
    if (err) *err = "tensor map: base must be 16-byte aligned, rows of whole 16-byte units";
    return false;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                  strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) {
      char buf[128];
      std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
      *err = buf;
    }
    return false;
  }
  return true;
}

bool encode_map_f32(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                    uint32_t box_cols, uint32_t box_rows, std::string *err) {
  auto fn = encode_fn(err);
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 4) % 16 != 0 || rows == 0 ||
      box_cols * 4 != 128 || box_rows == 0 || box_rows > 256) {
    if (err) *err = "tensor map: base must be 16-byte aligned, rows of whole 16-byte units";
    return false;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 4};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides,
                  box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) {
      char buf[128];
      std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
      *err = buf;
    }
    return false;
  }
  return true;
}

bool encode_map_f16_images(CUtensorMap *map, const void *base, uint64_t cols, uint64_t n_images,
                           uint32_t box_rows, std::string *err) {
  auto fn = encode_fn(err);
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0 || n_images == 0 ||
      box_rows == 0 || box_rows > 256) {
    if (err) *err = "tensor map: base must be 16-byte aligned, rows of whole 16-byte units";
    return false;
  }
  const cuuint64_t dims[3] = {cols, static_cast<cuuint64_t>(kTokens), n_images};
  const cuuint64_t strides[2] = {cols * 2, cols * 2 * kTokens};
  const cuuint32_t box[3] = {64, box_rows, 1};
  const cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims,
                  strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) {
      char buf[128];
      std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
      *err = buf;
    }
    return false;
  }
  return true;
}

// 3D f32 view [slabs][rows][cols] of split-K partial slabs, box = 32 columns (128 bytes) x
// box_rows x 1 slab, 128-byte swizzle: stores past `rows` are clipped inside each slab.
bool encode_map_f32_slabs(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                          uint64_t slabs, uint32_t box_rows, std::string *err) {
  auto fn = encode_fn(err);
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 4) % 16 != 0 || rows == 0 ||
      slabs == 0 || box_rows == 0 || box_rows > 256) {
    if (err) *err = "tensor map: base must be 16-byte aligned, rows of whole 16-byte units";
    return false;
  }
  const cuuint64_t dims[3] = {cols, rows, slabs};
  const cuuint64_t strides[2] = {cols * 4, cols * 4 * rows};
  const cuuint32_t box[3] = {32, box_rows, 1};
  const cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void *>(base), dims,
                  strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) {
      char buf[128];
      std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
      *err = buf;
    }
    return false;
  }
  return true;
}

}  // namespace dv3
