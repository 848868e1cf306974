// Host helpers: TMA tensor maps and the per-device error slot of the
// bounded-wait protocol (see sm100.cuh).
#pragma once

#include <ATen/ATen.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "sm100.cuh"

namespace eb {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status);
    TORCH_CHECK(err == cudaSuccess && status == cudaDriverEntryPointSuccess && ptr != nullptr,
                "cuTensorMapEncodeTiled is unavailable");
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

// The tensor-map encoder is a driver entry point: it needs a CUDA context
// current on the calling thread. A fresh thread (the autograd engine's device
// thread running a backward as its first CUDA work) may not have one yet, so
// bind the current device's primary context explicitly before encoding.
inline void bind_primary_context() {
  int device = 0;
  cudaGetDevice(&device);
  cudaSetDevice(device);
}

// bf16 tensor [B, L, H, D] viewed as (D, H, L, B); boxes of 64 x 1 x rows x 1
// with 128-byte swizzle (the canonical K-major / MN-major UMMA atom).
inline CUtensorMap make_bhld_map(void* base, int batch, int length, int heads, int dim, int rows) {
  bind_primary_context();
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(length), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(dim) * 2, static_cast<cuuint64_t>(heads) * dim * 2,
                           static_cast<cuuint64_t>(length) * heads * dim * 2};
  cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(rows), 1};
  cuuint32_t elem[4] = {1, 1, 1, 1};
  CUresult res = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box, elem,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with ", static_cast<int>(res));
  return map;
}

// Row-major bf16 matrix [rows, cols] (cols contiguous) with boxes of
// 64 columns x box_rows rows, 128-byte swizzle.
inline CUtensorMap make_matrix_map(const void* base, int64_t rows, int64_t cols, int64_t row_stride_elems,
                                   int box_rows) {
  bind_primary_context();
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t elem[2] = {1, 1};
  CUresult res = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                                      strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with ", static_cast<int>(res));
  return map;
}

// bf16 tensor [planes, rows, cols] (cols contiguous, dense) with boxes of
// 64 columns x box_rows rows x 1 plane, 128-byte swizzle. `base` may be a
// peer GPU's memory mapped into this process (plain tiled loads only).
inline CUtensorMap make_plane_map(const void* base, int64_t planes, int64_t rows, int64_t cols, int box_rows) {
  bind_primary_context();
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((cols * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(planes)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 2, static_cast<cuuint64_t>(rows) * cols * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult res = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                                      strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with ", static_cast<int>(res));
  return map;
}

// bf16 tensor [planes, rows, cols] (cols contiguous, dense) for TMA stores of
// unswizzled boxes of box_cols x box_rows x 1 (rows packed in shared memory).
// `base` may be a peer GPU's memory mapped into this process.
inline CUtensorMap make_store_plane_map(const void* base, int64_t planes, int64_t rows, int64_t cols, int box_cols,
                                        int box_rows) {
  bind_primary_context();
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((cols * 2) % 16 == 0 && (box_cols * 2) % 16 == 0, "TMA rows must be multiples of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(planes)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 2, static_cast<cuuint64_t>(rows) * cols * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult res = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                                      strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with ", static_cast<int>(res));
  return map;
}

// GEMM output [planes, rows, cols] (cols contiguous, row stride `ld` elements,
// plane stride `plane` elements; fp32 or bf16) for TMA stores / reductions of
// 32-row boxes whose rows are one swizzle span wide: 128 bytes (32 fp32 columns,
// 128-byte swizzle) for fp32, 64 bytes (32 bf16 columns, 64-byte swizzle) for bf16.
inline CUtensorMap make_epilogue_map(const void* base, int64_t planes, int64_t rows, int64_t cols, int64_t ld,
                                     int64_t plane, bool fp32) {
  bind_primary_context();
  const int elem = fp32 ? 4 : 2;
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * elem) % 16 == 0 && (plane * elem) % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(planes)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * elem, static_cast<cuuint64_t>(plane) * elem};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t unit[3] = {1, 1, 1};
  CUresult res = tensor_map_encoder()(&map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                      3, const_cast<void*>(base), dims, strides, box, unit,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                                      fp32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with ", static_cast<int>(res));
  return map;
}

// One error slot per device, allocated on first use and kept for the process
// (defined in attention/gated_entry.cu).
sm100::ErrorSlot* device_error_slot(int device);

}  // namespace eb
