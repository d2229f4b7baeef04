// Host-side TMA tensor-map construction.
//
// cuTensorMapEncodeTiled is a driver-API entry point; it is fetched through
// cudaGetDriverEntryPoint so that the extension does not link libcuda
// directly (the library then imports on machines without a GPU driver).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace pm {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Driver-API calls need the primary context current on the calling thread.
// Autograd's backward threads may not have it yet: cudaSetDevice makes it current.
inline void ensure_context() {
  static thread_local bool ready = false;
  if (!ready) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaSetDevice(dev);
    ready = true;
  }
}

inline EncodeTiledFn encode_tiled_fn() {
  ensure_context();
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || p == nullptr || q != cudaDriverEntryPointSuccess)
      throw std::runtime_error("placemoe_b200: cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Row-major bf16 matrix [rows, cols] with leading dimension `ld` (elements);
// box = {box_cols, box_rows}, 128-byte swizzle (64-byte for 32-column boxes).
inline CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols,
                                     uint32_t box_rows) {
  const CUtensorMapSwizzle swz = box_cols * 2 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((ld * 2) % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled(2d) failed: " + std::to_string((int)r));
  return m;
}

// Batched row-major bf16 matrices [batch, rows, cols]; box = {box_cols, box_rows, 1}.
inline CUtensorMap make_tmap_3d_bf16(const void* base, uint64_t batch, uint64_t rows, uint64_t cols, uint64_t ld,
                                     uint64_t batch_stride, uint32_t box_cols, uint32_t box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((ld * 2) % 16 != 0 || (batch_stride * 2) % 16 != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {cols, rows, batch};
  cuuint64_t strides[2] = {ld * 2, batch_stride * 2};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled(3d) failed: " + std::to_string((int)r));
  return m;
}

// fp32 output [rows, cols] (2-D) or [batch, rows, cols] (3-D) for TMA store / reduce-add,
// box = 32 x 32 (x 1) elements, 128-byte swizzle.
inline CUtensorMap make_tmap_f32_out(void* base, uint64_t batch, uint64_t rows, uint64_t cols, uint64_t ld,
                                     uint64_t batch_stride, bool three_d) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((ld * 4) % 16 != 0 || (three_d && (batch_stride * 4) % 16 != 0))
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  const cuuint32_t rank = three_d ? 3 : 2;
  cuuint64_t dims[3] = {cols, rows, batch};
  cuuint64_t strides[2] = {ld * 4, batch_stride * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, base, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled(f32 out) failed: " + std::to_string((int)r));
  return m;
}

// bf16 epilogue boxes: 32 rows x 32 columns, 64-byte swizzle.
inline CUtensorMap make_tmap_bf16_epi(const void* base, uint64_t rows, uint64_t cols, uint64_t ld) {
  return make_tmap_2d_bf16(base, rows, cols, ld, 32, 32);
}

}  // namespace pm
