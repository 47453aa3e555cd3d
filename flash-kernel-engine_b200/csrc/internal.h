// Host-side helpers shared by the kernel files of libflash_engine_b200.so:
// the device error word, cached device properties, the TMA descriptor encoder
// (resolved through the runtime's driver entry point, so the library does not
// link libcuda directly) and a one-time per-device smem opt-in.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fe {

// Device address of the library's error word on the current device
// (a __device__ variable in errors.cu). nullptr if it cannot be resolved.
unsigned* device_error_word();

// Number of SMs of the current device (cached per device).
int sm_count();

// Current device ordinal (cudaGetDevice) or 0.
int current_device();

// Encodes a 2-D tiled TMA descriptor with 128-byte swizzle over a row-major
// [rows, cols] matrix of 2-byte elements (row stride = row_stride_elems).
// box = {box_cols, box_rows}; box_cols * 2 must be <= 128 bytes.
cudaError_t encode_tma_2d_b16(CUtensorMap* map, const void* base, bool bf16, uint64_t cols,
                              uint64_t rows, uint64_t row_stride_elems, uint32_t box_cols,
                              uint32_t box_rows, bool swizzle128 = true);

// 3-D tiled TMA descriptor, 128-byte swizzle, over a contiguous [outer, rows, cols]
// tensor of 2-byte elements; box = {box_cols, box_rows, 1}. Rows past `rows` of an
// outer index read as zeros (they do not spill into the next outer slice).
cudaError_t encode_tma_3d_b16(CUtensorMap* map, const void* base, bool bf16, uint64_t cols,
                              uint64_t rows, uint64_t outer, uint32_t box_cols,
                              uint32_t box_rows);

// The same over fp32 elements (box_cols * 4 must be <= 128 bytes).
cudaError_t encode_tma_3d_f32(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                              uint64_t outer, uint32_t box_cols, uint32_t box_rows);

// Calls cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per
// (function, device).
cudaError_t ensure_smem_optin(const void* func, int bytes);

inline cudaError_t stream_ok(void* stream) {
  (void)stream;
  return cudaSuccess;
}

}  // namespace fe
