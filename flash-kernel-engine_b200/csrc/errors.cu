// Library-wide device state and host helpers (see internal.h).
#include <cudaTypedefs.h>

#include <mutex>
#include <stdio.h>

#include "internal.h"
#include "../../include/flash_engine_c.h"

namespace fe {

// OR-ed error bits written by kernels (ptx.cuh: kErrWaitTimeout, kErrBadBlock,
// kErrTmem). One word per device.
__device__ unsigned g_error_word = 0;

namespace {
constexpr int kMaxDevices = 64;
unsigned* g_err_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
std::mutex g_mu;

struct SmemOptin {
  const void* func;
  int device;
  int bytes;
};
SmemOptin g_optin[512];
int g_n_optin = 0;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
}  // namespace

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return 0;
  return d;
}

unsigned* device_error_word() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[d]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) return nullptr;
    g_err_ptr[d] = static_cast<unsigned*>(p);
  }
  return g_err_ptr[d];
}

int sm_count() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sm_count[d]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[d] = n;
  }
  return g_sm_count[d];
}

cudaError_t ensure_smem_optin(const void* func, int bytes) {
  const int d = current_device();
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (int i = 0; i < g_n_optin; ++i)
      if (g_optin[i].func == func && g_optin[i].device == d && g_optin[i].bytes >= bytes)
        return cudaSuccess;
  }
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_n_optin < 512) g_optin[g_n_optin++] = SmemOptin{func, d, bytes};
  return cudaSuccess;
}

cudaError_t encode_tma_2d_b16(CUtensorMap* map, const void* base, bool bf16, uint64_t cols,
                              uint64_t rows, uint64_t row_stride_elems, uint32_t box_cols,
                              uint32_t box_rows, bool swizzle128) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess || !fn)
        return cudaErrorNotSupported;
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return cudaErrorInvalidValue;
  if ((row_stride_elems * 2) % 16 != 0) return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

static cudaError_t encode_tma_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt,
                                 uint64_t elem, uint64_t cols, uint64_t rows, uint64_t outer,
                                 uint32_t box_cols, uint32_t box_rows) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess || !fn)
        return cudaErrorNotSupported;
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (cols * elem) % 16 != 0)
    return cudaErrorInvalidValue;
  cuuint64_t dims[3] = {cols, rows, outer};
  cuuint64_t strides[2] = {cols * elem, rows * cols * elem};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t encode_tma_3d_b16(CUtensorMap* map, const void* base, bool bf16, uint64_t cols,
                              uint64_t rows, uint64_t outer, uint32_t box_cols,
                              uint32_t box_rows) {
  return encode_tma_3d(map, base,
                       bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                       2, cols, rows, outer, box_cols, box_rows);
}

cudaError_t encode_tma_3d_f32(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                              uint64_t outer, uint32_t box_cols, uint32_t box_rows) {
  return encode_tma_3d(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, cols, rows, outer,
                       box_cols, box_rows);
}

}  // namespace fe

extern "C" int fe_get_device_errors(unsigned int* errors_out) {
  unsigned v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemcpyFromSymbol(&v, fe::g_error_word, sizeof(v));
  if (e != cudaSuccess) return static_cast<int>(e);
  const unsigned zero = 0;
  e = cudaMemcpyToSymbol(fe::g_error_word, &zero, sizeof(zero));
  if (errors_out) *errors_out = v;
  return static_cast<int>(e);
}

extern "C" const char* fe_get_version(void) { return "1.2.0-b200"; }

extern "C" int fe_print_device_info(int device_id) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device_id);
  if (e != cudaSuccess) return static_cast<int>(e);
  printf("Device %d: %s\n", device_id, prop.name);
  printf("  compute capability : %d.%d\n", prop.major, prop.minor);
  printf("  SMs                : %d\n", prop.multiProcessorCount);
  printf("  warp size          : %d\n", prop.warpSize);
  printf("  smem per block opt : %zu bytes\n", prop.sharedMemPerBlockOptin);
  printf("  smem per SM        : %zu bytes\n", prop.sharedMemPerMultiprocessor);
  printf("  L2 cache           : %d bytes\n", prop.l2CacheSize);
  printf("  global memory      : %zu bytes\n", prop.totalGlobalMem);
  return 0;
}
