// Library-wide C-ABI entry points: version, error reporting, device status,
// and the host helpers (tensor maps, SM count) the kernels' launchers share.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <utility>

#include "common.cuh"
#include "host.hpp"

namespace npu_b200 {

__device__ uint32_t g_device_error = 0;

namespace {
thread_local char t_error[1024] = {0};
}

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_error, sizeof(t_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { t_error[0] = 0; }

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return NPU_B200_OK;
  return set_error(e == cudaErrorMemoryAllocation ? NPU_B200_E_NOMEM : NPU_B200_E_CUDA,
                   "%s failed: %s (%d)", what, cudaGetErrorString(e), static_cast<int>(e));
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int make_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                       uint32_t box_rows, uint32_t box_cols) {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error(NPU_B200_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(NPU_B200_E_INVALID, "tensor map base %p is not 16-byte aligned", base);
  if ((cols * 2) % 16 != 0)
    return set_error(NPU_B200_E_INVALID, "row pitch %llu B is not a multiple of 16",
                     static_cast<unsigned long long>(cols * 2));
  if (box_cols * 2 > 128 || box_rows > 256 || box_rows == 0 || box_cols == 0)
    return set_error(NPU_B200_E_INVALID, "bad TMA box %ux%u", box_rows, box_cols);
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NPU_B200_E_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu",
                     static_cast<int>(r), static_cast<unsigned long long>(rows),
                     static_cast<unsigned long long>(cols));
  return NPU_B200_OK;
}

int make_tensor_map_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                       uint64_t planes, uint64_t plane_bytes, uint32_t box_rows,
                       uint32_t box_cols) {
  CUtensorMap probe;
  int rc = make_tensor_map_2d(&probe, base, 1, cols, 1, box_cols);  // loads the encoder, checks base/pitch
  if (rc) return rc;
  if (plane_bytes % 16 != 0 || plane_bytes < rows * cols * 2)
    return set_error(NPU_B200_E_INVALID, "plane pitch %llu B is not a multiple of 16 or too small",
                     static_cast<unsigned long long>(plane_bytes));
  if (box_rows > 256 || box_rows == 0 || rows == 0 || planes == 0)
    return set_error(NPU_B200_E_INVALID, "bad 3-D TMA box %u rows over %llu x %llu", box_rows,
                     static_cast<unsigned long long>(rows), static_cast<unsigned long long>(planes));
  cuuint64_t dims[3] = {cols, rows, planes};
  cuuint64_t strides[2] = {cols * 2, plane_bytes};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NPU_B200_E_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", static_cast<int>(r));
  return NPU_B200_OK;
}

}  // namespace npu_b200

using namespace npu_b200;

extern "C" int npu_b200_abi_version(void) { return NPU_B200_ABI_VERSION; }

extern "C" const char* npu_b200_last_error(void) { return t_error; }

extern "C" int npu_b200_device_status(uint32_t* h_bits) {
  if (!h_bits) return set_error(NPU_B200_E_INVALID, "h_bits is null");
  NPU_TRY_CUDA(cudaDeviceSynchronize());
  uint32_t bits = 0, zero = 0;
  NPU_TRY_CUDA(cudaMemcpyFromSymbol(&bits, g_device_error, sizeof(bits)));
  NPU_TRY_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
  *h_bits = bits;
  if (bits) return set_error(NPU_B200_E_DEVICE, "device error bits 0x%x", bits);
  return NPU_B200_OK;
}
