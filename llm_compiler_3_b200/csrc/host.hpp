// Host-side helpers shared by the C-ABI translation units of libnpu_b200.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/npu_b200.h"

namespace npu_b200 {

// Thread-local error message behind npu_b200_last_error().
int set_error(int code, const char* fmt, ...);
void clear_error();

// Returns NPU_B200_E_CUDA with a message if `e` is an error.
int check_cuda(cudaError_t e, const char* what);

#define NPU_TRY_CUDA(expr)                                   \
  do {                                                       \
    int _rc = ::npu_b200::check_cuda((expr), #expr);         \
    if (_rc != NPU_B200_OK) return _rc;                      \
  } while (0)

#define NPU_REQUIRE(cond, ...)                                       \
  do {                                                               \
    if (!(cond)) return ::npu_b200::set_error(NPU_B200_E_INVALID, __VA_ARGS__); \
  } while (0)

// Number of SMs of the current device (cached per device).
int sm_count();

// 2-D tensor map over a row-major FP16 matrix [rows, cols] with a box of
// box_cols x box_rows elements and the 128-byte swizzle.  box_cols * 2 must be
// <= 128.  The base must be 16-byte aligned and cols * 2 a multiple of 16.
int make_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                       uint32_t box_rows, uint32_t box_cols);

// 3-D tensor map over `planes` row-major FP16 matrices [rows, cols], plane_bytes
// apart, box box_cols x box_rows x 1, 128-byte swizzle.  Elements past `rows`
// in a plane (or past the last plane) load as zero.
int make_tensor_map_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                       uint64_t planes, uint64_t plane_bytes, uint32_t box_rows,
                       uint32_t box_cols);

// Graph plans (graph.cu): the state a context holds once npu_b200_load_graph
// succeeded, freed by graph_free; runtime.cu owns the context and exposes its
// device and graph slot.
struct GraphState;
void graph_free(GraphState* g);
int ctx_device(const npu_b200_ctx* c);
GraphState*& ctx_graph(npu_b200_ctx* c);

// Launch helper: enables programmatic dependent launch when `pdl` is set.
struct LaunchCfg {
  dim3 grid, block;
  size_t smem = 0;
  cudaStream_t stream = nullptr;
  bool pdl = false;
  int cluster = 1;  // thread-block cluster size along x (1 = no cluster)
};

template <typename... KArgs, typename... Args>
int launch(const LaunchCfg& c, void (*kernel)(KArgs...), Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = c.grid;
  cfg.blockDim = c.block;
  cfg.dynamicSmemBytes = c.smem;
  cfg.stream = c.stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (c.pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (c.cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = c.cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = n ? attr : nullptr;
  cfg.numAttrs = n;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...),
                    "cudaLaunchKernelEx");
}

}  // namespace npu_b200
