// Host-side helpers: TMA tensor-map encoding through the driver entry point
// (so the extension does not link libcuda directly and still imports on a
// machine without a GPU), plus argument checks shared by the launchers.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>
#include <utility>

namespace gsb {

// Message building avoids <sstream>: the toolchain's libstdc++ differs from
// the one loaded at run time, and iostream objects crossed that boundary badly.
inline void gsb_str_append(std::string& s, const char* v) { s += v; }
inline void gsb_str_append(std::string& s, const std::string& v) { s += v; }
template <typename T>
inline void gsb_str_append(std::string& s, const T& v) { s += std::to_string(v); }
template <typename... Ts>
inline std::string gsb_str(const Ts&... vs) {
  std::string s;
  (gsb_str_append(s, vs), ...);
  return s;
}

#define GSB_CHECK(cond, ...)                                                     \
  do {                                                                           \
    if (!(cond)) {                                                               \
      throw std::runtime_error(::gsb::gsb_str("granite_switch_b200: ", __VA_ARGS__, \
                                              " (", __FILE__, ":", __LINE__, ")")); \
    }                                                                            \
  } while (0)

#define GSB_CUDA_CHECK(expr)                                                  \
  do {                                                                        \
    cudaError_t _e = (expr);                                                  \
    GSB_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " in " #expr); \
  } while (0)

bool pdl_enabled();
void count_launch();

// Launches `kernel` as a programmatic dependent of the kernel before it in `st` when
// programmatic launch is enabled: it may start while that kernel finishes, so it must
// execute griddepcontrol.wait (griddep_wait) before it reads anything an earlier kernel
// writes or writes anything an earlier kernel reads.
template <typename... KArgs, typename... Args>
inline void launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  count_launch();
  GSB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

inline PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    GSB_CHECK(e == cudaSuccess && p != nullptr && q == cudaDriverEntryPointSuccess,
              "cuTensorMapEncodeTiled is not available from the driver");
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with the given row
// stride (elements). The box is [box_rows, box_cols]; box_cols * 2 bytes must
// equal the swizzle span (128 B for SW128, 64 B for SW64).
inline CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t rows, uint64_t cols,
                                     uint64_t row_stride_elems, uint32_t box_cols,
                                     uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  GSB_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  GSB_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tma_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr),
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  GSB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r, " rows=",
            rows, " cols=", cols, " box=", box_rows, "x", box_cols);
  return m;
}

// 2-D tensor map of any element type (uint8 fp8 bytes, fp32 scales): [rows, cols]
// with the given row stride in elements; box [box_rows, box_cols].
inline CUtensorMap make_tmap_2d(const void* ptr, CUtensorMapDataType dtype, uint32_t elem_bytes, uint64_t rows,
                                uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows,
                                CUtensorMapSwizzle swizzle) {
  GSB_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  GSB_CHECK((row_stride_elems * elem_bytes) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tma_encode_fn()(&m, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  GSB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r, " rows=", rows, " cols=", cols);
  return m;
}

// 3-D bf16 tensor map over a stack of row-major matrices [planes, rows, cols]
// (contiguous); box [1, box_rows, box_cols].
inline CUtensorMap make_tmap_bf16_3d(const void* ptr, uint64_t planes, uint64_t rows, uint64_t cols,
                                     uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  GSB_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  GSB_CHECK((cols * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {cols, rows, planes};
  cuuint64_t strides[2] = {cols * 2, rows * cols * 2};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = tma_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides,
                               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  GSB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3-D) failed with code ", (int)r);
  return m;
}

}  // namespace gsb
