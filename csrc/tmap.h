// Host helpers: TMA tensor-map encoding through the driver entry point, and
// small launch utilities shared by the .cu files.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <mutex>
#include <set>
#include <utility>
#include <stdexcept>
#include <string>

namespace nq {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || p == nullptr) throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix [rows, cols] (cols contiguous,
// row stride `ld` elements), box {box_cols, box_rows}, 128-byte swizzle.
inline CUtensorMap make_tmap_2d_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld,
                                     int box_cols, int box_rows,
                                     CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base not 16B aligned");
  if ((ld * 2) % 16 != 0) throw std::runtime_error("TMA row stride not a multiple of 16 bytes");
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return m;
}

// 3-D bf16 tensor map: dims {d0 (contiguous), d1, d2} with byte strides s1, s2.
inline CUtensorMap make_tmap_3d_bf16(const void* base, int64_t d0, int64_t d1, int64_t d2,
                                     int64_t s1_elems, int64_t s2_elems, int b0, int b1, int b2,
                                     CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1),
                        static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1_elems) * 2,
                           static_cast<cuuint64_t>(s2_elems) * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(b0), static_cast<cuuint32_t>(b1),
                       static_cast<cuuint32_t>(b2)};
  cuuint32_t estr[3] = {1, 1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base not 16B aligned");
  if ((s1_elems * 2) % 16 != 0 || (s2_elems * 2) % 16 != 0)
    throw std::runtime_error("TMA stride not a multiple of 16 bytes");
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled(3d) failed: " + std::to_string(r));
  return m;
}

// 2-D fp32 tensor map over a row-major matrix [rows, cols] with row stride
// `ld` elements (TMA store / reduce-add destinations).
inline CUtensorMap make_tmap_2d_f32(const void* base, int64_t rows, int64_t cols, int64_t ld,
                                    int box_cols, int box_rows,
                                    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base not 16B aligned");
  if ((ld * 4) % 16 != 0) throw std::runtime_error("TMA row stride not a multiple of 16 bytes");
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled(2d f32) failed: " + std::to_string(r));
  return m;
}

// 3-D fp32 tensor map (used as the destination of TMA bulk reductions).
inline CUtensorMap make_tmap_3d_f32(const void* base, int64_t d0, int64_t d1, int64_t d2,
                                    int64_t s1_elems, int64_t s2_elems, int b0, int b1, int b2,
                                    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1),
                        static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1_elems) * 4,
                           static_cast<cuuint64_t>(s2_elems) * 4};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(b0), static_cast<cuuint32_t>(b1),
                       static_cast<cuuint32_t>(b2)};
  cuuint32_t estr[3] = {1, 1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base not 16B aligned");
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled(3d f32) failed: " + std::to_string(r));
  return m;
}

// Device-side error block shared by all kernels of the extension (int32
// words, one block per device): word 0 is the error code a kernel writes when
// it gives up on a bounded wait; words 2-3 hold the mbarrier wait limit and
// words 4-5 the peer-flag wait limit, in nanoseconds (u64), which the waits in
// sm100.cuh / peer.cuh read at run time.  Host code reads the code with
// `error_flag_read` (tests, watchdog), resets it with `error_flag_clear` and
// changes the limits with `wait_limits_set`.
int* error_flag_ptr();

#define NQ_CHECK_CUDA(expr)                                                          \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    if (_e != cudaSuccess) throw std::runtime_error(std::string("CUDA error: ") +    \
                                                    cudaGetErrorString(_e) + " at " + \
                                                    __FILE__ + ":" + std::to_string(__LINE__)); \
  } while (0)

constexpr int kMaxDevices = 64;

// Current device ordinal, checked against the per-device tables' size.
inline int current_device() {
  int dev = 0;
  NQ_CHECK_CUDA(cudaGetDevice(&dev));
  TORCH_CHECK(dev >= 0 && dev < kMaxDevices, "device ordinal ", dev, " beyond the library's limit of ",
              kMaxDevices);
  return dev;
}

// SM count of the current device (cached per device).
inline int num_sms() {
  static int n[kMaxDevices] = {};
  const int dev = current_device();
  if (n[dev] == 0) {
    int v = 0;
    NQ_CHECK_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
    n[dev] = v;
  }
  return n[dev];
}

// Raise a kernel's dynamic shared-memory limit on the current device.  The
// attribute belongs to the device's context, so a process that launches the
// kernel on several GPUs must set it on each; done once per (kernel, device).
inline void set_max_smem_once(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({kernel, dev})) return;
  NQ_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert({kernel, dev});
}

inline void check_bf16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bf16");
}

}  // namespace nq
