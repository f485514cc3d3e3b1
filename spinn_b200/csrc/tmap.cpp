// tmap.cpp -- TMA tensor-map encoding, per-device properties, error state.
#include <cstdarg>
#include <mutex>
#include <vector>

#include "internal.h"

namespace spinn {

// ------------------------------------------------------------------ error state
static thread_local char g_err[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
const char* get_error() { return g_err; }

// ------------------------------------------------------------------ driver entry points
using PFN_tiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
using PFN_im2col = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const int*, const int*, cuuint32_t, cuuint32_t,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_tiled g_tiled = nullptr;
static PFN_im2col g_im2col = nullptr;
static int g_driver_version = 0;
static std::once_flag g_once;

static void load_entry_points() {
  cudaDriverEntryPointQueryResult q;
  void* p = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_tiled = reinterpret_cast<PFN_tiled>(p);
  p = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_im2col = reinterpret_cast<PFN_im2col>(p);
  cudaDriverGetVersion(&g_driver_version);
}

// Drivers up to 13.1 encode tensors smaller than 128 KiB with a bit that has to be cleared
// (the same adjustment CUTLASS makes in cute/atom/copy_traits_sm90_tma.hpp and
// copy_traits_sm90_im2col.hpp).
static void small_tensor_fixup(CUtensorMap* map, uint64_t span_bytes) {
  if (g_driver_version <= 13010 && span_bytes < 131072) {
    reinterpret_cast<uint64_t*>(map)[1] &= ~(1ull << 21);
  }
}

int encode_tiled_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swizzle) {
  std::call_once(g_once, load_entry_points);
  if (!g_tiled) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return SPINN_CUDA_ECUDA;
  }
  SPINN_CHECK_ARG((reinterpret_cast<uintptr_t>(base) & 15) == 0, "tensor map base %p not 16-B aligned", base);
  SPINN_CHECK_ARG(row_stride_bytes % 16 == 0, "tensor map row stride %llu not a multiple of 16",
                  (unsigned long long)row_stride_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): dims %llu x %llu stride %llu box %u x %u", (int)r,
              (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)row_stride_bytes, box_inner,
              box_outer);
    return SPINN_CUDA_ECUDA;
  }
  small_tensor_fixup(map, row_stride_bytes * outer);
  return 0;
}

int encode_tiled_3d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t planes,
                    uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  std::call_once(g_once, load_entry_points);
  if (!g_tiled) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return SPINN_CUDA_ECUDA;
  }
  SPINN_CHECK_ARG((reinterpret_cast<uintptr_t>(base) & 15) == 0, "tensor map base %p not 16-B aligned", base);
  SPINN_CHECK_ARG(row_stride_bytes % 16 == 0, "tensor map row stride not a multiple of 16");
  cuuint64_t dims[3] = {inner, outer, planes};
  cuuint64_t strides[2] = {row_stride_bytes, row_stride_bytes * outer};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    return SPINN_CUDA_ECUDA;
  }
  small_tensor_fixup(map, row_stride_bytes * outer * planes);
  return 0;
}

int encode_nhwc_window(CUtensorMap* map, const void* base, int n, int h, int w, int cpad, uint32_t box_c,
                       uint32_t box_w, uint32_t box_h) {
  std::call_once(g_once, load_entry_points);
  if (!g_tiled) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return SPINN_CUDA_ECUDA;
  }
  SPINN_CHECK_ARG((reinterpret_cast<uintptr_t>(base) & 15) == 0, "tensor map base %p not 16-B aligned", base);
  SPINN_CHECK_ARG(cpad % 4 == 0 && (box_c * 4) % 16 == 0, "NHWC window: channel stride %d / box %u", cpad, box_c);
  cuuint64_t dims[4] = {(cuuint64_t)cpad, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)n};
  cuuint64_t strides[3] = {(cuuint64_t)cpad * 4, (cuuint64_t)cpad * 4 * w, (cuuint64_t)cpad * 4 * w * h};
  cuuint32_t box[4] = {box_c, box_w, box_h, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (NHWC window) failed (%d): nhwc %d %d %d %d box %u %u %u", (int)r, n, h, w,
              cpad, box_c, box_w, box_h);
    return SPINN_CUDA_ECUDA;
  }
  small_tensor_fixup(map, (uint64_t)cpad * 4 * w * h * n);
  return 0;
}

int encode_im2col_4d(CUtensorMap* map, const void* base, int n, int h, int w, int c, int lower_w, int lower_h,
                     int upper_w, int upper_h, int channels_per_pixel, int pixels_per_column, int stride_w,
                     int stride_h, CUtensorMapSwizzle swizzle) {
  std::call_once(g_once, load_entry_points);
  if (!g_im2col) {
    set_error("cuTensorMapEncodeIm2col unavailable from the driver");
    return SPINN_CUDA_ECUDA;
  }
  SPINN_CHECK_ARG((reinterpret_cast<uintptr_t>(base) & 15) == 0, "im2col base %p not 16-B aligned", base);
  SPINN_CHECK_ARG((c * 4) % 16 == 0, "im2col channel count %d not a multiple of 4", c);
  SPINN_CHECK_ARG(lower_w >= -128 && lower_w <= 127 && lower_h >= -128 && lower_h <= 127 && upper_w >= -128 &&
                      upper_w <= 127 && upper_h >= -128 && upper_h <= 127,
                  "im2col corners out of range");
  SPINN_CHECK_ARG(stride_w >= 1 && stride_w <= 8 && stride_h >= 1 && stride_h <= 8, "im2col stride out of range");
  cuuint64_t dims[4] = {(cuuint64_t)c, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)n};
  cuuint64_t strides[3] = {(cuuint64_t)c * 4, (cuuint64_t)c * 4 * w, (cuuint64_t)c * 4 * w * h};
  int lower[2] = {lower_w, lower_h};
  int upper[2] = {upper_w, upper_h};
  cuuint32_t estr[4] = {1, (cuuint32_t)stride_w, (cuuint32_t)stride_h, 1};
  CUresult r = g_im2col(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, lower,
                        upper, (cuuint32_t)channels_per_pixel, (cuuint32_t)pixels_per_column, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeIm2col failed (%d): nhwc %d %d %d %d corners (%d,%d)/(%d,%d) cpp %d ppc %d", (int)r,
              n, h, w, c, lower_w, lower_h, upper_w, upper_h, channels_per_pixel, pixels_per_column);
    return SPINN_CUDA_ECUDA;
  }
  small_tensor_fixup(map, (uint64_t)c * 4 * w * h * n);
  return 0;
}

// ------------------------------------------------------------------ device properties / error flags
static std::mutex g_dev_mu;
static std::vector<int> g_sm_counts;
static std::vector<int*> g_err_flags;

int sm_count(int device) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if ((int)g_sm_counts.size() <= device) g_sm_counts.resize(device + 1, 0);
  if (!g_sm_counts[device]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    g_sm_counts[device] = v > 0 ? v : 148;
  }
  return g_sm_counts[device];
}

int* device_error_flag(int device) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if ((int)g_err_flags.size() <= device) g_err_flags.resize(device + 1, nullptr);
  if (!g_err_flags[device]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    g_err_flags[device] = p;
  }
  return g_err_flags[device];
}

int check_device_error_flag(int device, cudaStream_t stream) {
  int* f = device_error_flag(device);
  if (!f) return 0;
  int h = 0;
  SPINN_CUDA_TRY(cudaMemcpyAsync(&h, f, sizeof(int), cudaMemcpyDeviceToHost, stream));
  SPINN_CUDA_TRY(cudaStreamSynchronize(stream));
  if (h) {
    cudaMemsetAsync(f, 0, sizeof(int), stream);
    cudaStreamSynchronize(stream);
    set_error("a kernel's bounded wait expired (device error code %d)", h);
    return SPINN_CUDA_ETIMEOUT;
  }
  return 0;
}

}  // namespace spinn
