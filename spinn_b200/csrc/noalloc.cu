// noalloc.cu -- spinn_cuda_conv2d_noalloc: the tensor-core convolution with every
// temporary (NHWC copies of the input and residual, the NHWC result, the transformed weights,
// the padded bias, the device error word) carved out of one fixed file-scope device array.
//
// Why: SPINN targets systems that plan all memory ahead of time and allocate nothing while
// running (its runtime uses one static arena, ennf2c emits programs with a static arena and
// embedded weights).  A host like that, or one whose device memory is owned by another
// allocator, cannot call cudaMalloc at inference time.  This entry point calls no cudaMalloc,
// cudaFree or allocating library routine; its scratch is the array below, which the CUDA
// loader places on every GPU that loads this library and which stays there until exit.
//
// Contract:
//  * x, w, bias, residual and y are device pointers supplied by the caller (NCHW fp32, weights
//    OIHW), group 1.  The problem's scratch need must fit kNoAllocScratchBytes; larger
//    problems are rejected with SPINN_CUDA_EINVAL before any GPU work.
//  * Every unsupported problem is refused with SPINN_CUDA_EINVAL before any GPU work is
//    queued: scratch need above kNoAllocScratchBytes, a batch above 65535 (the layout
//    kernels put the image index in grid.z), a geometry the tensor-core kernel does not take
//    (stride above 8, im2col corners outside [-128, 127]), or a stream of another device.
//  * `stream` must belong to the current device (NULL: that device's legacy default stream).
//  * The first call on a device resolves the array's device address with
//    cudaGetSymbolAddress (with that device current).  Under lazy module loading (the CUDA
//    default since 12.2) that first call, and the first call that needs a kernel variant not
//    launched before, also loads code onto the GPU, which allocates device memory.  A host
//    that must not allocate at inference time therefore makes one call per device, of each
//    shape it will use, during its setup, or runs with CUDA_MODULE_LOADING=EAGER.
//  * Never call it while its stream (or any stream, under a global-mode capture) is being
//    captured: every call copies the device error word into host memory and waits for the
//    stream, and neither may happen inside a capture.
//  * Every call shares the array and overwrites it.  Calls that overlap on the GPU (other
//    streams, other host threads, the same device) race on it: serialize them.
//  * The call is synchronous: it waits for its stream and reports a kernel timeout as
//    SPINN_CUDA_ETIMEOUT.
#include <algorithm>
#include <mutex>
#include <string>

#include "internal.h"
#include "ptx.cuh"

namespace spinn {
namespace {

constexpr size_t kNoAllocScratchBytes = 32ull << 20;  // 32 MiB per GPU
constexpr size_t kErrSlot = 256;                      // first 256 B: the error word

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_addr[64] = {nullptr};

// Device address of the scratch array on the current device (resolved once per device).
int scratch_address(int dev, unsigned char** out) {
  if (dev < 0 || dev >= 64) {
    set_error("conv2d_noalloc: device ordinal %d out of range", dev);
    return SPINN_CUDA_EINVAL;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error("conv2d_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return SPINN_CUDA_ECUDA;
    }
    g_addr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_addr[dev]);
  return 0;
}

// OIHW weights -> [ocpad][kpad], k = (r*kw + s)*cpad + c, tf32 round-to-nearest; every
// element is written, padding with zeros, so nothing from an earlier call survives.
__global__ void weight_km_kernel(const float* __restrict__ w, float* __restrict__ out, int oc, int c, int kh, int kw,
                                 int cpad, int ocpad, int kpad) {
  const long total = (long)ocpad * kpad;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int o = (int)(i / kpad);
    const int k = (int)(i - (long)o * kpad);
    const int tap = k / cpad, ch = k - tap * cpad;
    float v = 0.0f;
    if (o < oc && ch < c && tap < kh * kw) {
      const int r = tap / kw, s = tap - r * kw;
      v = to_tf32_rna(w[(((size_t)o * c + ch) * kh + r) * kw + s]);
    }
    out[i] = v;
  }
}

size_t up256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace

extern "C" __attribute__((visibility("default"))) int spinn_cuda_conv2d_noalloc(
    const float* x, const float* w, const float* bias, const float* residual, float* y, int n, int c, int h, int wd,
    int oc, int kh, int kw, int stride_h, int stride_w, int pad_h, int pad_w, int fused_act, void* stream) {
  SPINN_CHECK_ARG(x && w && y, "conv2d_noalloc: x, w and y are required");
  SPINN_CHECK_ARG(n > 0 && c > 0 && h > 0 && wd > 0 && oc > 0 && kh > 0 && kw > 0 && stride_h > 0 && stride_w > 0 &&
                      pad_h >= 0 && pad_w >= 0,
                  "conv2d_noalloc: bad geometry");
  SPINN_CHECK_ARG(fused_act == 0 || fused_act == 1 || fused_act == 3 || fused_act == 4 || fused_act == 5,
                  "conv2d_noalloc: fused_act %d not supported", fused_act);
  const bool has_res = fused_act == 4 || fused_act == 5;
  SPINN_CHECK_ARG(!has_res || residual, "conv2d_noalloc: fused_act %d needs a residual", fused_act);
  const int oh = (h + 2 * pad_h - kh) / stride_h + 1, ow = (wd + 2 * pad_w - kw) / stride_w + 1;
  SPINN_CHECK_ARG(oh > 0 && ow > 0, "conv2d_noalloc: empty output");
  const int cpad = (c + 3) & ~3, ocpad = (oc + 3) & ~3;
  const int kpad = tc_num_kb(kh * kw * cpad) * 32;
  const size_t xb = up256((size_t)n * h * wd * cpad * 4), yb = up256((size_t)n * oh * ow * ocpad * 4);
  const size_t wb = up256((size_t)ocpad * kpad * 4), bb = up256((size_t)ocpad * 4);
  const size_t need = kErrSlot + xb + wb + bb + yb + (has_res ? yb : 0);
  if (need > kNoAllocScratchBytes) {
    set_error("conv2d_noalloc: problem needs %zu bytes of scratch; the fixed scratch is %zu bytes (32 MiB)", need,
              kNoAllocScratchBytes);
    return SPINN_CUDA_EINVAL;
  }
  SPINN_CHECK_ARG(n <= 65535, "conv2d_noalloc: batch %d above 65535", n);
  int dev = 0;
  SPINN_CUDA_TRY(cudaGetDevice(&dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (st) {
    int sdev = -1;
    SPINN_CUDA_TRY(cudaStreamGetDevice(st, &sdev));
    SPINN_CHECK_ARG(sdev == dev, "conv2d_noalloc: stream belongs to device %d, the current device is %d", sdev, dev);
  }
  unsigned char* base = nullptr;
  int rc = scratch_address(dev, &base);
  if (rc) return rc;
  int* err = reinterpret_cast<int*>(base);
  float* xs = reinterpret_cast<float*>(base + kErrSlot);
  float* ws = reinterpret_cast<float*>(base + kErrSlot + xb);
  float* bs = reinterpret_cast<float*>(base + kErrSlot + xb + wb);
  float* ys = reinterpret_cast<float*>(base + kErrSlot + xb + wb + bb);
  float* rs = has_res ? reinterpret_cast<float*>(base + kErrSlot + xb + wb + bb + yb) : nullptr;

  TcGemmArgs a;
  a.a_mode = 0;
  a.x = xs;
  a.n = n;
  a.h = h;
  a.w = wd;
  a.cpad = cpad;
  a.kh = kh;
  a.kw = kw;
  a.sh = stride_h;
  a.sw = stride_w;
  a.ph = pad_h;
  a.pw = pad_w;
  a.oh = oh;
  a.ow = ow;
  a.M = n * oh * ow;
  a.K = kh * kw * cpad;
  a.wt = ws;
  a.kpad = kpad;
  a.N = ocpad;
  a.bias = bias ? bs : nullptr;
  a.res = rs;
  a.ldr = ocpad;
  a.y = ys;
  a.ldy = ocpad;
  a.act = fused_act;
  a.err = err;
  std::string why;
  if (!tc_gemm_supported(a, &why)) {
    set_error("conv2d_noalloc: %s", why.c_str());
    return SPINN_CUDA_EINVAL;
  }

  // from here on GPU work is queued
  SPINN_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), st));
  rc = launch_nchw_to_nhwc(x, xs, n, c, h, wd, cpad, st, /*round_tf32=*/1);
  if (rc) return rc;
  const long wtotal = (long)ocpad * kpad;
  weight_km_kernel<<<(int)std::min<long>((wtotal + 255) / 256, 148 * 8), 256, 0, st>>>(w, ws, oc, c, kh, kw, cpad,
                                                                                       ocpad, kpad);
  SPINN_CUDA_TRY(cudaGetLastError());
  SPINN_CUDA_TRY(cudaMemsetAsync(bs, 0, (size_t)ocpad * 4, st));
  if (bias) SPINN_CUDA_TRY(cudaMemcpyAsync(bs, bias, (size_t)oc * 4, cudaMemcpyDeviceToDevice, st));
  if (has_res) {
    rc = launch_nchw_to_nhwc(residual, rs, n, oc, oh, ow, ocpad, st);
    if (rc) return rc;
  }
  rc = tc_gemm_launch(a, st);
  if (rc) return rc;
  rc = launch_nhwc_to_nchw(ys, y, n, oc, oh, ow, ocpad, st);
  if (rc) return rc;
  int h_err = 0;
  SPINN_CUDA_TRY(cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, st));
  SPINN_CUDA_TRY(cudaStreamSynchronize(st));
  if (h_err) {
    set_error("conv2d_noalloc: a kernel's bounded wait expired");
    return SPINN_CUDA_ETIMEOUT;
  }
  return 0;
}

}  // namespace spinn
