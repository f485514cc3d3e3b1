// diag.cu -- tcgen05 instruction-rate diagnostic.
//
// Measures what one kind::tf32 MMA of shape M x N x 8 costs when both operands already sit in
// shared memory: one thread per CTA issues `iters` MMAs into one TMEM accumulator, cycling
// through the 32-float K extent of a row group, commits, and waits (bounded).  Every SM runs
// one CTA at once, so the figure is the per-SM issue cost under full-chip load.  The tile
// planner's cost model and the design of the narrow (N <= 64) layers rest on these numbers.
#include "internal.h"
#include "ptx.cuh"

namespace spinn {

namespace {

constexpr int kDiagABytes = 16384;  // 128 rows x 128 B
constexpr int kDiagBBytes = 32768;  // 256 rows x 128 B
// Dynamic shared memory per CTA: the operands, 1 KB for alignment, and padding that keeps
// one CTA per SM (two would not fit beside each other), so TMEM is never contended.
constexpr int kDiagSmem = 120 * 1024;

__global__ void __launch_bounds__(128, 1)
    mma_rate_kernel(int m, int n, int layout, int iters, long long* cycles, int* err) {
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = sm;
  uint8_t* sb = sm + kDiagABytes;
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tslot;
  __shared__ volatile int abort_flag;
  const int warp = threadIdx.x >> 5;
  float* f = reinterpret_cast<float*>(sm);
  for (int i = threadIdx.x; i < (kDiagABytes + kDiagBBytes) / 4; i += blockDim.x) f[i] = 0.001f * (i & 31);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tslot, 256);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tslot;
  if (threadIdx.x == 0) {
    // K-major operands.  layout 0: no swizzle, core matrices [row group][k core][8 rows x 16 B]
    // (LBO 128 B, SBO 1 KB, a k-step is two cores = 256 B).  layout 1/2/3: 32/64/128-byte
    // swizzle, one row of 32/64/128 B per output row, 8-row atoms (SBO = 8 rows), a k-step
    // advances 32 B inside the row.  All footprints fit 128 x 128 B (A) and 256 x 128 B (B).
    uint32_t lay, sbo, kadv, ksteps;
    if (layout == 0) {
      lay = kSwNone, sbo = 1024, kadv = 256, ksteps = 4;
    } else if (layout == 1) {
      lay = kSw32, sbo = 256, kadv = 0, ksteps = 1;
    } else if (layout == 2) {
      lay = kSw64, sbo = 512, kadv = 32, ksteps = 2;
    } else {
      lay = kSw128, sbo = 1024, kadv = 32, ksteps = 4;
    }
    const uint32_t lbo = layout == 0 ? 128 : 16;
    const uint64_t ad0 = make_smem_desc(smem_u32(sa), lbo, sbo, lay);
    const uint64_t bd0 = make_smem_desc(smem_u32(sb), lbo, sbo, lay);
    const uint32_t idesc = make_idesc_tf32((uint32_t)m, (uint32_t)n);
    const long long t0 = clock64();
    for (int i = 0; i < iters; ++i) {
      const uint32_t ks = ((uint32_t)(i % (int)ksteps) * kadv) >> 4;
      umma_tf32(tbase, ad0 + ks, bd0 + ks, idesc, i > 0 ? 1u : 0u);
    }
    umma_commit(&bar);
    const bool ok = mbar_wait(&bar, 0, &abort_flag, 1000000000ull);
    const long long t1 = clock64();
    cycles[blockIdx.x] = ok ? (t1 - t0) : -1;
    if (!ok) atomicExch(err, 2);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
  }
}

}  // namespace

int run_mma_rate_probe(int device, int m, int n, int layout, int iters, int* err, cudaStream_t s,
                       double* cycles_per_mma) {
  SPINN_CHECK_ARG(m == 64 || m == 128, "mma rate: M=%d (64 or 128)", m);
  SPINN_CHECK_ARG(n >= 16 && n <= 256 && n % 16 == 0, "mma rate: N=%d (16..256, multiple of 16)", n);
  SPINN_CHECK_ARG(layout >= 0 && layout <= 3, "mma rate: layout %d (0 none, 1/2/3 = 32/64/128 B swizzle)",
                  layout);
  SPINN_CHECK_ARG(iters >= 1 && iters <= (1 << 20), "mma rate: %d iterations outside [1, 2^20]", iters);
  SPINN_CHECK_ARG(cycles_per_mma != nullptr && err != nullptr, "mma rate: null output");
  const int grid = sm_count(device);
  SPINN_CHECK_ARG(grid > 0, "mma rate: no SM count for device %d", device);
  SPINN_CUDA_TRY(cudaFuncSetAttribute(mma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDiagSmem));
  long long* d_cycles = nullptr;
  SPINN_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&d_cycles), sizeof(long long) * grid, s));
  mma_rate_kernel<<<grid, 128, kDiagSmem, s>>>(m, n, layout, iters, d_cycles, err);
  cudaError_t le = cudaGetLastError();
  long long* h = new long long[grid];
  cudaError_t ce = le == cudaSuccess
                       ? cudaMemcpyAsync(h, d_cycles, sizeof(long long) * grid, cudaMemcpyDeviceToHost, s)
                       : le;
  cudaError_t fe = cudaFreeAsync(d_cycles, s);
  cudaError_t se = cudaStreamSynchronize(s);
  long long mx = 0;
  bool expired = false;
  for (int i = 0; ce == cudaSuccess && se == cudaSuccess && i < grid; ++i) {
    if (h[i] < 0) expired = true;
    mx = h[i] > mx ? h[i] : mx;
  }
  delete[] h;
  SPINN_CUDA_TRY(le);
  SPINN_CUDA_TRY(ce);
  SPINN_CUDA_TRY(fe);
  SPINN_CUDA_TRY(se);
  *cycles_per_mma = expired ? -1.0 : (double)mx / iters;
  return 0;
}

}  // namespace spinn
