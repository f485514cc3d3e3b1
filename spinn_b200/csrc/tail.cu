// tail.cu -- the end of one ResNet bottleneck block and the start of the next in one kernel.
//
//   y = act_e( t2 * W3^T + b3 + x )          (1x1 expand, fused residual; act_e: ReLU or none)
//   t = act_r( y * W1^T + b1 )               (the next block's 1x1 reduce; act_r: ReLU or none)
//
// These are two consecutive Conv nodes of a converted ResNet (graph_opt.c's Conv+Add(+ReLU)
// fusion on the expand, SPINN/graph_opt.c:304-421, and Conv+ReLU on the reduce, :235-288),
// each an op_conv2d call in the reference (SPINN/run_time/ops/conv/conv2d.c:92-232).  Run as
// two launches, the 1x1 reduce reads y back from HBM right after the expand wrote it; y is the
// widest tensor of the block (4x the channels of t2 and t).  Here a CTA owns 128 rows (pixels)
// and walks y's channels in chunks of 128:
//
//   E_j   y[:, 128j .. 128j+127] into a TMEM accumulator (two, alternating), K = channels of t2
//   epilogue E_j: bias, residual, activation, tf32 rounding; the chunk goes to shared memory in
//         the 128-B swizzled K-major layout -- which is both a TMA store box (y is written to
//         HBM once, for the next residual) and the A operand layout of the next MMA
//   R_j   t += y[:, chunk j] * W1[:, chunk j]^T into a third TMEM accumulator
//
// so y never comes back from HBM.  The accumulation order over K of every output element is
// the one the two separate launches use (k-blocks in increasing order), as is the epilogue
// arithmetic, so the results are those of the unfused path.
//
// Warp roles (384 threads, one persistent CTA per SM):
//   warp 0      TMA producer: a ring of 32 KiB stages in the order the MMA warp consumes them
//               (E_0, E_1, R_0, E_2, R_1, ..., R_last): an E stage holds a 128x32 box of t2
//               and a 128x32 box of W3, an R stage a N2x32 box of W1
//   warp 1      MMA issuer (E_{j+1} is issued before R_j, so the tensor pipe runs the next
//               expand chunk while the epilogue warps turn chunk j into the R operand)
//   warp 2      TMEM allocator (512 columns: acc_E x 2 = 256, acc_R <= 256)
//   warp 3      residual producer: x in 128x32 boxes through a 4-slot ring
//   warps 4..11 epilogue, two groups of four (one warp per TMEM lane quarter); group g takes
//               the 32-column blocks c with c % 2 == g of every chunk, then the same blocks of t
//
// Every mbarrier wait is bounded (4 s); on expiry the CTA drains what it issued, frees TMEM
// and returns with the device error flag set.
#include <algorithm>
#include <atomic>

#include "internal.h"
#include "ptx.cuh"

namespace spinn {
namespace {

constexpr int kBM = 128;
constexpr uint64_t kTimeoutNs = 4000000000ull;
constexpr uint64_t kDrainNs = 200000000ull;
constexpr uint32_t kSub = kBM * 32 * 4;    // one 128-row x 32-column fp32 block: 16 KiB
constexpr uint32_t kStage = 2 * kSub;      // 32 KiB
constexpr int kStages = 3;
constexpr uint32_t kYbuf = 4 * kSub;       // one 128-channel chunk of y: 64 KiB
constexpr int kResSlots = 4;               // two per epilogue group
constexpr int kThreads = 384;
constexpr uint32_t kSmem = kStages * kStage + kYbuf + kResSlots * kSub + 1024 + 1024;

struct TailParams {
  int M;          // rows (pixels)
  int k1_blocks;  // channels of t2 / 32
  int nch;        // channels of y / 128
  int n2;         // channels of t (32..256, multiple of 32)
  int act_e, act_r, round_out;
  const float* b3;  // [channels of y] or null
  const float* b1;  // [n2] or null
  int* err;
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t ns) {
  const bool ok = mbar_wait(bar, parity, abort, ns);
  return __all_sync(0xffffffffu, ok);
}
__device__ __forceinline__ bool warp_wait_backoff(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t ns) {
  const bool ok = mbar_wait_backoff(bar, parity, abort, ns);
  return __all_sync(0xffffffffu, ok);
}
__device__ __forceinline__ bool warp_aborted(volatile int* abort) { return __any_sync(0xffffffffu, *abort != 0); }

// K-major, 128-B swizzled operand of 32-column blocks `sub` bytes apart: descriptor of the
// 8-wide K slice k (k = 0 .. 4 * blocks - 1) starting at `addr`.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr, uint32_t sub, int k) {
  return make_smem_desc(addr + (uint32_t)((8 * k) / 32) * sub + (uint32_t)((8 * k) % 32) * 4, 16, 8 * 32 * 4, kSw128);
}

__global__ void __launch_bounds__(kThreads, 1)
    tail_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapW3,
                const __grid_constant__ CUtensorMap mapW1, const __grid_constant__ CUtensorMap mapR,
                const __grid_constant__ CUtensorMap mapY, const __grid_constant__ CUtensorMap mapT,
                const TailParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sRing = smem;                   // [kStages][32 KiB]
  uint8_t* sY = sRing + kStages * kStage;  // [4][16 KiB]: chunk j of y, K-major, swizzled
  uint8_t* sRes = sY + kYbuf;              // [kResSlots][16 KiB]
  uint64_t* full = reinterpret_cast<uint64_t*>(sRes + kResSlots * kSub);
  uint64_t* empty = full + kStages;
  uint64_t* tfullE = empty + kStages;  // [2] expand accumulator ready
  uint64_t* temptyE = tfullE + 2;      // [2] expand accumulator drained
  uint64_t* tfullR = temptyE + 2;      // reduce accumulator ready (per tile)
  uint64_t* temptyR = tfullR + 1;      // reduce accumulator drained (per tile)
  uint64_t* yfull = temptyR + 1;       // chunk of y in shared memory (per chunk)
  uint64_t* yempty = yfull + 1;        // its reduce MMAs have read it (per chunk)
  uint64_t* rfull = yempty + 1;        // [kResSlots]
  uint64_t* rempty = rfull + kResSlots;
  uint64_t* drain = rempty + kResSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (p.M + kBM - 1) / kBM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfullE[b], 1);
      mbar_init(&temptyE[b], 8);
    }
    mbar_init(tfullR, 1);
    mbar_init(temptyR, 8);
    mbar_init(yfull, 8);
    mbar_init(yempty, 1);
    for (int r = 0; r < kResSlots; ++r) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&mapA);
    prefetch_tmap(&mapW3);
    prefetch_tmap(&mapW1);
    prefetch_tmap(&mapR);
    prefetch_tmap(&mapY);
    prefetch_tmap(&mapT);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    int s = 0;
    uint32_t ph = 0;
    uint32_t armed = 0, armed_ph = 0;
    bool ok = true;
    auto next_stage = [&](uint32_t bytes) -> uint8_t* {
      if (!warp_wait(&empty[s], ph ^ 1, abort_flag, kTimeoutNs)) {
        ok = false;
        return nullptr;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], bytes);
        armed |= 1u << s;
        armed_ph = (armed_ph & ~(1u << s)) | (ph << s);
      }
      return sRing + s * kStage;
    };
    auto advance = [&]() {
      __syncwarp();
      if (++s == kStages) {
        s = 0;
        ph ^= 1;
      }
    };
    auto load_e = [&](int m0, int j) {
      for (int kb = 0; ok && kb < p.k1_blocks; ++kb) {
        uint8_t* st = next_stage(kStage);
        if (!ok) return;
        if (lane == 0) {
          tma_load_2d(&mapA, &full[s], st, kb * 32, m0);
          tma_load_2d(&mapW3, &full[s], st + kSub, kb * 32, j * 128);
        }
        advance();
      }
    };
    auto load_r = [&](int j) {
      for (int kb = 0; ok && kb < 4; ++kb) {
        uint8_t* st = next_stage((uint32_t)p.n2 * 128);
        if (!ok) return;
        if (lane == 0) tma_load_2d(&mapW1, &full[s], st, j * 128 + kb * 32, 0);
        advance();
      }
    };
    for (int t = blockIdx.x; ok && t < tiles && !warp_aborted(abort_flag); t += gridDim.x) {
      const int m0 = t * kBM;
      load_e(m0, 0);
      for (int j = 1; ok && j < p.nch; ++j) {
        load_e(m0, j);
        load_r(j - 1);
      }
      load_r(p.nch - 1);
    }
    if (warp_aborted(abort_flag) && lane == 0) {
      volatile int dummy = 0;
      for (int st = 0; st < kStages; ++st)
        if (armed & (1u << st)) mbar_wait(&full[st], (armed_ph >> st) & 1, &dummy, kDrainNs);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idescE = make_idesc_tf32(kBM, 128);
    const uint32_t idescR = make_idesc_tf32(kBM, (uint32_t)p.n2);
    const uint32_t ring = smem_u32(sRing), ybase = smem_u32(sY);
    int s = 0;
    uint32_t ph = 0;
    int ecnt = 0, rcnt = 0, tcnt = 0;
    bool ok = true, issued = false;
    auto issue_e = [&]() {
      const int b = ecnt & 1;
      if (!warp_wait(&temptyE[b], ((ecnt >> 1) & 1) ^ 1, abort_flag, kTimeoutNs)) {
        ok = false;
        return;
      }
      tc_fence_after();
      const uint32_t d = tmem_base + b * 128;
      for (int kb = 0; kb < p.k1_blocks; ++kb) {
        if (!warp_wait(&full[s], ph, abort_flag, kTimeoutNs)) {
          ok = false;
          return;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t st = ring + s * kStage;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_tf32(d, kmajor_desc(st, kSub, k), kmajor_desc(st + kSub, kSub, k), idescE, (kb | k) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        __syncwarp();
        issued = true;
        if (++s == kStages) {
          s = 0;
          ph ^= 1;
        }
      }
      if (lane == 0) umma_commit(&tfullE[b]);
      __syncwarp();
      ++ecnt;
    };
    auto issue_r = [&](int j) {
      if (j == 0 && !warp_wait(temptyR, (tcnt & 1) ^ 1, abort_flag, kTimeoutNs)) {
        ok = false;
        return;
      }
      if (!warp_wait(yfull, rcnt & 1, abort_flag, kTimeoutNs)) {
        ok = false;
        return;
      }
      tc_fence_after();
      const uint32_t d = tmem_base + 256;
      for (int kb = 0; kb < 4; ++kb) {
        if (!warp_wait(&full[s], ph, abort_flag, kTimeoutNs)) {
          ok = false;
          return;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t st = ring + s * kStage;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_tf32(d, kmajor_desc(ybase, kSub, kb * 4 + k), kmajor_desc(st, kSub, k), idescR,
                      (j | kb | k) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        __syncwarp();
        if (++s == kStages) {
          s = 0;
          ph ^= 1;
        }
      }
      if (lane == 0) umma_commit(yempty);
      __syncwarp();
      ++rcnt;
    };
    for (int t = blockIdx.x; ok && t < tiles && !warp_aborted(abort_flag); t += gridDim.x) {
      issue_e();
      for (int j = 1; ok && j < p.nch; ++j) {
        issue_e();
        if (ok) issue_r(j - 1);
      }
      if (ok) issue_r(p.nch - 1);
      if (ok && lane == 0) umma_commit(tfullR);
      __syncwarp();
      ++tcnt;
    }
    if (warp_aborted(abort_flag) && issued && lane == 0) {
      volatile int dummy = 0;
      umma_commit(drain);
      mbar_wait(drain, 0, &dummy, kDrainNs);
    }
    __syncwarp();
  } else if (warp == 3) {
    // ------------------------------------------------------------ residual producer
    if (lane == 0) {
      int count[2] = {0, 0};
      uint32_t armed = 0, armed_ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles && !*abort_flag; t += gridDim.x) {
        const int m0 = t * kBM;
        for (int j = 0; ok && j < p.nch; ++j)
          for (int c = 0; c < 4; ++c) {
            const int g = c & 1;
            const int slot = g * 2 + (count[g] & 1);
            const uint32_t ph = (count[g] >> 1) & 1;
            if (!mbar_wait(&rempty[slot], ph ^ 1, abort_flag, kTimeoutNs)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&rfull[slot], kSub);
            armed |= 1u << slot;
            armed_ph = (armed_ph & ~(1u << slot)) | (ph << slot);
            tma_load_2d(&mapR, &rfull[slot], sRes + slot * kSub, j * 128 + c * 32, m0);
            ++count[g];
          }
      }
      if (*abort_flag) {
        volatile int dummy = 0;
        for (int r = 0; r < kResSlots; ++r)
          if (armed & (1u << r)) mbar_wait(&rfull[r], (armed_ph >> r) & 1, &dummy, kDrainNs);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3, eg = (warp - 4) >> 2;
    int ecnt = 0, rc = 0, tcnt = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
      const int m0 = t * kBM, row0 = m0 + wq * 32;
      const bool rows_live = row0 < p.M;
      const int r = wq * 32 + lane;  // row inside the tile = TMEM lane
      // ---- chunks of y
      for (int j = 0; ok && j < p.nch; ++j) {
        const int b = ecnt & 1;
        float bias_reg[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) bias_reg[i] = p.b3 ? __ldg(p.b3 + j * 128 + (eg + 2 * i) * 32 + lane) : 0.0f;
        if (!warp_wait_backoff(&tfullE[b], (ecnt >> 1) & 1, abort_flag, kTimeoutNs)) {
          ok = false;
          break;
        }
        // the previous chunk's reduce MMAs have read the y buffer
        if (ecnt > 0 && !warp_wait_backoff(yempty, (ecnt - 1) & 1, abort_flag, kTimeoutNs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) tma_store_wait_read0();  // this warp's earlier stores have read their rows
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int c = eg + 2 * i;  // 32-column block of the chunk
          const int slot = eg * 2 + (rc & 1);
          if (!warp_wait(&rfull[slot], (rc >> 1) & 1, abort_flag, kTimeoutNs)) {
            ok = false;
            break;
          }
          uint8_t* blk = sY + c * kSub;
          if (rows_live) {
            uint32_t a[32];
            tmem_ld_32x32b_x32(tmem_base + b * 128 + c * 32 + ((uint32_t)(wq * 32) << 16), a);
            tmem_ld_wait();
            float v[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(a[k]) + __shfl_sync(0xffffffffu, bias_reg[i], k);
            const float* res_row = reinterpret_cast<const float*>(sRes + slot * kSub) + r * 32;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 x = *reinterpret_cast<const float4*>(res_row + ((q ^ (r & 7)) * 4));
              v[4 * q + 0] += x.x;
              v[4 * q + 1] += x.y;
              v[4 * q + 2] += x.z;
              v[4 * q + 3] += x.w;
            }
            if (p.act_e == 5) {
#pragma unroll
              for (int k = 0; k < 32; ++k) v[k] = v[k] < 0.0f ? 0.0f : v[k];
            }
            if (p.round_out) {
#pragma unroll
              for (int k = 0; k < 32; ++k) v[k] = to_tf32_rna(v[k]);
            }
            float* row = reinterpret_cast<float*>(blk) + r * 32;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<float4*>(row + ((q ^ (r & 7)) * 4)) =
                  make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          } else {
            // rows past the end of the tensor: zeros, so the reduce MMA reads defined values
            float* row = reinterpret_cast<float*>(blk) + r * 32;
#pragma unroll
            for (int q = 0; q < 8; ++q) *reinterpret_cast<float4*>(row + q * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&rempty[slot]);
          ++rc;
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && rows_live) {
            tma_store_2d(&mapY, blk + wq * 32 * 128, j * 128 + c * 32, row0);
            tma_store_commit();
          }
        }
        if (!ok) break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&temptyE[b]);
          mbar_arrive(yfull);
        }
        ++ecnt;
      }
      if (!ok) break;
      // ---- t = act_r(acc_R + b1), staged through the y buffer once its last reduce is done
      if (!warp_wait_backoff(tfullR, tcnt & 1, abort_flag, kTimeoutNs) ||
          !warp_wait_backoff(yempty, (ecnt - 1) & 1, abort_flag, kTimeoutNs)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int c = eg; c < p.n2 / 32; c += 2) {
        uint8_t* blk = sY + (c & 3) * kSub;
        if (lane == 0) tma_store_wait_read0();
        __syncwarp();
        if (rows_live) {
          const float bias_lane = p.b1 ? __ldg(p.b1 + c * 32 + lane) : 0.0f;
          uint32_t a[32];
          tmem_ld_32x32b_x32(tmem_base + 256 + c * 32 + ((uint32_t)(wq * 32) << 16), a);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(a[k]) + __shfl_sync(0xffffffffu, bias_lane, k);
          if (p.act_r == 1) {
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = v[k] < 0.0f ? 0.0f : v[k];
          }
          if (p.round_out) {
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = to_tf32_rna(v[k]);
          }
          float* row = reinterpret_cast<float*>(blk) + r * 32;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(row + ((q ^ (r & 7)) * 4)) =
                make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&mapT, blk + wq * 32 * 128, c * 32, row0);
            tma_store_commit();
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(temptyR);
      ++tcnt;
    }
    if (lane == 0) tma_store_wait_read0();  // global writes complete with the grid
    __syncwarp();
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (threadIdx.x == 0 && *abort_flag && p.err) atomicExch(p.err, 1);
}

}  // namespace

bool tail_fused_supported(const TailArgs& a, std::string* why) {
  auto fail = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (a.M <= 0) return fail("empty problem");
  if (a.k1 < 32 || a.k1 % 32) return fail("expand input channels must be a positive multiple of 32");
  if (a.n1 < 128 || a.n1 % 128) return fail("expand output channels must be a positive multiple of 128");
  if (a.n2 < 32 || a.n2 > 256 || a.n2 % 32) return fail("reduce output channels must be 32..256 in steps of 32");
  if (a.kpad3 != a.k1 || a.kpad1 != a.n1) return fail("weight K padding must equal the input channels");
  if ((a.act_e != 4 && a.act_e != 5) || (a.act_r != 0 && a.act_r != 1)) return fail("unsupported activations");
  for (const void* q : {(const void*)a.t2, (const void*)a.x, (const void*)a.w3, (const void*)a.w1, (const void*)a.y,
                        (const void*)a.t})
    if (!q || (reinterpret_cast<uintptr_t>(q) & 15)) return fail("operand missing or not 16-byte aligned");
  return true;
}

int tail_fused_launch(const TailArgs& a, cudaStream_t stream) {
  std::string why;
  if (!tail_fused_supported(a, &why)) {
    set_error("bottleneck tail: %s", why.c_str());
    return SPINN_CUDA_EINVAL;
  }
  int dev = 0;
  SPINN_CUDA_TRY(cudaGetDevice(&dev));
  CUtensorMap mA, mW3, mW1, mR, mY, mT;
  int rc = encode_tiled_2d(&mA, a.t2, (uint64_t)a.k1, (uint64_t)a.M, (uint64_t)a.k1 * 4, 32, kBM,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_tiled_2d(&mW3, a.w3, (uint64_t)a.kpad3, (uint64_t)a.n1, (uint64_t)a.kpad3 * 4, 32, 128,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_tiled_2d(&mW1, a.w1, (uint64_t)a.kpad1, (uint64_t)a.n2, (uint64_t)a.kpad1 * 4, 32,
                                (uint32_t)a.n2, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_tiled_2d(&mR, a.x, (uint64_t)a.n1, (uint64_t)a.M, (uint64_t)a.n1 * 4, 32, kBM,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_tiled_2d(&mY, a.y, (uint64_t)a.n1, (uint64_t)a.M, (uint64_t)a.n1 * 4, 32, 32,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_tiled_2d(&mT, a.t, (uint64_t)a.n2, (uint64_t)a.M, (uint64_t)a.n2 * 4, 32, 32,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    SPINN_CUDA_TRY(cudaFuncSetAttribute(tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    configured.fetch_or(bit);
  }
  TailParams p{};
  p.M = a.M;
  p.k1_blocks = a.k1 / 32;
  p.nch = a.n1 / 128;
  p.n2 = a.n2;
  p.act_e = a.act_e;
  p.act_r = a.act_r;
  p.round_out = a.round_out;
  p.b3 = a.b3;
  p.b1 = a.b1;
  p.err = a.err ? a.err : device_error_flag(dev);
  const int tiles = (a.M + kBM - 1) / kBM;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min(tiles, sm_count(dev)), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = getenv("SPINN_NO_PDL") ? 0 : 1;
  SPINN_CUDA_TRY(cudaLaunchKernelEx(&cfg, tail_kernel, mA, mW3, mW1, mR, mY, mT, p));
  SPINN_CUDA_TRY(cudaGetLastError());
  return 0;
}

}  // namespace spinn
